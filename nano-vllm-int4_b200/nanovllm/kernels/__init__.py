"""sm_100a kernels behind the reference kernel module names."""
