"""Linear layers of the quantized path."""
