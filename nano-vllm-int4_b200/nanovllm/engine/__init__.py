"""Engine: requests, scheduler, model runner."""
