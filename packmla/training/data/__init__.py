"""Training data: the hash-bound state cache, device staging, and capture from packmla's model."""
