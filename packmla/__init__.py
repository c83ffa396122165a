"""packmla: Blackwell-native (sm_100a) serving framework for MLA models with compressed
sparse attention and Packed (256-of-512) C4 KV records."""

__version__ = "0.1.0"
