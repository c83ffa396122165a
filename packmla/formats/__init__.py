"""Record formats: ABI constants and the CPU oracle codec."""
from . import abi, codec  # noqa: F401
