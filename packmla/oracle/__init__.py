"""fp32 CPU references used as test oracles."""
from . import attention  # noqa: F401
