"""Operators: sm_100a CUDA kernels for CUDA tensors, fp32 oracle for CPU tensors."""
from ._ext import check_errors, error_word, ext  # noqa: F401
from . import kv, attention  # noqa: F401
