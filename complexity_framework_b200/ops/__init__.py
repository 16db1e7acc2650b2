"""sm_100a operators (autograd-aware wrappers around the CUDA extension)."""
from ._ext import available, check_errors, load, require

__all__ = ["available", "check_errors", "load", "require"]
