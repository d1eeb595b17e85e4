"""Hand-written sm_100a kernels and their plain-PyTorch reference forms."""
from ._ext import available, ext  # noqa: F401
