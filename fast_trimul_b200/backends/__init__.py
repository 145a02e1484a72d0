"""Importing this package registers the backends: "torch" (universal) and "cuda"
(the sm_100a kernels through the C ABI), as fast_trimul/backends/__init__.py does."""

from . import torch_ref  # noqa: F401
from . import cuda_b200  # noqa: F401
