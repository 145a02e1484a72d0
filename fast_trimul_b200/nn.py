"""Backward-compatible re-exports (fast_trimul/nn.py:9-12)."""

from .integrations.loaders import _OPENFOLD_TO_FAST  # noqa: F401
from .ops.triangle import FastTriangleMultiplication

__all__ = ["FastTriangleMultiplication"]
