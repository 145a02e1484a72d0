"""One-line integration (fast_trimul/integrations/patch.py:20-64): swap a library's
TriMul classes for adapters built on FastTriangleMultiplication. The adapter takes
the library constructor `(c_z, c_hidden=None, ...)`, ignores extra forward kwargs
and returns delta only (residual=False; the library adds its own residual).
Call before the library builds its model."""

import importlib

from ..ops.triangle import FastTriangleMultiplication


def _adapter(mode):
    class _FastTriMul(FastTriangleMultiplication):
        def __init__(self, c_z, c_hidden=None, *args, **kwargs):
            super().__init__(d_z=c_z, d_c=c_hidden or c_z, mode=mode, residual=False)

        def forward(self, z, mask=None, **kwargs):
            return super().forward(z, mask=mask)

    _FastTriMul.__name__ = f"FastTriMul_{mode}"
    return _FastTriMul


def _patch(module_path, outgoing, incoming):
    module = importlib.import_module(module_path)
    for names, mode in ((outgoing, "outgoing"), (incoming, "incoming")):
        for name in names:
            if hasattr(module, name):
                setattr(module, name, _adapter(mode))
    return module


def patch_openfold3():
    return _patch("openfold3.core.model.latent.base_blocks",
                  ["TriangleMultiplicationOutgoing", "FusedTriangleMultiplicationOutgoing"],
                  ["TriangleMultiplicationIncoming", "FusedTriangleMultiplicationIncoming"])


def patch_openfold():
    return _patch("openfold.model.evoformer",
                  ["TriangleMultiplicationOutgoing", "FusedTriangleMultiplicationOutgoing"],
                  ["TriangleMultiplicationIncoming", "FusedTriangleMultiplicationIncoming"])


def patch_boltz():
    return _patch("boltz.model.layers.pairformer",
                  ["TriangleMultiplicationOutgoing"], ["TriangleMultiplicationIncoming"])


def patch_protenix():
    return _patch("protenix.model.modules.pairformer",
                  ["TriangleMultiplicationOutgoing"], ["TriangleMultiplicationIncoming"])
