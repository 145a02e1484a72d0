"""fast_trimul_b200: the AlphaFold-family triangle multiplicative update on
hand-written sm_100a (B200) kernels, with the operator surface of fast_trimul.

- `FastTriangleMultiplication` -- the drop-in module (outgoing / incoming).
- `functional.triangle_multiplication` -- functional entry point.
- `accelerate` / `accelerated` -- scoped backend preference.
- `verify`, `list_backends`, `patch_openfold*`, `patch_boltz`, `patch_protenix`.
- `distributed.RowShardedTriMul` -- i-row sharding over GPUs with NCCL.

The kernels live in libfast_trimul_b200.so (C ABI: include/fast_trimul_b200.h).
"""

from . import functional
from . import backends
from . import integrations
from .ops.triangle import FastTriangleMultiplication
from .core.decorators import accelerate, accelerated
from .core.registry import list_backends
from .integrations.checks import verify
from .integrations.patch import patch_boltz, patch_openfold, patch_openfold3, patch_protenix
from . import nn

__all__ = ["FastTriangleMultiplication", "accelerate", "accelerated", "verify", "list_backends",
           "patch_openfold", "patch_openfold3", "patch_boltz", "patch_protenix", "functional",
           "backends", "integrations", "nn"]
__version__ = "0.1.0"
