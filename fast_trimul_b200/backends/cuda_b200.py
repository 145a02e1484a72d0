"""The "cuda" backend: the sm_100a kernels behind the C ABI.

Replaces the reference's CuTe-DSL backend (fast_trimul/backends/cuda_cute.py:19-25):
same registration (N % 8 == 0, fp16/bf16/fp32 in, output in z's dtype), but the
work is one `ftm_trimul_fwd` call -- input stage, contraction, output stage --
with the mask and the casts folded into the kernels. fp32 z is converted to fp16
first, exactly where the reference calls `.half()` (functional.py:23).

A missing library raises `NativeLibraryMissing` (the dispatcher does not hide it);
shapes the kernels do not cover (d_z or d_c != 128) raise `NativeDeclined`, which
the dispatcher treats like a guard miss.
"""

import torch

from .. import _lib
from ..core.registry import backend

_FLOATS = {torch.float16, torch.bfloat16, torch.float32}


@backend("cuda", dtypes=_FLOATS, min_align=8, supports_graph=True)
class CudaB200Backend:
    def __init__(self, caps):
        self.caps = caps

    def execute(self, inp, params):
        z = inp.tensor
        if not z.is_cuda:
            raise _lib.NativeDeclined("cuda backend needs a CUDA tensor")
        _lib.load()
        if not params.native_supported():
            raise _lib.NativeDeclined("native kernels need d_z == d_c == 128")
        return params(z, inp.mask)
