"""The universal backend: pure-torch triangle multiply on any device, the last link
of every fallback chain (fast_trimul/backends/torch_ref.py:18-35): cast z to the
weights' dtype, mask, `_torch_forward`, mask, cast back."""

import torch

from ..core.registry import backend

_ALL_FLOATS = {torch.float16, torch.bfloat16, torch.float32}


@backend("torch", dtypes=_ALL_FLOATS, min_align=1, supports_graph=False)
class TorchReferenceBackend:
    def __init__(self, caps):
        self.caps = caps

    def execute(self, inp, params):
        z = inp.tensor
        out_dtype = z.dtype
        wdt = params.proj_a.weight.dtype
        z = z.to(wdt)
        if inp.mask is not None:
            z = z * inp.mask.unsqueeze(-1).to(wdt)
        out = params._torch_forward(z, params._params())
        if inp.mask is not None:
            out = out * inp.mask.unsqueeze(-1).to(out.dtype)
        return out.to(out_dtype)
