"""Low-level functional entry point, same contract as fast_trimul/functional.py:7-26.

    out = triangle_multiplication(z, params, mask=None)

z: (B, N, N, d_z) pair representation, any float dtype; params: the layer's
weights (`FastTriangleMultiplication._impl`); mask: optional (B, N, N).
Returns z's dtype. Semantics kept from the reference: z is multiplied by the mask
before the input LayerNorm, and the result is multiplied by the mask again.

On a CUDA tensor this is one C-ABI call (three sm_100a kernels) with the mask
product, the dtype casts and the residual done inside the kernels; elsewhere it
runs the torch formula with the reference's casts.
"""

import torch


def triangle_multiplication(z: torch.Tensor, params, mask: torch.Tensor = None) -> torch.Tensor:
    if z.is_cuda:
        return params(z, mask)      # native kernels (autograd-aware module forward)
    orig = z.dtype
    wdt = params.proj_a.weight.dtype
    if mask is not None:
        z = z * mask.unsqueeze(-1).to(z.dtype)
    out = params._torch_forward(z.to(wdt), params._params()).to(orig)
    if mask is not None:
        out = out * mask.unsqueeze(-1).to(out.dtype)
    return out
