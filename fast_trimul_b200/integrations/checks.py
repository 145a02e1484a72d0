"""`verify(source, reference)`: load a library module's weights through the `source`
remap and compare on a random probe (fast_trimul/integrations/checks.py:20-36;
N=128, atol = rtol = 1e-2, all-ones mask, residual=False)."""

import torch

from ..ops.triangle import FastTriangleMultiplication


def verify(source: str, reference, n: int = 128, d_z: int = 128, d_c: int = 128,
           mode: str = "outgoing", atol: float = 1e-2, rtol: float = 1e-2) -> bool:
    device = next(reference.parameters()).device
    fast = FastTriangleMultiplication(d_z=d_z, d_c=d_c, mode=mode, residual=False).to(device).eval()
    fast.load_weights(reference.state_dict(), source)
    z = torch.randn(1, n, n, d_z, device=device)
    mask = torch.ones(1, n, n, device=device)
    with torch.no_grad():
        want = reference(z, mask=mask).float()
        got = fast(z, mask=mask).float()
    return bool(torch.allclose(want, got, atol=atol, rtol=rtol))
