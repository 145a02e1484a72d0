"""The PairFormer-style trunk on the GPU (the trunk configuration's layers at a smaller
N): the trunk whose 16 TriMul layers are FastTriangleMultiplication (native kernels)
agrees with the trunk whose TriMul layers are plain PyTorch, same weights, with and
without a padding mask. Both trunks run in bf16, so the bound is the trunk's own bf16
noise level, not the single-layer tolerance."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")
@pytest.mark.parametrize("masked", [False, True])
def test_trunk_fast_equals_torch_on_gpu(masked):
    from fast_trimul_b200 import _lib
    from fast_trimul_b200.pairformer import (PairFormerTrunk, copy_trimul_weights, fast_trimul,
                                             torch_trimul)
    torch.manual_seed(0)
    n, blocks = 128, 2
    ref = PairFormerTrunk(blocks, 384, 128, torch_trimul).cuda().to(torch.bfloat16).eval()
    fast = PairFormerTrunk(blocks, 384, 128, fast_trimul).cuda().to(torch.bfloat16).eval()
    for mod in fast.modules():
        if hasattr(mod, "_impl"):
            mod._impl.half()
    copy_trimul_weights(ref, fast)
    g = torch.Generator(device="cuda").manual_seed(9)
    s = torch.randn(1, n, 384, device="cuda", generator=g).to(torch.bfloat16)
    z = torch.randn(1, n, n, 128, device="cuda", generator=g).to(torch.bfloat16)
    mask = torch.ones(1, n, n, device="cuda", dtype=torch.bfloat16)
    if masked:
        mask[:, 112:] = 0
        mask[:, :, 112:] = 0
    calls = _lib.stats["calls"]
    with torch.no_grad():
        s1, z1 = ref(s, z, mask)
        s2, z2 = fast(s, z, mask)
    assert _lib.stats["calls"] >= calls + 2 * blocks      # the native layers ran
    for a, b in ((z1, z2), (s1, s2)):
        a, b = a.float(), b.float()
        assert torch.isfinite(b).all()
        rel = ((a - b).abs().mean() / a.abs().mean()).item()
        assert rel < 2e-2, rel
