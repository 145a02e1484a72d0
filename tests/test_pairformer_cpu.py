"""The PairFormer-style trunk harness on CPU: swapping the TriMul layers for
FastTriangleMultiplication (same weights) leaves the trunk's output unchanged
within fp16 tolerance."""

import torch

from fast_trimul_b200.pairformer import (PairFormerTrunk, TriMulTorch, copy_trimul_weights,
                                         fast_trimul, torch_trimul)


def test_trimul_torch_matches_fast_layer():
    torch.manual_seed(0)
    ref = TriMulTorch(32, 32, "incoming")
    src = PairFormerTrunk(1, 16, 32, torch_trimul)
    dst = PairFormerTrunk(1, 16, 32, fast_trimul)
    src.blocks[0].tri_in = ref
    copy_trimul_weights(src, dst)
    z = torch.randn(1, 12, 12, 32)
    mask = torch.ones(1, 12, 12)
    mask[:, 10:] = 0
    mask[:, :, 10:] = 0
    with torch.no_grad():
        for mk in (None, mask):
            want = ref(z, mask=mk)
            got = dst.blocks[0].tri_in(z, mask=mk)
            assert (got.float() - want).abs().max() < 2e-2


def test_trunk_swap_preserves_output():
    torch.manual_seed(0)
    ref = PairFormerTrunk(2, 32, 32, torch_trimul)
    fast = PairFormerTrunk(2, 32, 32, fast_trimul)
    copy_trimul_weights(ref, fast)
    s = torch.randn(1, 12, 32)
    z = torch.randn(1, 12, 12, 32)
    mask = torch.ones(1, 12, 12)
    with torch.no_grad():
        s1, z1 = ref(s, z, mask)
        s2, z2 = fast(s, z, mask)
    rel = ((z2 - z1).abs().mean() / z1.abs().mean()).item()
    assert rel < 5e-3, rel
    assert ((s2 - s1).abs().mean() / s1.abs().mean()).item() < 5e-3
