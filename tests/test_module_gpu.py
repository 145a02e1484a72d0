"""Module-level GPU checks, mirroring the reference's own GPU tests
(fast_trimul tests/test_kernel_gpu.py:14-76 and tests/test_trimul.py:72-78): the
functional entry point equals the module, CUDA-graph replay equals eager, the
residual-free layer keeps shape and dtype, an N the kernels do not cover (N % 8 != 0)
falls back to the torch path, and gradients through the native forward are finite."""

import pytest
import torch

from tests.helpers import MAX_ABS, MEAN_REL, compare, make_layer, oracle_out

pytestmark = pytest.mark.gpu
needs_gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")


def _inputs(n, seed, dtype=torch.bfloat16, tail=5):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(1, n, n, 128, generator=g).to(dtype)
    mask = torch.ones(1, n, n)
    mask[:, :, n - tail:] = 0
    return z, mask


@needs_gpu
@pytest.mark.parametrize("mode", ["outgoing", "incoming"])
def test_functional_equals_module(mode):
    from fast_trimul_b200 import _lib
    from fast_trimul_b200.functional import triangle_multiplication
    m = make_layer(mode, True).cuda()
    z, mask = _inputs(64, 31)
    z, mask = z.cuda(), mask.cuda()
    with torch.no_grad():
        calls = _lib.stats["calls"]
        a = m(z, mask=mask)
        b = triangle_multiplication(z, m._impl, mask=mask)
    assert _lib.stats["calls"] >= calls + 2          # both went through the native kernels
    assert a.dtype == b.dtype == z.dtype and a.shape == z.shape
    assert torch.equal(a, b)


@needs_gpu
def test_graph_replay_equals_eager():
    m = make_layer("outgoing", True).cuda()
    z1, mask = _inputs(96, 32)
    z2, _ = _inputs(96, 33)
    z1, z2, mask = z1.cuda(), z2.cuda(), mask.cuda()
    with torch.no_grad():
        eager = m(z2, mask=mask).clone()
        m.graphed(z1, mask=mask)
        replay = m(z2, mask=mask)
    torch.cuda.synchronize()
    assert torch.equal(replay, eager)


@needs_gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_residual_false_shape_and_dtype(dtype):
    m = make_layer("outgoing", False).cuda()
    z, mask = _inputs(40, 34, dtype=dtype)
    with torch.no_grad():
        out = m(z.cuda(), mask=mask.cuda())
    assert out.shape == z.shape and out.dtype == dtype
    max_abs, mean_rel = compare(out.float().cpu(), oracle_out(m, z, mask))
    # the output is stored in z's dtype: rounding to bf16 alone contributes ~1e-3 mean-rel
    # on an output without the residual, so the bound here is the storage format's
    assert max_abs <= MAX_ABS and mean_rel <= (3e-3 if dtype == torch.bfloat16 else MEAN_REL), \
        (max_abs, mean_rel)


@needs_gpu
def test_unaligned_n_falls_back_to_torch():
    """N = 30 is not a multiple of 8 (the reference's min_align): the dispatcher routes
    it to the torch path, so the native kernels are not called."""
    from fast_trimul_b200 import _lib
    m = make_layer("outgoing", True).cuda()
    z, mask = _inputs(30, 35, tail=3)
    calls = _lib.stats["calls"]
    with torch.no_grad():
        out = m(z.cuda(), mask=mask.cuda())
    assert _lib.stats["calls"] == calls
    assert out.shape == z.shape and out.dtype == z.dtype
    max_abs, _ = compare(out.float().cpu(), oracle_out(m, z, mask))
    assert max_abs < 5e-2


@needs_gpu
def test_gradients_are_finite():
    m = make_layer("incoming", True).cuda()
    z, mask = _inputs(32, 36)
    z = z.cuda().requires_grad_(True)
    out = m(z, mask=mask.cuda())
    out.float().square().mean().backward()
    assert z.grad is not None and torch.isfinite(z.grad).all()
    grads = [p.grad for p in m._impl.parameters()]
    assert all(g is not None and torch.isfinite(g).all() for g in grads)


@needs_gpu
@pytest.mark.parametrize("backward", ["native", "recompute"])
@pytest.mark.parametrize("masked", [True, False])
@pytest.mark.parametrize("mode", ["outgoing", "incoming"])
def test_gradients_match_fp32_autograd(mode, masked, backward, monkeypatch):
    """Gradients of z and of all 16 parameters through the layer's training path match
    torch autograd of the fp32 module (the reference formula, _kernels.py:532-547, on
    fp32 copies of the same fp16 weights) with the same mask rules. Tolerance: the
    gradient's max-abs error relative to its largest entry, at fp16-storage level."""
    if backward == "recompute":
        monkeypatch.setenv("FTM_BACKWARD", "recompute")
    m = make_layer(mode, True).cuda()
    z, mask = _inputs(48, 37, dtype=torch.float32)
    z, mask = z.cuda(), mask.cuda()
    if not masked:
        mask = torch.ones_like(mask)
    g = torch.Generator(device="cuda").manual_seed(38)
    gout = torch.randn(z.shape, device="cuda", generator=g)
    zq = z.clone().requires_grad_(True)
    out = m(zq, mask=mask)
    out.float().backward(gout)
    got = [zq.grad] + [p.grad for p in m._impl._params()]

    ref = make_layer(mode, True).cuda()
    ref._impl.load_state_dict({k: v.float() for k, v in m._impl.state_dict().items()})
    ref._impl.float()
    params = [p.detach().clone().requires_grad_(True) for p in ref._impl._params()]
    zr = z.clone().requires_grad_(True)
    mm = mask.unsqueeze(-1)
    o = ref._impl._torch_forward(zr * mm, params) * mm
    o.backward(gout)
    want = [zr.grad] + [p.grad for p in params]
    from oracle.trimul_oracle import PARAM_NAMES       # the _params() order
    names = ["z"] + list(PARAM_NAMES)
    for name, a, b in zip(names, got, want):
        assert a is not None and torch.isfinite(a).all(), name
        scale = b.abs().max().item()
        err = (a.float() - b).abs().max().item()
        assert err <= 2e-2 * scale + 1e-6, (name, err, scale)
