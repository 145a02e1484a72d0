"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle.

Tolerance (stated by the north star): max-abs <= 2e-2 and mean-relative <= 1e-3
against an fp32 reference of the same fp16 weights, measured on fp32 output (the
kernels can write fp32 directly; bf16 output rounding alone is ~1.4e-3 mean-rel).
"""

import numpy as np
import pytest
import torch

from tests.helpers import MAX_ABS, MEAN_REL, compare, make_layer, make_mask, oracle_out

pytestmark = pytest.mark.gpu

needs_gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")


def _native(m, z, mask, out_dtype=torch.float32):
    from fast_trimul_b200 import _lib
    m._impl.packed_params()                 # one-time weight packing (its own launch)
    n0 = _lib.stats["kernel_launches"]
    with torch.no_grad():
        out = m._impl._forward_native(z, mask, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert _lib.stats["kernel_launches"] - n0 == 3, "native path did not launch its kernels"
    return out


CASES = [
    # (mode, B, N, residual, mask kind, z dtype)
    ("outgoing", 1, 64, True, None, torch.float32),
    ("incoming", 1, 64, True, None, torch.float32),
    ("outgoing", 1, 8, True, "tail", torch.bfloat16),
    ("incoming", 1, 16, False, None, torch.float16),
    ("outgoing", 2, 24, False, "pad", torch.bfloat16),
    ("incoming", 2, 40, True, "pad", torch.bfloat16),
    ("outgoing", 1, 72, False, "tail", torch.float32),
    ("incoming", 1, 136, True, "tail", torch.bfloat16),
    ("outgoing", 1, 200, True, "frac", torch.float16),
    ("incoming", 1, 256, True, "tail", torch.bfloat16),     # config C2
    ("outgoing", 1, 256, False, "tail", torch.bfloat16),
    ("outgoing", 2, 128, True, "pad", torch.bfloat16),
]


@needs_gpu
@pytest.mark.parametrize("mode,B,N,residual,mkind,dt", CASES)
def test_native_matches_oracle(mode, B, N, residual, mkind, dt):
    m = make_layer(mode, residual).cuda()
    gen = torch.Generator().manual_seed(1)
    z = torch.randn(B, N, N, 128, generator=gen).to(dt)
    mask = make_mask(mkind, B, N, gen)
    ref = oracle_out(m, z, mask)
    out = _native(m, z.cuda(), None if mask is None else mask.cuda())
    assert out.dtype == torch.float32 and out.shape == z.shape
    max_abs, mean_rel = compare(out, ref)
    assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, (max_abs, mean_rel)


@needs_gpu
@pytest.mark.parametrize("mode", ["outgoing", "incoming"])
def test_native_c3_shape(mode):
    """Config C3: B=2, N=512, z*0.5, padding masks with lengths in [384, 512]."""
    m = make_layer(mode, True).cuda()
    gen = torch.Generator().manual_seed(3)
    z = (0.5 * torch.randn(2, 512, 512, 128, generator=gen)).to(torch.bfloat16)
    r = torch.zeros(2, 512)
    for b in range(2):
        r[b, :int(torch.randint(384, 513, (1,), generator=gen))] = 1
    mask = r[:, :, None] * r[:, None, :]
    ref = oracle_out(m, z, mask)
    out = _native(m, z.cuda(), mask.cuda())
    max_abs, mean_rel = compare(out, ref)
    assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, (max_abs, mean_rel)


@needs_gpu
@pytest.mark.parametrize("mode,mkind", [("outgoing", None), ("incoming", None),
                                        ("outgoing", "tail"), ("incoming", "pad")])
def test_native_c5_n2048(mode, mkind):
    """Config C5, the size every benchmark number is quoted on: B=1, N=2048, bf16
    z ~ N(0,1), random-init weights (all-ones mask as in C5, plus masked variants).
    The checker is the fp32 formula of the reference's torch path evaluated on 24 rows
    spread over the output (fast_trimul_b200.parity, pinned to the oracle by
    test_api_cpu.py::test_parity_rows_checker_matches_oracle); the full forward on
    the host would take minutes."""
    from fast_trimul_b200.parity import error_metrics, reference_rows, sample_rows
    m = make_layer(mode, True, ln_noise=False).cuda()
    N = 2048
    gen = torch.Generator(device="cuda").manual_seed(51)
    z = torch.randn(1, N, N, 128, device="cuda", generator=gen).to(torch.bfloat16)
    mask = make_mask(mkind, 1, N, torch.Generator().manual_seed(52))
    mask = torch.ones(1, N, N) if mask is None else mask
    mask = mask.cuda()
    out = _native(m, z, mask)
    rows = sample_rows(N, 24)
    ref = reference_rows(m._impl, z, mask, rows)
    max_abs, mean_rel = error_metrics(out[:, rows], ref)
    assert torch.isfinite(out).all()
    assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, (max_abs, mean_rel)


@needs_gpu
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_half_outputs(out_dtype):
    m = make_layer("outgoing", True).cuda()
    z = torch.randn(1, 96, 96, 128, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    ref = oracle_out(m, z, None)
    out = _native(m, z.cuda(), None, out_dtype=out_dtype)
    assert out.dtype == out_dtype
    max_abs, mean_rel = compare(out, ref)
    assert max_abs <= MAX_ABS and mean_rel <= 4e-3, (max_abs, mean_rel)


@needs_gpu
def test_golden_fixtures_d128():
    """The fixtures made by running the reference itself (tests/golden/)."""
    import glob
    import os
    from tests.test_oracle_golden import load_fixture
    files = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*d128*.npz")))
    assert files
    for f in files:
        fx = load_fixture(f)
        m = make_layer(fx["mode"], fx["residual"], ln_noise=False)
        m._impl.load_state_dict({k: torch.from_numpy(v) for k, v in fx["params"].items()})
        m = m.cuda()
        z = torch.from_numpy(fx["z"]).to(fx["z_dtype"])
        mask = None if fx["mask"] is None else torch.from_numpy(fx["mask"]).cuda()
        out = _native(m, z.cuda(), mask)
        max_abs, mean_rel = compare(out, fx["out_ref_fp32"].astype(np.float64))
        assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, (f, max_abs, mean_rel)


def _select_contraction(kernel, monkeypatch):
    """pair: 256 x 256 CTA-pair tiles; pair_wide: 256 x 512 (FTM_CT_NH=2); single: 128 x 256."""
    monkeypatch.setenv("FTM_CONTRACTION", "single" if kernel == "single" else "pair")
    monkeypatch.setenv("FTM_CT_NH", "2" if kernel == "pair_wide" else "1")


@needs_gpu
@pytest.mark.parametrize("kernel", ["pair", "pair_wide", "single"])
@pytest.mark.parametrize("L,m,n,k", [(3, 64, 64, 64), (2, 200, 136, 72), (4, 256, 512, 1024),
                                     (1, 1024, 1024, 1024), (2, 8, 8, 8), (3, 384, 640, 200)])
def test_contraction_vs_matmul(L, m, n, k, kernel, monkeypatch):
    """ftm_contraction alone against an fp32 matmul of the same fp16 operands."""
    _select_contraction(kernel, monkeypatch)
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(7)
    A = torch.randn(L, m, k, device="cuda", generator=g).half()
    B = torch.randn(L, n, k, device="cuda", generator=g).half()
    X = torch.full((L, m, n), float("nan"), device="cuda", dtype=torch.half)
    err = torch.zeros(64, dtype=torch.int32, device="cuda")
    st = lib.ftm_contraction(A.data_ptr(), B.data_ptr(), X.data_ptr(), L, m, k, n, 1,
                             err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 0, _lib.status_string(st)
    assert lib.ftm_check_error(err.data_ptr(), None, torch.cuda.current_stream().cuda_stream) == 0
    ref = torch.bmm(A.float(), B.float().transpose(1, 2))
    assert torch.isfinite(X).all()
    rel = ((X.float() - ref).abs().max() / ref.abs().max()).item()
    assert rel < 2e-3, rel


@needs_gpu
@pytest.mark.parametrize("kernel", ["pair", "pair_wide", "single"])
def test_contraction_blocked_b(kernel, monkeypatch):
    """B given as row blocks (the layout an all-gather of row shards produces)."""
    _select_contraction(kernel, monkeypatch)
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    L, m, k, rpb, blocks = 3, 256, 512, 256, 2
    g = torch.Generator(device="cuda").manual_seed(8)
    A = torch.randn(L, m, k, device="cuda", generator=g).half()
    Bb = torch.randn(blocks, L, rpb, k, device="cuda", generator=g).half()
    X = torch.empty(L, m, rpb * blocks, device="cuda", dtype=torch.half)
    err = torch.zeros(64, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.ftm_contraction(A.data_ptr(), Bb.data_ptr(), X.data_ptr(), L, m, k, rpb, blocks,
                               err.data_ptr(), s) == 0
    assert lib.ftm_check_error(err.data_ptr(), None, s) == 0
    Bfull = Bb.permute(1, 0, 2, 3).reshape(L, blocks * rpb, k)
    ref = torch.bmm(A.float(), Bfull.float().transpose(1, 2))
    rel = ((X.float() - ref).abs().max() / ref.abs().max()).item()
    assert rel < 2e-3, rel


@needs_gpu
def test_contraction_blocked_a_and_x():
    """A and X as row blocks too (the channel-sharded multi-GPU layout)."""
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    L, rpb, blocks, k = 3, 256, 3, 520
    g = torch.Generator(device="cuda").manual_seed(9)
    Ab = torch.randn(blocks, L, rpb, k, device="cuda", generator=g).half()
    Bb = torch.randn(blocks, L, rpb, k, device="cuda", generator=g).half()
    X = torch.empty(blocks, L, rpb, rpb * blocks, device="cuda", dtype=torch.half)
    err = torch.zeros(64, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.ftm_contraction_blocked(Ab.data_ptr(), Bb.data_ptr(), X.data_ptr(), L, rpb, blocks,
                                       k, rpb, blocks, err.data_ptr(), s) == 0
    assert lib.ftm_check_error(err.data_ptr(), None, s) == 0
    A = Ab.permute(1, 0, 2, 3).reshape(L, blocks * rpb, k).float()
    B = Bb.permute(1, 0, 2, 3).reshape(L, blocks * rpb, k).float()
    ref = torch.bmm(A, B.transpose(1, 2)).view(L, blocks, rpb, -1).permute(1, 0, 2, 3)
    rel = ((X.float() - ref).abs().max() / ref.abs().max()).item()
    assert rel < 2e-3, rel


@needs_gpu
@pytest.mark.parametrize("kernel", ["pair", "pair_wide"])
def test_contraction_kblocked(kernel, monkeypatch):
    """k split into source blocks (incoming mode's channel shards): A, B as
    [k block][L][m][k_rpb], X blocked by row owner."""
    _select_contraction(kernel, monkeypatch)
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    L, n, rows, blocks = 3, 512, 256, 2
    g = torch.Generator(device="cuda").manual_seed(10)
    Ab = torch.randn(blocks, L, n, rows, device="cuda", generator=g).half()
    Bb = torch.randn(blocks, L, n, rows, device="cuda", generator=g).half()
    X = torch.full((n // rows, L, rows, n), float("nan"), device="cuda", dtype=torch.half)
    err = torch.zeros(64, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.ftm_contraction_kblocked(Ab.data_ptr(), Bb.data_ptr(), X.data_ptr(), L, n, n, rows,
                                        blocks, rows, err.data_ptr(), s) == 0
    assert lib.ftm_check_error(err.data_ptr(), None, s) == 0
    A = Ab.permute(1, 2, 0, 3).reshape(L, n, blocks * rows).float()
    B = Bb.permute(1, 2, 0, 3).reshape(L, n, blocks * rows).float()
    ref = torch.bmm(A, B.transpose(1, 2)).view(L, n // rows, rows, n).permute(1, 0, 2, 3)
    assert torch.isfinite(X).all()
    rel = ((X.float() - ref).abs().max() / ref.abs().max()).item()
    assert rel < 2e-3, rel


@needs_gpu
@pytest.mark.parametrize("case", ["row_blocks_padded", "k_blocks_row_offset", "x_column_window"])
def test_contraction_general_strided(case):
    """ftm_contraction_general on the partial problems the sharded pipeline issues:
    A / B in 128-row blocks with padded row strides, k split into 128-wide blocks with
    A starting at a row offset inside each block, and X written into a column window of
    a wider matrix -- against an fp32 matmul of the same operands."""
    import ctypes
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(13)
    s = torch.cuda.current_stream().cuda_stream
    err = torch.zeros(64, dtype=torch.int32, device="cuda")
    d = _lib.ContractionLayout()
    L = 3
    if case == "row_blocks_padded":
        m, n, k, rpb, pad = 256, 384, 200, 128, 8
        Ab = torch.randn(m // rpb, L, rpb, k + pad, device="cuda", generator=g).half()
        Bb = torch.randn(n // rpb, L, rpb, k + pad, device="cuda", generator=g).half()
        A = Ab[..., :k].permute(1, 0, 2, 3).reshape(L, m, k)
        B = Bb[..., :k].permute(1, 0, 2, 3).reshape(L, n, k)
        X = torch.full((L, m, n), float("nan"), device="cuda", dtype=torch.half)
        d.L, d.m, d.n, d.k, d.k_per_block = L, m, n, k, 0
        d.a, d.a_rows_per_block = Ab.data_ptr(), rpb
        d.a_block_stride, d.a_l_stride, d.a_row_stride = L * rpb * (k + pad), rpb * (k + pad), k + pad
        d.b, d.b_rows_per_block = Bb.data_ptr(), rpb
        d.b_block_stride, d.b_l_stride, d.b_row_stride = L * rpb * (k + pad), rpb * (k + pad), k + pad
        d.x, d.x_rows_per_block, d.x_l_stride, d.x_row_stride = X.data_ptr(), 0, m * n, n
        got = X
    elif case == "k_blocks_row_offset":
        kb, nkb, rows_all, off, m = 128, 3, 512, 256, 256
        Ab = torch.randn(nkb, L, rows_all, kb, device="cuda", generator=g).half()
        Bb = torch.randn(nkb, L, rows_all, kb, device="cuda", generator=g).half()
        A = Ab[:, :, off:off + m].permute(1, 2, 0, 3).reshape(L, m, nkb * kb)
        B = Bb.permute(1, 2, 0, 3).reshape(L, rows_all, nkb * kb)
        X = torch.full((L, m, rows_all), float("nan"), device="cuda", dtype=torch.half)
        d.L, d.m, d.n, d.k, d.k_per_block = L, m, rows_all, nkb * kb, kb
        d.a, d.a_rows_per_block = Ab.data_ptr() + off * kb * 2, 0
        d.a_l_stride, d.a_row_stride, d.a_kblock_stride = rows_all * kb, kb, L * rows_all * kb
        d.b, d.b_rows_per_block = Bb.data_ptr(), 0
        d.b_l_stride, d.b_row_stride, d.b_kblock_stride = rows_all * kb, kb, L * rows_all * kb
        d.x, d.x_l_stride, d.x_row_stride = X.data_ptr(), m * rows_all, rows_all
        got = X
    else:
        m, n, k, wide, col0 = 128, 256, 256, 768, 256
        A = torch.randn(L, m, k, device="cuda", generator=g).half()
        B = torch.randn(L, n, k, device="cuda", generator=g).half()
        Xw = torch.full((L, m, wide), 5.0, device="cuda", dtype=torch.half)
        d.L, d.m, d.n, d.k, d.k_per_block = L, m, n, k, 0
        d.a, d.a_l_stride, d.a_row_stride = A.data_ptr(), m * k, k
        d.b, d.b_l_stride, d.b_row_stride = B.data_ptr(), n * k, k
        d.x, d.x_l_stride, d.x_row_stride = Xw.data_ptr() + col0 * 2, m * wide, wide
        got = Xw[:, :, col0:col0 + n]
    st = lib.ftm_contraction_general(ctypes.byref(d), err.data_ptr(), s)
    assert st == 0, _lib.status_string(st)
    assert lib.ftm_check_error(err.data_ptr(), None, s) == 0
    ref = torch.bmm(A.float(), B.float().transpose(1, 2))
    assert torch.isfinite(got).all()
    rel = ((got.float() - ref).abs().max() / ref.abs().max()).item()
    assert rel < 2e-3, rel
    if case == "x_column_window":        # nothing outside the window was written
        assert (Xw[:, :, :col0] == 5.0).all() and (Xw[:, :, col0 + n:] == 5.0).all()


@needs_gpu
@pytest.mark.parametrize("a_mn,b_mn", [(0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("L,m,n,k", [(3, 256, 256, 320), (2, 384, 128, 512), (1, 200, 136, 72)])
def test_contraction_mn_major_operands(a_mn, b_mn, L, m, n, k):
    """MN-major A and/or B (rows contiguous, k strided): the operand forms of the
    backward's dA = dX B and dB = dX^T A, against an fp32 matmul."""
    import ctypes
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(14)
    mp, np_ = (m + 7) // 8 * 8, (n + 7) // 8 * 8            # padded contiguous extents
    A = torch.randn(L, m, k, device="cuda", generator=g).half()
    B = torch.randn(L, n, k, device="cuda", generator=g).half()
    d = _lib.ContractionLayout()
    d.L, d.m, d.n, d.k, d.k_per_block = L, m, n, k, 0
    if a_mn:
        As = torch.zeros(L, k, mp, device="cuda", dtype=torch.half)
        As[:, :, :m] = A.transpose(1, 2)
        d.a, d.a_mn_major, d.a_l_stride, d.a_row_stride = As.data_ptr(), 1, k * mp, mp
    else:
        As = A.contiguous()
        d.a, d.a_l_stride, d.a_row_stride = As.data_ptr(), m * k, k
    if b_mn:
        Bs = torch.zeros(L, k, np_, device="cuda", dtype=torch.half)
        Bs[:, :, :n] = B.transpose(1, 2)
        d.b, d.b_mn_major, d.b_l_stride, d.b_row_stride = Bs.data_ptr(), 1, k * np_, np_
    else:
        Bs = B.contiguous()
        d.b, d.b_l_stride, d.b_row_stride = Bs.data_ptr(), n * k, k
    X = torch.full((L, m, n), float("nan"), device="cuda", dtype=torch.half)
    d.x, d.x_l_stride, d.x_row_stride = X.data_ptr(), m * n, n
    err = torch.zeros(64, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    st = lib.ftm_contraction_general(ctypes.byref(d), err.data_ptr(), s)
    assert st == 0, _lib.status_string(st)
    assert lib.ftm_check_error(err.data_ptr(), None, s) == 0
    ref = torch.bmm(A.float(), B.float().transpose(1, 2))
    assert torch.isfinite(X).all()
    rel = ((X.float() - ref).abs().max() / ref.abs().max()).item()
    assert rel < 2e-3, rel


@needs_gpu
def test_input_stage_incoming_row_shard():
    """Incoming mode on a non-square row shard (rows != cols): the transposed planes
    [c][i][k] of this shard's rows k, against the torch stand-in of the same stage."""
    from fast_trimul_b200 import _lib
    from fast_trimul_b200.distributed import NativeStageOps, TorchStageOps
    m = make_layer("incoming", True).cuda()
    rows, n = 128, 384
    g = torch.Generator(device="cuda").manual_seed(12)
    z = torch.randn(1, rows, n, 128, device="cuda", generator=g).to(torch.bfloat16)
    mask = torch.ones(1, rows, n, device="cuda")
    mask[:, :, n - 20:] = 0
    prob = m._impl.problem(z, torch.bfloat16)
    plane = 128 * rows * n
    a = torch.empty(plane, dtype=torch.float16, device="cuda")
    b = torch.empty_like(a)
    ops = NativeStageOps(m._impl, z.device)
    ops.input_stage(prob, z, mask, a, b)
    ops.check()
    ra, rb = torch.empty(plane, dtype=torch.float32, device="cuda"), torch.empty(plane, device="cuda")
    TorchStageOps(m._impl).input_stage(prob, z, mask, ra, rb)
    for got, ref in ((a, ra), (b, rb)):
        d = (got.float() - ref).abs()
        assert d.max().item() < 2e-2 and d.mean().item() / ref.abs().mean().item() < 3e-3


@needs_gpu
def test_output_canaries_and_error_word():
    """Writes stay inside `out` (guard regions untouched) and no wait timed out."""
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    m = make_layer("incoming", True).cuda()
    N, guard = 40, 4096
    z = torch.randn(1, N, N, 128, device="cuda").half()
    buf = torch.full((guard * 2 + z.numel(),), 7.0, device="cuda", dtype=torch.float32)
    out = buf[guard:guard + z.numel()].view(z.shape)
    packed, _ = m._impl.packed_params()
    prob = m._impl.problem(z, torch.float32)
    nbytes = lib.ftm_workspace_bytes(prob)
    ws = torch.empty(nbytes + 512, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    st = lib.ftm_trimul_fwd(prob, z.data_ptr(), None, packed.data_ptr(), out.data_ptr(),
                            ws.data_ptr(), nbytes, s)
    assert st == 0
    detail = __import__("ctypes").c_int(0)
    assert lib.ftm_check_error(lib.ftm_workspace_error_word(prob, ws.data_ptr()),
                               __import__("ctypes").byref(detail), s) == 0, detail.value
    assert (buf[:guard] == 7.0).all() and (buf[-guard:] == 7.0).all()
    assert torch.isfinite(out).all()


@needs_gpu
def test_bad_arguments_return_status():
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    m = make_layer("outgoing", True).cuda()
    z = torch.randn(1, 12, 12, 128, device="cuda").half()     # N % 8 != 0
    prob = m._impl.problem(z, torch.float32)
    assert lib.ftm_workspace_bytes(prob) == 0
    assert lib.ftm_trimul_fwd(prob, z.data_ptr(), None, z.data_ptr(), z.data_ptr(),
                              z.data_ptr(), 0, None) == _lib.BAD_SHAPE
