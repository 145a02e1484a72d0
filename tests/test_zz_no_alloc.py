"""The allocation-free entry point, ftm_trimul_fwd_static_scratch.

It exists for callers that cannot give the library a workspace: hosts that get a fixed
device-memory budget at start-up, or that must not call cudaMalloc mid-run because it
can synchronise the device. Its scratch is a device array built into the library.
These tests call it through the C ABI twice in a row (different inputs, so stale
contents from the first call would show) and compare each result with ftm_trimul_fwd
on the same inputs. Both run the same three kernels on the same inputs, so the results
must be bit-identical (torch.equal): any tolerance would hide a stale-scratch or offset
bug smaller than it. The file name makes pytest collect it last.
"""

import ctypes

import pytest
import torch

from tests.helpers import make_layer, make_mask

pytestmark = pytest.mark.gpu

needs_gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")


def _bind(lib):
    fn = lib.ftm_trimul_fwd_static_scratch
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6
    return fn


def _error_word(lib):
    fn = lib.ftm_static_scratch_error_word
    fn.restype = ctypes.c_void_p
    fn.argtypes = []
    return fn()


def _with_workspace(lib, m, z, mask, out_dtype):
    prob = m._impl.problem(z, out_dtype)
    packed, _ = m._impl.packed_params()
    nbytes = lib.ftm_workspace_bytes(prob)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    out = torch.empty(z.shape, dtype=out_dtype, device="cuda")
    st = lib.ftm_trimul_fwd(prob, z.data_ptr(), None if mask is None else mask.data_ptr(),
                            packed.data_ptr(), out.data_ptr(), ws.data_ptr(), nbytes,
                            torch.cuda.current_stream().cuda_stream)
    assert st == 0
    return out


@needs_gpu
@pytest.mark.parametrize("mode", ["outgoing", "incoming"])
def test_static_scratch_matches_workspace_path(mode):
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    fn = _bind(lib)
    m = make_layer(mode, True).cuda()
    packed, _ = m._impl.packed_params()
    gen = torch.Generator().manual_seed(11)
    for call, (B, N, mkind) in enumerate([(1, 256, "tail"), (2, 72, "pad")]):
        z = torch.randn(B, N, N, 128, generator=gen).to(torch.bfloat16).cuda()
        mask = make_mask(mkind, B, N, gen).float().cuda()
        want = _with_workspace(lib, m, z, mask, torch.float32)
        got = torch.full_like(want, float("nan"))
        prob = m._impl.problem(z, torch.float32)
        st = fn(ctypes.addressof(prob), z.data_ptr(), mask.data_ptr(), packed.data_ptr(),
                got.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert st == 0, _lib.status_string(st)
        assert lib.ftm_last_launch_count() == 3
        errw = _error_word(lib)
        assert errw
        s = torch.cuda.current_stream().cuda_stream
        assert lib.ftm_check_error(errw, None, s) == _lib.OK
        assert torch.equal(got, want), (call, (got - want).abs().max().item())


@needs_gpu
def test_static_scratch_rejects_oversized_problem():
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    fn = _bind(lib)
    m = make_layer("outgoing", True).cuda()
    z = torch.empty(1, 264, 264, 128, dtype=torch.bfloat16, device="cuda")  # > 65,536 positions
    prob = m._impl.problem(z, torch.float32)
    st = fn(ctypes.addressof(prob), z.data_ptr(), None, z.data_ptr(), z.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    assert st == _lib.BAD_WORKSPACE


@needs_gpu
def test_static_scratch_rejects_bad_arguments_before_queueing():
    """Null or misaligned buffers are rejected up front, with no launch."""
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    fn = _bind(lib)
    m = make_layer("outgoing", True).cuda()
    packed, _ = m._impl.packed_params()
    z = torch.randn(1, 64, 64, 128, device="cuda").to(torch.bfloat16)
    out = torch.empty(z.shape, dtype=torch.float32, device="cuda")
    prob = m._impl.problem(z, torch.float32)
    s = torch.cuda.current_stream().cuda_stream
    assert fn(ctypes.addressof(prob), z.data_ptr(), None, packed.data_ptr(), None, s) == _lib.BAD_ARGUMENT
    assert fn(ctypes.addressof(prob), z.data_ptr(), None, packed.data_ptr(), out.data_ptr() + 4,
              s) == _lib.BAD_ALIGN
    assert lib.ftm_last_launch_count() == 0
