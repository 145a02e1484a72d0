"""Failure detection on the GPU without a fault: a test switch (FTM_TEST_STALL=input)
makes the input stage withhold one tile load, so the bounded waits on it expire after
~2 s. The kernel must record the failing kernel / role / site in the device error word,
drain, free its tensor memory and exit; the host reads FTM_TIMEOUT; and the same CUDA
context must then run a normal forward correctly."""

import ctypes

import pytest
import torch

from tests.helpers import MAX_ABS, MEAN_REL, compare, make_layer, oracle_out

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")
def test_bounded_wait_expires_and_context_survives(monkeypatch):
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    m = make_layer("outgoing", True).cuda()
    z = torch.randn(1, 64, 64, 128, generator=torch.Generator().manual_seed(2)).half()
    zc = z.cuda()
    packed, _ = m._impl.packed_params()
    prob = m._impl.problem(zc, torch.float32)
    nbytes = lib.ftm_workspace_bytes(prob)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    out = torch.empty(zc.shape, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    errw = lib.ftm_workspace_error_word(prob, ws.data_ptr())
    assert errw

    # the input stage alone, with its own error word and buffers
    plane = 128 * 64 * 64
    a_cm = torch.empty(plane, dtype=torch.float16, device="cuda")
    b_cm = torch.empty(plane, dtype=torch.float16, device="cuda")
    zst = torch.empty(64 * 64 * 2, dtype=torch.float32, device="cuda")
    err = torch.zeros(64, dtype=torch.int32, device="cuda")
    monkeypatch.setenv("FTM_TEST_STALL", "input")
    assert lib.ftm_input_stage(prob, zc.data_ptr(), None, packed.data_ptr(), a_cm.data_ptr(),
                               b_cm.data_ptr(), zst.data_ptr(), err.data_ptr(), s) == _lib.OK
    detail = ctypes.c_int(0)
    st = lib.ftm_check_error(err.data_ptr(), ctypes.byref(detail), s)
    assert st == _lib.TIMEOUT, st
    kernel, role = detail.value >> 8, (detail.value >> 4) & 15
    assert kernel == 1, hex(detail.value)              # input stage
    assert role in (2, 3, 4), hex(detail.value)        # a consumer of the withheld tile
    assert lib.ftm_check_error(err.data_ptr(), None, s) == _lib.OK   # read-and-clear

    monkeypatch.delenv("FTM_TEST_STALL")
    assert lib.ftm_trimul_fwd(prob, zc.data_ptr(), None, packed.data_ptr(), out.data_ptr(),
                              ws.data_ptr(), nbytes, s) == _lib.OK
    assert lib.ftm_check_error(errw, None, s) == _lib.OK
    max_abs, mean_rel = compare(out, oracle_out(m, z, None))
    assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, (max_abs, mean_rel)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")
def test_module_forward_raises_after_device_timeout(monkeypatch):
    """The product path: a forward whose input stage waits expire raises
    NativeKernelError on that layer's next call (or at `check()`), with no
    synchronisation in the forward itself; afterwards the layer computes correctly."""
    from fast_trimul_b200 import _lib
    m = make_layer("outgoing", True).cuda()
    z = torch.randn(1, 64, 64, 128, generator=torch.Generator().manual_seed(3)).half()
    zc = z.cuda()
    with torch.no_grad():
        m(zc)
    m.check()
    monkeypatch.setenv("FTM_TEST_STALL", "input")
    with torch.no_grad():
        m(zc)                               # queued; its waits expire on the device
    torch.cuda.synchronize()
    with pytest.raises(_lib.NativeKernelError):
        with torch.no_grad():
            m(zc)                           # sees the recorded error before launching
    monkeypatch.delenv("FTM_TEST_STALL")
    m.check()                               # the error was reported once and cleared
    with torch.no_grad():
        out = m._impl._forward_native(zc, None, out_dtype=torch.float32)
    m.check()
    max_abs, mean_rel = compare(out, oracle_out(m, z, None))
    assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, (max_abs, mean_rel)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")
def test_static_scratch_error_word_reports_timeout(monkeypatch):
    """The allocation-free entry point reports an expired wait through its error word."""
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    m = make_layer("outgoing", True).cuda()
    z = torch.randn(1, 64, 64, 128, device="cuda").half()
    packed, _ = m._impl.packed_params()
    out = torch.empty(z.shape, dtype=torch.float32, device="cuda")
    prob = m._impl.problem(z, torch.float32)
    s = torch.cuda.current_stream().cuda_stream
    monkeypatch.setenv("FTM_TEST_STALL", "input")
    assert lib.ftm_trimul_fwd_static_scratch(prob, z.data_ptr(), None, packed.data_ptr(),
                                             out.data_ptr(), s) == _lib.OK
    errw = lib.ftm_static_scratch_error_word()
    assert errw
    detail = ctypes.c_int(0)
    assert lib.ftm_check_error(errw, ctypes.byref(detail), s) == _lib.TIMEOUT
    assert detail.value >> 8 == 1, hex(detail.value)
    monkeypatch.delenv("FTM_TEST_STALL")
    assert lib.ftm_trimul_fwd_static_scratch(prob, z.data_ptr(), None, packed.data_ptr(),
                                             out.data_ptr(), s) == _lib.OK
    assert lib.ftm_check_error(errw, None, s) == _lib.OK
