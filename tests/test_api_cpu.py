"""Host-side API, CPU only. Mirrors the reference's own unit tests
(tests/test_{registry,context,dispatch,decorators,loaders,patch,smoke}.py of fast_trimul)
against this package's implementation of the same interface."""

import sys
import types

import numpy as np
import pytest
import torch

import fast_trimul_b200 as ftm
from fast_trimul_b200.core import dispatch, registry
from fast_trimul_b200.core.context import BackendCapabilities, NormalizedInput, normalize
from fast_trimul_b200.core.decorators import accelerate, accelerated, active_backend
from fast_trimul_b200.core.registry import get_loader
from fast_trimul_b200.integrations import patch
from fast_trimul_b200.integrations.loaders import _OPENFOLD_TO_FAST
from fast_trimul_b200.ops.triangle import FastTriangleMultiplication


# ------------------------------------------------------------------ smoke / API
def test_public_api_exported():
    for name in ("FastTriangleMultiplication", "accelerate", "accelerated", "verify",
                 "list_backends", "patch_openfold", "patch_openfold3", "patch_boltz",
                 "patch_protenix", "functional"):
        assert hasattr(ftm, name)
    assert isinstance(ftm.__version__, str) and ftm.__version__
    assert hasattr(ftm.functional, "triangle_multiplication")
    assert {"torch", "cuda"} <= set(ftm.list_backends())


# ------------------------------------------------------------------ input guard
def _caps(dtypes, align=1):
    return BackendCapabilities(dtypes=dtypes, min_align=align)


def test_guard_rejects_non_4d_and_misaligned():
    assert normalize(torch.randn(4, 4), None, _caps({torch.float16})) is None
    assert normalize(torch.randn(1, 12, 12, 4), None, _caps({torch.float32}, 8)) is None
    assert normalize(torch.randn(1, 3, 3, 4), None, _caps({torch.float32})) is not None


def test_guard_accepts_and_casts():
    out = normalize(torch.randn(1, 8, 8, 4), None, _caps({torch.float32}, 8))
    assert isinstance(out, NormalizedInput) and out.shape == (1, 8, 8, 4)
    assert normalize(torch.randn(1, 8, 8, 4), None, _caps({torch.float16}, 8)).tensor.dtype == torch.float16
    z = torch.randn(1, 8, 8, 4).half()
    assert normalize(z, None, _caps({torch.float32}, 8)).tensor.dtype == torch.float32
    zb = torch.randn(1, 8, 8, 4).bfloat16()
    assert normalize(zb, None, _caps({torch.float16}, 8)).tensor.dtype == torch.float16


def test_guard_makes_contiguous():
    z = torch.randn(1, 8, 8, 4).transpose(1, 2)
    m = torch.ones(1, 8, 8).transpose(1, 2)
    out = normalize(z, m, _caps({torch.float32}, 8))
    assert out.tensor.is_contiguous() and out.mask.is_contiguous()
    assert all(isinstance(s, int) for s in out.strides)


# ------------------------------------------------------------------ dispatcher
def test_dispatch_order():
    cpu, gpu = torch.device("cpu"), torch.device("cuda")
    assert dispatch._order(cpu, "torch") == ["torch"]
    assert dispatch._order(cpu, "cuda") == ["cuda", "torch"]
    assert dispatch._order(cpu, "auto") == ["torch"]
    assert dispatch._order(gpu, "auto") == ["cuda", "torch"]
    with accelerated("torch"):
        assert dispatch._order(gpu, "auto") == ["torch"]


def test_dispatch_runs_registered_backend_and_falls_back():
    marker = object()

    @registry.backend("__ok", dtypes={torch.float32}, min_align=1)
    class _Ok:
        def __init__(self, caps):
            self.caps = caps

        def execute(self, inp, params):
            return marker

    @registry.backend("__bad", dtypes={torch.float32}, min_align=1)
    class _Bad:
        def __init__(self, caps):
            self.caps = caps

        def execute(self, inp, params):
            raise ValueError("declines")

    try:
        assert dispatch.run(torch.randn(1, 8, 8, 4), None, None, prefer="__ok") is marker
        # a generic failure falls to "torch", which then needs real params
        layer = FastTriangleMultiplication(4, 4, "outgoing")
        out = dispatch.run(torch.randn(1, 8, 8, 4), None, layer._impl, prefer="__bad")
        assert out.shape == (1, 8, 8, 4)
    finally:
        registry._BACKENDS.pop("__ok", None)
        registry._BACKENDS.pop("__bad", None)
    with pytest.raises(RuntimeError):
        dispatch.run(torch.randn(2, 2), None, None, prefer="torch")


def test_dispatch_does_not_hide_missing_native_library():
    from fast_trimul_b200 import _lib

    @registry.backend("__missing", dtypes={torch.float32}, min_align=1)
    class _Missing:
        def __init__(self, caps):
            self.caps = caps

        def execute(self, inp, params):
            raise _lib.NativeLibraryMissing("no .so")

    try:
        with pytest.raises(_lib.NativeLibraryMissing):
            dispatch.run(torch.randn(1, 8, 8, 4), None, None, prefer="__missing")
    finally:
        registry._BACKENDS.pop("__missing", None)


# ------------------------------------------------------------------ decorators
def test_scoped_backend():
    assert active_backend() == "auto"
    with accelerated("cuda"):
        assert active_backend() == "cuda"
        with accelerated("torch"):
            assert active_backend() == "torch"
        assert active_backend() == "cuda"
    assert active_backend() == "auto"

    @accelerate(backend="torch")
    def where():
        return active_backend()

    @accelerate
    def where_auto():
        return active_backend()

    assert where() == "torch" and where_auto() == "auto" and active_backend() == "auto"


# ------------------------------------------------------------------ registry / loaders
def test_registry_roundtrip():
    @registry.weights_for("__src")
    def _l(sd):
        return sd

    try:
        assert registry.get_loader("__src") is _l
    finally:
        registry._LOADERS.pop("__src", None)
    with pytest.raises(KeyError):
        registry.get_loader("__nope__")
    assert registry.get_backend("__nope__") is None
    for src in ("openfold", "openfold3", "protenix", "boltz", "chai"):
        assert callable(get_loader(src))


def test_openfold_and_protenix_rename():
    out = get_loader("openfold")({"layer_norm_in.weight": torch.zeros(2),
                                  "linear_a_p.weight": torch.zeros(2, 2),
                                  "linear_z.weight": torch.zeros(2, 2)})
    assert {"norm_in.weight", "proj_a.weight", "proj_out.weight"} <= set(out)
    assert "gate_a.weight" in get_loader("protenix")({"linear_a_g.weight": torch.zeros(2, 2)})
    assert _OPENFOLD_TO_FAST["linear_a_p"] == "proj_a"
    assert get_loader("chai") is get_loader("boltz")


def test_boltz_and_openfold3_split():
    d = 4
    p_in = torch.arange(2 * d * d).reshape(2 * d, d).float()
    sd = {"norm_in.weight": torch.zeros(d), "norm_in.bias": torch.zeros(d),
          "norm_out.weight": torch.zeros(d), "norm_out.bias": torch.zeros(d),
          "p_in.weight": p_in, "g_in.weight": torch.zeros(2 * d, d),
          "p_out.weight": torch.zeros(d, d), "g_out.weight": torch.zeros(d, d)}
    out = get_loader("boltz")(sd)
    assert torch.equal(out["proj_a.weight"], p_in[:d]) and torch.equal(out["proj_b.weight"], p_in[d:])
    of3 = {"layer_norm_in.weight": torch.zeros(d), "layer_norm_in.bias": torch.zeros(d),
           "layer_norm_out.weight": torch.zeros(d), "layer_norm_out.bias": torch.zeros(d),
           "linear_ab_p.weight": p_in, "linear_ab_g.weight": torch.zeros(2 * d, d),
           "linear_ab_p.bias": torch.arange(2 * d).float(),
           "linear_z.weight": torch.zeros(d, d), "linear_g.weight": torch.zeros(d, d)}
    out = get_loader("openfold3")(of3)
    assert torch.equal(out["proj_b.weight"], p_in[d:]) and out["proj_b.bias"].shape == (d,)
    assert "proj_a.weight" in get_loader("openfold3")({"linear_a_p.weight": torch.zeros(2, 2)})


def test_load_weights_zeroes_missing_biases_and_rejects_unknown_keys():
    d = 8
    m = FastTriangleMultiplication(d, d, "outgoing")
    sd = {"norm_in.weight": torch.ones(d), "norm_in.bias": torch.zeros(d),
          "norm_out.weight": torch.ones(d), "norm_out.bias": torch.zeros(d),
          "p_in.weight": torch.randn(2 * d, d), "g_in.weight": torch.randn(2 * d, d),
          "p_out.weight": torch.randn(d, d), "g_out.weight": torch.randn(d, d)}
    m.load_boltz_state_dict(sd)
    assert torch.all(m._impl.proj_a.bias == 0) and torch.all(m._impl.proj_out.bias == 0)
    with pytest.raises(KeyError):
        m.load_weights({"bogus.weight": torch.zeros(1)}, "openfold")


# ------------------------------------------------------------------ patchers
def test_patch_swaps_classes_and_ignores_missing():
    mod = types.ModuleType("__fake_stack")

    class TriangleMultiplicationOutgoing:
        pass

    mod.TriangleMultiplicationOutgoing = TriangleMultiplicationOutgoing
    sys.modules["__fake_stack"] = mod
    try:
        patch._patch("__fake_stack", ["TriangleMultiplicationOutgoing", "NotPresent"],
                     ["TriangleMultiplicationIncoming"])
        cls = mod.TriangleMultiplicationOutgoing
        assert issubclass(cls, FastTriangleMultiplication)
        assert not hasattr(mod, "NotPresent") and not hasattr(mod, "TriangleMultiplicationIncoming")
        layer = cls(16, 8, some_library_kwarg=1)
        assert layer._impl.residual is False and layer.mode == "outgoing"
        z = torch.randn(1, 8, 8, 16)
        assert layer(z, mask=torch.ones(1, 8, 8), chunk_size=4).shape == z.shape
    finally:
        sys.modules.pop("__fake_stack", None)
    for name in ("patch_openfold", "patch_openfold3", "patch_boltz", "patch_protenix"):
        assert callable(getattr(ftm, name))


# ------------------------------------------------------------------ torch path vs oracle
@pytest.mark.parametrize("mode", ["outgoing", "incoming"])
def test_torch_backend_matches_oracle(mode):
    from tests.helpers import compare, make_layer, make_mask, oracle_out
    m = make_layer(mode, residual=True, d=32)
    gen = torch.Generator().manual_seed(4)
    z = torch.randn(1, 16, 16, 32, generator=gen)
    mask = make_mask("tail", 1, 16, gen)
    with torch.no_grad():
        out = m(z, mask=mask)
    assert out.dtype == z.dtype
    max_abs, mean_rel = compare(out, oracle_out(m, z, mask))
    assert max_abs < 2e-2 and mean_rel < 3e-3


# ------------------------------------------------------------------ C ABI
def test_c_abi_exports_every_declared_symbol():
    """The shared library loads (no GPU needed) and exports each function the header
    declares; nothing is called that needs a device."""
    import ctypes
    import os
    import re
    from fast_trimul_b200 import _lib
    header = open(os.path.join(os.path.dirname(os.path.dirname(__file__)), "include",
                               "fast_trimul_b200.h")).read()
    declared = set(re.findall(r"\b(ftm_[a-z_0-9]+)\s*\(", header))
    assert len(declared) >= 13
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in sorted(declared):
        assert hasattr(lib, name), name
    _lib.load()
    assert _lib.status_string(0) == "ok"
    assert set(_lib.SIGNATURES) <= declared


def test_clock_sampler_summary_reads_nvml_reason_bits():
    """The bench's clock record: median SM clock under load and the NVML clock-event
    reasons seen during the timed region (sw_power_cap kept, slowdowns reported)."""
    import sys, os
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from bench import ClockSampler
    c = ClockSampler(0)
    c.samples = [(1965, 1965, 0x0), (1900, 1965, 0x4), (345, 1965, 0x1), (1930, 1965, 0x4 | 0x40)]
    s = c.summary()
    assert s["samples"] == 4 and s["sm_max_mhz"] == 1965.0
    assert s["sm_mhz"] == 1930.0                       # idle sample (345) left out
    assert s["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]
    assert ClockSampler(0).summary()["samples"] == 0


def test_c_abi_rejects_bad_arguments_before_touching_a_device():
    """Argument checks of the multi-GPU and blocked entry points run on the host and
    return a status before any device call (here, without a GPU, valid arguments stop at
    FTM_UNSUPPORTED_ARCH); nothing is launched."""
    import ctypes
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    fake = ctypes.c_void_p(1 << 20)          # 16-byte aligned, never dereferenced
    err = ctypes.c_void_p(1 << 20)

    def prob(rows, cols, mode=_lib.OUTGOING):
        return _lib.Problem(1, rows, cols, 128, 128, mode, 1, _lib.BF16, _lib.BF16, 1e-5, 1e-5)

    planes = _lib.PeerPlanes.make(2, 0, [1 << 20, 2 << 20])
    bad_world = _lib.PeerPlanes.make(3, 0, [1 << 20, 2 << 20, 3 << 20])   # 128 % 3 != 0
    null_plane = _lib.PeerPlanes.make(2, 1, [1 << 20, 0])
    p_ok, p_in_ragged = prob(256, 512), prob(12, 512, _lib.INCOMING)
    scatter = lib.ftm_input_stage_scatter
    assert scatter(None, fake, None, fake, ctypes.byref(planes), ctypes.byref(planes), fake, err, None) \
        == _lib.BAD_ARGUMENT
    assert scatter(ctypes.byref(p_ok), fake, None, fake, ctypes.byref(bad_world),
                   ctypes.byref(bad_world), fake, err, None) == _lib.BAD_ARGUMENT
    assert scatter(ctypes.byref(p_ok), fake, None, fake, ctypes.byref(null_plane),
                   ctypes.byref(null_plane), fake, err, None) == _lib.BAD_ARGUMENT
    assert scatter(ctypes.byref(p_in_ragged), fake, None, fake, ctypes.byref(planes),
                   ctypes.byref(planes), fake, err, None) == _lib.BAD_SHAPE
    assert scatter(ctypes.byref(p_ok), fake, None, fake, ctypes.byref(planes), ctypes.byref(planes),
                   fake, err, None) == _lib.UNSUPPORTED_ARCH
    cs = lib.ftm_contraction_scatter
    assert cs(fake, fake, ctypes.byref(planes), 1, 128, 256, 512, _lib.OUTGOING, err, None) \
        == _lib.UNSUPPORTED_ARCH
    assert cs(fake, fake, ctypes.byref(planes), 1, 128, 200, 400, _lib.OUTGOING, err, None) \
        == _lib.BAD_SHAPE                                  # rows % 256
    assert cs(fake, fake, ctypes.byref(planes), 1, 128, 256, 1024, _lib.OUTGOING, err, None) \
        == _lib.BAD_SHAPE                                  # n != P * rows
    assert cs(fake, fake, ctypes.byref(planes), 1, 128, 256, 512, 7, err, None) == _lib.BAD_ARGUMENT
    kb = lib.ftm_contraction_kblocked
    assert kb(fake, fake, fake, 3, 512, 512, 100, 2, 256, err, None) == _lib.BAD_SHAPE   # k block % 64
    assert kb(fake, fake, fake, 3, 512, 512, 256, 2, 200, err, None) == _lib.BAD_SHAPE   # x blocks
    assert kb(None, fake, fake, 3, 512, 512, 256, 2, 256, err, None) == _lib.BAD_ARGUMENT
    assert kb(fake, fake, fake, 3, 512, 512, 256, 2, 256, err, None) == _lib.UNSUPPORTED_ARCH


def test_bench_line_has_every_contract_key():
    """bench.py's JSON line, built from a stand-in measurement on the CPU: every key the
    contract names, the roofline fractions and vs_baseline derived consistently."""
    import argparse
    import json
    import sys, os
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    args = argparse.Namespace(n=2048, gpus=1, steps=10, warmup=3, mode="outgoing")
    res = {"ms_per_step": 3.2, "stage_ms": {"input_stage": 0.75, "contraction": 1.65, "output_stage": 0.8},
           "clocks": {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 5},
           "e2e": {"value": 130.0, "unit": "TFLOP/s", "h2d_bytes_per_step": 1, "d2h_bytes_per_step": 1},
           "gpu_launches": 30}
    line = json.loads(json.dumps(bench.build_line(args, res, 1)))
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "roofline", "clocks", "e2e",
              "gpu_launches"):
        assert k in line, k
    assert line["value"] == round(bench.trimul_flops(1, 2048) / 3.2e-3 / 1e12, 3)
    rf = line["roofline"]
    assert rf["frac"] == round(rf["achieved"] / rf["peak"], 3)
    assert rf["bound"] == "tensor" and rf["unit"] == "TFLOP/s"
    assert abs(rf["achieved"] - 2 * 128 * 2048 ** 3 / 1.65e-3 / 1e12) < 0.1
    assert line["vs_baseline"] == round(line["value"] / 24.65, 2)
    assert line["config"]["workload"].startswith("C5 outgoing")
    assert set(line["stages"]) == {"input_stage", "contraction", "output_stage"}


def test_c_caller_compiles_against_the_header_and_links():
    """The boundary from plain C: tests/c_abi/abi_host_check.c includes only the public
    header, links libfast_trimul_b200.so and checks sizes, status strings and argument
    validation (host-side paths only; nothing is launched)."""
    import os
    import shutil
    import subprocess
    import tempfile
    from fast_trimul_b200 import _lib
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    libdir = os.path.dirname(_lib.LIB_PATH)
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "abi_host_check")
        subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(root, "include"),
                        os.path.join(root, "tests", "c_abi", "abi_host_check.c"),
                        "-L", libdir, "-l:libfast_trimul_b200.so", "-Wl,-rpath," + libdir,
                        "-o", exe], check=True, capture_output=True, text=True)
        r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all host-side checks passed" in r.stdout


@pytest.mark.parametrize("mode", ["outgoing", "incoming"])
@pytest.mark.parametrize("residual", [True, False])
def test_parity_rows_checker_matches_oracle(mode, residual):
    """The fp32 row-sampled checker used at N = 2048 (fast_trimul_b200.parity) equals
    the oracle on the rows it evaluates."""
    from fast_trimul_b200.parity import reference_rows, sample_rows
    from tests.helpers import make_layer, make_mask, oracle_out
    m = make_layer(mode, residual, d=32)
    gen = torch.Generator().manual_seed(4)
    B, N = 2, 24
    z = torch.randn(B, N, N, 32, generator=gen).to(torch.bfloat16)
    mask = make_mask("pad", B, N, gen)
    rows = sample_rows(N, 5)
    got = reference_rows(m._impl, z, mask, rows, chunk_rows=7)
    ref = oracle_out(m, z, mask)[:, rows]
    assert np.abs(got.numpy() - ref).max() < 1e-4


@pytest.mark.parametrize("mode", ["outgoing", "incoming"])
def test_backward_plane_layout_on_cpu(mode, monkeypatch):
    """The training backward (fast_trimul_b200.backward) with its native product swapped
    for torch.bmm on the same planes: the gradients of z and of all parameters equal
    autograd of the reference formula -- this pins the plane layouts of both modes."""
    import torch.nn.functional as F
    from fast_trimul_b200 import backward as bw
    from tests.helpers import make_layer, make_mask

    def torch_grads(dx, a, b):
        return torch.bmm(dx, b.float()), torch.bmm(dx.transpose(1, 2), a.float())

    monkeypatch.setattr(bw, "native_plane_grads", torch_grads)
    m = make_layer(mode, True, d=16)
    imp = m._impl.float()
    gen = torch.Generator().manual_seed(6)
    B, N, C = 2, 8, 16
    z = torch.randn(B, N, N, C, generator=gen)
    mask = make_mask("pad", B, N, gen)
    gout = torch.randn(B, N, N, C, generator=gen)
    params = [p.detach() for p in imp._params()]
    # the forward's planes, as the native forward would keep them
    with torch.no_grad():
        mm = mask.unsqueeze(-1)
        zn = F.layer_norm(z * mm, (C,), params[0], params[1], 1e-5)
        a = F.linear(zn, params[4], params[5]) * torch.sigmoid(F.linear(zn, params[6], params[7]))
        b = F.linear(zn, params[8], params[9]) * torch.sigmoid(F.linear(zn, params[10], params[11]))
        a16 = bw._planes(a, mode).contiguous()
        b16 = bw._planes(b, mode).contiguous()
        x16 = torch.matmul(a16, b16.transpose(-1, -2))
    gz, gp = bw.backward(imp, z, mask, params, (a16, b16, x16), gout)
    zr = z.clone().requires_grad_(True)
    pr = [p.clone().requires_grad_(True) for p in params]
    out = imp._torch_forward(zr * mm, pr) * mm
    want = torch.autograd.grad(out, [zr] + pr, gout)
    for g, w in zip([gz] + gp, want):
        assert torch.allclose(g, w, atol=1e-4, rtol=1e-3), (g - w).abs().max()
