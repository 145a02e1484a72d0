"""Benchmark of the TriMul forward on B200 (one JSON line on rank 0).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Workload (the benchmark's large single-layer configuration): one outgoing TriMul, B=1, N=2048, c_z=c_h=128,
bf16 z ~ N(0,1), all-ones pair mask, random-init weights. One step = one forward.
N=1 runs it on one GPU; N>1 shards the i-rows over N ranks, which exchange the
projections over NVLink (fast_trimul_b200.distributed), so total work is fixed
("scaling": "strong").

Metric: TFLOP/s by the reference's FLOP formula (fast_trimul/benchmark.py:77-83)
over the device time of K steps (CUDA events, barrier + synchronize on both sides,
max over ranks). z (1.07 GB) is larger than L2, so no flush is needed between steps.
`e2e` is the same metric through the public module API with the input copied from
pinned host memory and the output copied back inside the timed region.

`--impl reference` times the reference's own CPU path -- its FastTriangleMultiplication
with backend="torch", imported unmodified from baseline/_ref -- on all host threads,
on a bounded sample of the same workload (the numpy port in oracle/ stands in only
when baseline/_ref is missing).

After timing, one forward of the same workload with fp32 output is checked against
the fp32 formula of the reference's torch path on sampled rows (`parity`).
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

C = 128
N_DEFAULT = 2048
# The reference's own published numbers for this metric (TriMul forward TFLOP/s, B=1,
# c=128, reference FLOP formula), single A100-SXM4-80GB, CUDA-graphed:
# reports/results/results_openfold3.md:32,36,44,52 of the reference checkout.
PUBLISHED_TFLOPS = {256: 12.36, 512: 14.46, 1024: 16.36, 2048: 24.65}
PUBLISHED_SOURCE = "reference's published A100-SXM4-80GB number (results_openfold3.md)"
MEASURED_PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) from one ncu
# capture of each kernel of this build at N=2048, B=1, outgoing.
NCU_TRAFFIC_N2048 = {"contraction": 4623865344, "input_stage": 3242864384,
                     "output_stage": 3234792960}


def trimul_flops(batch, n, c_z=C, c_h=C):
    m = batch * n * n
    return 4 * 2 * m * c_z * c_h + 2 * m * c_z * c_z + 2 * m * c_h * c_z + 2 * batch * c_h * n ** 3


def stage_model(batch, n, rows=None, world=1):
    """Algorithmic FLOPs and bytes per launch of each kernel (rows = local i-rows)."""
    rows = n if rows is None else rows
    pos = batch * rows * n
    return {
        # read z (2c) + mask (4), write a and b (2 * 2c) per position
        "input_stage": {"flops": 2 * pos * C * 4 * C, "bytes": pos * (2 * C + 4 + 4 * C)},
        # read a (local rows) and b (all rows), write x
        "contraction": {"flops": 2 * batch * C * rows * n * n,
                        "bytes": 2 * batch * C * (rows * n + n * n + rows * n)},
        # read z, mask, x; write out (bf16)
        "output_stage": {"flops": 2 * pos * C * 2 * C, "bytes": pos * (2 * C + 4 + 2 * C + 2 * C)},
    }


def load_peaks():
    try:
        with open(MEASURED_PEAKS) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled DURING the timed region.

    NVML is read from a background thread every 10 ms (read-only queries; nothing is set),
    so even a timed region of a few tens of milliseconds gets samples; nvidia-smi's
    200 ms loop is the fallback when NVML is unavailable. `index` is the CUDA device
    ordinal of this process; the NVML handle is found by the device's UUID so that
    CUDA_VISIBLE_DEVICES remapping cannot pick the wrong GPU."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_S = 0.01

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.thread = None
        self.samples = []          # (sm_mhz, max_mhz, reasons bitmask)
        self.lines = []

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID("GPU-" + uuid if not uuid.startswith("GPU-") else uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self._stop = threading.Event()

            def loop():
                while not self._stop.is_set():
                    try:
                        self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), mx,
                                             nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
                    except Exception:
                        pass
                    self._stop.wait(self.PERIOD_S)

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    # NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}

    def summary(self):
        sm, mx, reasons = [], None, set()
        for clk, mxc, bits in self.samples:
            sm.append(float(clk))
            mx = float(mxc)
            for name, bit in self.REASON_BITS.items():
                if bits & bit:
                    reasons.add(name)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        loaded = [x for x in sm if x > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvml" if self.samples else "nvidia-smi"}


# --------------------------------------------------------------------------- reference
REF_ROOT = os.path.join(ROOT, "baseline", "_ref")


def import_reference():
    """The reference package, unmodified, from baseline/_ref. Two runtime shims and no
    edits: the CLI-only `cutlass.testing` import of its GEMM harness gets a stub module,
    and on a host without a GPU `torch.cuda.get_device_properties` (called when its
    kernel module is imported) returns a stand-in. Returns (FastTriangleMultiplication,
    None) or (None, reason)."""
    import types
    import torch
    if not os.path.isdir(os.path.join(REF_ROOT, "fast_trimul")):
        return None, "baseline/_ref/fast_trimul missing"
    try:
        import cutlass
        if "cutlass.testing" not in sys.modules:
            stub = types.ModuleType("cutlass.testing")
            sys.modules["cutlass.testing"] = stub
            cutlass.testing = stub
    except ImportError as e:
        return None, f"nvidia-cutlass-dsl not importable: {e}"
    if not torch.cuda.is_available():
        props = types.SimpleNamespace(multi_processor_count=148, max_threads_per_multi_processor=2048)
        torch.cuda.get_device_properties = lambda *a, **k: props
    if REF_ROOT not in sys.path:
        sys.path.insert(0, REF_ROOT)
    try:
        import fast_trimul as ref
        from fast_trimul import FastTriangleMultiplication
    except Exception as e:                       # noqa: BLE001 -- reported, not hidden
        return None, f"reference import failed: {type(e).__name__}: {e}"
    if not os.path.abspath(ref.__file__).startswith(REF_ROOT):
        return None, "a different fast_trimul shadows baseline/_ref"
    return FastTriangleMultiplication, None


def reference_cpu_forward(n, seed=0):
    """One outgoing forward of the workload at size n through the reference's own CPU
    path: FastTriangleMultiplication(128, 128, 'outgoing', backend='torch') (fp16
    weights, its mask/cast rules, its `_torch_forward`), bf16 z ~ N(0,1), ones mask.
    Returns (callable, kind, threads)."""
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)           # torchrun sets OMP_NUM_THREADS=1; use every core
    FTM, why = import_reference()
    if FTM is None:
        return _oracle_cpu_forward(n, seed), "port", threads, why
    torch.manual_seed(seed)
    m = FTM(C, C, mode="outgoing", backend="torch").eval()
    gen = torch.Generator().manual_seed(seed + 1)
    z = torch.randn(1, n, n, C, generator=gen).to(torch.bfloat16)
    mask = torch.ones(1, n, n)

    def fn():
        with torch.no_grad():
            return m(z, mask=mask)
    return fn, "reference", torch.get_num_threads(), None


def _oracle_cpu_forward(n, seed=0):
    """Stand-in when the reference package is absent: the numpy port in oracle/."""
    import numpy as np
    from oracle.trimul_oracle import trimul_forward
    rng = np.random.default_rng(seed)
    p = {}
    for ln in ("norm_in", "norm_out"):
        p[ln + ".weight"] = np.ones(C, np.float32)
        p[ln + ".bias"] = np.zeros(C, np.float32)
    for lin in ("proj_a", "gate_a", "proj_b", "gate_b", "proj_g", "proj_out"):
        bound = C ** -0.5
        p[lin + ".weight"] = rng.uniform(-bound, bound, (C, C)).astype(np.float32)
        p[lin + ".bias"] = rng.uniform(-bound, bound, C).astype(np.float32)
    z = rng.standard_normal((1, n, n, C)).astype(np.float32)
    mask = np.ones((1, n, n), np.float32)
    return lambda: trimul_forward(z, p, "outgoing", True, mask)


def _timed_calls(fn, steps, warmup, budget_s=None, max_calls=1000):
    for _ in range(warmup):
        fn()
    ts = []
    t_end = None if budget_s is None else time.perf_counter() + budget_s
    while len(ts) < steps or (t_end is not None and time.perf_counter() < t_end and len(ts) < max_calls):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return ts


CPU_SAMPLE_N = 1024


def run_reference(args):
    """The contract's reference arm: the reference's CPU path on this host's cores. Each
    step is one N=1024 forward (a bounded sample of the N=2048 workload); after the K
    timed steps, one full N=2048 forward is timed once (`same_config_once`)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    fn, kind, cores, why = reference_cpu_forward(CPU_SAMPLE_N)
    ts = _timed_calls(fn, args.steps, args.warmup)[:args.steps]
    sec = sum(ts) / len(ts)
    tflops = trimul_flops(1, CPU_SAMPLE_N) / sec / 1e12
    full = None
    if not args.no_full_reference:
        fn_full, _, _, _ = reference_cpu_forward(args.n)
        t0 = time.perf_counter()
        fn_full()
        dt = time.perf_counter() - t0
        full = {"n": args.n, "s": round(dt, 3), "tflops": round(trimul_flops(1, args.n) / dt / 1e12, 5)}
    src = ("the reference's FastTriangleMultiplication(backend='torch') from baseline/_ref"
           if kind == "reference" else f"numpy port of the reference's torch path ({why})")
    sample = (f"one outgoing forward at N={CPU_SAMPLE_N} (B=1, c_z=c_h=128, bf16 z, ones mask) per "
              f"step, {src}, {cores} threads; TFLOP/s by the reference formula")
    line = {
        "metric": "trimul_fwd_tflops", "value": round(tflops, 5), "unit": "TFLOP/s",
        "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16" if kind == "reference" else "f32", "data": "synthetic",
        "config": {"workload": f"C5 outgoing TriMul B=1 N={args.n} c=128 (CPU sample N={CPU_SAMPLE_N})",
                   "batch": 1, "n": args.n, "c_z": C, "c_h": C, "mode": "outgoing"},
        "cpu_baseline": {"value": round(tflops, 5), "unit": "TFLOP/s", "cores": cores,
                         "kind": kind, "sample": sample, "same_config_once": full},
        "e2e": {"value": round(tflops, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_line(budget_s=15.0):
    """`cpu_baseline` of the main line: the reference's CPU path, N=1024 forwards for
    about `budget_s` seconds on all host threads."""
    fn, kind, cores, why = reference_cpu_forward(CPU_SAMPLE_N)
    ts = _timed_calls(fn, 2, 1, budget_s=budget_s, max_calls=50)
    sec = statistics.median(ts)
    src = ("the reference's FastTriangleMultiplication(backend='torch') from baseline/_ref"
           if kind == "reference" else f"numpy port of the reference's torch path ({why})")
    return {"value": round(trimul_flops(1, CPU_SAMPLE_N) / sec / 1e12, 5), "unit": "TFLOP/s",
            "cores": cores, "kind": kind,
            "sample": f"{src}: one outgoing N={CPU_SAMPLE_N} forward (bf16 z, ones mask), median of "
                      f"{len(ts)} runs (~{budget_s:.0f} s), {cores} threads"}


# --------------------------------------------------------------------------- ours, 1 GPU
def make_layer(device, mode="outgoing"):
    import torch
    from fast_trimul_b200 import FastTriangleMultiplication
    torch.manual_seed(0)
    return FastTriangleMultiplication(C, C, mode=mode, residual=True).to(device).eval()


def bench_single(args, torch):
    from fast_trimul_b200.plan import TriMulPlan
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = args.n
    layer = make_layer(dev, getattr(args, "mode", "outgoing"))
    gen = torch.Generator(device=dev).manual_seed(1)
    z = torch.randn(1, n, n, C, device=dev, generator=gen).to(torch.bfloat16)
    mask = torch.ones(1, n, n, device=dev)
    plan = TriMulPlan(layer._impl, 1, n, torch.bfloat16)
    out = plan.out_like()
    for _ in range(args.warmup):
        plan(z, mask, out=out)
    plan.check_error()
    K = args.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        t0.record()
        for k in range(K):
            plan(z, mask, out=out, stage_events=evs[k])
        t1.record()
        torch.cuda.synchronize()
    plan.check_error()
    total_ms = t0.elapsed_time(t1)
    stage_ms = {
        "input_stage": sum(e[0].elapsed_time(e[1]) for e in evs) / K,
        "contraction": sum(e[1].elapsed_time(e[2]) for e in evs) / K,
        "output_stage": sum(e[2].elapsed_time(e[3]) for e in evs) / K,
    }
    res = {"ms_per_step": total_ms / K, "stage_ms": stage_ms, "clocks": clk.summary(),
           "gpu_launches": 3 * K}
    res["parity"] = parity_single(torch, layer, z, mask, out)
    del plan
    res["contraction_n1024"] = contraction_alone(torch, 1024)
    res["e2e"] = bench_e2e(args, torch, layer, dev, n)
    res["sweep"] = bench_sweep(args, torch, layer, dev) if not args.no_sweep else None
    res["trunk"] = bench_trunk(args, torch, dev) if not args.no_trunk else None
    res["train"] = bench_train(torch, dev) if not args.no_trunk else None
    res["small_n"] = bench_small_n(torch, dev) if not args.no_sweep else None
    return res


def bench_small_n(torch, dev, ns=(64, 128, 256)):
    """Latency of one outgoing layer call through the public module API at small N
    (B=1, bf16 z, ones mask): eager (`layer(z, mask)`: dispatch, a workspace from the
    caching allocator, three launches) and after `layer.graphed(z, mask)` (replay of the
    three launches, z already in the graph's input buffer). Median of 50 CUDA-event timed
    calls each, back to back (z is small enough to stay in L2: this is a latency figure)."""
    from fast_trimul_b200 import FastTriangleMultiplication
    rows = []
    for n in ns:
        torch.manual_seed(0)
        layer = FastTriangleMultiplication(C, C, mode="outgoing").to(dev).eval()
        z = torch.randn(1, n, n, C, device=dev).to(torch.bfloat16)
        mask = torch.ones(1, n, n, device=dev)

        def timed(fn):
            for _ in range(5):
                fn()
            ts = []
            for _ in range(50):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                fn()
                b.record()
                torch.cuda.synchronize()
                ts.append(a.elapsed_time(b))
            return statistics.median(ts)

        with torch.no_grad():
            eager = timed(lambda: layer(z, mask=mask))
            layer.graphed(z, mask)
            zin = layer.graph_input()
            graphed = timed(lambda: layer(zin, mask=mask))
        rows.append({"n": n, "eager_ms": round(eager, 4), "graphed_ms": round(graphed, 4)})
        del layer, z
    return rows

def bench_train(torch, dev, ns=(384, 1024)):
    """Forward + backward of one outgoing layer (B=1, bf16 z, all-ones mask, loss =
    sum(out * g) for a fixed random g): this library's training path (native forward
    keeping a, b, x; contraction gradients on the native kernel; per-position parts in
    fp32 autograd) against the same layer run through the torch backend (the reference's
    `_torch_forward` under autograd, fp16 weights). Median of 5 CUDA-event timed steps."""
    from fast_trimul_b200 import FastTriangleMultiplication
    rows = []
    for n in ns:
        for backend in ("cuda", "torch"):
            torch.manual_seed(0)
            layer = FastTriangleMultiplication(C, C, mode="outgoing", backend=backend).to(dev)
            z = torch.randn(1, n, n, C, device=dev).to(torch.bfloat16).requires_grad_(True)
            mask = torch.ones(1, n, n, device=dev)
            g = torch.randn(1, n, n, C, device=dev)

            def step():
                out = layer(z, mask=mask)
                (out.float() * g).sum().backward()

            try:
                for _ in range(2):
                    step()
                torch.cuda.synchronize()
                ts = []
                for _ in range(5):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    step()
                    b.record()
                    torch.cuda.synchronize()
                    ts.append(a.elapsed_time(b))
                rows.append({"n": n, "path": backend, "fwd_bwd_ms": round(statistics.median(ts), 3)})
            except torch.cuda.OutOfMemoryError:
                rows.append({"n": n, "path": backend, "fwd_bwd_ms": None, "note": "out of memory"})
            del layer, z, g
            torch.cuda.empty_cache()
    return rows


PARITY_ROWS = 16


def parity_single(torch, layer, z, mask, out_bench):
    """One more forward of the benchmarked workload with fp32 output, compared on
    PARITY_ROWS sampled rows with the fp32 formula of the reference's torch path
    (fast_trimul_b200.parity), under the stated tolerance; the benchmark's own bf16
    output is compared on the same rows for information (its bf16 rounding alone is
    ~1.4e-3 mean-relative)."""
    from fast_trimul_b200.parity import error_metrics, reference_rows, sample_rows
    from fast_trimul_b200.plan import TriMulPlan
    n = z.shape[1]
    plan = TriMulPlan(layer._impl, z.shape[0], n, z.dtype, out_dtype=torch.float32)
    out = plan(z, mask)
    plan.check_error()
    rows = sample_rows(n, PARITY_ROWS)
    ref = reference_rows(layer._impl, z, mask, rows)
    max_abs, mean_rel = error_metrics(out[:, rows], ref)
    b_abs, b_rel = error_metrics(out_bench[:, rows].float(), ref)
    return {"max_abs": round(max_abs, 6), "mean_rel": round(mean_rel, 7), "rows_checked": len(rows),
            "tolerance": {"max_abs": 2e-2, "mean_rel": 1e-3},
            "ok": bool(max_abs <= 2e-2 and mean_rel <= 1e-3),
            "checker": "fp32 torch formula of the reference's torch path on the GPU, sampled rows",
            "output": "fp32 (same kernels; the timed steps write bf16)",
            "bf16_output": {"max_abs": round(b_abs, 6), "mean_rel": round(b_rel, 7)}}


def contraction_alone(torch, n, reps=10):
    """The contraction kernel alone at N=n (128 channels of N x N x N, fp16 operands in
    HBM): median of `reps` CUDA-event timed launches after warm-up."""
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    s = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(C, n, n, device="cuda", generator=g).half()
    B = torch.randn(C, n, n, device="cuda", generator=g).half()
    X = torch.empty(C, n, n, device="cuda", dtype=torch.half)
    err = torch.zeros(64, dtype=torch.int32, device="cuda")

    def launch():
        _lib.check(lib.ftm_contraction(A.data_ptr(), B.data_ptr(), X.data_ptr(), C, n, n, n, 1,
                                       err.data_ptr(), s), "ftm_contraction")
    for _ in range(5):
        launch()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    ev[0].record()
    for i in range(reps):
        launch()
        ev[i + 1].record()
    torch.cuda.synchronize()
    if lib.ftm_check_error(err.data_ptr(), None, s) != _lib.OK:
        raise _lib.NativeKernelError("contraction wait expired")
    ms = statistics.median(ev[i].elapsed_time(ev[i + 1]) for i in range(reps))
    peaks, src = load_peaks()
    tf = 2 * C * n ** 3 / (ms * 1e-3) / 1e12
    return {"n": n, "ms": round(ms, 4), "tflops": round(tf, 1),
            "frac": round(tf / float(peaks["bf16_tflops"]), 3),
            "peak": f"{src} bf16 dense burst", "launches_timed": reps,
            "note": "back-to-back launches; operands 0.54 GB > L2 is not guaranteed, L2 not flushed"}


def reference_gpu_subprocess(ns=(64, 128, 256, 2048), timeout_s=300):
    """Times the reference's own GPU kernels (its FastTriangleMultiplication with CUDA-graph
    capture, from baseline/_ref) on this GPU in a child process, so its JIT-compiled
    CuTe kernels cannot disturb this process. Returns a list of per-N results or an
    `unavailable` reason."""
    cmd = [sys.executable, os.path.abspath(__file__), "--reference-gpu-sweep"] + [str(n) for n in ns]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"reference GPU sweep exceeded {timeout_s} s"}
    rows = []
    for ln in r.stdout.splitlines():
        try:
            d = json.loads(ln)
        except ValueError:
            continue
        if "unavailable" in d and "n" not in d:
            return {"unavailable": d["unavailable"]}
        rows.append(d)
    if not rows:
        return {"unavailable": f"rc={r.returncode}: {r.stderr.strip()[-300:]}"}
    return rows


def bench_trunk(args, torch, dev, n=384, blocks=8):
    """The trunk configuration: 8 PairFormer-style blocks, N=384, c_s=384, c_z=128, bf16,
    all-ones masks, random weights; ms per trunk forward with plain-PyTorch TriMul
    layers vs with FastTriangleMultiplication, everything else identical."""
    from fast_trimul_b200.pairformer import (PairFormerTrunk, copy_trimul_weights, fast_trimul,
                                             torch_trimul, trunk_flops_trimul)
    torch.manual_seed(0)
    ref = PairFormerTrunk(blocks, 384, C, torch_trimul).to(dev).to(torch.bfloat16).eval()
    fast = PairFormerTrunk(blocks, 384, C, fast_trimul).to(dev).to(torch.bfloat16).eval()
    for m in fast.modules():
        if hasattr(m, "_impl"):
            m._impl.half()                      # the TriMul weights stay fp16, as in the reference
    copy_trimul_weights(ref, fast)
    gen = torch.Generator(device=dev).manual_seed(3)
    s = torch.randn(1, n, 384, device=dev, generator=gen).to(torch.bfloat16)
    z = torch.randn(1, n, n, C, device=dev, generator=gen).to(torch.bfloat16)
    mask = torch.ones(1, n, n, device=dev, dtype=torch.bfloat16)

    def timed(model):
        with torch.no_grad():
            for _ in range(3):
                model(s, z, mask)
            torch.cuda.synchronize()
            ts = []
            for _ in range(10):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                out = model(s, z, mask)
                b.record()
                torch.cuda.synchronize()
                ts.append(a.elapsed_time(b))
        return statistics.median(ts), out

    def trimul_layers_ms(model):
        """The trunk's 16 TriMul layers alone, each on the trunk's input z and mask."""
        layers = [m for blk in model.blocks for m in (blk.tri_out, blk.tri_in)]
        with torch.no_grad():
            for lay in layers:
                lay(z, mask=mask)
            torch.cuda.synchronize()
            ts = []
            for _ in range(5):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for lay in layers:
                    lay(z, mask=mask)
                b.record()
                torch.cuda.synchronize()
                ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    ms_ref, (s_ref, z_ref) = timed(ref)
    ms_fast, (s_fast, z_fast) = timed(fast)
    tri_ref, tri_fast = trimul_layers_ms(ref), trimul_layers_ms(fast)
    dz = ((z_fast.float() - z_ref.float()).abs().mean() / z_ref.float().abs().mean()).item()
    return {"config": "C4 PairFormer-style trunk, 8 blocks, N=384, c_s=384, c_z=128, bf16",
            "ms_per_fwd_torch_trimul": round(ms_ref, 3), "ms_per_fwd_fast_trimul": round(ms_fast, 3),
            "speedup": round(ms_ref / ms_fast, 3),
            "trimul_layers_ms": {"torch": round(tri_ref, 3), "fast": round(tri_fast, 3)},
            "trimul_share_of_trunk": {"torch": round(tri_ref / ms_ref, 3),
                                      "fast": round(tri_fast / ms_fast, 3)},
            "mask_semantics": "both trunks: z * mask before the input LayerNorm, output * mask",
            "trimul_tflop_per_fwd": round(trunk_flops_trimul(n, C, blocks) / 1e12, 4),
            "z_out_mean_rel_diff": round(dz, 5)}


def bench_e2e(args, torch, layer, dev, n):
    """Public API (module forward) with pinned host input copied in and the full output
    copied back every step. Steps are pipelined across three streams -- H2D of step
    k+1, the forward of step k and D2H of step k-1 overlap -- with double-buffered
    device tensors; the timed region covers all copies of all steps."""
    gen = torch.Generator().manual_seed(2)
    z_host = torch.randn(1, n, n, C, generator=gen).to(torch.bfloat16).pin_memory()
    mask_host = torch.ones(1, n, n).pin_memory()
    out_host = torch.empty_like(z_host).pin_memory()
    steps = max(3, min(args.steps, 20))
    h2d, comp, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    zd = [torch.empty(z_host.shape, dtype=z_host.dtype, device=dev) for _ in range(2)]
    md = [torch.empty(mask_host.shape, dtype=mask_host.dtype, device=dev) for _ in range(2)]
    od = [None, None]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]

    def run(k_steps):
        for k in range(k_steps + 2):
            if k < k_steps:                       # H2D of step k
                i = k & 1
                h2d.wait_event(ev_free[i])
                with torch.cuda.stream(h2d):
                    zd[i].copy_(z_host, non_blocking=True)
                    md[i].copy_(mask_host, non_blocking=True)
                    ev_in[i].record(h2d)
            if 1 <= k <= k_steps:                 # forward of step k-1
                i = (k - 1) & 1
                comp.wait_event(ev_in[i])
                with torch.cuda.stream(comp), torch.no_grad():
                    od[i] = layer(zd[i], mask=md[i])
                    ev_out[i].record(comp)
            if 2 <= k:                            # D2H of step k-2
                i = (k - 2) & 1
                d2h.wait_event(ev_out[i])
                with torch.cuda.stream(d2h):
                    out_host.copy_(od[i], non_blocking=True)
                    od[i].record_stream(d2h)
                    ev_free[i].record(d2h)

    run(2)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(h2d)
    run(steps)
    t1.record(d2h)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    return {"value": round(trimul_flops(1, n) / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
            "ms_per_step": round(ms, 3), "steps": steps, "pipelined": True,
            "h2d_bytes_per_step": z_host.numel() * 2 + mask_host.numel() * 4,
            "d2h_bytes_per_step": out_host.numel() * 2}


def bench_sweep(args, torch, layer, dev):
    """Latency / TFLOP/s at the other sizes the metric names (median of per-step events)."""
    from fast_trimul_b200.plan import TriMulPlan
    rows = []
    mode0 = layer._impl.mode
    for n, mode in ((256, "outgoing"), (256, "incoming"), (512, "outgoing"), (1024, "outgoing"),
                    (1024, "incoming"), (2048, "incoming")):
        layer._impl.mode = mode
        z = torch.randn(1, n, n, C, device=dev).to(torch.bfloat16)
        mask = torch.ones(1, n, n, device=dev)
        plan = TriMulPlan(layer._impl, 1, n, torch.bfloat16)
        out = plan.out_like()
        for _ in range(5):
            plan(z, mask, out=out)
        ts = []
        for _ in range(20):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            plan(z, mask, out=out)
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        plan.check_error()
        ms = statistics.median(ts)
        rows.append({"n": n, "mode": mode, "ms": round(ms, 4),
                     "tflops": round(trimul_flops(1, n) / (ms * 1e-3) / 1e12, 2)})
        del plan, z, out
    layer._impl.mode = mode0
    return rows


def contraction_vs_cublas(ns, launches=150):
    """The contraction kernel alone against cuBLAS (torch.bmm) on the same batched problem
    X[l] = A[l] B[l]^T, 128 channels of N x N x N, fp16 operands, fp32 accumulation.
    Short runs: median of 10 back-to-back launches (CUDA events). Sustained runs:
    `launches` back-to-back launches with NVML energy and SM clocks sampled during them
    (both kernels hit the 1 kW power cap; energy per launch decides the clock)."""
    import time
    import torch
    from fast_trimul_b200 import _lib
    lib = _lib.load()
    s = torch.cuda.current_stream().cuda_stream
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + str(torch.cuda.get_device_properties(0).uuid))
    except Exception:
        h = None
    for n in ns:
        L = C
        A = torch.randn(L, n, n, device="cuda").half()
        B = torch.randn(L, n, n, device="cuda").half()
        X = torch.empty(L, n, n, device="cuda", dtype=torch.half)
        err = torch.zeros(64, dtype=torch.int32, device="cuda")
        kernels = {
            "ftm_contraction": lambda: lib.ftm_contraction(A.data_ptr(), B.data_ptr(), X.data_ptr(), L, n,
                                                           n, n, 1, err.data_ptr(), s),
            "cublas_bmm": lambda: torch.bmm(A, B.transpose(1, 2), out=X),
        }
        flops = 2 * L * n ** 3
        for name, f in kernels.items():
            for _ in range(5):
                f()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(11)]
            ev[0].record()
            for i in range(10):
                f()
                ev[i + 1].record()
            torch.cuda.synchronize()
            short = statistics.median(ev[i].elapsed_time(ev[i + 1]) for i in range(10))
            time.sleep(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            j0 = pynvml.nvmlDeviceGetTotalEnergyConsumption(h) if h is not None else None
            with ClockSampler(0) as clk:
                e0.record()
                for _ in range(launches):
                    f()
                e1.record()
                torch.cuda.synchronize()
            j1 = pynvml.nvmlDeviceGetTotalEnergyConsumption(h) if h is not None else None
            sus = e0.elapsed_time(e1) / launches
            lib.ftm_check_error(err.data_ptr(), None, s)
            print(json.dumps({"kernel": name, "n": n, "short_ms": round(short, 4),
                              "short_tflops": round(flops / short / 1e9, 1),
                              "sustained_ms": round(sus, 4),
                              "sustained_tflops": round(flops / sus / 1e9, 1),
                              "joules_per_launch": None if j0 is None else round((j1 - j0) / 1e3 / launches, 3),
                              "clocks": clk.summary()}))
        del A, B, X


def reference_gpu_sweep(ns):
    """The reference's own FastTriangleMultiplication (its CuTe-DSL Ampere kernels, fp16)
    on this GPU, imported unmodified from baseline/_ref (see import_reference). Same
    workload as the main line: outgoing, B=1, c=128, bf16 z, ones mask; median of 10
    CUDA-event timed calls after warm-up, eager and after its own `graphed()` capture."""
    import torch
    RefTriMul, why = import_reference()
    if RefTriMul is None:
        print(json.dumps({"impl": "reference-gpu", "unavailable": why}))
        return
    for n in ns:
        try:
            torch.manual_seed(0)
            m = RefTriMul(C, C, "outgoing").cuda().eval()
            z = torch.randn(1, n, n, C, device="cuda").to(torch.bfloat16)
            mask = torch.ones(1, n, n, device="cuda")

            def timed():
                ts = []
                for _ in range(10):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    m(z, mask=mask)
                    b.record()
                    torch.cuda.synchronize()
                    ts.append(a.elapsed_time(b))
                return statistics.median(ts)

            with torch.no_grad():
                for _ in range(3):
                    m(z, mask=mask)
                torch.cuda.synchronize()
                eager = timed()
                m.graphed(z, mask)
                graphed = timed()
        except Exception as e:                    # noqa: BLE001 -- reported in the line
            print(json.dumps({"impl": "reference-gpu", "n": n,
                              "unavailable": f"{type(e).__name__}: {str(e)[:200]}"}), flush=True)
            continue
        print(json.dumps({"impl": "reference-gpu", "n": n, "eager_ms": round(eager, 3),
                          "graphed_ms": round(graphed, 3),
                          "graphed_tflops": round(trimul_flops(1, n) / graphed / 1e9, 2)}), flush=True)
        del m, z, mask
        torch.cuda.empty_cache()


def profile_case(args):
    """A small fixed case for profilers: a few forwards at N=args.profile_case."""
    import torch
    from fast_trimul_b200.plan import TriMulPlan
    dev = torch.device("cuda", 0)
    n = args.profile_case
    if args.profile_shard:
        return profile_shard(args, torch, dev, n, args.profile_shard)
    layer = make_layer(dev, getattr(args, "mode", "outgoing"))
    layer._impl.mode = args.mode
    z = torch.randn(1, n, n, C, device=dev).to(torch.bfloat16)
    mask = torch.ones(1, n, n, device=dev)
    plan = TriMulPlan(layer._impl, 1, n, torch.bfloat16)
    out = plan.out_like()
    for _ in range(max(2, args.steps if args.steps < 10 else 2)):
        plan(z, mask, out=out)
    plan.check_error()
    print("profile case ok", n, args.mode)


def profile_shard(args, torch, dev, n, P):
    """One rank's kernels of the P-way channel-sharded forward (alltoall schemes):
    input stage on N/P rows, the contraction of 128/P channels over all N rows with A,
    B and X in the blocked layouts, and the output stage on N/P rows."""
    from fast_trimul_b200 import _lib
    from fast_trimul_b200.distributed import RowShardedTriMul, TorchStageOps  # noqa: F401
    lib = _lib.load()
    layer = make_layer(dev, getattr(args, "mode", "outgoing"))
    R = n // P
    z = torch.randn(1, R, n, C, device=dev).to(torch.bfloat16)
    mask = torch.ones(1, R, n, device=dev)
    plane = C * R * n
    a, b, x = (torch.empty(plane, dtype=torch.float16, device=dev) for _ in range(3))
    ar = torch.randn(plane, device=dev).half()
    br = torch.randn(plane, device=dev).half()
    out = torch.empty_like(z)
    packed = layer._impl.packed_params()[0]
    prob = layer._impl.problem(z, torch.bfloat16)
    err = torch.zeros(64, dtype=torch.int32, device=dev)
    zst = torch.empty(R * n * 2, dtype=torch.float32, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        _lib.check(lib.ftm_input_stage(prob, z.data_ptr(), mask.data_ptr(), packed.data_ptr(),
                                       a.data_ptr(), b.data_ptr(), zst.data_ptr(), err.data_ptr(), s),
                   "input")
        _lib.check(lib.ftm_contraction_blocked(ar.data_ptr(), br.data_ptr(), x.data_ptr(), C // P,
                                               R, P, n, R, P, err.data_ptr(), s), "contraction")
        _lib.check(lib.ftm_output_stage(prob, z.data_ptr(), mask.data_ptr(), x.data_ptr(),
                                        zst.data_ptr(), packed.data_ptr(), out.data_ptr(),
                                        err.data_ptr(), s), "output")
    torch.cuda.synchronize()
    print("profile shard ok", n, P)


# --------------------------------------------------------------------------- main
def build_line(args, res, world):
    """The contract's JSON line from a measurement result `res` (ms per step, per-stage
    CUDA-event times, clocks, e2e, launch count, optional sweep / trunk / comm)."""
    n = args.n
    flops = trimul_flops(1, n)
    ms = res["ms_per_step"]
    peaks, peak_src = load_peaks()
    model = stage_model(1, n, rows=res.get("rows_per_rank"), world=world)
    dom = "contraction"
    dom_ms = res["stage_ms"][dom]
    achieved = model[dom]["flops"] / (dom_ms * 1e-3) / 1e12
    peak = float(peaks["bf16_tflops"])
    traffic = NCU_TRAFFIC_N2048.get(dom) if world == 1 and n == N_DEFAULT else None
    stages = {}
    for name, st in model.items():
        t = res["stage_ms"][name] * 1e-3
        stages[name] = {"ms": round(res["stage_ms"][name], 4),
                        "tflops": round(st["flops"] / t / 1e12, 1),
                        "gbs": round(st["bytes"] / t / 1e9, 1),
                        "tensor_frac": round(st["flops"] / t / 1e12 / peak, 3),
                        "hbm_frac": round(st["bytes"] / t / 1e9 / float(peaks["hbm_gbs"]), 3)}
    res_value = round(flops / (ms * 1e-3) / 1e12, 3)
    line = {
        "metric": "trimul_fwd_tflops", "value": res_value,
        "unit": "TFLOP/s", "n_gpus": max(world, args.gpus), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": (round(res_value / PUBLISHED_TFLOPS[n], 2) if n in PUBLISHED_TFLOPS else None),
        "vs_baseline_ref": ({"tflops": PUBLISHED_TFLOPS[n], "source": PUBLISHED_SOURCE}
                            if n in PUBLISHED_TFLOPS else None),
        "dtype": "f16",
        "data": "synthetic (z ~ N(0,1) bf16, ones mask, seeded random-init weights)",
        "config": {"workload": f"C5 {args.mode} TriMul B=1 N={n} c_z=c_h=128", "batch": 1, "n": n,
                   "c_z": C, "c_h": C, "mode": args.mode, "z_dtype": "bf16",
                   "parallelism": f"i-row shards x{max(world, args.gpus)}" if world > 1 else "single",
                   "l2": "inputs larger than L2 (z = %.2f GB)" % (n * n * C * 2 / 1e9)},
        "roofline": {"kernel": dom, "bound": "tensor", "achieved": round(achieved, 1),
                     "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 3),
                     "peak_source": f"{peak_src} bf16 dense burst (MEASURED_PEAKS.json)",
                     # the same kernel against the measured sustained (power-capped) peak,
                     # the denominator for a kernel timed inside long runs of steps
                     "peak_sustained": peaks.get("bf16_tflops_sustained"),
                     "frac_of_sustained": (round(achieved / float(peaks["bf16_tflops_sustained"]), 3)
                                           if peaks.get("bf16_tflops_sustained") else None),
                     "traffic": traffic, "algorithmic_bytes": model[dom]["bytes"]},
        "stages": stages,
        "clocks": res["clocks"],
        "e2e": res.get("e2e"),
        "gpu_launches": res["gpu_launches"],
    }
    if res.get("sweep"):
        line["sweep"] = res["sweep"]
    if res.get("trunk"):
        line["trunk"] = res["trunk"]
    if res.get("train"):
        line["train"] = res["train"]
    if res.get("comm"):
        line["comm"] = res["comm"]
    if res.get("trace"):
        line["trace"] = res["trace"]
    if res.get("stage_note"):
        line["stages_note"] = res["stage_note"]
    for key in ("parity", "contraction_n1024", "small_n"):
        if res.get(key):
            line[key] = res[key]
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--n", type=int, default=N_DEFAULT)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-trunk", action="store_true")
    ap.add_argument("--no-full-reference", action="store_true",
                    help="reference arm: skip the one full-size CPU forward")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own GPU kernels (reference_gpu key)")
    ap.add_argument("--trace-timed", action="store_true",
                    help="N>1: keep the timeline markers on during the timed steps (diagnostic)")
    ap.add_argument("--trace", action="store_true",
                    help="N>1: add the device-clock timeline of one forward per rank (trace key)")
    ap.add_argument("--push", default=None, choices=["ce", "sm"],
                    help="N>1: pushes of the native pipeline by copy engines (ce) or by a kernel "
                         "of vector stores (sm)")
    ap.add_argument("--row-chunks", type=int, default=None,
                    help="input-stage row chunks of the native sharded pipeline (N>1)")
    ap.add_argument("--chunks", type=int, default=None,
                    help="channel chunks of the exchange (N>1; default 4 for all-gather, 2 for all-to-all)")
    ap.add_argument("--scheme", default=None,
                    choices=["p2p_allgather", "p2p_alltoall", "allgather", "alltoall", "allgather_ce",
                             "alltoall_ce", "fused"],
                    help="multi-GPU exchange (default: the native pipeline, p2p_allgather at 2 GPUs "
                         "in outgoing mode, p2p_alltoall otherwise)")
    ap.add_argument("--profile-case", type=int, default=0, metavar="N",
                    help="run a few plain forwards at this N (for ncu captures) and exit")
    ap.add_argument("--mode", default="outgoing", choices=["outgoing", "incoming"])
    ap.add_argument("--reference-gpu-sweep", type=int, nargs="*", default=None, metavar="N",
                    help="time the reference's own GPU kernels (baseline/_ref, CUDA-graphed) at "
                         "these N and print one JSON line each")
    ap.add_argument("--contraction-vs-cublas", type=int, nargs="*", default=None, metavar="N",
                    help="time the contraction kernel alone against cuBLAS bmm (short and "
                         "sustained, with energy and clocks) at these N and exit")
    ap.add_argument("--profile-shard", type=int, default=0, metavar="P",
                    help="with --profile-case: run one rank's kernels of the P-way channel-sharded "
                         "forward on this GPU (no communication)")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args)
        return
    if args.contraction_vs_cublas is not None:
        contraction_vs_cublas(args.contraction_vs_cublas or [1024, 2048])
        return
    if args.reference_gpu_sweep is not None:
        reference_gpu_sweep(args.reference_gpu_sweep or [256, 512, 1024, 2048])
        return
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    if args.push:
        os.environ["FTM_SHARD_PUSH"] = args.push
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 or args.gpus > 1:
        from fast_trimul_b200.distributed import bench_sharded
        res = bench_sharded(args, torch)
        if res is None:      # non-zero ranks
            return
    else:
        res = bench_single(args, torch)

    line = build_line(args, res, world)
    if world == 1 and not args.no_reference_gpu:
        rg = reference_gpu_subprocess()
        if isinstance(rg, list):
            ours = {r["n"]: r["ms"] for r in (line.get("sweep") or []) if r["mode"] == "outgoing"}
            ours.update({r["n"]: r["graphed_ms"] for r in (res.get("small_n") or [])})   # graphed vs graphed
            ours[args.n] = line["ms_per_step"]
            for r in rg:
                if r.get("n") in ours and r.get("graphed_ms"):
                    r["ours_ms"] = ours[r["n"]]
                    r["speedup_vs_graphed"] = round(r["graphed_ms"] / ours[r["n"]], 2)
        line["reference_gpu"] = rg
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_line()
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
