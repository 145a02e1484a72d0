"""Build libfast_trimul_b200.so in-tree with nvcc for sm_100a.

    python -m fast_trimul_b200.csrc.build          # or:  python fast_trimul_b200/csrc/build.py

The library depends only on the CUDA runtime (linked statically); it has no
PyTorch dependency, so any host language can load it through the C ABI in
include/fast_trimul_b200.h.
"""

import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "libfast_trimul_b200.so")
SOURCES = ["ftm_api.cu", "ftm_pack.cu", "ftm_input_stage.cu", "ftm_contraction.cu", "ftm_contraction2.cu",
           "ftm_output_stage.cu", "ftm_shard.cu", "ftm_backward.cu", "ftm_noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
          "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA toolkit on PATH)")


def _stale(obj, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose=False, ptxas_info=False, force=False):
    """Compile every kernel for sm_100a and link the shared library. Returns its path."""
    cc = nvcc()
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    headers = [os.path.join(HERE, h) for h in os.listdir(HERE) if h.endswith((".cuh", ".h"))]
    headers.append(os.path.join(ROOT, "include", "fast_trimul_b200.h"))
    jobs = []
    for src in SOURCES:
        s = os.path.join(HERE, src)
        o = os.path.join(objdir, src.replace(".cu", ".o"))
        if force or _stale(o, [s] + headers):
            cmd = [cc] + ARCH + CFLAGS + (["-Xptxas", "-v"] if ptxas_info else []) + ["-c", s, "-o", o]
            jobs.append((src, cmd))
    objs = [os.path.join(objdir, s.replace(".cu", ".o")) for s in SOURCES]

    def run(job):
        name, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return name, r

    with concurrent.futures.ThreadPoolExecutor(max_workers=len(jobs) or 1) as ex:
        for name, r in ex.map(run, jobs):
            if verbose or ptxas_info or r.returncode:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode:
                raise RuntimeError(f"nvcc failed on {name}")
    if force or jobs or _stale(LIB, objs):
        cmd = [cc] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", LIB] + objs + ["-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc link failed")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv, force="-f" in sys.argv))
