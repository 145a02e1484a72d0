"""Generate the golden fixtures in this folder by running the REFERENCE itself.

Run in a container that has the reference checkout (read-only) and a CPU torch:

    python tests/golden/make_golden.py /path/to/fast_trimul_checkout

The reference has no golden vectors of its own (all its parity tests compare seeded
random inputs against its in-repo torch math), so the fixtures are produced here from:

* `FastTriangleMultiplication(..., backend="torch")` -- the reference's production
  CPU path: fp16 weights (ops/triangle.py:39), mask before/after and dtype casts
  (backends/torch_ref.py:26-35), `_torch_forward` (_kernels.py:532-547);
* the same module's `_torch_forward` run with fp32 copies of its fp16-rounded
  parameters -- the "fp32 reference" the tolerance is stated against.

Two runtime shims, no edits to the reference: the CLI-only `cutlass.testing`
import (_tensorop_gemm.py:41) gets a stub module, and `torch.cuda.get_device_properties`
(called at import by _kernels.py:300) returns a stand-in when no GPU is present.
"""

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, B, N, d_z, d_c, mode, residual, mask kind, input dtype)
CASES = [
    ("out_n16_d32_res", 1, 16, 32, 32, "outgoing", True, None, torch.float32),
    ("in_n16_d32_res", 1, 16, 32, 32, "incoming", True, None, torch.float32),
    ("out_n24_d32_delta_tailmask", 1, 24, 32, 32, "outgoing", False, "tail", torch.float32),
    ("in_n24_d32_delta_tailmask", 1, 24, 32, 32, "incoming", False, "tail", torch.float32),
    ("out_b2_n8_d16_res_padmask", 2, 8, 16, 16, "outgoing", True, "pad", torch.float32),
    ("in_b2_n8_d16_res_padmask", 2, 8, 16, 16, "incoming", True, "pad", torch.float32),
    ("out_n16_d128_res_tailmask_bf16", 1, 16, 128, 128, "outgoing", True, "tail", torch.bfloat16),
    ("in_n16_d128_delta_bf16", 1, 16, 128, 128, "incoming", False, None, torch.bfloat16),
    ("in_n24_d128_res_padmask", 1, 24, 128, 128, "incoming", True, "pad", torch.float32),
]


def _shim_and_import(ref_root):
    import cutlass  # noqa: F401  (nvidia-cutlass-dsl)
    if "cutlass.testing" not in sys.modules:
        stub = types.ModuleType("cutlass.testing")
        sys.modules["cutlass.testing"] = stub
        cutlass.testing = stub
    if not torch.cuda.is_available():
        props = types.SimpleNamespace(multi_processor_count=148,
                                      max_threads_per_multi_processor=2048)
        torch.cuda.get_device_properties = lambda *a, **k: props
    sys.path.insert(0, ref_root)
    import fast_trimul                         # the reference package
    from fast_trimul import FastTriangleMultiplication
    assert os.path.dirname(fast_trimul.__file__).startswith(os.path.abspath(ref_root))
    return FastTriangleMultiplication


def _mask(kind, B, N, gen):
    if kind is None:
        return None
    if kind == "tail":                         # residue mask with the last 10% zero
        r = torch.ones(B, N)
        r[:, int(0.9 * N):] = 0
    else:                                      # per-sample padding lengths
        r = torch.zeros(B, N)
        for b in range(B):
            L = int(torch.randint(N // 2, N + 1, (1,), generator=gen))
            r[b, :L] = 1
    return r[:, :, None] * r[:, None, :]


def main(ref_root):
    FTM = _shim_and_import(ref_root)
    for name, B, N, dz, dc, mode, residual, mkind, dt in CASES:
        torch.manual_seed(0)
        mod = FTM(dz, dc, mode=mode, residual=residual, backend="torch").eval()
        # non-trivial LayerNorm affine so gamma/beta handling is pinned too
        with torch.no_grad():
            for ln in (mod._impl.norm_in, mod._impl.norm_out):
                ln.weight.copy_(1.0 + 0.1 * torch.randn_like(ln.weight))
                ln.bias.copy_(0.1 * torch.randn_like(ln.bias))
        gen = torch.Generator().manual_seed(1)
        z = torch.randn(B, N, N, dz, generator=gen).to(dt)
        mask = _mask(mkind, B, N, gen)
        with torch.no_grad():
            out16 = mod(z, mask=mask)                               # production path
            impl32 = mod._impl.float()                              # fp16-rounded values in fp32
            zf = z.float() if mask is None else z.float() * mask[..., None]
            out32 = impl32._torch_forward(zf, impl32._params())
            if mask is not None:
                out32 = out32 * mask[..., None]
            mod._impl.half()
        sd = {k: v.detach().float().numpy() for k, v in mod._impl.state_dict().items()}
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            z=z.float().numpy(), z_dtype=str(dt).replace("torch.", ""),
            mask=(mask.numpy() if mask is not None else np.zeros(0, np.float32)),
            has_mask=mask is not None, mode=mode, residual=residual,
            out_ref_fp16_path=out16.float().numpy(), out_ref_fp32=out32.numpy(),
            **{"p:" + k: v for k, v in sd.items()})
        print(name, tuple(z.shape), float(out32.abs().mean()))


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FAST_TRIMUL_REFERENCE")
    if not ref:
        sys.exit("usage: make_golden.py <reference checkout> (or set FAST_TRIMUL_REFERENCE)")
    main(ref)
