"""CPU oracle for the triangle multiplicative update forward (TEST INFRASTRUCTURE).

This module is the checker, never the product: only `tests/`, `__graft_entry__.smoke()`
and `bench.py`'s CPU-baseline / reference arm may import it. The product path
(`fast_trimul_b200`) never calls into it and fails loudly if its CUDA library is missing.

It restates, in numpy float32 (or float64), the reference's pure-torch forward:

* `_torch_forward`  -- fast_trimul/_kernels.py:532-547 (param order :512-517,
  LayerNorm eps = nn.LayerNorm default 1e-5, :503/:508)
* mask handling     -- fast_trimul/functional.py:19-26 and
  fast_trimul/backends/torch_ref.py:26-35: z is multiplied by the pair mask
  BEFORE the input LayerNorm, and the result is multiplied by the mask again.
* outgoing / incoming contraction -- _kernels.py:541-544
  ('bikc,bjkc->bijc' and 'bkic,bjkc->bijc').
* residual flag     -- _kernels.py:547 (z + delta, or delta only).

Parity pin: tests/golden/*.npz were produced by importing the reference itself
(tests/golden/make_golden.py); tests/test_oracle_golden.py checks this module
against them (fp32 reference math to ~1e-5, the reference's fp16 production path
to fp16 tolerance).
"""

import numpy as np

# parameter names in the reference's state_dict (_kernels.py:503-510)
PARAM_NAMES = (
    "norm_in.weight", "norm_in.bias", "norm_out.weight", "norm_out.bias",
    "proj_a.weight", "proj_a.bias", "gate_a.weight", "gate_a.bias",
    "proj_b.weight", "proj_b.bias", "gate_b.weight", "gate_b.bias",
    "proj_g.weight", "proj_g.bias", "proj_out.weight", "proj_out.bias",
)


def layer_norm(x, w, b, eps=1e-5):
    """nn.LayerNorm over the last dim: biased variance, eps inside the sqrt."""
    mean = x.mean(axis=-1, keepdims=True)
    xc = x - mean
    var = (xc * xc).mean(axis=-1, keepdims=True)
    return xc / np.sqrt(var + eps) * w + b


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def linear(x, w, b):
    """x @ w^T + b over the last dim (as a single 2-D BLAS call)."""
    lead = x.shape[:-1]
    y = x.reshape(-1, x.shape[-1]) @ w.T
    y += b
    return y.reshape(*lead, w.shape[0])


def contract(a, b, mode):
    """x[b,i,j,c] = sum_k a[b,i,k,c] b[b,j,k,c] (outgoing) or
    sum_k a[b,k,i,c] b[b,k,j,c] (incoming); _kernels.py:541-544.
    Done as a batched matmul over (batch, channel) so BLAS does the work."""
    A = np.ascontiguousarray(np.transpose(a, (0, 3, 1, 2)))   # (B, C, N, N)
    Bm = np.ascontiguousarray(np.transpose(b, (0, 3, 1, 2)))
    if mode == "outgoing":
        x = A @ np.swapaxes(Bm, -1, -2)                          # [i,k]·[j,k]^T
    elif mode == "incoming":
        x = np.swapaxes(A, -1, -2) @ Bm                          # [k,i]^T·[k,j]
    else:
        raise ValueError(f"mode must be 'outgoing' or 'incoming', got {mode!r}")
    return np.ascontiguousarray(np.transpose(x, (0, 2, 3, 1)))  # (B, N, N, C)


def torch_forward(z, p, mode, residual, eps_in=1e-5, eps_out=1e-5):
    """Restatement of _kernels.py:532-547 (`p` maps PARAM_NAMES to arrays)."""
    zc = layer_norm(z, p["norm_in.weight"], p["norm_in.bias"], eps_in)
    a = linear(zc, p["proj_a.weight"], p["proj_a.bias"]) * sigmoid(
        linear(zc, p["gate_a.weight"], p["gate_a.bias"]))
    b = linear(zc, p["proj_b.weight"], p["proj_b.bias"]) * sigmoid(
        linear(zc, p["gate_b.weight"], p["gate_b.bias"]))
    m = contract(a, b, mode)
    mc = layer_norm(m, p["norm_out.weight"], p["norm_out.bias"], eps_out)
    g = sigmoid(linear(zc, p["proj_g.weight"], p["proj_g.bias"]))
    delta = g * linear(mc, p["proj_out.weight"], p["proj_out.bias"])
    return z + delta if residual else delta


def trimul_forward(z, params, mode="outgoing", residual=True, mask=None,
                   dtype=np.float32):
    """The reference's functional / torch-backend semantics in `dtype` arithmetic.

    z: (B, N, N, c_z) array, mask: (B, N, N) or None, params: dict of arrays
    (for an fp32 reference of the reference's fp16 module, pass the fp16-rounded
    values cast up). Returns (B, N, N, c_z) in `dtype`.
    """
    z = np.asarray(z, dtype=dtype)
    p = {k: np.asarray(params[k], dtype=dtype) for k in PARAM_NAMES}
    if z.ndim != 4:
        raise ValueError("z must be (B, N, N, c_z)")
    if mask is not None:
        m = np.asarray(mask, dtype=dtype)[..., None]
        z = z * m
    out = torch_forward(z, p, mode, residual)
    if mask is not None:
        out = out * m
    return out


def trimul_flops(batch, n, c_z, c_h):
    """Algorithmic FLOPs of one forward (fast_trimul/benchmark.py:77-83)."""
    m = batch * n * n
    gemm = 4 * 2 * m * c_z * c_h + 2 * m * c_z * c_z + 2 * m * c_h * c_z
    return gemm + 2 * batch * c_h * n ** 3


def error_metrics(got, ref):
    """max-abs and mean-relative (mean|got-ref| / mean|ref|) errors."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(got - ref)
    denom = float(np.abs(ref).mean())
    return float(d.max()) if d.size else 0.0, (float(d.mean()) / denom if denom > 0 else float(d.mean()))
