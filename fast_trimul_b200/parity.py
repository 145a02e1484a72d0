"""fp32 evaluation of selected output rows, for parity checks at sizes where a full
fp32 forward on the host is too slow.

The formula is the reference's pure-torch forward (fast_trimul/_kernels.py:532-547)
with the functional entry's mask rules (fast_trimul/functional.py:19-26: z is
multiplied by the pair mask before the input LayerNorm, and the result again), run
in fp32 on whatever device the inputs live on, with TF32 off. Only the rows asked
for are contracted and projected, so an N = 2048 check costs one pass of the input
projections over all positions plus `len(rows)` row contractions.

Outgoing row i needs a[i, :, :] and all of b; incoming row i needs a[:, i, :] (the
column) and all of b -- both are taken from the full fp32 projections.
"""

import torch
import torch.nn.functional as F


def _params32(impl):
    return [t.detach().float() for t in impl._params()]


@torch.no_grad()
def reference_rows(impl, z, mask, rows, chunk_rows=256):
    """fp32 output rows `rows` (a list of i) of every batch element: (B, len(rows), N, c_z).

    impl: the parameter module (`FastTriangleMultiplication._impl`); z: (B, N, N, c_z)
    in the dtype the kernels see; mask: (B, N, N) or None.
    """
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return _reference_rows(impl, z, mask, list(rows), chunk_rows)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _reference_rows(impl, z, mask, rows, chunk_rows):
    p = _params32(impl)
    eps_in, eps_out = impl.norm_in.eps, impl.norm_out.eps
    B, N, _, dz = z.shape
    dc = p[4].shape[0]
    outgoing = impl.mode == "outgoing"
    ridx = torch.tensor(rows, device=z.device, dtype=torch.long)
    outs = []
    for bi in range(B):
        m = None if mask is None else mask[bi].float()
        # b over all positions (k-major per row j), and the a rows / columns needed
        bfull = torch.empty(N, N, dc, device=z.device, dtype=torch.float32)
        a_sel = torch.empty(len(rows), N, dc, device=z.device, dtype=torch.float32)
        for r0 in range(0, N, chunk_rows):
            r1 = min(N, r0 + chunk_rows)
            zz = z[bi, r0:r1].float()
            if m is not None:
                zz = zz * m[r0:r1, :, None]
            zn = F.layer_norm(zz, (dz,), p[0], p[1], eps_in)
            bfull[r0:r1] = F.linear(zn, p[8], p[9]) * torch.sigmoid(F.linear(zn, p[10], p[11]))
            a = F.linear(zn, p[4], p[5]) * torch.sigmoid(F.linear(zn, p[6], p[7]))
            if outgoing:
                for t, i in enumerate(rows):
                    if r0 <= i < r1:
                        a_sel[t] = a[i - r0]
            else:
                a_sel[:, r0:r1] = a[:, ridx].permute(1, 0, 2)      # a[k, i, :] for k in chunk
        # outgoing: x[t, j, c] = sum_k a_sel[t, k, c] * b[j, k, c];
        # incoming: x[t, j, c] = sum_k a_sel[t, k, c] * b[k, j, c]
        bk = bfull.permute(2, 1, 0) if outgoing else bfull.permute(2, 0, 1)     # (c, k, j)
        x = torch.bmm(a_sel.permute(2, 0, 1), bk).permute(1, 2, 0)
        xn = F.layer_norm(x, (dc,), p[2], p[3], eps_out)
        zz = z[bi, ridx].float()
        if m is not None:
            zz = zz * m[ridx][:, :, None]
        zn = F.layer_norm(zz, (dz,), p[0], p[1], eps_in)
        delta = torch.sigmoid(F.linear(zn, p[12], p[13])) * F.linear(xn, p[14], p[15])
        o = zz + delta if impl.residual else delta
        if m is not None:
            o = o * m[ridx][:, :, None]
        outs.append(o)
    return torch.stack(outs)


def error_metrics(got, ref):
    """(max-abs, mean-relative) of `got` against `ref`: mean|got - ref| / mean|ref|."""
    d = (got.double() - ref.double()).abs()
    denom = ref.double().abs().mean().item()
    return d.max().item(), d.mean().item() / denom if denom > 0 else d.mean().item()


def sample_rows(n, count, lo=0):
    """`count` distinct rows spread evenly over [lo, lo + n), first and last included."""
    count = max(1, min(count, n))
    if count == 1:
        return [lo]
    return sorted({lo + round(t * (n - 1) / (count - 1)) for t in range(count)})
