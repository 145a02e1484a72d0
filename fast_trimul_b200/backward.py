"""Training path: native forward, backward with the contraction's gradients on the
sm_100a tensor-core kernel.

The reference trains through `_TrainableTriMul` (fast_trimul/_kernels.py:468-488): its
backward re-runs the whole forward in PyTorch (`_torch_forward`, :532-547) and
differentiates that, so every backward pays one extra N^3 contraction and two more
for the gradients, all through torch.einsum.

Here the forward is the three native kernels, and it keeps the fp16 channel-major
planes a, b (the contraction's operands) and x (its result). The backward then

* recomputes only the per-position parts (input LayerNorm, the four projections and
  gates, the output LayerNorm, projection and gate) with torch autograd, in the
  weights' dtype (fp16 for the module, like the reference's backward; fp32 weights give
  an fp32 recompute);
* takes x from the forward instead of recomputing the contraction;
* computes the contraction's gradients natively, on the tcgen05 contraction kernel
  with MN-major operands (no transpose pass) --
      dA[c][i][k] = sum_j dX[c][i][j] B[c][j][k]      (A = dX K-major, B MN-major)
      dB[c][j][k] = sum_i dX[c][i][j] A[c][i][k]      (A = dX MN-major, B MN-major)
  -- on the planes as stored, which is the same product in both modes (incoming mode's
  planes are the transposed ones the forward contracted).

dX is rescaled to a maximum magnitude of 1 before it is rounded to fp16 (and the
products scaled back in fp32), so small loss gradients neither underflow nor lose
precision in the fp16 operand.
"""

import ctypes

import torch
import torch.nn.functional as F

from . import _lib


def _planes(t, mode):
    """(B, N, N, C) position-major -> the (B, C, N, N) channel-major plane view the
    contraction reads: outgoing [c][i][k] = t[i, k, c]; incoming [c][i][k] = t[k, i, c]."""
    return t.permute(0, 3, 1, 2) if mode == "outgoing" else t.permute(0, 3, 2, 1)


def native_plane_grads(dx_plane, a_plane, b_plane):
    """dA = dX B and dB = dX^T A per channel plane on the native kernel.

    dx_plane: (L, N, N) gradient of X[l][i][j]; a_plane, b_plane: (L, N, N) fp16
    contiguous operands of the forward (A[l][i][k], B[l][j][k]). Returns (dA, dB) in
    dx_plane's dtype."""
    lib = _lib.load()
    L, N, _ = dx_plane.shape
    scale = dx_plane.abs().amax().float()
    if scale.item() == 0.0:
        return torch.zeros_like(dx_plane), torch.zeros_like(dx_plane)
    dx16 = (dx_plane.float() / scale).to(torch.float16).contiguous()
    dA = torch.empty(L, N, N, dtype=torch.float16, device=dx_plane.device)
    dB = torch.empty_like(dA)
    err = _lib_err(dx_plane.device)
    s = torch.cuda.current_stream(dx_plane.device).cuda_stream
    for out, a, a_mn, b in ((dA, dx16, 0, b_plane), (dB, dx16, 1, a_plane)):
        d = _lib.ContractionLayout()
        d.L, d.m, d.n, d.k, d.k_per_block = L, N, N, N, 0
        d.a, d.a_l_stride, d.a_row_stride, d.a_mn_major = a.data_ptr(), N * N, N, a_mn
        d.b, d.b_l_stride, d.b_row_stride, d.b_mn_major = b.data_ptr(), N * N, N, 1
        d.x, d.x_l_stride, d.x_row_stride = out.data_ptr(), N * N, N
        _lib.check(lib.ftm_contraction_general(ctypes.byref(d), err, s), "ftm_contraction_general")
        _lib.stats["kernel_launches"] += 1
    return (dA.float() * scale).to(dx_plane.dtype), (dB.float() * scale).to(dx_plane.dtype)


def _lib_err(device):
    from ._module import device_error_word
    return device_error_word(device).ptr


class _SavedContraction(torch.autograd.Function):
    """x from the native forward; the gradients of its operands from native_plane_grads."""

    @staticmethod
    def forward(ctx, a_pl, b_pl, x16, a16, b16):
        ctx.save_for_backward(a16, b16)
        return x16.to(a_pl.dtype)

    @staticmethod
    def backward(ctx, dx):
        a16, b16 = ctx.saved_tensors
        B, C, N, _ = dx.shape
        dA, dB = native_plane_grads(dx.reshape(B * C, N, N), a16.view(B * C, N, N),
                                    b16.view(B * C, N, N))
        return dA.view(B, C, N, N), dB.view(B, C, N, N), None, None, None


def backward(mod, z, mask, params, planes, grad_out):
    """Gradients of z and of the 16 parameters (in `_params()` order) for one forward.

    planes: (a16, b16, x16), the forward's fp16 channel-major planes (B, C, N, N)."""
    a16, b16, x16 = planes
    eps_in, eps_out = mod.norm_in.eps, mod.norm_out.eps
    # the per-position parts run in the weights' dtype (fp16 for the module, as the
    # reference's own backward does), fp32 when the weights are fp32
    ct = params[0].dtype if params[0].dtype in (torch.float16, torch.bfloat16) else torch.float32
    with torch.enable_grad():
        zq = z.detach().to(ct).requires_grad_(True)
        p = [t.detach().to(ct).requires_grad_(True) for t in params]
        m = None if mask is None else mask.to(ct).expand(z.shape[:3]).unsqueeze(-1)
        zm = zq if m is None else zq * m
        zn = F.layer_norm(zm, (zm.shape[-1],), p[0], p[1], eps_in)
        a = F.linear(zn, p[4], p[5]) * torch.sigmoid(F.linear(zn, p[6], p[7]))
        b = F.linear(zn, p[8], p[9]) * torch.sigmoid(F.linear(zn, p[10], p[11]))
        xp = _SavedContraction.apply(_planes(a, mod.mode), _planes(b, mod.mode), x16, a16, b16)
        x = xp.permute(0, 2, 3, 1)                       # (B, N, N, C): x[b, i, j, c]
        xn = F.layer_norm(x, (x.shape[-1],), p[2], p[3], eps_out)
        delta = torch.sigmoid(F.linear(zn, p[12], p[13])) * F.linear(xn, p[14], p[15])
        out = zm + delta if mod.residual else delta
        if m is not None:
            out = out * m
    grads = torch.autograd.grad(out, [zq] + p, grad_out.to(ct), allow_unused=True)
    gz = grads[0].to(z.dtype)
    gp = [g.to(t.dtype) if g is not None else None for g, t in zip(grads[1:], params)]
    return gz, gp
