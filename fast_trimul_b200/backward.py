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


# --------------------------------------------------------------------------- native
_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


def _mm32(a, b):
    """a @ b of fp16 operands with an fp32 result (fp32 accumulation in cuBLAS)."""
    try:
        return torch.mm(a, b, out_dtype=torch.float32)
    except (TypeError, RuntimeError):
        return torch.mm(a.float(), b.float())


def native_plane_grads_pos(dx_plane, a16, b16, mode):
    """Gradients of the contraction's operands as fp16 planes in position order.

    dx_plane: (L, N, N) fp32 dX[l][i][j]; a16, b16: (L, N, N) fp16 planes of the forward.
    Returns (dA, dB, scale) with scale a one-element device tensor: dA[l][u][v] * scale is
    the gradient of a at position (u, v) of channel l (likewise dB) in both modes --
    incoming mode's transposed planes are undone by choosing the operand order
    (dA^T = B^T dX^T is computed directly), so no transpose pass is needed. The scale
    stays on the device: no host synchronisation."""
    lib = _lib.load()
    L, N, _ = dx_plane.shape
    # max |dX|, kept away from zero so an all-zero gradient gives zeros, not NaNs
    scale = dx_plane.abs().amax().clamp_min(1e-30).reshape(1)
    dA = torch.empty(L, N, N, dtype=torch.float16, device=dx_plane.device)
    dB = torch.empty_like(dA)
    dx16 = (dx_plane / scale).to(torch.float16)
    err = _lib_err(dx_plane.device)
    s = torch.cuda.current_stream(dx_plane.device).cuda_stream
    if mode == "outgoing":
        # dA[i][k] = sum_j dX[i][j] B[j][k];  dB[j][k] = sum_i dX[i][j] A[i][k]
        jobs = ((dA, dx16, 0, b16, 1), (dB, dx16, 1, a16, 1))
    else:
        # transposed: dA^T[k][i] = sum_j B[j][k] dX[i][j];  dB^T[k][j] = sum_i A[i][k] dX[i][j]
        jobs = ((dA, b16, 1, dx16, 0), (dB, a16, 1, dx16, 1))
    for out, a, a_mn, b, b_mn in jobs:
        d = _lib.ContractionLayout()
        d.L, d.m, d.n, d.k, d.k_per_block = L, N, N, N, 0
        d.a, d.a_l_stride, d.a_row_stride, d.a_mn_major = a.data_ptr(), N * N, N, a_mn
        d.b, d.b_l_stride, d.b_row_stride, d.b_mn_major = b.data_ptr(), N * N, N, b_mn
        d.x, d.x_l_stride, d.x_row_stride = out.data_ptr(), N * N, N
        _lib.check(lib.ftm_contraction_general(ctypes.byref(d), err, s), "ftm_contraction_general")
        _lib.stats["kernel_launches"] += 1
    return dA, dB, scale


def backward_native(mod, z, mask, params, planes, grad_out):
    """Gradients of z and of the 16 parameters (`_params()` order): per-position GEMMs on
    cuBLAS (fp16 operands, fp32 accumulation), the N^3 products on the native
    contraction kernel, everything elementwise in the ftm_bwd_* kernels. The output
    gradient is divided by its largest magnitude first and every result multiplied back,
    so the fp16 intermediates neither underflow nor overflow."""
    lib = _lib.load()
    dev = z.device
    s = torch.cuda.current_stream(dev).cuda_stream
    a16, b16, x16 = planes
    B, N = z.shape[0], z.shape[1]
    C = 128
    P = B * N * N
    L = B * C
    p = params
    W_all = torch.cat([p[4], p[6], p[8], p[10], p[12]]).to(torch.float16).contiguous()
    b_in = torch.cat([p[5], p[7], p[9], p[11]]).float().contiguous()
    b_g, W_o, b_o = p[13].float().contiguous(), p[14].to(torch.float16).contiguous(), p[15].float().contiguous()
    g_in, be_in = p[0].float().contiguous(), p[1].float().contiguous()
    g_out, be_out = p[2].float().contiguous(), p[3].float().contiguous()
    zc = z if z.dtype in _DT else z.float()
    zc = zc.contiguous()
    m = None if mask is None else mask.to(device=dev, dtype=torch.float32).expand(B, N, N).contiguous()
    mp = None if m is None else m.data_ptr()
    gout = grad_out.contiguous()
    if gout.dtype not in _DT:
        gout = gout.float()
    # largest |dout| as a device scalar (no host synchronisation), kept away from zero
    gmax = gout.abs().amax().float().clamp_min(1e-30).reshape(1)
    gsc = (1.0 / gmax).contiguous()
    chk = _lib.check

    zn = torch.empty(P, C, dtype=torch.float16, device=dev)
    zst = torch.empty(P, 2, dtype=torch.float32, device=dev)
    chk(lib.ftm_bwd_ln_in(zc.data_ptr(), _DT[zc.dtype], mp, g_in.data_ptr(), be_in.data_ptr(),
                          float(mod.norm_in.eps), zn.data_ptr(), zst.data_ptr(), P, s), "ftm_bwd_ln_in")
    H = zn @ W_all.t()                                          # (P, 640) without biases
    xn = torch.empty(P, C, dtype=torch.float16, device=dev)
    xst = torch.empty(P, 2, dtype=torch.float32, device=dev)
    chk(lib.ftm_bwd_x_ln(x16.data_ptr(), g_out.data_ptr(), be_out.data_ptr(), float(mod.norm_out.eps),
                         xn.data_ptr(), xst.data_ptr(), B, N, s), "ftm_bwd_x_ln")
    O = xn @ W_o.t()
    dO = torch.empty(P, C, dtype=torch.float16, device=dev)
    dPGZ = torch.empty(P, 640, dtype=torch.float16, device=dev)
    nb = lib.ftm_bwd_partial_blocks()
    part_g = torch.empty(nb, 2 * C, dtype=torch.float32, device=dev)
    chk(lib.ftm_bwd_gate(O.data_ptr(), b_o.data_ptr(), H.data_ptr(), b_g.data_ptr(), gout.data_ptr(),
                         _DT[gout.dtype], gsc.data_ptr(), mp, dO.data_ptr(), dPGZ.data_ptr(), part_g.data_ptr(),
                         P, s), "ftm_bwd_gate")
    del O
    dxn = dO @ W_o
    dW_o = _mm32(dO.t(), xn)
    sg = part_g.sum(0)
    db_o, db_gz = sg[:C], sg[C:]
    part = torch.empty(nb, 2 * C, dtype=torch.float32, device=dev)
    dxp = torch.empty(L, N, N, dtype=torch.float32, device=dev)
    chk(lib.ftm_bwd_x_ln_bwd(x16.data_ptr(), xst.data_ptr(), dxn.data_ptr(), g_out.data_ptr(),
                             dxp.data_ptr(), part.data_ptr(), B, N, s), "ftm_bwd_x_ln_bwd")
    pg = part.sum(0)
    dg_out, db_out = pg[:C], pg[C:]
    del dxn, xn, dO
    dA, dB, dsc = native_plane_grads_pos(dxp, a16.reshape(L, N, N), b16.reshape(L, N, N), mod.mode)
    del dxp
    part_in = torch.empty(nb, 4 * C, dtype=torch.float32, device=dev)
    chk(lib.ftm_bwd_gates_in(dA.data_ptr(), dB.data_ptr(), dsc.data_ptr(), H.data_ptr(), b_in.data_ptr(),
                             dPGZ.data_ptr(), part_in.data_ptr(), B, N, s), "ftm_bwd_gates_in")
    del dA, dB, H
    dzn = dPGZ @ W_all                                          # (P, 128)
    dW_all = _mm32(dPGZ.t(), zn)                                # (640, 128)
    db_all = torch.cat([part_in.sum(0), db_gz])
    del dPGZ, zn
    dz = torch.empty(z.shape, dtype=zc.dtype, device=dev)
    part2 = torch.empty(nb, 2 * C, dtype=torch.float32, device=dev)
    chk(lib.ftm_bwd_ln_in_bwd(zc.data_ptr(), _DT[zc.dtype], mp, zst.data_ptr(), dzn.data_ptr(),
                              g_in.data_ptr(), gout.data_ptr(), _DT[gout.dtype], gsc.data_ptr(),
                              1 if mod.residual else 0, dz.data_ptr(), _DT[dz.dtype],
                              part2.data_ptr(), P, s), "ftm_bwd_ln_in_bwd")
    pg2 = part2.sum(0)
    _lib.stats["kernel_launches"] += 6
    grads32 = [pg2[:C], pg2[C:], dg_out, db_out]
    for q in range(4):
        grads32 += [dW_all[q * C:(q + 1) * C], db_all[q * C:(q + 1) * C]]
    grads32 += [dW_all[4 * C:], db_all[4 * C:], dW_o, db_o]
    gp = [(g * gmax).to(t.dtype) for g, t in zip(grads32, params)]
    dz = dz.mul_(gmax).to(z.dtype)
    return dz, gp
