"""The parameter-holding module behind `FastTriangleMultiplication._impl`.

Same parameter names, order and init as the reference's
`TriangleMultiplicativeUpdateKernelFused` (fast_trimul/_kernels.py:491-552), so
state_dicts and the weight loaders carry over unchanged:
norm_in, proj_a, gate_a, proj_b, gate_b, norm_out, proj_g, proj_out.

Forward paths:
* `_forward_native` -- the three sm_100a kernels through the C ABI (CUDA tensors);
* `_torch_forward`  -- the pure-torch formula (the "torch" backend and the
  backward recompute), same math as _kernels.py:532-547;
* with grad enabled, `_TrainableTriMul` pairs the native forward with a torch
  recompute for the backward, like _kernels.py:468-488.
"""

import ctypes
import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib

_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


def _linear(d_in, d_out):
    lin = nn.Linear(d_in, d_out)
    # nn.Linear default init, spelled out as in _kernels.py:170-175
    nn.init.kaiming_uniform_(lin.weight, a=math.sqrt(5))
    nn.init.uniform_(lin.bias, -d_in ** -0.5, d_in ** -0.5)
    return lin


class DeviceErrorWord:
    """The sticky error word every module call on one GPU passes to its kernels.

    A kernel whose bounded wait expires records `(kernel << 8) | (role << 4) | site`
    there and drains instead of hanging. After each call an asynchronous 4-byte copy
    moves the word into pinned host memory, followed by an event; the next call reads
    that copy once its event has completed (`poll`, no synchronisation) and raises.
    `check` synchronises and reads the word itself. Both clear the word when they
    report it. Nothing is polled or recorded while the stream is being captured."""

    def __init__(self, device):
        self.device = device
        self.dev = torch.zeros(64, dtype=torch.int32, device=device)
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event = None
        self.side = None
        self.ptr = self.dev.data_ptr()

    def after_launch(self):
        if torch.cuda.is_current_stream_capturing() or _NO_ASYNC_CHECK:
            return
        # the copy runs on a side stream that waits for this point of the calling stream,
        # so a busy copy engine can never hold up the work queued after the call
        if self.side is None:
            self.side = torch.cuda.Stream(self.device)
        done = torch.cuda.Event()
        done.record()
        self.side.wait_event(done)
        with torch.cuda.stream(self.side):
            self.host.copy_(self.dev[:1], non_blocking=True)
            self.event = torch.cuda.Event()
            self.event.record(self.side)

    def _raise(self, code):
        self.dev.zero_()
        self.host.zero_()
        self.event = None
        raise _lib.NativeKernelError(
            f"a bounded device wait expired in a native TriMul kernel (code 0x{code:x}: kernel "
            f"{code >> 8}, role {(code >> 4) & 15}, site {code & 15}); its output is invalid")

    def poll(self):
        if self.event is None or torch.cuda.is_current_stream_capturing():
            return
        if self.event.query():
            code = int(self.host[0])
            self.event = None
            if code:
                self._raise(code)

    def check(self):
        torch.cuda.synchronize(self.device)
        code = int(self.dev[0].item())
        self.event = None
        if code:
            self._raise(code)


_ERROR_WORDS = {}
# FTM_ERROR_POLL=0: no per-call copy of the word (errors then surface at check() only)
_NO_ASYNC_CHECK = __import__("os").environ.get("FTM_ERROR_POLL") == "0"


def device_error_word(device):
    """The process-wide DeviceErrorWord of `device` (created on first use)."""
    device = torch.device(device)
    key = device.index if device.index is not None else torch.cuda.current_device()
    w = _ERROR_WORDS.get(key)
    if w is None:
        w = _ERROR_WORDS[key] = DeviceErrorWord(torch.device("cuda", key))
    return w


class TriangleMultiplicativeUpdateKernelFused(nn.Module):
    """Weights + mode of one TriMul layer (the reference's fused-kernel module)."""

    def __init__(self, d_z: int = 128, d_c: int = 128, mode: str = "outgoing",
                 residual: bool = True):
        super().__init__()
        if mode not in ("outgoing", "incoming"):
            raise ValueError("Mode must be 'outgoing' or 'incoming'")
        self.mode = mode
        self.residual = residual
        self.norm_in = nn.LayerNorm(d_z)
        self.proj_a = _linear(d_z, d_c)
        self.gate_a = _linear(d_z, d_c)
        self.proj_b = _linear(d_z, d_c)
        self.gate_b = _linear(d_z, d_c)
        self.norm_out = nn.LayerNorm(d_c)
        self.proj_g = _linear(d_z, d_z)
        self.proj_out = _linear(d_c, d_z)
        self._packed = None
        self._packed_key = None

    @property
    def d_z(self):
        return self.norm_in.normalized_shape[0]

    @property
    def d_c(self):
        return self.norm_out.normalized_shape[0]

    def _params(self):
        """Parameters in the reference's _params() order (_kernels.py:512-517)."""
        return [self.norm_in.weight, self.norm_in.bias,
                self.norm_out.weight, self.norm_out.bias,
                self.proj_a.weight, self.proj_a.bias, self.gate_a.weight, self.gate_a.bias,
                self.proj_b.weight, self.proj_b.bias, self.gate_b.weight, self.gate_b.bias,
                self.proj_g.weight, self.proj_g.bias, self.proj_out.weight, self.proj_out.bias]

    # ------------------------------------------------------------------ torch path
    def _torch_forward(self, z, p):
        dz, dc = z.shape[-1], p[4].shape[0]
        zn = F.layer_norm(z, (dz,), p[0], p[1], self.norm_in.eps)
        a = F.linear(zn, p[4], p[5]) * torch.sigmoid(F.linear(zn, p[6], p[7]))
        b = F.linear(zn, p[8], p[9]) * torch.sigmoid(F.linear(zn, p[10], p[11]))
        if self.mode == "outgoing":
            x = torch.einsum("bikc,bjkc->bijc", a, b)
        else:
            x = torch.einsum("bkic,bkjc->bijc", a, b)
        xn = F.layer_norm(x, (dc,), p[2], p[3], self.norm_out.eps)
        g = torch.sigmoid(F.linear(zn, p[12], p[13]))
        delta = g * F.linear(xn, p[14], p[15])
        return z + delta if self.residual else delta

    # ----------------------------------------------------------------- native path
    def native_supported(self):
        return self.d_z == 128 and self.d_c == 128

    def packed_params(self):
        """Device buffer of folded weights (ftm_pack_params), rebuilt only when a
        parameter changes (tracked through tensor version counters)."""
        ps = self._params()
        key = (ps[0].device, ps[0].dtype) + tuple((t.data_ptr(), t._version) for t in ps)
        if self._packed is not None and self._packed_key == key:
            return self._packed
        lib = _lib.load()
        dt = ps[0].dtype
        if dt not in (torch.float16, torch.float32) or any(t.dtype != dt for t in ps):
            ps = [t.detach().float().contiguous() for t in ps]
            dt = torch.float32
        else:
            ps = [t.detach().contiguous() for t in ps]
        nbytes = lib.ftm_packed_params_bytes(self.d_z, self.d_c)
        buf = torch.empty(nbytes, dtype=torch.uint8, device=ps[0].device)
        ptrs = (ctypes.c_void_p * 16)(*[t.data_ptr() for t in ps])
        st = lib.ftm_pack_params(ptrs, _DT[dt], self.d_z, self.d_c, buf.data_ptr(),
                                 torch.cuda.current_stream(buf.device).cuda_stream)
        _lib.check(st, "ftm_pack_params")
        _lib.record_launches()
        self._packed, self._packed_key = (buf, ps), key   # keep the sources alive
        return self._packed

    def problem(self, z, out_dtype, rows=None):
        B, R, S, _ = z.shape
        return _lib.Problem(B, R if rows is None else rows, S, self.d_z, self.d_c,
                            _lib.OUTGOING if self.mode == "outgoing" else _lib.INCOMING,
                            1 if self.residual else 0, _DT[z.dtype], _DT[out_dtype],
                            float(self.norm_in.eps), float(self.norm_out.eps))

    def _forward_native(self, z, mask=None, out_dtype=None, keep_planes=False):
        """z: (B, N, N, d_z) CUDA tensor (fp16/bf16; fp32 is converted to fp16 like
        functional.py:23); mask: (B, N, N) or None. Returns z's dtype unless
        `out_dtype` says otherwise. Mask semantics are applied inside the kernels.

        The three stages are launched through the C ABI on the current stream, with
        a, b, x and the LayerNorm statistics in a workspace from torch's caching
        allocator and the device error word of this GPU (`device_error_word`): a
        bounded device wait that expired in an earlier call raises
        `NativeKernelError` here, without a synchronisation."""
        lib = _lib.load()
        if not self.native_supported():
            raise _lib.NativeDeclined(f"native kernels need d_z == d_c == 128, got "
                                      f"{self.d_z}/{self.d_c}")
        out_dtype = z.dtype if out_dtype is None else out_dtype
        if z.dtype not in (torch.float16, torch.bfloat16):
            z = z.to(torch.float16)
        z = z.contiguous()
        if mask is not None:
            mask = mask.to(device=z.device, dtype=torch.float32).expand(z.shape[:3]).contiguous()
        errw = device_error_word(z.device)
        errw.poll()
        packed, _ = self.packed_params()
        prob = self.problem(z, out_dtype)
        if lib.ftm_workspace_bytes(prob) == 0:
            raise _lib.NativeDeclined(f"unsupported problem {tuple(z.shape)}")
        B, N = z.shape[0], z.shape[2]
        plane = (B * self.d_c * N * N * 2 + 255) // 256 * 256
        ws = torch.empty(3 * plane + B * N * N * 8, dtype=torch.uint8, device=z.device)
        base = ws.data_ptr()
        a, b, x, zst = base, base + plane, base + 2 * plane, base + 3 * plane
        out = torch.empty(z.shape, dtype=out_dtype, device=z.device)
        s = torch.cuda.current_stream(z.device).cuda_stream
        mptr = None if mask is None else mask.data_ptr()
        e = errw.ptr
        _lib.check(lib.ftm_input_stage(prob, z.data_ptr(), mptr, packed.data_ptr(), a, b, zst, e, s),
                   "ftm_input_stage")
        _lib.check(lib.ftm_contraction(a, b, x, B * self.d_c, N, N, N, 1, e, s), "ftm_contraction")
        _lib.check(lib.ftm_output_stage(prob, z.data_ptr(), mptr, x, zst, packed.data_ptr(),
                                        out.data_ptr(), e, s), "ftm_output_stage")
        errw.after_launch()
        _lib.stats["calls"] += 1
        _lib.stats["kernel_launches"] += 3
        if keep_planes:
            # fp16 channel-major a, b, x (B, C, N, N) for the backward (views of ws)
            n_el = B * self.d_c * N * N
            views = tuple(ws[off:off + 2 * n_el].view(torch.float16).view(B, self.d_c, N, N)
                          for off in (0, plane, 2 * plane))
            return out, views
        return out

    def check(self, device=None):
        """Synchronise this layer's GPU and raise `NativeKernelError` if a bounded device
        wait expired in any native call since the last check."""
        dev = self.proj_a.weight.device if device is None else torch.device(device)
        if dev.type == "cuda":
            device_error_word(dev).check()

    def forward(self, z: torch.Tensor, mask: torch.Tensor = None) -> torch.Tensor:
        """The fused module's forward (used by `functional.triangle_multiplication`):
        native kernels on CUDA, with a torch-recompute backward when grad is needed."""
        if torch.is_grad_enabled() and (z.requires_grad or any(t.requires_grad for t in self._params())):
            return _TrainableTriMul.apply(self, z, mask, *self._params())
        return self._forward_native(z, mask)


class _TrainableTriMul(torch.autograd.Function):
    """Native forward that keeps the planes a, b, x; native backward: the contraction's
    gradients on the tcgen05 kernel, per-position GEMMs on cuBLAS, the elementwise and
    LayerNorm parts in the ftm_bwd_* kernels (fast_trimul_b200.backward). Replaces the
    reference's recompute-everything backward (_kernels.py:468-488)."""

    @staticmethod
    def forward(ctx, mod, z, mask, *params):
        ctx.mod = mod
        ctx.has_mask = mask is not None
        with torch.no_grad():
            out, planes = mod._forward_native(z, mask, keep_planes=True)
        ctx.save_for_backward(z, *([mask] if mask is not None else []), *params, *planes)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        import os
        from . import backward as bw
        saved = ctx.saved_tensors
        z = saved[0]
        mask = saved[1] if ctx.has_mask else None
        first = 2 if ctx.has_mask else 1
        params = list(saved[first:first + 16])
        planes = saved[first + 16:first + 19]
        # FTM_BACKWARD=recompute: the per-position parts through torch autograd instead
        if os.environ.get("FTM_BACKWARD") == "recompute":
            gz, gp = bw.backward(ctx.mod, z, mask, params, planes, grad_out)
        else:
            gz, gp = bw.backward_native(ctx.mod, z, mask, params, planes, grad_out)
        return (None, gz, None, *gp)
