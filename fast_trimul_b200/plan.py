"""Pre-planned forward: fixed shape, buffers allocated once, stages launched through
the C ABI with no per-call allocation (what a serving loop or a benchmark wants).

    plan = TriMulPlan(layer._impl, batch=1, n=2048, z_dtype=torch.bfloat16)
    out = plan(z, mask)                      # three kernel launches, no allocation
    plan(z, mask, out=out, stage_events=ev)  # ev: 4 CUDA events bracketing the stages
"""

import torch

from . import _lib


class TriMulPlan:
    def __init__(self, impl, batch, n, z_dtype=torch.bfloat16, out_dtype=None, device=None,
                 rows=None):
        self.impl = impl
        self.device = torch.device(device) if device is not None else impl.proj_a.weight.device
        self.z_dtype = z_dtype
        self.out_dtype = z_dtype if out_dtype is None else out_dtype
        self.batch, self.n = batch, n
        self.rows = n if rows is None else rows
        lib = _lib.load()
        self.lib = lib
        if not impl.native_supported():
            raise _lib.NativeDeclined("native kernels need d_z == d_c == 128")
        probe = torch.empty(batch, self.rows, n, impl.d_z, dtype=z_dtype, device="meta")
        self.prob = impl.problem(probe, self.out_dtype)
        plane = batch * impl.d_c * self.rows * n
        self.a = torch.empty(plane, dtype=torch.float16, device=self.device)
        self.b = torch.empty(plane, dtype=torch.float16, device=self.device)
        self.x = torch.empty(plane, dtype=torch.float16, device=self.device)
        self.zstats = torch.empty(batch * self.rows * n * 2, dtype=torch.float32, device=self.device)
        from ._module import device_error_word
        self.errw = device_error_word(self.device)
        self.err = self.errw.dev
        self.packed = impl.packed_params()[0]

    def out_like(self):
        return torch.empty(self.batch, self.rows, self.n, self.impl.d_z, dtype=self.out_dtype,
                           device=self.device)

    def check_error(self):
        """Synchronise and raise `NativeKernelError` if a bounded device wait expired."""
        self.errw.check()

    def __call__(self, z, mask=None, out=None, stage_events=None):
        if z.dtype != self.z_dtype or tuple(z.shape) != (self.batch, self.rows, self.n, self.impl.d_z):
            raise ValueError("input does not match the plan")
        if out is None:
            out = self.out_like()
        s = torch.cuda.current_stream(self.device).cuda_stream
        lib, p = self.lib, self.prob
        mptr = None if mask is None else mask.data_ptr()
        ev = stage_events
        if ev is not None:
            ev[0].record()
        _lib.check(lib.ftm_input_stage(p, z.data_ptr(), mptr, self.packed.data_ptr(),
                                       self.a.data_ptr(), self.b.data_ptr(), self.zstats.data_ptr(),
                                       self.err.data_ptr(), s), "ftm_input_stage")
        if ev is not None:
            ev[1].record()
        L = self.batch * self.impl.d_c
        _lib.check(lib.ftm_contraction(self.a.data_ptr(), self.b.data_ptr(), self.x.data_ptr(),
                                       L, self.rows, self.n, self.n, 1, self.err.data_ptr(), s),
                   "ftm_contraction")
        if ev is not None:
            ev[2].record()
        _lib.check(lib.ftm_output_stage(p, z.data_ptr(), mptr, self.x.data_ptr(),
                                        self.zstats.data_ptr(), self.packed.data_ptr(), out.data_ptr(),
                                        self.err.data_ptr(), s), "ftm_output_stage")
        if ev is not None:
            ev[3].record()
        _lib.stats["calls"] += 1
        _lib.stats["kernel_launches"] += 3
        return out


class GraphedTriMul:
    """One CUDA graph of a plan's three launches at a fixed shape.

    The graph reads z and the mask from staging buffers the object owns and writes
    its own output buffer; a, b, x and the statistics are the plan's. Nothing else is
    captured: no allocation, no casts, no torch ops. `run(z, mask)` copies z (and the
    mask) into the staging buffers unless they already are those buffers -- a caller
    that writes its next input into `staging_input()` replays with no copy at all --
    then replays and returns the output buffer, which the next replay overwrites.
    """

    def __init__(self, impl, z, mask=None):
        if not z.is_cuda:
            raise ValueError("graph capture needs CUDA tensors")
        zdt = z.dtype if z.dtype in (torch.float16, torch.bfloat16) else torch.float16
        B, N = z.shape[0], z.shape[2]
        self.out_dtype = z.dtype
        self.plan = TriMulPlan(impl, B, N, zdt, out_dtype=z.dtype, device=z.device)
        self.z = torch.empty(z.shape, dtype=zdt, device=z.device)
        self.z.copy_(z)
        self.mask = None
        if mask is not None:
            self.mask = torch.empty(z.shape[:3], dtype=torch.float32, device=z.device)
            self.mask.copy_(mask.expand(z.shape[:3]))
        self.out = self.plan.out_like()
        # one eager run: validates the arguments and does every one-time host set-up
        self.plan(self.z, self.mask, out=self.out)
        self.plan.check_error()
        self.graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(z.device)
        side.wait_stream(torch.cuda.current_stream(z.device))
        with torch.cuda.stream(side):
            with torch.cuda.graph(self.graph, stream=side):
                self.plan(self.z, self.mask, out=self.out)
        torch.cuda.current_stream(z.device).wait_stream(side)

    def staging_input(self):
        """The buffer the graph reads z from (write the next input here to skip a copy)."""
        return self.z

    def run(self, z, mask=None):
        if tuple(z.shape) != tuple(self.z.shape):
            raise ValueError(f"graph captured for {tuple(self.z.shape)}, got {tuple(z.shape)}")
        if (mask is None) != (self.mask is None):
            raise ValueError("the mask must be given on every call iff it was given at capture")
        if z.data_ptr() != self.z.data_ptr():
            self.z.copy_(z)
        if mask is not None and mask.data_ptr() != self.mask.data_ptr():
            self.mask.copy_(mask.expand(self.mask.shape))
        self.plan.errw.poll()
        self.graph.replay()
        _lib.stats["calls"] += 1
        _lib.stats["kernel_launches"] += 3
        return self.out
