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
        self.err = torch.zeros(64, dtype=torch.int32, device=self.device)
        self.packed = impl.packed_params()[0]

    def out_like(self):
        return torch.empty(self.batch, self.rows, self.n, self.impl.d_z, dtype=self.out_dtype,
                           device=self.device)

    def check_error(self):
        """Synchronise and raise if a bounded device wait expired."""
        import ctypes
        detail = ctypes.c_int(0)
        st = self.lib.ftm_check_error(self.err.data_ptr(), ctypes.byref(detail),
                                      torch.cuda.current_stream(self.device).cuda_stream)
        if st != _lib.OK:
            raise _lib.NativeKernelError(f"device wait expired (code 0x{detail.value:x})")

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
