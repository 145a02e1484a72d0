"""i-row sharding of the outgoing triangle multiplicative update over GPUs.

Output row i needs a's row i and ALL rows of b (x[c,i,j] = sum_k a[c,i,k] b[c,j,k]),
so with rank r owning z rows I_r (N/P of them):

  1. input stage on the local rows -> a_loc, b_loc  (B*C, N/P, N) channel-major, fp16;
  2. NCCL all-gather of b_loc, split into channel chunks, each gathered into a
     (P, chunk, N/P, N) buffer -- the block-major layout ftm_contraction reads
     directly (B row j lives in block j // (N/P));
  3. per chunk: wait for its all-gather, contract local rows x all rows;
     all-gathers are queued back to back on NCCL's stream, so chunk k+1 crosses
     NVLink while chunk k is on the tensor cores;
  4. output stage on the local rows -> this rank's rows of the output.

The reference has no multi-GPU path; this follows the row-sharding scheme the
benchmark's multi-GPU configuration names (B=1, N=2048, outgoing). Incoming mode
needs a column exchange instead and is not sharded here.

`StageOps` isolates the three compute steps so the host-side logic (partitioning,
buffer layout, chunked exchange) runs with torch stand-ins on CPU / gloo in tests.
"""

import os

import torch
import torch.distributed as dist

from . import _lib

C = 128


def row_range(n, world, rank):
    """Rows [lo, hi) of an N-row problem owned by `rank` (equal blocks)."""
    if n % world:
        raise ValueError(f"N={n} must be divisible by the number of ranks ({world})")
    per = n // world
    return rank * per, (rank + 1) * per


class NativeStageOps:
    """The sm_100a kernels through the C ABI."""

    def __init__(self, impl, device):
        self.impl = impl
        self.lib = _lib.load()
        self.packed = impl.packed_params()[0]
        self.err = torch.zeros(64, dtype=torch.int32, device=device)

    def _s(self):
        return torch.cuda.current_stream().cuda_stream

    def input_stage(self, prob, z, mask, a, b):
        _lib.check(self.lib.ftm_input_stage(prob, z.data_ptr(), None if mask is None else mask.data_ptr(),
                                            self.packed.data_ptr(), a.data_ptr(), b.data_ptr(),
                                            self.err.data_ptr(), self._s()), "ftm_input_stage")

    def contraction(self, a, bblk, x, L, rows, n, blocks):
        _lib.check(self.lib.ftm_contraction(a.data_ptr(), bblk.data_ptr(), x.data_ptr(), L, rows, n,
                                            rows, blocks, self.err.data_ptr(), self._s()),
                   "ftm_contraction")

    def output_stage(self, prob, z, mask, x, out):
        _lib.check(self.lib.ftm_output_stage(prob, z.data_ptr(), None if mask is None else mask.data_ptr(),
                                             x.data_ptr(), self.packed.data_ptr(), out.data_ptr(),
                                             self.err.data_ptr(), self._s()), "ftm_output_stage")

    def check(self):
        import ctypes
        d = ctypes.c_int(0)
        if self.lib.ftm_check_error(self.err.data_ptr(), ctypes.byref(d), self._s()) != _lib.OK:
            raise _lib.NativeKernelError(f"device wait expired (code 0x{d.value:x})")


class TorchStageOps:
    """fp32 torch stand-ins for the three stages (CPU tests of the sharding logic);
    same buffer layouts as the native kernels."""

    def __init__(self, impl, device=None):
        self.impl = impl

    def _proj(self, z, mask):
        import torch.nn.functional as F
        im = self.impl
        p = [t.detach().float() for t in im._params()]
        zz = z.float() if mask is None else z.float() * mask[..., None]
        zn = F.layer_norm(zz, (zz.shape[-1],), p[0], p[1], im.norm_in.eps)
        return zz, zn, p

    def input_stage(self, prob, z, mask, a, b):
        import torch.nn.functional as F
        _, zn, p = self._proj(z, mask)
        av = F.linear(zn, p[4], p[5]) * torch.sigmoid(F.linear(zn, p[6], p[7]))
        bv = F.linear(zn, p[8], p[9]) * torch.sigmoid(F.linear(zn, p[10], p[11]))
        a.copy_(av.permute(0, 3, 1, 2).reshape(-1).to(a.dtype))
        b.copy_(bv.permute(0, 3, 1, 2).reshape(-1).to(b.dtype))

    def contraction(self, a, bblk, x, L, rows, n, blocks):
        A = a.view(L, rows, n).float()
        Bf = bblk.view(blocks, L, rows, n).permute(1, 0, 2, 3).reshape(L, blocks * rows, n).float()
        x.view(L, rows, blocks * rows).copy_(torch.bmm(A, Bf.transpose(1, 2)).to(x.dtype))

    def output_stage(self, prob, z, mask, x, out):
        import torch.nn.functional as F
        im = self.impl
        zz, zn, p = self._proj(z, mask)
        Bsz, R, S, _ = z.shape
        xv = x.view(Bsz, C, R, S).permute(0, 2, 3, 1).float()
        xn = F.layer_norm(xv, (C,), p[2], p[3], im.norm_out.eps)
        delta = torch.sigmoid(F.linear(zn, p[12], p[13])) * F.linear(xn, p[14], p[15])
        o = zz + delta if im.residual else delta
        if mask is not None:
            o = o * mask[..., None]
        out.copy_(o.to(out.dtype))

    def check(self):
        pass


class RowShardedTriMul:
    """Outgoing TriMul with z's rows sharded over the ranks of `group`.

    Call with this rank's rows: z_local (B, N/P, N, C), mask_local (B, N/P, N) or None;
    returns this rank's rows of the output. `chunks` channel chunks pipeline the
    all-gather of b with the contraction.
    """

    def __init__(self, impl, batch, n, group=None, z_dtype=torch.bfloat16, out_dtype=None,
                 chunks=4, device=None, ops=None):
        if impl.mode != "outgoing":
            raise NotImplementedError("row sharding covers outgoing mode")
        self.impl, self.group = impl, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.batch, self.n = batch, n
        self.rows = n // self.world
        row_range(n, self.world, self.rank)
        native = ops is None or isinstance(ops, NativeStageOps)
        if native and self.world > 1 and self.rows % 256:
            # ftm_contraction reads gathered b blocks whole 256-row tiles at a time
            raise ValueError("each rank's row block must be a multiple of 256 rows")
        L = batch * C
        if L % chunks:
            raise ValueError("channel chunks must divide batch * 128")
        self.L, self.chunks, self.lc = L, chunks, L // chunks
        dev = torch.device(device) if device is not None else impl.proj_a.weight.device
        self.device = dev
        self.z_dtype = z_dtype
        self.out_dtype = z_dtype if out_dtype is None else out_dtype
        self.ops = ops if ops is not None else NativeStageOps(impl, dev)
        probe = torch.empty(batch, self.rows, n, C, dtype=z_dtype, device="meta")
        self.prob = impl.problem(probe, self.out_dtype)
        plane = L * self.rows * n
        self.a = torch.empty(plane, dtype=torch.float16, device=dev)
        self.b = torch.empty(plane, dtype=torch.float16, device=dev)
        self.x = torch.empty(plane, dtype=torch.float16, device=dev)
        # gathered b, chunk-major: [chunk][rank][lc][rows][n]
        self.bg = torch.empty(chunks * self.world * self.lc * self.rows * n, dtype=torch.float16,
                              device=dev)

    def comm_bytes_per_step(self):
        """Bytes each rank receives over the interconnect per forward."""
        return (self.world - 1) * self.L * self.rows * self.n * 2

    def __call__(self, z_local, mask_local=None, out=None, events=None):
        if out is None:
            out = torch.empty(z_local.shape, dtype=self.out_dtype, device=z_local.device)
        ev = events
        if ev is not None:
            ev[0].record()
        self.ops.input_stage(self.prob, z_local, mask_local, self.a, self.b)
        if ev is not None:
            ev[1].record()
        blk = self.lc * self.rows * self.n
        works = []
        for k in range(self.chunks):
            src = self.b[k * blk:(k + 1) * blk]
            dst = self.bg[k * self.world * blk:(k + 1) * self.world * blk]
            if self.world > 1:
                works.append(dist.all_gather_into_tensor(dst, src, group=self.group, async_op=True))
            else:
                works.append(None)
                dst.copy_(src)
        for k in range(self.chunks):
            if works[k] is not None:
                works[k].wait()
            bsrc = self.bg[k * self.world * blk:(k + 1) * self.world * blk]
            self.ops.contraction(self.a[k * blk:(k + 1) * blk], bsrc,
                                 self.x[k * self.lc * self.rows * self.n:(k + 1) * self.lc * self.rows * self.n],
                                 self.lc, self.rows, self.n, self.world)
        if ev is not None:
            ev[2].record()
        self.ops.output_stage(self.prob, z_local, mask_local, self.x, out)
        if ev is not None:
            ev[3].record()
        if isinstance(self.ops, NativeStageOps):
            _lib.stats["calls"] += 1
            _lib.stats["kernel_launches"] += 2 + self.chunks
        return out


# --------------------------------------------------------------------------- bench
def _flops(n, batch=1):
    m = batch * n * n
    return 12 * m * C * C + 2 * batch * C * n ** 3


def bench_sharded(args, torch_mod):
    """bench.py's multi-GPU arm: one N x N outgoing TriMul, rows sharded over ranks.
    Returns the timing dict on rank 0, None elsewhere."""
    from fast_trimul_b200 import FastTriangleMultiplication
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if not dist.is_initialized():
        dist.init_process_group("nccl", device_id=dev)
    n = args.n
    torch.manual_seed(0)
    layer = FastTriangleMultiplication(C, C, mode="outgoing", residual=True).to(dev).eval()
    lo, hi = row_range(n, world, rank)
    gen = torch.Generator(device=dev).manual_seed(1 + rank)
    z = torch.randn(1, hi - lo, n, C, device=dev, generator=gen).to(torch.bfloat16)
    mask = torch.ones(1, hi - lo, n, device=dev)
    sh = RowShardedTriMul(layer._impl, 1, n, chunks=getattr(args, "chunks", 4) or 4, device=dev)
    out = torch.empty_like(z)
    for _ in range(args.warmup):
        sh(z, mask, out=out)
    sh.ops.check()
    K = args.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    from bench import ClockSampler
    dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0.record()
        for k in range(K):
            sh(z, mask, out=out, events=evs[k])
        t1.record()
        torch.cuda.synchronize()
    dist.barrier()
    sh.ops.check()
    ms = torch.tensor([t0.elapsed_time(t1) / K], device=dev)
    st = torch.tensor([sum(e[0].elapsed_time(e[1]) for e in evs) / K,
                       sum(e[1].elapsed_time(e[2]) for e in evs) / K,
                       sum(e[2].elapsed_time(e[3]) for e in evs) / K], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    dist.all_reduce(st, op=dist.ReduceOp.MAX)
    clocks = clk.summary()
    # end to end through the same public object: this rank's z rows from pinned host
    # memory in, its output rows back out, inside the timed region
    z_host = z.cpu().pin_memory()
    m_host = mask.cpu().pin_memory()
    o_host = torch.empty_like(z_host).pin_memory()
    e2e_steps = max(3, min(K, 20))

    def e2e_step():
        zd = z_host.to(dev, non_blocking=True)
        md = m_host.to(dev, non_blocking=True)
        o_host.copy_(sh(zd, md), non_blocking=True)

    for _ in range(2):
        e2e_step()
    dist.barrier()
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    for _ in range(e2e_steps):
        e2e_step()
    a1.record()
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([a0.elapsed_time(a1) / e2e_steps], device=dev)
    dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    res = None
    if rank == 0:
        res = {"ms_per_step": ms.item(), "rows_per_rank": hi - lo,
               "stage_ms": {"input_stage": st[0].item(), "contraction": st[1].item(),
                            "output_stage": st[2].item()},
               "clocks": clocks, "gpu_launches": (2 + sh.chunks) * K,
               "comm": {"all_gather_bytes_recv_per_rank_per_step": sh.comm_bytes_per_step(),
                        "chunks": sh.chunks,
                        "note": "contraction stage time includes waiting for the chunked all-gather"},
               "e2e": {"value": round(_flops(n) / (e2e_ms.item() * 1e-3) / 1e12, 3),
                       "unit": "TFLOP/s", "ms_per_step": round(e2e_ms.item(), 3),
                       "steps": e2e_steps,
                       "h2d_bytes_per_step": world * (z_host.numel() * 2 + m_host.numel() * 4),
                       "d2h_bytes_per_step": world * o_host.numel() * 2},
               "sweep": None}
    dist.barrier()
    dist.destroy_process_group()
    return res
