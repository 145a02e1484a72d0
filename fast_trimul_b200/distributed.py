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
(x[c,i,j] = sum_k a[c,k,i] b[c,k,j], k = z row) shards the same way through the
channel-sharded schemes: each rank's input stage writes the transposed planes of its own
rows k, the all-to-all hands every rank its channels with k split by source rank, and
the contraction reduces over those k blocks (`ftm_contraction_kblocked`).

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
        self.zstats = None

    def _stats(self, z):
        n = z.shape[0] * z.shape[1] * z.shape[2] * 2
        if self.zstats is None or self.zstats.numel() < n:
            self.zstats = torch.empty(n, dtype=torch.float32, device=z.device)
        return self.zstats.data_ptr()

    def _s(self):
        return torch.cuda.current_stream().cuda_stream

    def input_stage(self, prob, z, mask, a, b):
        _lib.check(self.lib.ftm_input_stage(prob, z.data_ptr(), None if mask is None else mask.data_ptr(),
                                            self.packed.data_ptr(), a.data_ptr(), b.data_ptr(),
                                            self._stats(z), self.err.data_ptr(), self._s()),
                   "ftm_input_stage")

    def contraction_kblocked(self, a, b, x, L, n, rows, blocks):
        """x (blocked by row owner) of incoming mode: k split into `blocks` source blocks."""
        _lib.check(self.lib.ftm_contraction_kblocked(a.data_ptr(), b.data_ptr(), x.data_ptr(), L, n, n,
                                                     rows, blocks, rows, self.err.data_ptr(), self._s()),
                   "ftm_contraction_kblocked")

    def contraction(self, a, bblk, x, L, rows, n, blocks, a_blocks=1):
        _lib.check(self.lib.ftm_contraction_blocked(a.data_ptr(), bblk.data_ptr(), x.data_ptr(), L,
                                                    rows, a_blocks, n, rows, blocks,
                                                    self.err.data_ptr(), self._s()),
                   "ftm_contraction_blocked")

    def output_stage(self, prob, z, mask, x, out):
        _lib.check(self.lib.ftm_output_stage(prob, z.data_ptr(), None if mask is None else mask.data_ptr(),
                                             x.data_ptr(), self._stats(z), self.packed.data_ptr(),
                                             out.data_ptr(),
                                             self.err.data_ptr(), self._s()), "ftm_output_stage")

    def input_stage_scatter(self, prob, z, mask, a_planes, b_planes, world, rank, group):
        """Input stage writing each channel group straight into its owner's receive
        plane (peer TMA stores; a_planes / b_planes: _lib.PeerPlanes)."""
        import ctypes
        _lib.check(self.lib.ftm_input_stage_scatter(
            prob, z.data_ptr(), None if mask is None else mask.data_ptr(), self.packed.data_ptr(),
            ctypes.byref(a_planes), ctypes.byref(b_planes), self._stats(z), self.err.data_ptr(),
            self._s()), "ftm_input_stage_scatter")

    def contraction_scatter(self, ar, br, x_planes, xr, batch, rows, n, world, rank, group,
                            mode="outgoing"):
        """Contraction of this rank's channel shard with every x row stored straight
        into its owner's x plane."""
        import ctypes
        _lib.check(self.lib.ftm_contraction_scatter(ar.data_ptr(), br.data_ptr(), ctypes.byref(x_planes),
                                                    batch, C, rows, n,
                                                    _lib.OUTGOING if mode == "outgoing" else _lib.INCOMING,
                                                    self.err.data_ptr(), self._s()),
                   "ftm_contraction_scatter")

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
        """Channel planes [b][c][i][j]; incoming mode writes them transposed, [b][c][i][k]
        with k the z row, as the native input stage does."""
        import torch.nn.functional as F
        _, zn, p = self._proj(z, mask)
        av = F.linear(zn, p[4], p[5]) * torch.sigmoid(F.linear(zn, p[6], p[7]))
        bv = F.linear(zn, p[8], p[9]) * torch.sigmoid(F.linear(zn, p[10], p[11]))
        perm = (0, 3, 1, 2) if self.impl.mode == "outgoing" else (0, 3, 2, 1)
        a.copy_(av.permute(*perm).reshape(-1).to(a.dtype))
        b.copy_(bv.permute(*perm).reshape(-1).to(b.dtype))

    def contraction_kblocked(self, a, b, x, L, n, rows, blocks):
        def unblock(t):      # [k block][L][n][rows] -> (L, n, blocks * rows)
            return t.view(blocks, L, n, rows).permute(1, 2, 0, 3).reshape(L, n, blocks * rows).float()
        X = torch.bmm(unblock(a), unblock(b).transpose(1, 2))               # (L, n, n)
        x.view(n // rows, L, rows, n).copy_(X.view(L, n // rows, rows, n).permute(1, 0, 2, 3).to(x.dtype))

    def contraction(self, a, bblk, x, L, rows, n, blocks, a_blocks=1):
        def unblock(t, nb):
            return t.view(nb, L, rows, n).permute(1, 0, 2, 3).reshape(L, nb * rows, n).float()
        A, Bf = unblock(a, a_blocks), unblock(bblk, blocks)
        X = torch.bmm(A, Bf.transpose(1, 2))                       # (L, a_blocks*rows, n)
        x.view(a_blocks, L, rows, n).copy_(X.view(L, a_blocks, rows, n).permute(1, 0, 2, 3).to(x.dtype))

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

    def input_stage_scatter(self, prob, z, mask, ar, br, world, rank, group):
        """Same receive layout as the native scatter -- [source rank][batch][C/P][rows][n]
        -- produced with an all-to-all instead of peer stores."""
        B, rows, n = z.shape[0], z.shape[1], z.shape[2]
        lq = C // world
        a = torch.empty(B * C * rows * n, dtype=ar.dtype, device=ar.device)
        b = torch.empty_like(a)
        self.input_stage(prob, z, mask, a, b)
        for src, dst in ((a, ar), (b, br)):
            send = src.view(B, world, lq, rows, n).permute(1, 0, 2, 3, 4).contiguous().view(-1)
            if world > 1:
                dist.all_to_all_single(dst, send, group=group)
            else:
                dst.copy_(send)

    def contraction_scatter(self, ar, br, x_planes, xr, batch, rows, n, world, rank, group,
                            mode="outgoing"):
        """X rows of this rank's channels returned to their owners' channel-major planes."""
        lq = C // world
        L = batch * lq
        xb = torch.empty(world * L * rows * n, dtype=xr.dtype, device=xr.device)
        if mode == "outgoing":
            self.contraction(ar, br, xb, L, rows, n, world, a_blocks=world)   # [owner][L][rows][n]
        else:
            self.contraction_kblocked(ar, br, xb, L, n, rows, world)
        recv = torch.empty_like(xb)                                        # [src][L][rows][n]
        if world > 1:
            dist.all_to_all_single(recv, xb, group=group)
        else:
            recv.copy_(xb)
        xr.view(batch, world, lq, rows, n).copy_(
            recv.view(world, batch, lq, rows, n).permute(1, 0, 2, 3, 4))

    def check(self):
        pass


SCHEMES = ("allgather", "alltoall", "allgather_ce", "alltoall_ce", "fused")


def default_scheme(world, mode="outgoing"):
    """Copy-engine exchanges; all-gather of b moves fewer bytes at 2 ranks, the
    channel-sharded all-to-all from 4 ranks on (measured N=2048: 2 GPUs 1408 vs
    1228 TFLOP/s, 4 GPUs 1961 vs 1662). Incoming mode always shards by channel."""
    return "allgather_ce" if world <= 2 and mode == "outgoing" else "alltoall_ce"


class PeerWindow:
    """A device buffer on every rank, with every peer's copy mapped into this process
    (CUDA IPC), so copy engines can write straight into a peer's buffer over NVLink."""

    def __init__(self, nbytes, device, group=None):
        from cuda.bindings import driver as drv
        from cuda.bindings import runtime as rt
        self.rt = rt
        self.tensor = torch.empty(nbytes, dtype=torch.uint8, device=device)
        ptr = self.tensor.data_ptr()
        err, base, _ = drv.cuMemGetAddressRange(ptr)
        if int(err) != 0:
            raise RuntimeError(f"cuMemGetAddressRange failed ({err})")
        err, handle = rt.cudaIpcGetMemHandle(int(base))
        if int(err) != 0:
            raise RuntimeError(f"cudaIpcGetMemHandle failed ({err})")
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        infos = [None] * world
        dist.all_gather_object(infos, (bytes(handle.reserved), ptr - int(base)), group=group)
        self.ptrs, self._opened = [], []
        for r, (hb, off) in enumerate(infos):
            if r == rank:
                self.ptrs.append(ptr)
                continue
            h = rt.cudaIpcMemHandle_t()
            h.reserved = hb
            err, p = rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess)
            if int(err) != 0:
                raise RuntimeError(f"cudaIpcOpenMemHandle failed ({err})")
            self._opened.append(int(p))
            self.ptrs.append(int(p) + off)

    def close(self):
        for p in self._opened:
            self.rt.cudaIpcCloseMemHandle(p)
        self._opened = []


def PeerWindow_rt():
    from cuda.bindings import runtime as rt
    return rt


def _copy_async(rt, dst, src, nbytes, stream):
    err, = rt.cudaMemcpyAsync(dst, src, nbytes, rt.cudaMemcpyKind.cudaMemcpyDefault,
                              rt.cudaStream_t(stream))
    if int(err) != 0:
        raise RuntimeError(f"cudaMemcpyAsync failed ({err})")


class RowShardedTriMul:
    """Outgoing TriMul with z's rows sharded over the ranks of `group`.

    Call with this rank's rows: z_local (B, N/P, N, C), mask_local (B, N/P, N) or None;
    returns this rank's rows of the output. `chunks` channel chunks pipeline the
    all-gather of b with the contraction.
    """

    def __init__(self, impl, batch, n, group=None, z_dtype=torch.bfloat16, out_dtype=None,
                 chunks=4, device=None, ops=None, scheme="allgather"):
        self.mode = impl.mode
        if impl.mode != "outgoing" and scheme not in ("alltoall", "alltoall_ce", "fused"):
            raise NotImplementedError("incoming mode is sharded by the channel-sharded schemes "
                                      "(alltoall, alltoall_ce, fused)")
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
        if scheme not in SCHEMES:
            raise ValueError(f"scheme must be one of {SCHEMES}")
        self.scheme = scheme
        if scheme == "fused":
            chunks = 1
            if C % self.world or (C // self.world) % 16:
                raise ValueError("the fused exchange needs 128 / P channels per rank, a multiple of 16")
        if L % (chunks * (self.world if scheme.startswith("alltoall") else 1)):
            raise ValueError("channel chunks (x ranks for alltoall) must divide batch * 128")
        self.L, self.chunks, self.lc = L, chunks, L // chunks
        dev = torch.device(device) if device is not None else impl.proj_a.weight.device
        self.device = dev
        self.z_dtype = z_dtype
        self.out_dtype = z_dtype if out_dtype is None else out_dtype
        self.ops = ops if ops is not None else NativeStageOps(impl, dev)
        probe = torch.empty(batch, self.rows, n, C, dtype=z_dtype, device="meta")
        self.prob = impl.problem(probe, self.out_dtype)
        plane = L * self.rows * n
        if scheme != "fused":     # the fused scheme's input stage writes the peers' planes
            self.a = torch.empty(plane, dtype=torch.float16, device=dev)
            self.b = torch.empty(plane, dtype=torch.float16, device=dev)
        if scheme == "allgather_ce":
            self.x = torch.empty(plane, dtype=torch.float16, device=dev)
            # gathered b window, chunk-major [chunk][src rank][lc][rows][n], written by
            # the peers' copy engines
            self.win_b = PeerWindow(chunks * self.world * self.lc * self.rows * n * 2, dev, group)
            self.bg = self.win_b.tensor.view(torch.float16)
            self.copy_stream = torch.cuda.Stream(dev)
            self.peer_streams = [torch.cuda.Stream(dev)]
            self.flag = torch.zeros(1, dtype=torch.float32, device=dev)
        elif scheme == "allgather":
            self.x = torch.empty(plane, dtype=torch.float16, device=dev)
            # gathered b, chunk-major: [chunk][rank][lc][rows][n]
            self.bg = torch.empty(chunks * self.world * self.lc * self.rows * n,
                                  dtype=torch.float16, device=dev)
        elif scheme == "fused":
            # receive planes written by the peers' kernels: a, b as
            # [source rank][batch][C/P][rows][n]; x as this rank's channel-major plane
            native_ops = isinstance(self.ops, NativeStageOps)
            if native_ops:
                self.win_a = PeerWindow(plane * 2, dev, group)
                self.win_b = PeerWindow(plane * 2, dev, group)
                self.win_x = PeerWindow(plane * 2, dev, group)
                self.ar = self.win_a.tensor.view(torch.float16)
                self.br = self.win_b.tensor.view(torch.float16)
                self.xr = self.win_x.tensor.view(torch.float16)
                P, r = self.world, self.rank
                self.a_planes = _lib.PeerPlanes.make(P, r, self.win_a.ptrs)
                self.b_planes = _lib.PeerPlanes.make(P, r, self.win_b.ptrs)
                self.x_planes = _lib.PeerPlanes.make(P, r, self.win_x.ptrs)
                self.flag = torch.zeros(1, dtype=torch.float32, device=dev)
            else:
                self.ar = torch.empty(plane, dtype=torch.float16, device=dev)
                self.br = torch.empty(plane, dtype=torch.float16, device=dev)
                self.xr = torch.empty(plane, dtype=torch.float16, device=dev)
                self.a_planes = self.b_planes = self.x_planes = None
        elif scheme == "alltoall_ce":
            # receive windows written by the peers' copy engines (CUDA IPC mappings)
            self.win_a = PeerWindow(plane * 2, dev, group)
            self.win_b = PeerWindow(plane * 2, dev, group)
            self.win_x = PeerWindow(plane * 2, dev, group)
            self.ar = self.win_a.tensor.view(torch.float16)
            self.br = self.win_b.tensor.view(torch.float16)
            self.xr = self.win_x.tensor.view(torch.float16)
            self.xb = torch.empty(plane, dtype=torch.float16, device=dev)
            self.copy_stream = torch.cuda.Stream(dev)
            self.peer_streams = [torch.cuda.Stream(dev)]   # local-block copies
            self.flag = torch.zeros(1, dtype=torch.float32, device=dev)
        else:
            # channel-sharded buffers (same size as a plane each): received a and b
            # [chunk][src rank][lc / P][rows][n], x blocked by row owner, x returned
            self.ar = torch.empty(plane, dtype=torch.float16, device=dev)
            self.br = torch.empty(plane, dtype=torch.float16, device=dev)
            self.xb = torch.empty(plane, dtype=torch.float16, device=dev)
            self.xr = torch.empty(plane, dtype=torch.float16, device=dev)

    def close(self):
        """Unmap the peers' receive windows (CUDA IPC handles). Call on every rank after
        the last forward, before the process group is destroyed."""
        for name in ("win_a", "win_b", "win_x"):
            w = getattr(self, name, None)
            if w is not None:
                w.close()

    def comm_bytes_per_step(self):
        """Bytes each rank receives over the interconnect per forward."""
        plane = self.L * self.rows * self.n * 2
        if self.scheme.startswith("allgather"):
            return (self.world - 1) * plane
        return 3 * plane * (self.world - 1) // self.world      # a, b in and x back

    def __call__(self, z_local, mask_local=None, out=None, events=None):
        if out is None:
            out = torch.empty(z_local.shape, dtype=self.out_dtype, device=z_local.device)
        ev = events
        if self.scheme == "fused":
            return self._forward_fused(z_local, mask_local, out, ev)
        if ev is not None:
            ev[0].record()
        self.ops.input_stage(self.prob, z_local, mask_local, self.a, self.b)
        if ev is not None:
            ev[1].record()
        if self.scheme == "allgather":
            self._exchange_allgather()
        elif self.scheme == "allgather_ce":
            self._exchange_allgather_ce()
        elif self.scheme == "alltoall":
            self._exchange_alltoall()
        else:
            self._exchange_alltoall_ce()
        if ev is not None:
            ev[2].record()
        self.ops.output_stage(self.prob, z_local, mask_local,
                              self.x if self.scheme.startswith("allgather") else self.xr, out)
        if ev is not None:
            ev[3].record()
        if isinstance(self.ops, NativeStageOps):
            _lib.stats["calls"] += 1
            _lib.stats["kernel_launches"] += 2 + self.chunks
        return out

    def _forward_fused(self, z_local, mask_local, out, ev):
        """Exchange fused into the kernels: the input stage stores each channel group of
        a and b into its owner's receive plane, the contraction stores each x row into
        its row owner's plane, and a device-side barrier separates the phases (a rank
        reads a plane only after every writer's kernel has finished). The barrier after
        the contraction also frees the a / b planes for the next call's input stage,
        and x planes are rewritten only after their owner's next input stage, which
        follows its output stage on the same stream."""
        P, r = self.world, self.rank
        native = isinstance(self.ops, NativeStageOps)
        if ev is not None:
            ev[0].record()
        self.ops.input_stage_scatter(self.prob, z_local, mask_local,
                                     self.a_planes if native else self.ar,
                                     self.b_planes if native else self.br, P, r, self.group)
        if native and P > 1:
            dist.all_reduce(self.flag, group=self.group)
        if ev is not None:
            ev[1].record()
        self.ops.contraction_scatter(self.ar, self.br, self.x_planes, self.xr, self.batch,
                                     self.rows, self.n, P, r, self.group, mode=self.mode)
        if native and P > 1:
            dist.all_reduce(self.flag, group=self.group)
        if ev is not None:
            ev[2].record()
        self.ops.output_stage(self.prob, z_local, mask_local, self.xr, out)
        if ev is not None:
            ev[3].record()
        if native:
            _lib.stats["calls"] += 1
            _lib.stats["kernel_launches"] += 3
        return out

    def _contract_shard(self, A, B, X, L):
        """This rank's channels over all rows, X blocked by row owner: outgoing reads row
        blocks of A and B; incoming reads the transposed planes with k split by source."""
        P = self.world
        if self.mode == "outgoing":
            self.ops.contraction(A, B, X, L, self.rows, self.n, P, a_blocks=P)
        else:
            self.ops.contraction_kblocked(A, B, X, L, self.n, self.rows, P)

    def _exchange_allgather(self):
        """All-gather b chunk by chunk; contract each chunk as soon as it lands."""
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
            self.ops.contraction(self.a[k * blk:(k + 1) * blk],
                                 self.bg[k * self.world * blk:(k + 1) * self.world * blk],
                                 self.x[k * blk:(k + 1) * blk], self.lc, self.rows, self.n,
                                 self.world)

    def _exchange_alltoall(self):
        """Row shards -> channel shards -> row shards. Chunk k moves channels
        [k*lc, (k+1)*lc), of which rank q receives [k*lc + q*lc/P, ...): one contiguous
        all_to_all_single per chunk for a and b, the contraction of this rank's channels
        over all N rows, and an all_to_all_single of x back to the row owners."""
        P, blk = self.world, self.lc * self.rows * self.n
        lq = self.lc // P
        ins = []
        for k in range(self.chunks):
            sl = slice(k * blk, (k + 1) * blk)
            ins.append((dist.all_to_all_single(self.ar[sl], self.a[sl], group=self.group, async_op=True),
                        dist.all_to_all_single(self.br[sl], self.b[sl], group=self.group, async_op=True)))
        outs = []
        for k in range(self.chunks):
            sl = slice(k * blk, (k + 1) * blk)
            ins[k][0].wait()
            ins[k][1].wait()
            # A and B: P row blocks (one per source rank) of lq channels; X blocked by row owner
            self._contract_shard(self.ar[sl], self.br[sl], self.xb[sl], lq)
            outs.append(dist.all_to_all_single(self.xr[sl], self.xb[sl], group=self.group,
                                               async_op=True))
        for w in outs:
            w.wait()

    def _barrier_on(self, stream):
        """Device-side barrier: a one-element NCCL all-reduce queued on `stream`
        completes on every rank only after all ranks' earlier work on it."""
        with torch.cuda.stream(stream):
            dist.all_reduce(self.flag, group=self.group)

    def _shifted_copies(self, src_event, copies, blk):
        """Copy blocks to every rank after `src_event`. NVLink copies run on the copy
        stream in shifted order -- round s goes to rank (me + s) % P -- so at any moment
        each GPU sends to one peer and receives from one (concurrent copies to several
        peers measured at ~half the aggregate bandwidth of this schedule). The local
        block is copied on a side stream. copies[q] = [(dst, src), ...] for rank q."""
        P, me, rt = self.world, self.rank, PeerWindow_rt()
        cs, side = self.copy_stream, self.peer_streams[0]
        cs.wait_event(src_event)
        side.wait_event(src_event)
        for dst, src in copies[me]:
            _copy_async(rt, dst, src, blk, side.cuda_stream)
        for sft in range(1, P):
            for dst, src in copies[(me + sft) % P]:
                _copy_async(rt, dst, src, blk, cs.cuda_stream)
        cs.wait_stream(side)

    def _exchange_allgather_ce(self):
        """All-gather of b by the copy engines: chunk k of this rank's b goes to block
        `me` of chunk k in every rank's window (shifted rounds), a device-side barrier
        per chunk, and the contraction of chunk k starts as soon as its barrier passes."""
        P, me = self.world, self.rank
        blk = self.lc * self.rows * self.n * 2
        comp = torch.cuda.current_stream()
        ev = torch.cuda.Event()
        ev.record(comp)
        b0 = self.b.data_ptr()
        done = []
        for k in range(self.chunks):
            self._shifted_copies(ev, [[(self.win_b.ptrs[q] + (k * P + me) * blk, b0 + k * blk)]
                                      for q in range(P)], blk)
            self._barrier_on(self.copy_stream)
            e = torch.cuda.Event()
            e.record(self.copy_stream)
            done.append(e)
        elems = self.lc * self.rows * self.n
        for k in range(self.chunks):
            comp.wait_event(done[k])
            self.ops.contraction(self.a[k * elems:(k + 1) * elems],
                                 self.bg[k * P * elems:(k + 1) * P * elems],
                                 self.x[k * elems:(k + 1) * elems], self.lc, self.rows, self.n, P)

    def _exchange_alltoall_ce(self):
        """Same data movement as _exchange_alltoall, done by the copy engines: each
        chunk's channel shards of a and b are copied straight into the owners' receive
        windows over NVLink (no SMs used), a device-side barrier orders them before the
        contraction, and x blocks are copied back to the row owners the same way."""
        P, me = self.world, self.rank
        rows, n = self.rows, self.n
        lq = self.lc // P
        blk = lq * rows * n * 2                     # bytes of one (rank, chunk) block
        comp = torch.cuda.current_stream()
        cs = self.copy_stream
        a0, b0, xb0 = self.a.data_ptr(), self.b.data_ptr(), self.xb.data_ptr()
        ev_ab = torch.cuda.Event()
        ev_ab.record(comp)                          # a, b written by the input stage
        done = []
        for k in range(self.chunks):
            self._shifted_copies(
                ev_ab, [[(self.win_a.ptrs[q] + (k * P + me) * blk, a0 + (k * P + q) * blk),
                         (self.win_b.ptrs[q] + (k * P + me) * blk, b0 + (k * P + q) * blk)]
                        for q in range(P)], blk)
            self._barrier_on(cs)
            ev = torch.cuda.Event()
            ev.record(cs)
            done.append(ev)
        for k in range(self.chunks):
            comp.wait_event(done[k])
            elems = self.lc * rows * n
            sl = slice(k * elems, (k + 1) * elems)
            self._contract_shard(self.ar[sl], self.br[sl], self.xb[sl], lq)
            ev = torch.cuda.Event()
            ev.record(comp)
            # x rows of owner p (my channels) -> p's channel-major x at my channel block
            self._shifted_copies(
                ev, [[(self.win_x.ptrs[p] + (k * P + me) * blk, xb0 + (k * P + p) * blk)]
                     for p in range(P)], blk)
        self._barrier_on(cs)
        comp.wait_stream(cs)


# ------------------------------------------------------------- native pipeline
PIPELINE_SCHEMES = ("p2p_alltoall", "p2p_allgather")


def default_pipeline_scheme(world, mode="outgoing"):
    """b all-gathered at 2 ranks (it sends (P-1)/P of one plane against 3(P-1)/P^2 for
    the all-to-all, fewer at P = 2), the channel all-to-all from 4 ranks on and for
    incoming mode."""
    return "p2p_allgather" if world == 2 and mode == "outgoing" else "p2p_alltoall"


def default_row_chunks(rows, batch=1, world=1):
    """Row chunks of the input stage: each chunk's exchange starts when it is done.
    Chunks of at least 128 rows (the contraction's row / k blocks), at most 4. At 8
    ranks one chunk: its pushes per peer are then 2x larger, which the copy engines
    move faster (measured 610 vs 450 GB/s), and the input stage is short."""
    if batch > 1 or world >= 8:
        return 1
    for rc in (4, 3, 2):
        if rows % rc == 0 and (rows // rc) % 128 == 0:
            return rc
    return 1


class ShardedTriMul:
    """Row-sharded forward on the library's native exchange pipeline (ftm_shard_forward).

    Each rank of `group` owns rows [rank * N/P, (rank + 1) * N/P) of z and of the output.
    One call queues this rank's whole forward on the current stream: the input stage in
    row chunks, copy-engine pushes of each chunk into the peers' receive windows (CUDA IPC
    mappings) with a flag raised in the receiver's memory after each push, bounded
    device-side waits on those flags, the contraction and the output stage. NCCL is used
    only here, at construction, to exchange the IPC handles. Every rank must make the
    same calls in the same order.
    """

    def __init__(self, impl, batch, n, group=None, z_dtype=torch.bfloat16, out_dtype=None,
                 device=None, scheme=None, row_chunks=None):
        from ._module import device_error_word
        import ctypes
        self.impl, self.group = impl, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.batch, self.n = batch, n
        lo, hi = row_range(n, self.world, self.rank)
        self.rows = hi - lo
        self.mode = impl.mode
        scheme = scheme or default_pipeline_scheme(self.world, self.mode)
        if scheme not in PIPELINE_SCHEMES:
            raise ValueError(f"scheme must be one of {PIPELINE_SCHEMES}")
        self.scheme = scheme
        dev = torch.device(device) if device is not None else impl.proj_a.weight.device
        self.device = dev
        self.z_dtype = z_dtype
        self.out_dtype = z_dtype if out_dtype is None else out_dtype
        self.row_chunks = row_chunks or default_row_chunks(self.rows, batch, self.world)
        lib = _lib.load()
        self.lib = lib
        probe = torch.empty(batch, self.rows, n, C, dtype=z_dtype, device="meta")
        self.errw = device_error_word(dev)
        self.packed = impl.packed_params()[0]
        cfg = _lib.ShardConfig()
        cfg.world, cfg.rank = self.world, self.rank
        cfg.scheme = _lib.SHARD_ALLTOALL if scheme == "p2p_alltoall" else _lib.SHARD_ALLGATHER
        cfg.row_chunks = self.row_chunks
        cfg.shard = impl.problem(probe, self.out_dtype)

        def nbytes(which):
            v = lib.ftm_shard_buffer_bytes(ctypes.byref(cfg), which)
            if v == 0:
                raise ValueError(f"unsupported sharded problem: B={batch} N={n} P={self.world} "
                                 f"row_chunks={self.row_chunks} scheme={scheme} mode={self.mode}")
            return v

        def buf(which):
            return torch.empty(nbytes(which), dtype=torch.uint8, device=dev)

        a2a = scheme == "p2p_alltoall"
        self.a_local = buf(_lib.SHARD_BUF_LOCAL)
        self.zstats = buf(_lib.SHARD_BUF_ZSTATS)
        self.x_blocks = buf(_lib.SHARD_BUF_XBLOCKS)
        self.windows = {}
        names = ("recv_a", "x_plane", "flags") if a2a else ("recv_b", "flags")
        sizes = {"recv_a": _lib.SHARD_BUF_RECV, "recv_b": _lib.SHARD_BUF_RECV,
                 "x_plane": _lib.SHARD_BUF_XPLANE, "flags": _lib.SHARD_BUF_FLAGS}
        for name in names:
            if self.world > 1:
                w = PeerWindow(nbytes(sizes[name]), dev, group)
            else:
                w = _LocalWindow(nbytes(sizes[name]), dev)
            self.windows[name] = w
        self.windows["flags"].tensor.zero_()
        torch.cuda.synchronize(dev)
        cfg.packed = self.packed.data_ptr()
        cfg.a_local = self.a_local.data_ptr()
        cfg.zstats = self.zstats.data_ptr()
        cfg.x_blocks = self.x_blocks.data_ptr()
        cfg.err_word = self.errw.ptr
        for name, w in self.windows.items():
            arr = getattr(cfg, name)
            for q, p in enumerate(w.ptrs):
                arr[q] = p
        self.cfg = cfg
        self.plan = ctypes.c_void_p()
        with torch.cuda.device(dev):
            _lib.check(lib.ftm_shard_plan_create(ctypes.byref(cfg), ctypes.byref(self.plan)),
                       "ftm_shard_plan_create")
        if self.world > 1:
            dist.barrier(group=group)         # every rank's flags are zero before any push

    def comm_bytes_per_step(self):
        """Bytes this rank sends over NVLink per forward."""
        plane = self.batch * C * self.rows * self.n * 2            # this rank's a (or b, or x)
        P = self.world
        if self.scheme == "p2p_allgather":
            return (P - 1) * plane
        return 3 * plane * (P - 1) // P

    def __call__(self, z_local, mask_local=None, out=None):
        shape = (self.batch, self.rows, self.n, C)
        if tuple(z_local.shape) != shape or z_local.dtype != self.z_dtype or not z_local.is_contiguous():
            raise ValueError(f"z_local must be a contiguous {self.z_dtype} tensor of shape {shape}")
        if mask_local is not None:
            mask_local = mask_local.to(device=self.device, dtype=torch.float32).expand(shape[:3]).contiguous()
        if out is None:
            out = torch.empty(shape, dtype=self.out_dtype, device=self.device)
        if out.dtype not in _DTYPES:
            raise ValueError(f"unsupported output dtype {out.dtype}")
        self.errw.poll()
        st = self.lib.ftm_shard_forward(self.plan, z_local.data_ptr(),
                                        None if mask_local is None else mask_local.data_ptr(),
                                        out.data_ptr(), _DTYPES[out.dtype],
                                        torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(st, "ftm_shard_forward")
        self.last_launches = self.lib.ftm_last_launch_count()
        self.errw.after_launch()
        _lib.stats["calls"] += 1
        _lib.stats["kernel_launches"] += self.last_launches
        return out

    def check(self):
        self.errw.check()

    TRACE_NAMES = {1: "start", 2: "input", 3: "pushed", 4: "ready", 5: "contracted", 6: "x_pushed",
                   7: "x_ready", 8: "output"}

    def enable_trace(self):
        """Record a device-clock timeline of each later forward (ftm_shard_set_trace)."""
        self._trace = torch.zeros(2 * 128, dtype=torch.int64, device=self.device)
        _lib.check(self.lib.ftm_shard_set_trace(self.plan, self._trace.data_ptr()), "ftm_shard_set_trace")

    def disable_trace(self):
        self.lib.ftm_shard_set_trace(self.plan, None)

    def read_trace(self):
        """[(microseconds since the forward's start, event, index)] of the last forward."""
        torch.cuda.synchronize(self.device)
        t = self._trace.view(-1, 2).cpu().tolist()
        pts = [(ts, tag) for ts, tag in t if tag]
        if not pts:
            return []
        t0 = min(ts for ts, tag in pts if tag >> 8 == 1)
        return sorted((round((ts - t0) / 1e3, 1), self.TRACE_NAMES.get(tag >> 8, str(tag >> 8)),
                       tag & 255) for ts, tag in pts)

    def close(self):
        """Destroy the plans and unmap the peers' windows; call on every rank after the
        last forward, before the process group is destroyed."""
        torch.cuda.synchronize(self.device)
        if self.plan:
            self.lib.ftm_shard_plan_destroy(self.plan)
            self.plan = None
        for w in self.windows.values():
            w.close()


_DTYPES = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


class _LocalWindow:
    """One rank: a plain device buffer in place of a peer window."""

    def __init__(self, nbytes, device):
        self.tensor = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self.ptrs = [self.tensor.data_ptr()]

    def close(self):
        pass


# --------------------------------------------------------------------------- bench
def _flops(n, batch=1):
    m = batch * n * n
    return 12 * m * C * C + 2 * batch * C * n ** 3


def _sharded_parity(impl, z, mask, out_f32, group, rows_total=16):
    """Checks this rank's fp32 output rows against the fp32 formula of the reference's
    torch path (fast_trimul_b200.parity) on rows spread over ALL ranks' rows: z is
    all-gathered so every rank can form b over all rows. Returns, on every rank, the
    max-abs and mean-relative error over the rows every rank checked."""
    from .parity import reference_rows, sample_rows
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, R, N, _ = z.shape
    parts = [torch.empty_like(z) for _ in range(world)]
    dist.all_gather(parts, z.contiguous(), group=group)
    zf = torch.cat(parts, dim=1)
    mf = None
    if mask is not None:
        mparts = [torch.empty_like(mask) for _ in range(world)]
        dist.all_gather(mparts, mask.contiguous(), group=group)
        mf = torch.cat(mparts, dim=1)
    per = max(2, rows_total // world)
    local = sample_rows(R, per)
    ref = reference_rows(impl, zf, mf, [rank * R + i for i in local])
    got = out_f32[:, local].double()
    d = (got - ref.double()).abs()
    stats = torch.tensor([d.max().item(), d.sum().item(), ref.double().abs().sum().item(),
                          float(len(local))], device=z.device, dtype=torch.float64)
    mx = stats[:1].clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
    dist.all_reduce(stats, group=group)
    max_abs, mean_rel = mx.item(), stats[1].item() / stats[2].item()
    del zf, parts
    return {"max_abs": round(max_abs, 6), "mean_rel": round(mean_rel, 7),
            "rows_checked": int(stats[3].item()), "ranks": world,
            "tolerance": {"max_abs": 2e-2, "mean_rel": 1e-3},
            "ok": bool(max_abs <= 2e-2 and mean_rel <= 1e-3),
            "checker": "fp32 torch formula of the reference's torch path on the all-gathered z, "
                       "rows sampled on every rank",
            "output": "fp32 (same sharded forward; the timed steps write bf16)"}


def _stages_alone(impl, n, world, dev, reps=10):
    """CUDA-event time of each of one rank's kernels run alone on local data (no
    exchange): the input stage on N/P rows, the contraction of this rank's share
    (128/P channels over all rows -- C R N^2 multiply-adds either way) and the output stage
    on N/P rows. The roofline of the sharded run is quoted on these."""
    lib = _lib.load()
    R = n // world
    s = torch.cuda.current_stream().cuda_stream
    z = torch.randn(1, R, n, C, device=dev).to(torch.bfloat16)
    mask = torch.ones(1, R, n, device=dev)
    plane = C * R * n
    a = torch.empty(plane, dtype=torch.float16, device=dev)
    b = torch.empty_like(a)
    x = torch.randn(plane, device=dev).half()
    A = torch.randn(C // world, n, n, device=dev).half()
    Bm = torch.randn(C // world, n, n, device=dev).half()
    X = torch.empty_like(A)
    out = torch.empty_like(z)
    zst = torch.empty(R * n * 2, dtype=torch.float32, device=dev)
    err = torch.zeros(64, dtype=torch.int32, device=dev)
    packed = impl.packed_params()[0]
    prob = impl.problem(z, torch.bfloat16)
    calls = {
        "input_stage": lambda: lib.ftm_input_stage(prob, z.data_ptr(), mask.data_ptr(), packed.data_ptr(),
                                                   a.data_ptr(), b.data_ptr(), zst.data_ptr(),
                                                   err.data_ptr(), s),
        "contraction": lambda: lib.ftm_contraction(A.data_ptr(), Bm.data_ptr(), X.data_ptr(), C // world,
                                                   n, n, n, 1, err.data_ptr(), s),
        "output_stage": lambda: lib.ftm_output_stage(prob, z.data_ptr(), mask.data_ptr(), x.data_ptr(),
                                                     zst.data_ptr(), packed.data_ptr(), out.data_ptr(),
                                                     err.data_ptr(), s),
    }
    res = {}
    for name, f in calls.items():
        for _ in range(3):
            _lib.check(f(), name)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
        ev[0].record()
        for i in range(reps):
            f()
            ev[i + 1].record()
        torch.cuda.synchronize()
        res[name] = sorted(ev[i].elapsed_time(ev[i + 1]) for i in range(reps))[reps // 2]
    if lib.ftm_check_error(err.data_ptr(), None, s) != _lib.OK:
        raise _lib.NativeKernelError("a stage timed alone reported an expired wait")
    return res


def bench_sharded(args, torch_mod):
    """bench.py's multi-GPU arm: one N x N TriMul, rows sharded over ranks.
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
    mode = getattr(args, "mode", "outgoing") or "outgoing"
    layer = FastTriangleMultiplication(C, C, mode=mode, residual=True).to(dev).eval()
    lo, hi = row_range(n, world, rank)
    gen = torch.Generator(device=dev).manual_seed(1 + rank)
    z = torch.randn(1, hi - lo, n, C, device=dev, generator=gen).to(torch.bfloat16)
    mask = torch.ones(1, hi - lo, n, device=dev)
    scheme = getattr(args, "scheme", None) or default_pipeline_scheme(world, mode)
    if scheme in PIPELINE_SCHEMES:
        sh = ShardedTriMul(layer._impl, 1, n, device=dev, scheme=scheme,
                           row_chunks=getattr(args, "row_chunks", None))
        run = sh
        check = sh.check
        detail = {"scheme": scheme, "row_chunks": sh.row_chunks,
                  "push": os.environ.get("FTM_SHARD_PUSH", "ce")}
    else:
        chunks = getattr(args, "chunks", None) or (4 if scheme.startswith("allgather") else 2)
        sh = RowShardedTriMul(layer._impl, 1, n, chunks=chunks, device=dev, scheme=scheme)
        run = sh
        check = sh.ops.check
        detail = {"scheme": scheme, "chunks": chunks}
    out = torch.empty_like(z)
    for _ in range(args.warmup):
        run(z, mask, out=out)
    check()
    K = args.steps
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    from bench import ClockSampler
    n_launch0 = _lib.stats["kernel_launches"]
    import time
    if getattr(args, "trace_timed", False) and hasattr(sh, "enable_trace"):
        sh.enable_trace()
    spans = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(K)]
    # the clock sampler starts (NVML set-up takes milliseconds) before the barrier, so
    # every rank enters the timed loop at the same moment: otherwise the first forward of
    # the fastest rank waits for the others' late start inside the timed region
    with ClockSampler(local) as clk:
        dist.barrier()
        torch.cuda.synchronize()
        t0.record()
        h0 = time.perf_counter()
        for k in range(K):
            spans[k][0].record()
            run(z, mask, out=out)
            spans[k][1].record()
        host_issue_ms = (time.perf_counter() - h0) * 1e3 / K
        t1.record()
        torch.cuda.synchronize()
    span_ms = sorted(a.elapsed_time(b) for a, b in spans)
    gap_ms = sorted(spans[k][1].elapsed_time(spans[k + 1][0]) for k in range(K - 1))
    if getattr(args, "trace_timed", False) and hasattr(sh, "disable_trace"):
        sh.disable_trace()
    launches = _lib.stats["kernel_launches"] - n_launch0
    dist.barrier()
    check()
    trace = None
    if getattr(args, "trace", False) and hasattr(sh, "enable_trace"):
        sh.enable_trace()
        for _ in range(3):
            run(z, mask, out=out)
        mine = sh.read_trace()
        allt = [None] * world
        dist.all_gather_object(allt, mine)
        trace = allt
        sh.disable_trace()
    ms = torch.tensor([t0.elapsed_time(t1) / K], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    clocks = clk.summary()
    # parity of the same sharded forward (fp32 output) on rows of every rank
    out32 = torch.empty(z.shape, dtype=torch.float32, device=dev)
    run(z, mask, out=out32)
    check()
    parity = _sharded_parity(layer._impl, z, mask, out32, None)
    del out32
    # end to end through the same public object: this rank's z rows from pinned host
    # memory in, its output rows back out, inside the timed region
    z_host = z.cpu().pin_memory()
    m_host = mask.cpu().pin_memory()
    o_host = torch.empty_like(z_host).pin_memory()
    e2e_steps = max(3, min(K, 20))
    zd, md = torch.empty_like(z), torch.empty_like(mask)

    def e2e_step():
        zd.copy_(z_host, non_blocking=True)
        md.copy_(m_host, non_blocking=True)
        o_host.copy_(run(zd, md, out=out), non_blocking=True)

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
    check()
    stage_ms = _stages_alone(layer._impl, n, world, dev)
    res = None
    if rank == 0:
        detail.update({"host_issue_ms_per_step": round(host_issue_ms, 3),
                       "forward_span_ms_median": round(span_ms[len(span_ms) // 2], 3),
                       "forward_span_ms": {"min": round(span_ms[0], 3), "mean": round(sum(span_ms) / K, 3),
                                           "max": round(span_ms[-1], 3),
                                           "in_order": [round(a.elapsed_time(b), 3) for a, b in spans]},
                       "gap_between_forwards_ms_median": round(gap_ms[len(gap_ms) // 2], 3),
                       "bytes_sent_per_rank_per_step": sh.comm_bytes_per_step(),
                       "nvlink_gbs_per_rank": round(sh.comm_bytes_per_step() / (ms.item() * 1e-3) / 1e9, 1)})
        res = {"ms_per_step": ms.item(), "rows_per_rank": hi - lo,
               "clocks": clocks, "gpu_launches": launches, "parity": parity,
               "trace": trace,
               "stage_ms": stage_ms, "stage_note": "each kernel of one rank timed alone on local "
                                                   "data; the step adds the exchange",
               "comm": detail,
               "e2e": {"value": round(_flops(n) / (e2e_ms.item() * 1e-3) / 1e12, 3),
                       "unit": "TFLOP/s", "ms_per_step": round(e2e_ms.item(), 3),
                       "steps": e2e_steps,
                       "h2d_bytes_per_step": world * (z_host.numel() * 2 + m_host.numel() * 4),
                       "d2h_bytes_per_step": world * o_host.numel() * 2},
               "sweep": None}
    dist.barrier()
    if hasattr(sh, "close"):
        sh.close()
    dist.barrier()
    dist.destroy_process_group()
    return res
