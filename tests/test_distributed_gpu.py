"""Row-sharded forward on real GPUs over NCCL (needs >= 2 GPUs; skipped otherwise):
each rank runs the native kernels on its rows with the chunked all-gather of b, and
the gathered output must match the single-GPU native forward and the oracle."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N = 512


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, path, scheme, mode="outgoing", row_chunks=None, push="ce"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      FTM_SHARD_PUSH=push)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from fast_trimul_b200.distributed import RowShardedTriMul, row_range
        from tests.helpers import make_layer
        m = make_layer(mode, True).to(dev)
        gen = torch.Generator().manual_seed(21)
        z = torch.randn(1, N, N, 128, generator=gen).to(torch.bfloat16)
        mask = torch.ones(1, N, N)
        mask[:, :, N - 40:] = 0
        lo, hi = row_range(N, world, rank)
        zl = z[:, lo:hi].contiguous().to(dev)
        ml = mask[:, lo:hi].contiguous().to(dev)
        if scheme.startswith("p2p_"):
            from fast_trimul_b200.distributed import ShardedTriMul
            sh = ShardedTriMul(m._impl, 1, N, device=dev, out_dtype=torch.float32, scheme=scheme,
                               row_chunks=row_chunks)
            # three forwards in a row: the receive windows alternate, flags count epochs
            for _ in range(3):
                out = sh(zl, ml)
            sh.check()
            sh.close()
        else:
            sh = RowShardedTriMul(m._impl, 1, N, chunks=4, device=dev, out_dtype=torch.float32,
                                  scheme=scheme)
            out = sh(zl, ml)
            sh.ops.check()
        parts = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(parts, out)
        if rank == 0:
            np.save(path, torch.cat(parts, dim=1).cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("scheme,mode", [("p2p_allgather", "outgoing"), ("p2p_alltoall", "outgoing"),
                                         ("p2p_alltoall", "incoming"), ("p2p_alltoall_sm", "outgoing"),
                                         ("allgather", "outgoing"), ("alltoall", "outgoing"),
                                         ("allgather_ce", "outgoing"), ("alltoall_ce", "outgoing"),
                                         ("fused", "outgoing"), ("alltoall_ce", "incoming"),
                                         ("fused", "incoming")])
def test_two_gpu_row_sharding(tmp_path, scheme, mode):
    from tests.helpers import MAX_ABS, MEAN_REL, compare, make_layer, oracle_out
    path = str(tmp_path / "o.npy")
    push = "sm" if scheme.endswith("_sm") else "ce"
    scheme = scheme[:-3] if scheme.endswith("_sm") else scheme
    mp.start_processes(_worker, args=(2, _free_port(), path, scheme, mode, None, push), nprocs=2,
                       join=True, start_method="spawn")
    got = torch.from_numpy(np.load(path))
    m = make_layer(mode, True)
    gen = torch.Generator().manual_seed(21)
    z = torch.randn(1, N, N, 128, generator=gen).to(torch.bfloat16)
    mask = torch.ones(1, N, N)
    mask[:, :, N - 40:] = 0
    max_abs, mean_rel = compare(got, oracle_out(m, z, mask))
    assert max_abs <= MAX_ABS and mean_rel <= MEAN_REL, (max_abs, mean_rel)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")
def test_single_rank_sharded_object_matches_plain_forward():
    """world = 1: the chunked path (blocks = 1) equals the plain forward bit for bit."""
    from fast_trimul_b200.distributed import RowShardedTriMul
    from tests.helpers import make_layer
    m = make_layer("outgoing", True).cuda()
    z = torch.randn(1, 256, 256, 128, device="cuda").to(torch.bfloat16)
    sh = RowShardedTriMul(m._impl, 1, 256, chunks=4, device="cuda", out_dtype=torch.float32)
    got = sh(z)
    with torch.no_grad():
        want = m._impl._forward_native(z, None, out_dtype=torch.float32)
    assert torch.equal(got, want)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")
@pytest.mark.parametrize("scheme,mode,row_chunks,push", [("p2p_alltoall", "outgoing", 2, "ce"),
                                                         ("p2p_alltoall", "incoming", 2, "ce"),
                                                         ("p2p_allgather", "outgoing", 2, "ce"),
                                                         ("p2p_alltoall", "outgoing", 1, "ce"),
                                                         ("p2p_alltoall", "outgoing", 2, "sm"),
                                                         ("p2p_allgather", "outgoing", 2, "sm")])
def test_single_rank_native_pipeline(scheme, mode, row_chunks, push, monkeypatch):
    """world = 1: the native pipeline (row-chunked input stage, copies into its own
    receive window, flag waits, strided contractions) equals the plain forward, over
    several forwards (alternating receive slots, increasing flag epochs)."""
    from fast_trimul_b200.distributed import ShardedTriMul
    from tests.helpers import make_layer
    monkeypatch.setenv("FTM_SHARD_PUSH", push)
    m = make_layer(mode, True).cuda()
    g = torch.Generator(device="cuda").manual_seed(22)
    sh = ShardedTriMul(m._impl, 1, 256, device="cuda", out_dtype=torch.float32, scheme=scheme,
                       row_chunks=row_chunks)
    for it in range(3):
        z = torch.randn(1, 256, 256, 128, device="cuda", generator=g).to(torch.bfloat16)
        mask = torch.ones(1, 256, 256, device="cuda")
        mask[:, :, 250:] = 0
        got = sh(z, mask)
        with torch.no_grad():
            want = m._impl._forward_native(z, mask, out_dtype=torch.float32)
        sh.check()
        d = (got - want).abs().max().item()
        assert d <= 2e-3, (it, d)
    sh.close()
