"""Row-sharded forward on CPU: world_size 2 gloo ranks run the sharding logic
(partitioning, chunked all-gather into the block-major layout, per-chunk
contraction) with torch stand-ins for the three kernels; the gathered result must
equal the unsharded CPU oracle."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, n, chunks, result_path, scheme, mode="outgoing"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fast_trimul_b200.distributed import RowShardedTriMul, TorchStageOps, row_range
        from tests.helpers import make_layer
        m = make_layer(mode, True, d=128)
        gen = torch.Generator().manual_seed(9)
        z = torch.randn(1, n, n, 128, generator=gen)
        mask = torch.ones(1, n, n)
        mask[:, :, n - 3:] = 0
        lo, hi = row_range(n, world, rank)
        sh = RowShardedTriMul(m._impl, 1, n, chunks=chunks, device="cpu",
                              z_dtype=torch.float32, out_dtype=torch.float32,
                              ops=TorchStageOps(m._impl), scheme=scheme)
        out = sh(z[:, lo:hi].contiguous(), mask[:, lo:hi].contiguous())
        parts = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(parts, out)
        if rank == 0:
            np.save(result_path, torch.cat(parts, dim=1).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,chunks,scheme,mode", [
    (2, 4, "allgather", "outgoing"), (2, 1, "allgather", "outgoing"),
    (2, 4, "alltoall", "outgoing"), (4, 2, "alltoall", "outgoing"),
    (2, 1, "fused", "outgoing"), (4, 1, "fused", "outgoing"),
    (2, 2, "alltoall", "incoming"), (4, 1, "alltoall", "incoming"), (2, 1, "fused", "incoming")])
def test_row_sharded_matches_oracle(tmp_path, world, chunks, scheme, mode):
    from tests.helpers import compare, make_layer, oracle_out
    n = 16
    path = str(tmp_path / "out.npy")
    mp.start_processes(_worker, args=(world, _free_port(), n, chunks, path, scheme, mode),
                       nprocs=world, join=True, start_method="spawn")
    got = torch.from_numpy(np.load(path))
    m = make_layer(mode, True, d=128)
    gen = torch.Generator().manual_seed(9)
    z = torch.randn(1, n, n, 128, generator=gen)
    mask = torch.ones(1, n, n)
    mask[:, :, n - 3:] = 0
    max_abs, mean_rel = compare(got, oracle_out(m, z, mask))
    assert max_abs < 2e-2 and mean_rel < 2e-3, (max_abs, mean_rel)


def test_row_range_and_constraints():
    from fast_trimul_b200.distributed import row_range
    assert row_range(2048, 8, 3) == (768, 1024)
    with pytest.raises(ValueError):
        row_range(100, 8, 0)


def test_incoming_sharding_needs_a_channel_sharded_scheme():
    """Incoming mode reduces over z rows, so an all-gather of b (outgoing's scheme) does not
    apply; the channel-sharded schemes accept it and the default picks one."""
    from fast_trimul_b200.distributed import RowShardedTriMul, TorchStageOps, default_scheme
    from tests.helpers import make_layer
    m = make_layer("incoming", True, d=128)
    for scheme in ("allgather", "allgather_ce"):
        with pytest.raises(NotImplementedError):
            RowShardedTriMul(m._impl, 1, 16, chunks=1, device="cpu", z_dtype=torch.float32,
                             ops=TorchStageOps(m._impl), scheme=scheme)
    assert default_scheme(2, "incoming") == "alltoall_ce"
    assert default_scheme(2, "outgoing") == "allgather_ce"
    assert default_scheme(8, "outgoing") == "alltoall_ce"
    with pytest.raises(ValueError):     # unknown scheme
        RowShardedTriMul(make_layer("outgoing", True, d=128)._impl, 1, 16, chunks=1, device="cpu",
                         z_dtype=torch.float32, ops=TorchStageOps(m._impl), scheme="unknown")
