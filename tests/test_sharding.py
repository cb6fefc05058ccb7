"""Host-side batch sharding: slice arithmetic and a world-size-2 gloo run on CPU.

The per-rank factorisation in the gloo test is a CPU stand-in (torch.geqrf), since these
tests run without a GPU; what is tested is the split/gather plumbing of the N > 1 path.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from qr_v2_b200_kernel_b200.sharding import gather_shards, shard_range


@pytest.mark.parametrize("batch,world", [(640, 8), (64, 8), (8, 8), (2, 8), (2, 2), (1, 4), (0, 3), (13, 4)])
def test_shard_range_covers_batch_once(batch, world):
    seen = []
    for r in range(world):
        lo, hi = shard_range(batch, world, r)
        assert 0 <= lo <= hi <= batch
        seen.extend(range(lo, hi))
    assert seen == list(range(batch))


def test_shard_range_matches_workload_plan():
    assert [shard_range(640, 8, r) for r in (0, 7)] == [(0, 80), (560, 640)]  # C2: 80 per GPU
    assert shard_range(2, 8, 1) == (1, 2) and shard_range(2, 8, 2) == (2, 2)  # C5: 6 ranks idle
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, batch, n, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        A = torch.randn((batch, n, n), generator=g)
        lo, hi = shard_range(batch, world, rank)
        H_local, tau_local = torch.geqrf(A[lo:hi])  # CPU stand-in for the per-GPU kernel
        H = gather_shards(H_local, batch)
        tau = gather_shards(tau_local, batch)
        if rank == 0:
            Hf, tf = torch.geqrf(A)
            out.put((bool(torch.allclose(H, Hf, atol=1e-5)), bool(torch.allclose(tau, tf, atol=1e-6)), tuple(H.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch", [5, 2])
def test_gloo_world2_split_and_gather(batch):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, 12, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    okH, oktau, shape = q.get(timeout=5)
    assert okH and oktau and shape == (batch, 12, 12)
