"""Host logic of the multi-GPU path on CPU: contiguous batch shards and the
gather of per-pair distances, run as two gloo ranks.  Each rank computes its
shard with the float64 oracle (standing in for its GPU), and the gathered
result must equal the unsharded one bit for bit."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from torchwarp_b200.sharding import shard_bounds


def test_shard_bounds_partition():
    for B in range(0, 23):
        for world in range(1, 9):
            spans = [shard_bounds(B, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            for (a0, b0), (a1, _) in zip(spans, spans[1:]):
                assert b0 == a1
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)
    with pytest.raises(ValueError):
        shard_bounds(-1, 2, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, B, out_path):
    import torch.distributed as dist

    import oracle
    from torchwarp_b200.sharding import gather_pairs, shard_bounds
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        rng = np.random.default_rng(7)
        X = rng.standard_normal((B, 9, 3))
        Y = rng.standard_normal((B, 11, 3))
        a, b = shard_bounds(B, world, rank)
        d, _, _ = oracle.soft_dtw(X[a:b], Y[a:b], gamma=0.5)
        full = gather_pairs(torch.from_numpy(np.asarray(d, dtype=np.float64)), B)
        if rank == 0:
            ref, _, _ = oracle.soft_dtw(X, Y, gamma=0.5)
            np.save(out_path, np.stack([full.numpy(), np.asarray(ref)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [5, 8])
def test_two_rank_gather_matches_unsharded(tmp_path, B):
    out = str(tmp_path / "res.npy")
    mp.start_processes(_rank_main, args=(2, _free_port(), B, out), nprocs=2, join=True,
                       start_method="spawn")
    got, ref = np.load(out)
    assert np.array_equal(got, ref)
