"""Multi-rank host logic on CPU (gloo, world size 2).

The SKA core shards over batch and heads with no exchange between ranks.  These
tests run two gloo ranks that each compute their own head (or batch) shard with
the oracle, gather the shards, and check that the result equals the whole
problem computed in one process; and that the timing reduction returns the
slowest rank's time.  No GPU is involved.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from koopman_mamba_b200.sharding import batch_shard, head_shard, max_over_ranks, shard_range
from oracle.ska_oracle import SkaParams, ska_core_fwd_bwd

WORLD = 2


def _inputs(seed, B=2, T=96, H=3, r=8, P=16):
    g = torch.Generator().manual_seed(seed)
    s = 1.0 / np.sqrt(64)
    z, zq, v = (torch.randn(B, T, H, n, generator=g, dtype=torch.float64) * s for n in (r, r, P))
    dy = torch.randn(B, T, H, P, generator=g, dtype=torch.float64)
    return z, zq, v, dy


PARAMS = SkaParams(chunk_size=32, ridge_eps=1e-3, power_K=2)


def _run(z, zq, v, dy):
    outs = ska_core_fwd_bwd(z.numpy(), zq.numpy(), v.numpy(), 1.1, dy.numpy(), PARAMS, np.float64)
    y, dz, dzq, dv, _ = outs
    return [torch.from_numpy(np.ascontiguousarray(a)) for a in (y, dz, dzq, dv)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, mode, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        z, zq, v, dy = _inputs(0)
        shard = head_shard if mode == "heads" else batch_shard
        mine = _run(*(shard(t, WORLD, rank) for t in (z, zq, v, dy)))
        gathered = []
        for out in mine:
            parts = [None] * WORLD
            dist.all_gather_object(parts, out)
            gathered.append(torch.cat(parts, dim=2 if mode == "heads" else 0))
        slowest = max_over_ranks(10.0 + rank)
        if rank == 0:
            torch.save({"outs": gathered, "slowest": slowest}, result_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["heads", "batch"])
def test_shards_reassemble_to_the_whole_problem(mode, tmp_path):
    path = str(tmp_path / "res.pt")
    mp.start_processes(_worker, args=(_free_port(), mode, path), nprocs=WORLD, start_method="spawn")
    res = torch.load(path)
    whole = _run(*_inputs(0))
    for got, want in zip(res["outs"], whole):
        assert got.shape == want.shape
        # every series is independent: the shards give the whole answer (up to the
        # fp64 rounding of numpy's batched reductions over differently shaped arrays)
        assert float((got - want).norm() / want.norm()) <= 1e-12
    assert res["slowest"] == 11.0


def test_shard_range_is_a_balanced_partition():
    for n in (0, 1, 7, 12, 16):
        for world in (1, 2, 3, 4, 8):
            parts = [shard_range(n, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_head_shard_is_a_view():
    x = torch.zeros(2, 5, 6, 4)
    s = head_shard(x, 3, 1)
    assert s.shape == (2, 5, 2, 4)
    assert s.data_ptr() == x[:, :, 2].data_ptr()
    assert s.stride() == x.stride()
    assert max_over_ranks(3.5) == 3.5   # no process group: identity
