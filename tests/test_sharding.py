"""Sequence sharding (metagross_b200/sharding.py) on the CPU: the LPT split
and the output gather, the latter over two real gloo ranks (127.0.0.1)."""
import os
import socket

import numpy as np
import pytest
import torch

from metagross_b200.sharding import ShardGather, lpt_shard, shard_loads


def test_lpt_partitions_every_sequence_once():
    g = np.random.default_rng(3)
    lens = g.lognormal(np.log(2048), 1.0, 1024).clip(1, 32768).astype(np.int64)
    for world in (1, 2, 4, 8):
        shards = lpt_shard(lens, world)
        assert len(shards) == world
        allidx = np.sort(np.concatenate(shards))
        np.testing.assert_array_equal(allidx, np.arange(lens.size))
        loads = shard_loads(lens, shards)
        lower = max(lens.sum() / world, lens.max())  # no split can beat this
        assert max(loads) / lower < 1.01  # many jobs, none dominant: LPT is within 1% of the bound


def test_lpt_is_deterministic_and_handles_small_cases():
    assert [s.tolist() for s in lpt_shard([5, 5, 5], 2)] == [[0, 2], [1]]
    assert [s.tolist() for s in lpt_shard([1, 9, 3], 4)] == [[1], [2], [0], []]
    assert [s.tolist() for s in lpt_shard([], 3)] == [[], [], []]
    a = lpt_shard([7, 3, 3, 8, 1], 2)
    b = lpt_shard([7, 3, 3, 8, 1], 2)
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
    with pytest.raises(ValueError):
        lpt_shard([1, 2], 0)
    with pytest.raises(ValueError):
        lpt_shard([1, -2], 2)


def test_lpt_equal_counts_keeps_sizes_and_balance():
    g = np.random.default_rng(5)
    lens = g.lognormal(np.log(2048), 1.0, 1024).clip(1, 32768).astype(np.int64)
    for world in (2, 4, 8):
        shards = lpt_shard(lens, world, equal_counts=True)
        assert [s.size for s in shards] == [1024 // world] * world
        np.testing.assert_array_equal(np.sort(np.concatenate(shards)), np.arange(lens.size))
        loads = shard_loads(lens, shards)
        assert max(loads) / max(lens.sum() / world, lens.max()) < 1.02
    assert [s.size for s in lpt_shard([9, 1, 1, 1, 1], 2, equal_counts=True)] == [3, 2]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_rank(rank, world, port, lens, q):
    import torch.distributed as dist

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        shards = lpt_shard(lens, world)
        glob = torch.arange(len(lens) * 6, dtype=torch.float32).view(len(lens), 2, 3)
        gather = ShardGather(shards, rank, (2, 3), torch.float32, "cpu")
        out = gather(glob[torch.as_tensor(shards[rank])])
        ok = torch.equal(out, glob)
        # a second step through the same buffers
        out2 = gather(2 * glob[torch.as_tensor(shards[rank])])
        ok = ok and torch.equal(out2, 2 * glob)
        # equal counts: each rank's block goes out as it is; the padded buffer in rank order
        eq = lpt_shard(lens, world, equal_counts=True)
        g2 = ShardGather(eq, rank, (2, 3), torch.float32, "cpu")
        raw = g2(glob[torch.as_tensor(eq[rank])].contiguous(), reorder=False)
        for r, sh in enumerate(eq):
            ok = ok and torch.equal(raw[r * g2.n_max:r * g2.n_max + g2.lengths[r]], glob[torch.as_tensor(sh)])
        ok = ok and torch.equal(g2(glob[torch.as_tensor(eq[rank])].contiguous()), glob)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("lens", [[300, 20, 1024, 7, 512, 512, 64], [5]])
def test_gather_restores_global_order_over_two_gloo_ranks(lens):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_rank, args=(r, 2, port, lens, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}, results
