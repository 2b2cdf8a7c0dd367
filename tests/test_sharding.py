"""Placement of independent sequences on ranks (batched decode, no collective): a partition
with equal counts and balanced total context, computed identically on every rank."""
import os

import numpy as np
import pytest
import torch.multiprocessing as mp

from soc_b200.sharding import balanced_shards


def _contexts():
    # the config-3 workload: 256 sequences, contexts U[128, 4096], seed 4
    return np.random.default_rng(4).integers(128, 4097, 256)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_partition_counts_and_balance(world):
    c = _contexts()
    parts = balanced_shards(c, world)
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(len(c)))
    counts = [len(p) for p in parts]
    assert max(counts) - min(counts) <= 1
    loads = [int(c[p].sum()) for p in parts]
    assert max(loads) / np.mean(loads) < 1.005
    # contiguous blocks of the same sizes are far less even at 8 ranks (1.17)
    if world == 8:
        per = len(c) // world
        blocks = [int(c[r * per:(r + 1) * per].sum()) for r in range(world)]
        assert max(blocks) / np.mean(blocks) > 1.1


def test_small_and_degenerate_inputs():
    assert balanced_shards([], 3) == [[], [], []]
    assert balanced_shards([5, 5], 4) == [[0], [1], [], []]
    assert balanced_shards([7, 1, 1, 1, 1, 1, 1, 1], 2) == [[0, 5, 6, 7], [1, 2, 3, 4]]
    assert balanced_shards([3, 3, 3, 3], 2) == [[0, 2], [1, 3]]
    with pytest.raises(ValueError):
        balanced_shards([1], 0)


def _rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    mine = balanced_shards(_contexts(), world)[rank]
    got = [None] * world
    dist.all_gather_object(got, mine)
    if rank == 0:
        q.put(got)
    dist.destroy_process_group()


def test_ranks_agree_without_exchange():
    """Two gloo ranks each compute their own shard; gathered, they are the single-process
    placement and a partition of all sequences."""
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    port = 29500 + os.getpid() % 200
    ps = [ctxm.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == balanced_shards(_contexts(), 2)
