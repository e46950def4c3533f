"""Host logic of the sharded path (no GPU): row shards, the length-balanced
batch split of the key-padding workload, and the single-rank identity of the
gradient all-reduce."""
import numpy as np
import pytest

from nnop import shards


@pytest.mark.parametrize("n,world", [(0, 1), (1, 2), (7, 3), (65536, 8), (65537, 8), (5, 8)])
def test_row_shard_covers_rows_once(n, world):
    parts = [shards.row_shard(n, r, world) for r in range(world)]
    assert parts[0].start == 0 and parts[-1].stop == n
    assert all(a.stop == b.start for a, b in zip(parts, parts[1:]))
    sizes = [p.stop - p.start for p in parts]
    assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 0


def test_row_shard_rejects_bad_rank():
    with pytest.raises(ValueError):
        shards.row_shard(10, 2, 2)
    with pytest.raises(ValueError):
        shards.row_shard(-1, 0, 1)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_balance_by_length_varlen_workload(world):
    # the key lengths of the variable-length workload: B = 16 per GPU, len in [256, 4096]
    rng = np.random.default_rng(4)
    lens = rng.integers(256, 4097, size=16 * world)
    split = shards.balance_by_length(lens, world)
    assert sorted(i for s in split for i in s) == list(range(len(lens)))
    assert all(s == sorted(s) for s in split)
    loads = [int(lens[s].sum()) for s in split]
    mean = lens.sum() / world
    assert max(loads) - mean < lens.max()          # the LPT bound
    assert max(loads) / mean < 1.02                # and, at 16 batches per rank, within 2 %
    assert split == shards.balance_by_length(list(lens), world)   # deterministic


def test_balance_by_length_edges():
    assert shards.balance_by_length([], 3) == [[], [], []]
    assert shards.balance_by_length([5], 2) == [[0], []]
    assert shards.balance_by_length([3, 3, 3, 3], 2) == [[0, 2], [1, 3]]
    with pytest.raises(ValueError):
        shards.balance_by_length([1, -1], 2)
    with pytest.raises(ValueError):
        shards.balance_by_length([1], 0)


def test_allreduce_single_rank_is_identity():
    import torch
    dw, db = torch.arange(4.0), torch.ones(4, dtype=torch.bfloat16)
    out = shards.allreduce_norm_grads(dw, db)
    assert out[0] is dw and out[1] is db
