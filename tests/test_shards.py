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


@pytest.mark.parametrize("B,KH,world", [(4, 8, 8), (4, 8, 3), (2, 4, 3), (1, 4, 2), (4, 8, 1), (3, 5, 4), (1, 2, 4),
                                        (8, 16, 8), (0, 4, 2)])
def test_shard_batch_heads_covers_units_once(B, KH, world):
    seen = []
    sizes = []
    for r in range(world):
        pieces = shards.shard_batch_heads(B, KH, r, world)
        assert len(pieces) <= 3
        n = 0
        for (b0, b1, h0, h1) in pieces:
            assert 0 <= b0 < b1 <= B and 0 <= h0 < h1 <= KH
            assert b1 - b0 == 1 or (h0, h1) == (0, KH)      # a partial batch is one batch
            seen += [(b, h) for b in range(b0, b1) for h in range(h0, h1)]
            n += (b1 - b0) * (h1 - h0)
        sizes.append(n)
    assert sorted(seen) == [(b, h) for b in range(B) for h in range(KH)]
    assert max(sizes) - min(sizes) <= 1


def test_shard_batch_heads_gqa_workload_over_8():
    """The GQA workload (B = 4, KH = 8): 8 ranks, each one batch x 4 kv heads."""
    assert [shards.shard_batch_heads(4, 8, r, 8) for r in range(8)] == [
        [(b, b + 1, h, h + 4)] for b in range(4) for h in (0, 4)]


def test_piece_views_are_the_pieces_slices():
    import torch
    B, QH, KH, L, E = 2, 6, 3, 5, 4
    q = torch.arange(B * QH * L * E, dtype=torch.float32).reshape(B, QH, L, E)
    k = torch.arange(B * KH * L * E, dtype=torch.float32).reshape(B, KH, L, E)
    pair = torch.arange(B * L * L * QH, dtype=torch.float32).reshape(B, L, L, QH)
    qv, kv, vv, pv = shards.piece_views((1, 2, 1, 3), 2, q, k, k, pair)
    assert torch.equal(qv, q[1:2, 2:6]) and qv.is_contiguous()
    assert torch.equal(kv, k[1:2, 1:3]) and torch.equal(vv, kv)
    assert torch.equal(pv, pair[1:2, :, :, 2:6]) and pv.is_contiguous()
