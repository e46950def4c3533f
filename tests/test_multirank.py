"""The N > 1 path of bench.py on CPU: two gloo ranks (one process per GPU on a
B200 box, here plain processes) checking the host-side logic -- per-rank batch
shards, the max-over-ranks timing reduction every rank takes part in, the
whole-job throughput, and that the reference arm runs on rank 0 only."""
import contextlib
import io
import os
import pathlib
import socket
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), LOCAL_RANK=str(rank),
                      WORLD_SIZE=str(world))
    sys.path.insert(0, str(ROOT))
    import datetime

    import torch.distributed as dist

    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        r, lr, w = bench.dist_env()
        # rank 1 is the slow one for the first value, rank 0 for the second
        got = bench.max_over_ranks([1.0 + r, 10.0 - r, 0.5], "cpu", w)
        tf = bench.job_tflops(2.0e12, w, got[0])
        seed = bench.rank_seed(r)
        # the reference arm prints only on rank 0
        buf = io.StringIO()
        if r != 0:
            with contextlib.redirect_stdout(buf):
                bench.run_reference(type("A", (), {"steps": 1, "warmup": 0, "gpus": w})())
        (pathlib.Path(out_dir) / f"rank{r}.txt").write_text(
            f"{r} {lr} {w} {got[0]} {got[1]} {got[2]} {tf} {seed} {len(buf.getvalue())}")
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    rows = [(tmp_path / f"rank{r}.txt").read_text().split() for r in range(2)]
    seeds = set()
    for r, row in enumerate(rows):
        rank, lrank, world = int(row[0]), int(row[1]), int(row[2])
        assert (rank, lrank, world) == (r, r, 2)
        # every rank sees the same maxima
        assert [float(x) for x in row[3:6]] == [2.0, 10.0, 0.5]
        # 2 ranks x 2e12 flop in 2 ms of the slowest rank = 2000 TFLOP/s
        assert float(row[6]) == pytest.approx(2000.0)
        seeds.add(int(row[7]))
        assert int(row[8]) == 0   # rank 1's reference arm printed nothing
    assert len(seeds) == 2       # each rank its own batch shard


def _norm_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), LOCAL_RANK=str(rank),
                      WORLD_SIZE=str(world))
    sys.path[:0] = [str(ROOT), str(ROOT / "onionop.jl_b200")]
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from nnop import shards
    from oracle import nnop_oracle as orc
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(11)            # the same full job on every rank
        n, emb = 37, 24                            # 37 rows: shards of 19 and 18
        x, dy = rng.standard_normal((n, emb)), rng.standard_normal((n, emb))
        w = 1 + 0.1 * rng.standard_normal(emb)
        rows = shards.row_shard(n, rank, world)
        _, dw_rms = orc.rms_norm_bwd(dy[rows], x[rows], w)
        _, dw_ln, db_ln = orc.layer_norm_bwd(dy[rows], x[rows], w)
        (dw_rms_t,) = shards.allreduce_norm_grads(torch.from_numpy(dw_rms).float())
        dw_ln_t, db_ln_t = shards.allreduce_norm_grads(torch.from_numpy(dw_ln).bfloat16(),
                                                       torch.from_numpy(db_ln).bfloat16())
        assert dw_ln_t.dtype == torch.bfloat16 and db_ln_t.shape == (emb,)
        np.savez(pathlib.Path(out_dir) / f"norm{rank}.npz", rows=np.array([rows.start, rows.stop]),
                 dw_rms=dw_rms_t.double().numpy(), dw_ln=dw_ln_t.double().numpy(), db_ln=db_ln_t.double().numpy())
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_norm_grads(tmp_path):
    import numpy as np
    import torch.multiprocessing as mp

    from oracle import nnop_oracle as orc
    port = _free_port()
    mp.start_processes(_norm_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    got = [np.load(tmp_path / f"norm{r}.npz") for r in range(2)]
    assert [tuple(g["rows"]) for g in got] == [(0, 19), (19, 37)]
    rng = np.random.default_rng(11)
    n, emb = 37, 24
    x, dy = rng.standard_normal((n, emb)), rng.standard_normal((n, emb))
    w = 1 + 0.1 * rng.standard_normal(emb)
    _, dw_rms = orc.rms_norm_bwd(dy, x, w)
    _, dw_ln, db_ln = orc.layer_norm_bwd(dy, x, w)
    for g in got:                                  # every rank holds the whole job's gradients
        np.testing.assert_allclose(g["dw_rms"], dw_rms, rtol=1e-5, atol=1e-5)
        # 16-bit partials: each rank's value rounded once, the sum rounded once
        np.testing.assert_allclose(g["dw_ln"], dw_ln, rtol=2e-2, atol=5e-2)
        np.testing.assert_allclose(g["db_ln"], db_ln, rtol=2e-2, atol=5e-2)
    assert all((got[0][k] == got[1][k]).all() for k in ("dw_rms", "dw_ln", "db_ln"))


def _attn_worker(rank, world, port, out_dir):
    """One rank of an attention job sharded by (batch, kv head): the oracle's
    forward and backward on this rank's pieces only, results sent to rank 0."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), LOCAL_RANK=str(rank),
                      WORLD_SIZE=str(world))
    sys.path[:0] = [str(ROOT), str(ROOT / "onionop.jl_b200")]
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from nnop import shards
    from oracle import nnop_oracle as orc
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q, k, v, do, pair = _attn_job()
        B, QH, L, E = q.shape
        KH = k.shape[1]
        n_rep = QH // KH
        out = {}
        for i, piece in enumerate(shards.shard_batch_heads(B, KH, rank, world)):
            qs, ks, vs, ps = (t.numpy() for t in shards.piece_views(piece, n_rep, *map(torch.from_numpy,
                                                                                    (q, k, v)), torch.from_numpy(pair)))
            (dos,) = (t.numpy() for t in shards.piece_views(piece, n_rep, torch.from_numpy(do)))
            o, _ = orc.attention_fwd(qs, ks, vs, ps, causal=True, scale=0.25)
            g = orc.attention_bwd(dos, qs, ks, vs, ps, causal=True, scale=0.25)
            for name, a in zip(("o", "dq", "dk", "dv", "dpair"), (o,) + tuple(g)):
                out[f"{i}_{name}"] = a
            out[f"{i}_piece"] = np.array(piece)
        np.savez(pathlib.Path(out_dir) / f"attn{rank}.npz", **out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _attn_job():
    import numpy as np
    rng = np.random.default_rng(21)
    B, QH, KH, L, E = 2, 8, 4, 12, 8
    q = rng.standard_normal((B, QH, L, E))
    k, v = rng.standard_normal((B, KH, L, E)), rng.standard_normal((B, KH, L, E))
    do = rng.standard_normal((B, QH, L, E))
    pair = rng.standard_normal((B, L, L, QH))
    return q, k, v, do, pair


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ranks_batch_head_shards_reassemble(tmp_path, world):
    """Ranks that each run only their (batch, kv-head) pieces produce, put back
    together, exactly the whole job's o, dq, dk, dv and dpair (GQA n_rep = 2,
    causal, pair bias): the split needs no cross-rank reduction."""
    import numpy as np
    import torch.multiprocessing as mp

    from oracle import nnop_oracle as orc
    port = _free_port()
    mp.start_processes(_attn_worker, args=(world, port, str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)
    q, k, v, do, pair = _attn_job()
    n_rep = q.shape[1] // k.shape[1]
    o_w, _ = orc.attention_fwd(q, k, v, pair, causal=True, scale=0.25)
    dq_w, dk_w, dv_w, dp_w = orc.attention_bwd(do, q, k, v, pair, causal=True, scale=0.25)
    got = {n: np.full_like(a, np.nan) for n, a in (("o", o_w), ("dq", dq_w), ("dk", dk_w), ("dv", dv_w),
                                                     ("dpair", dp_w))}
    for r in range(world):
        f = np.load(tmp_path / f"attn{r}.npz")
        i = 0
        while f"{i}_piece" in f:
            b0, b1, h0, h1 = f[f"{i}_piece"]
            got["o"][b0:b1, h0 * n_rep:h1 * n_rep] = f[f"{i}_o"]
            got["dq"][b0:b1, h0 * n_rep:h1 * n_rep] = f[f"{i}_dq"]
            got["dk"][b0:b1, h0:h1] = f[f"{i}_dk"]
            got["dv"][b0:b1, h0:h1] = f[f"{i}_dv"]
            got["dpair"][b0:b1, :, :, h0 * n_rep:h1 * n_rep] = f[f"{i}_dpair"]
            i += 1
    for n, want in (("o", o_w), ("dq", dq_w), ("dk", dk_w), ("dv", dv_w), ("dpair", dp_w)):
        assert not np.isnan(got[n]).any(), n          # every element produced by some rank
        np.testing.assert_allclose(got[n], want, rtol=1e-12, atol=1e-12, err_msg=n)
