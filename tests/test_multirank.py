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
