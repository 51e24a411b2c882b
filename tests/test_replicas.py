"""The multi-GPU path of bench.py on the CPU: replicas (one sequence set per rank, no data-path collective) meet only
for the timing barrier and the max over ranks. Two gloo ranks as processes on 127.0.0.1:

- every rank gets the slowest rank's times (device and wall), so the whole-job rate is all ranks' units over the
  slowest time (weak scaling);
- the reference arm's non-zero ranks do no work and print nothing.
"""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out: str) -> None:
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dist.barrier()
        # rank r's own timings: device seconds and wall seconds (rank 1 is the slow one on the device, rank 0 on the host)
        dev, wall = bench.max_over_ranks([1.0 + rank, 3.0 - rank], dist)
        rate = bench.whole_job_rate(world, 512 * 5, dev)
        Path(out).write_text(json.dumps({"rank": rank, "dev": dev, "wall": wall, "rate": rate}))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_rate_on_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    port = _free_port()
    outs = [str(tmp_path / f"r{r}.json") for r in range(2)]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, outs[r])) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = [json.loads(Path(o).read_text()) for o in outs]
    for r in res:
        assert r["dev"] == 2.0 and r["wall"] == 3.0  # the slowest rank's device time and wall time, on every rank
        assert r["rate"] == pytest.approx(2 * 512 * 5 / 2.0)


def test_one_process_is_its_own_max():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.max_over_ranks([0.5, 0.25]) == [0.5, 0.25]
    assert bench.whole_job_rate(1, 100, 2.0) == 50.0


def test_reference_arm_other_ranks_do_nothing():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    p = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], env=env, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0 and p.stdout.strip() == ""
