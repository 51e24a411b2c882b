"""The page sweep's scheduler on the host (historic-htr-ocr_b200/pages.py), without a GPU.

Config 5 reads 512 pages with one model replica per GPU and no data-path collective: the ranks share only the
process group's key-value store (claims, ownership, heartbeats). These tests run the scheduler with a CPU stand-in for
a GPU's page engine (slots that spend a page's budget one step at a time), as gloo ranks in separate processes:
- every page is read exactly once, and both ranks take part;
- a rank that dies between steps while holding pages (its process exits) has its unfinished pages requeued by the
  survivor, which reads them: every page still read exactly once (the failure is made on the host, no GPU involved);
- the seeded page set has the config's ranges.
"""
from __future__ import annotations

import json
import multiprocessing as mp
import os
import socket
import time

import pytest


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n_pages, die_rank, die_after, out_path):
    import datetime
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "historic-htr-ocr_b200"))
    import torch.distributed as dist

    from pages import PageQueue, run_worker

    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=60))
    store = dist.distributed_c10d._get_default_store()
    q = PageQueue(store, rank, world, n_pages, ns="t/", hb_timeout=1.5)
    read_here = []

    def read(claim, done):
        # a stand-in page engine: 4 slots, a page of budget 3 + p % 5 steps, 2 ms per step
        slots = []
        while True:
            while len(slots) < 4:
                p = claim()
                if p is None:
                    break
                slots.append([p, 3 + p % 5])
            if not slots:
                return
            time.sleep(0.002)
            for s in slots:
                s[1] -= 1
            for s in [s for s in slots if s[1] <= 0]:
                slots.remove(s)
                done(s[0], 10 + s[0])
                read_here.append(s[0])
                if rank == die_rank and len(read_here) == die_after:
                    # dies between steps, holding the pages in its other slots
                    with open(out_path + f".held{rank}", "w") as f:
                        json.dump([x[0] for x in slots], f)
                    os._exit(3)

    run_worker(read, q, poll=0.05, deadline=60.0)
    owners = {p: store.get(f"t/done/{p}").decode() for p in range(n_pages)}
    with open(out_path + f".rank{rank}", "w") as f:
        json.dump({"read": read_here, "n_done": q.n_done(), "tokens": q.tokens(), "owners": owners}, f)
    q.leave()
    os._exit(0)


def _run(tmp_path, world, n_pages, die_rank=-1, die_after=0):
    port = _free_port()
    out = str(tmp_path / "sweep")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n_pages, die_rank, die_after, out))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    results = {}
    for r in range(world):
        path = out + f".rank{r}"
        if os.path.exists(path):
            with open(path) as f:
                results[r] = json.load(f)
    held = None
    if die_rank >= 0 and os.path.exists(out + f".held{die_rank}"):
        with open(out + f".held{die_rank}") as f:
            held = json.load(f)
    return codes, results, held


def test_two_ranks_read_every_page_once(tmp_path):
    n = 40
    codes, res, _ = _run(tmp_path, 2, n)
    assert codes == [0, 0]
    r0, r1 = res[0], res[1]
    assert r0["n_done"] == n and r0["tokens"] == sum(10 + p for p in range(n))
    assert sorted(r0["read"] + r1["read"]) == list(range(n))  # each page read once, by one rank
    assert r0["read"] and r1["read"]


def test_dead_rank_pages_are_requeued_and_read(tmp_path):
    n = 40
    codes, res, held = _run(tmp_path, 2, n, die_rank=1, die_after=5)
    assert codes == [0, 3], codes  # rank 1 exited between steps; rank 0 finished the sweep
    r0 = res[0]
    assert 1 not in res
    assert held, "rank 1 died holding pages"
    assert r0["n_done"] == n and r0["tokens"] == sum(10 + p for p in range(n))
    # the pages rank 1 held when it died were read by rank 0
    assert all(r0["owners"][str(p)] == "0" for p in held)
    assert all(p in r0["read"] for p in held)
    owners = r0["owners"]
    assert sorted(int(p) for p, o in owners.items() if o == "0") == sorted(r0["read"])


def test_page_specs_are_seeded_in_range():
    import pages as P

    a, b = P.page_specs(123), P.page_specs(123)
    assert a == b and len(a) == P.N_PAGES
    assert all(P.PREFIX_MIN <= s.prefix <= P.PREFIX_MAX and P.GEN_MIN <= s.new <= P.GEN_MAX for s in a)
    assert all(0 <= s.row0 and s.row0 + s.prefix <= P.POOL_ROWS for s in a)
    assert len({s.prefix for s in a}) > 100 and len({s.new for s in a}) > 100


def test_local_queue_single_rank():
    import pages as P

    q = P.PageQueue(P.LocalStore(), 0, 1, 7)
    got = []
    P.run_worker(lambda claim, done: [got.append(p) or done(p, 1) for p in iter(claim, None)], q, poll=0.01,
                 deadline=10)
    assert sorted(got) == list(range(7)) and q.n_done() == 7
