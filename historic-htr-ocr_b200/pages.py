"""pages.py — the page sweep across GPUs: one replica of the model per GPU (one process each), pages claimed from a
shared queue, each GPU reading its pages through its session's slots (ocr_read_pages, continuous batching).

The reference reads one page per Engine::read_text (app/crates/ocr-wgpu/src/engine.rs:447-524) on one device; pages
are independent, so a box of GPUs reads them in parallel with no data-path collective. The ranks share only a small
key-value store (torch.distributed's rendezvous store, or any object with its set / get / add / compare_set / check
methods):

    <ns>next              claims of fresh pages (an atomic counter)
    <ns>own/<p>           the rank that holds page p
    <ns>done/<p>          set once page p is read; <ns>n_done counts them, <ns>tokens sums their tokens
    <ns>hb/<r>            rank r's heartbeat (wall time); <ns>fin/<r> once rank r has nothing left to read
    <ns>rq_n, <ns>rq/<i>  pages given back: a dead rank's unfinished pages
    <ns>rqc/<i>           the claim of requeued entry i (first compare_set wins)
    <ns>reaped/<r>        the survivor that requeued dead rank r's pages (first compare_set wins)
    <ns>left/<r>          rank r is gone (the store's host waits for the others before it goes)

A rank whose heartbeat is older than `hb_timeout` and that has not declared itself finished is dead: the first
survivor to notice it requeues the pages it held and did not finish, and every rank keeps claiming until all pages are
done. Failures are detected on the host only (a rank that exits or stops); no GPU is faulted or waited on.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable, Optional

import numpy as np

import ocr_b200 as ocr

# 512 pages, prefix rows uniform on [1500, 3072], tokens uniform on [800, 1500]
N_PAGES, PREFIX_MIN, PREFIX_MAX, GEN_MIN, GEN_MAX = 512, 1500, 3072, 800, 1500
POOL_ROWS = 16384  # the seeded table the pages' prefix rows are cut from


@dataclass
class PageSpec:
    page: int
    prefix: int    # prefix rows (embedding rows: image positions and prompt, as config 3's)
    new: int       # tokens to generate
    row0: int      # the first of its rows in the seeded table


def page_specs(seed: int, n_pages: int = N_PAGES) -> list[PageSpec]:
    """the sweep's pages, seeded: prefix and generation lengths uniform on their ranges, each page's rows a distinct
    window of one seeded N(0,1) table (the rows' values do not change a page's work)"""
    z = ocr.splitmix64_at(seed, np.arange(3 * n_pages, dtype=np.uint64))
    u = (z >> np.uint64(11)).astype(np.float64) / float(1 << 53)
    out = []
    for p in range(n_pages):
        pre = PREFIX_MIN + int(u[3 * p] * (PREFIX_MAX - PREFIX_MIN + 1))
        new = GEN_MIN + int(u[3 * p + 1] * (GEN_MAX - GEN_MIN + 1))
        row0 = int(u[3 * p + 2] * (POOL_ROWS - pre + 1))
        out.append(PageSpec(p, pre, new, row0))
    return out


def page_pool(seed: int, dim: int) -> np.ndarray:
    return ocr.gauss(ocr.substream(seed, 300000), POOL_ROWS * dim, 1.0).reshape(POOL_ROWS, dim)


class LocalStore:
    """the store's interface in one process (a single GPU, or tests): set / get / add / compare_set / check"""

    def __init__(self):
        self.kv: dict[str, bytes] = {}

    def set(self, k, v):
        self.kv[k] = v.encode() if isinstance(v, str) else bytes(v)

    def get(self, k):
        return self.kv[k]

    def add(self, k, n):
        v = int(self.kv.get(k, b"0")) + n
        self.kv[k] = str(v).encode()
        return v

    def compare_set(self, k, expected, desired):
        cur = self.kv.get(k)
        exp = expected.encode() if isinstance(expected, str) else expected
        if (cur is None and exp == b"") or cur == exp:
            self.kv[k] = desired.encode() if isinstance(desired, str) else desired
        return self.kv.get(k, b"")

    def check(self, keys):
        return all(k in self.kv for k in keys)


class PageQueue:
    """the ranks' shared view of the sweep (see the module docstring for the keys)"""

    def __init__(self, store, rank: int, world: int, n_pages: int, ns: str = "pages/", hb_timeout: float = 30.0):
        self.s, self.rank, self.world, self.n, self.ns, self.hb_timeout = store, rank, world, n_pages, ns, hb_timeout
        self.rq_seen = 0  # requeued entries this rank has looked at
        self.heartbeat()

    def _k(self, *parts) -> str:
        return self.ns + "/".join(str(p) for p in parts)

    def _has(self, key: str) -> bool:
        return self.s.check([key])

    def heartbeat(self) -> None:
        self.s.set(self._k("hb", self.rank), repr(time.time()))

    def claim(self) -> Optional[int]:
        """the next page to read (a requeued one first), now owned by this rank; None when there is none"""
        self.heartbeat()
        n_rq = self.s.add(self._k("rq_n"), 0)
        while self.rq_seen < n_rq:
            i = self.rq_seen
            self.rq_seen += 1
            if self.s.compare_set(self._k("rqc", i), "", str(self.rank)).decode() == str(self.rank):
                p = int(self.s.get(self._k("rq", i)))
                self.s.set(self._k("own", p), str(self.rank))
                return p
        p = self.s.add(self._k("next"), 1) - 1
        if p >= self.n:
            return None
        self.s.set(self._k("own", p), str(self.rank))
        return p

    def done(self, p: int, n_tokens: int) -> None:
        if self.s.compare_set(self._k("done", p), "", str(self.rank)).decode() == str(self.rank):
            self.s.add(self._k("n_done"), 1)
            self.s.add(self._k("tokens"), int(n_tokens))
        self.heartbeat()

    def n_done(self) -> int:
        return self.s.add(self._k("n_done"), 0)

    def tokens(self) -> int:
        return self.s.add(self._k("tokens"), 0)

    def finish(self) -> None:
        """this rank has nothing left to read (it keeps watching for requeued pages)"""
        self.s.set(self._k("fin", self.rank), "1")

    def unfinish(self) -> None:
        self.s.set(self._k("fin", self.rank), "0")

    def _finished(self, r: int) -> bool:
        return self._has(self._k("fin", r)) and self.s.get(self._k("fin", r)) == b"1"

    def reap_dead(self) -> int:
        """requeue the unfinished pages of every rank whose heartbeat stopped (once per dead rank, by the first
        survivor to see it); returns how many pages this call requeued"""
        now, n = time.time(), 0
        for r in range(self.world):
            if r == self.rank or self._finished(r):
                continue
            hb = self._k("hb", r)
            if self._has(hb) and now - float(self.s.get(hb)) < self.hb_timeout:
                continue
            if not self._has(hb):
                continue  # not started yet
            if self.s.compare_set(self._k("reaped", r), "", str(self.rank)).decode() != str(self.rank):
                continue
            for p in range(self.n):
                own = self._k("own", p)
                if self._has(own) and self.s.get(own) == str(r).encode() and not self._has(self._k("done", p)):
                    i = self.s.add(self._k("rq_n"), 1) - 1
                    self.s.set(self._k("rq", i), str(p))
                    n += 1
        return n

    def pending_requeued(self) -> bool:
        return self.s.add(self._k("rq_n"), 0) > self.rq_seen

    def leave(self, host_rank: int = 0, poll: float = 0.05, deadline: float = 60.0) -> None:
        """the end of this rank's part: it marks itself gone; the rank that hosts the store (rank 0 of a
        torch.distributed rendezvous) waits until every other rank is gone or dead before it returns, so the store
        outlives their last reads"""
        self.s.set(self._k("left", self.rank), "1")
        if self.rank != host_rank:
            return
        t_end = time.time() + deadline
        while time.time() < t_end:
            pending = [r for r in range(self.world) if r != self.rank and not self._has(self._k("left", r))]
            now = time.time()
            alive = [r for r in pending
                     if self._has(self._k("hb", r)) and now - float(self.s.get(self._k("hb", r))) < self.hb_timeout]
            if not alive:
                return
            time.sleep(poll)


def run_worker(read: Callable[[Callable[[], Optional[int]], Callable[[int, int], bool]], None], q: PageQueue,
               poll: float = 0.2, deadline: float = 3600.0) -> int:
    """one rank's part of the sweep: `read(claim, done)` reads pages (claim() → a page or None; done(page, tokens))
    until none is left; then the rank watches for dead peers, reading any page they leave, until every page is done.
    Returns the pages this rank read."""
    mine = [0]

    def claim():
        return q.claim()

    def done(p, n_tokens):
        q.done(p, n_tokens)
        mine[0] += 1
        return True

    t_end = time.time() + deadline
    while time.time() < t_end:
        q.unfinish()
        read(claim, done)
        q.finish()
        while time.time() < t_end:
            if q.n_done() >= q.n:
                return mine[0]
            q.heartbeat()
            if q.reap_dead() or q.pending_requeued():
                break
            time.sleep(poll)
    raise TimeoutError(f"rank {q.rank}: the sweep did not finish within {deadline} s ({q.n_done()} of {q.n} pages)")
