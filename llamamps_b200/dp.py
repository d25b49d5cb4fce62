"""Data-parallel decode scheduling with dead-worker detection and requeue.

Decode shards by independent sequences: one process per GPU runs its own
engine over batches of prompts, with no collective on the data path (the
reference runs one sequence on one device, runners/engine.py:157-181; here
that forward is replicated, not split).  The ranks share only a key-value
store -- the process group's TCPStore under torchrun, or one made by
:func:`make_store` -- through which they

* claim batches: a shared counter hands out batch indices, and the claim is
  confirmed by an atomic compare-and-set of the batch's owner key;
* publish each finished batch's result (pickled) under its own key;
* beat a per-rank counter from a background thread every ``heartbeat``
  seconds, while the rank's work runs.

A rank that has no new batch to claim watches the unfinished ones.  A batch
is taken over (its owner key moved to the watcher by compare-and-set, so
exactly one survivor wins) and run again when

* its owner's heartbeat has not moved for ``dead_after`` seconds -- the
  process exited, was killed, or never started -- or
* it has been held for more than ``batch_timeout`` seconds (a live rank
  stuck in its work), when that limit is given, or
* it was counted as claimed but has had no owner key for ``dead_after``
  seconds (a rank that died between taking the index and confirming it).

The work of a batch must be a deterministic function of its index (greedy
decode, or sampling with a per-batch seed): a batch that two ranks end up
running gives the same result twice, and whichever copy lands is kept.
Nothing here waits on a collective, so a dead rank cannot block the others;
every wait is bounded by ``timeout``.  The process that hosts the store
(rank 0) must outlive the others: it leaves only after every rank has left
or been found dead.
"""
from __future__ import annotations

import datetime
import pickle
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Sequence

import numpy as np

_jobs = 0  # schedulers made with the default prefix in this process
_jobs_lock = threading.Lock()


def _next_job_prefix() -> str:
    global _jobs
    with _jobs_lock:
        _jobs += 1
        return f"dp{_jobs}"


def make_store(host: str, port: int, rank: int, world_size: int, timeout: float = 60.0):
    """A TCPStore shared by ``world_size`` ranks (rank 0 hosts it).  The host
    does not wait for the others to connect, so a rank that never starts
    cannot hold up the rest."""
    import torch.distributed as dist
    return dist.TCPStore(host, port, world_size, is_master=(rank == 0),
                         timeout=datetime.timedelta(seconds=timeout), wait_for_workers=False)


def default_store():
    """The store of the initialised default process group (torchrun's)."""
    from torch.distributed import distributed_c10d
    return distributed_c10d._get_default_store()


@dataclass
class DPReport:
    """What one rank saw: every batch's result (when collected), the batches
    it ran, those it took over from another rank, and the ranks it found
    stalled or gone."""
    results: Dict[int, Any] = field(default_factory=dict)
    ran: List[int] = field(default_factory=list)
    taken_over: List[int] = field(default_factory=list)
    dead: List[int] = field(default_factory=list)


class DPScheduler:
    """One rank's side of the shared batch queue (see the module docstring).

    ``store``: a key-value store shared by all ranks (``add``, ``set``,
    ``get``, ``check``, ``compare_set``: a torch.distributed Store).
    ``n_batches``: batches 0 .. n_batches-1, the same count on every rank.
    ``prefix`` keeps the keys of separate jobs on one store apart; by
    default each scheduler this process makes gets the next job number
    (dp1, dp2, ..), which names the same job on every rank as long as the
    ranks make their schedulers in the same order (one SPMD program).  A
    job's keys stay in the store; a prefix must not be reused on one store.
    """

    def __init__(self, store, rank: int, world_size: int, n_batches: int, *, prefix: Optional[str] = None,
                 heartbeat: float = 0.25, dead_after: float = 5.0, batch_timeout: Optional[float] = None,
                 poll: float = 0.02, timeout: float = 600.0):
        if world_size < 1 or not 0 <= rank < world_size:
            raise ValueError(f"rank {rank} outside a world of {world_size}")
        if n_batches < 0:
            raise ValueError("n_batches must be >= 0")
        if heartbeat <= 0 or dead_after < 2 * heartbeat:
            raise ValueError("dead_after must cover at least two heartbeats")
        if batch_timeout is not None and batch_timeout <= 0:
            raise ValueError("batch_timeout must be positive")
        self.store, self.rank, self.world, self.n = store, rank, world_size, n_batches
        self.prefix = prefix if prefix is not None else _next_job_prefix()
        self.heartbeat, self.dead_after = heartbeat, dead_after
        self.batch_timeout, self.poll, self.timeout = batch_timeout, poll, timeout
        self._lock = threading.Lock()  # one request at a time on the shared client
        self._stop = threading.Event()

    # -- store access -------------------------------------------------
    def _k(self, *parts) -> str:
        return "/".join((self.prefix,) + tuple(str(p) for p in parts))

    def _add(self, key: str, n: int) -> int:
        with self._lock:
            return int(self.store.add(key, n))

    def _set(self, key: str, value) -> None:
        with self._lock:
            self.store.set(key, value)

    def _has(self, key: str) -> bool:
        with self._lock:
            return bool(self.store.check([key]))

    def _get(self, key: str) -> bytes:
        with self._lock:
            return self.store.get(key)

    def _cas(self, key: str, expected: str, desired: str) -> bool:
        """Atomically move ``key`` from ``expected`` ('' = absent) to
        ``desired``; True when this call made the move (owner values carry
        the rank, so no other rank asks for the same ``desired``)."""
        with self._lock:
            got = self.store.compare_set(key, expected, desired)
        return (got.decode() if isinstance(got, bytes) else str(got)) == desired

    # -- heartbeat ----------------------------------------------------
    def _beat(self) -> None:
        key = self._k("hb", self.rank)
        self._add(key, 1)
        while not self._stop.wait(self.heartbeat):
            try:
                self._add(key, 1)
            except Exception:  # the store is gone: the job is ending
                return

    def _run_one(self, b: int, work: Callable[[int], Any], rep: DPReport) -> None:
        result = work(b)
        self._set(self._k("res", b), pickle.dumps(result, protocol=pickle.HIGHEST_PROTOCOL))
        rep.ran.append(b)

    # -- the rank's loop ----------------------------------------------
    def run(self, work: Callable[[int], Any], collect: bool = True) -> DPReport:
        """Claim and run batches until the queue is empty, then watch the
        unfinished ones and take over those whose owner stalled, until every
        batch has a result.  Returns this rank's report; with ``collect``
        its ``results`` hold every batch's result.  An exception from
        ``work`` ends this rank (it propagates) after the rank has marked
        itself gone; the others then take its batch over."""
        rep = DPReport()
        t0 = time.monotonic()
        self._stop.clear()
        beat = threading.Thread(target=self._beat, name=f"dp-heartbeat-{self.rank}", daemon=True)
        beat.start()
        try:
            while True:  # fresh batches, in counter order
                b = self._add(self._k("next"), 1) - 1
                if b >= self.n:
                    break
                if self._cas(self._k("own", b), "", f"{self.rank}.0"):
                    self._run_one(b, work, rep)
            self._watch(work, rep, t0)
            if collect:
                rep.results = {b: pickle.loads(self._get(self._k("res", b))) for b in range(self.n)}
        finally:
            self._stop.set()
            beat.join()
            try:
                self._set(self._k("left", self.rank), "1")
                if self.rank == 0:
                    self._wait_for_others(rep, t0)
            except Exception:
                pass
        return rep

    def _refresh(self, hb: Dict[int, tuple], now: float) -> None:
        """hb[r] = (heartbeat count, local time the count last moved)."""
        for r in range(self.world):
            if r != self.rank:
                c = self._add(self._k("hb", r), 0)
                if r not in hb or hb[r][0] != c:
                    hb[r] = (c, now)

    def _watch(self, work: Callable[[int], Any], rep: DPReport, t0: float) -> None:
        pending = set(range(self.n))
        seen: Dict[int, tuple] = {}  # batch -> (owner value, local time it was first seen)
        hb: Dict[int, tuple] = {}
        while True:
            for b in list(pending):
                if self._has(self._k("res", b)):
                    pending.discard(b)
            if not pending:
                return
            now = time.monotonic()
            if now - t0 > self.timeout:
                raise TimeoutError(f"data-parallel rank {self.rank}: batches {sorted(pending)} "
                                   f"unfinished after {self.timeout} s")
            self._refresh(hb, now)
            for b in sorted(pending):
                key = self._k("own", b)
                owner = self._get(key).decode() if self._has(key) else ""
                if seen.get(b, (None,))[0] != owner:
                    seen[b] = (owner, now)
                held = now - seen[b][1]
                if owner:
                    r, gen = (int(x) for x in owner.split("."))
                    if r == self.rank:
                        continue
                    stalled = now - hb[r][1] > self.dead_after
                    stuck = self.batch_timeout is not None and held > self.batch_timeout
                    if not (stalled or stuck):
                        continue
                    desired = f"{self.rank}.{gen + 1}"
                else:  # claimed by the counter, never confirmed
                    if held <= self.dead_after:
                        continue
                    r, stalled, desired = -1, False, f"{self.rank}.1"
                if self._cas(key, owner, desired):
                    if stalled and r not in rep.dead:
                        rep.dead.append(r)
                    rep.taken_over.append(b)
                    self._run_one(b, work, rep)
                    pending.discard(b)
            time.sleep(self.poll)

    def _wait_for_others(self, rep: DPReport, t0: float) -> None:
        """Rank 0 hosts the store: stay until every other rank has left or
        its heartbeat has stopped for ``dead_after`` seconds (bounded by
        ``timeout``)."""
        hb: Dict[int, tuple] = {}
        while True:
            now = time.monotonic()
            self._refresh(hb, now)
            gone = {r for r in range(1, self.world) if self._has(self._k("left", r))}
            waiting = [r for r in range(1, self.world) if r not in gone and now - hb[r][1] <= self.dead_after]
            if not waiting or now - t0 > self.timeout:
                for r in range(1, self.world):
                    if r not in gone and r not in waiting and r not in rep.dead:
                        rep.dead.append(r)
                return
            time.sleep(self.poll)


def batch_spans(n_seqs: int, batch_size: int) -> List[tuple]:
    """[lo, hi) sequence ranges of the batches, in order."""
    if batch_size < 1:
        raise ValueError("batch_size must be >= 1")
    return [(lo, min(n_seqs, lo + batch_size)) for lo in range(0, n_seqs, batch_size)]


def generate_dp(engine, prompts: Sequence[Sequence[int]], max_new_tokens: int, store, rank: int, world_size: int,
                *, batch_size: Optional[int] = None, temperature: float = 0.0, top_k: int = 0, seed: int = 0,
                **scheduler_kw):
    """Continuations of equal-length ``prompts`` shared out over the ranks,
    each rank running ``engine.generate_batch`` on the batches it claims;
    batch b samples with seed ``seed + b``, so a batch gives the same ids
    whichever rank runs it.  Returns (int32 [n_prompts, max_new_tokens] on
    every rank, this rank's DPReport)."""
    p = np.asarray(prompts)
    if p.ndim != 2 or len(p) == 0:
        raise ValueError("prompts must be a non-empty [n, length] array of token ids")
    spans = batch_spans(len(p), batch_size or engine.max_batch)

    def work(b: int):
        lo, hi = spans[b]
        return np.asarray(engine.generate_batch(p[lo:hi], max_new_tokens, temperature, top_k, seed + b),
                          dtype=np.int32)

    rep = DPScheduler(store, rank, world_size, len(spans), **scheduler_kw).run(work)
    return np.concatenate([rep.results[b] for b in range(len(spans))]), rep
