"""Data-parallel batch queue with dead-worker detection (llamamps_b200/dp.py),
run as separate CPU processes sharing one TCPStore.  Failures are made on
the host, never on a GPU: a rank that exits in the middle of a batch, a rank
whose work raises, a rank that never starts, and a live rank stuck in one
batch.  Every batch's result must arrive on the surviving ranks, equal to
the work function's answer, and the batch of the failed rank must be run
again by exactly one survivor.  The work stands in for a rank's engine
(generate_batch on the batch's prompts): a deterministic function of the
batch index, as the scheduler requires."""
import hashlib
import os
import pickle
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

N_BATCHES = 9
FAST = dict(heartbeat=0.1, dead_after=1.0, poll=0.01, timeout=60.0)


def _ids(b: int) -> np.ndarray:
    """The batch's 'generated ids': 4 sequences x 6 tokens from its index."""
    h = hashlib.sha256(f"batch {b}".encode()).digest()
    return np.frombuffer(h[:24], dtype=np.uint8).astype(np.int32).reshape(4, 6)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, fail, out_dir, kw):
    """One rank: meet the others at a start line (so every rank is live
    before the queue opens), then run the queue.  ``fail`` = (rank, how)."""
    from llamamps_b200.dp import DPScheduler, make_store
    store = make_store("127.0.0.1", port, rank, world, timeout=30.0)
    store.add("start", 1)
    t = time.monotonic()
    while int(store.add("start", 0)) < world - (1 if fail and fail[1] == "never" else 0):
        if time.monotonic() - t > 30:
            raise TimeoutError("ranks did not meet")
        time.sleep(0.01)
    first = [True]

    def work(b):
        time.sleep(0.15)  # long enough that every rank takes a batch
        if fail and fail[0] == rank and first[0]:
            first[0] = False
            if fail[1] == "exit":
                os._exit(3)  # killed mid-batch: no cleanup, heartbeat stops
            if fail[1] == "raise":
                raise RuntimeError("worker failure")
            if fail[1] == "stuck":
                time.sleep(3.0)  # alive (heartbeat beats) but far past batch_timeout
        return _ids(b)

    sched = DPScheduler(store, rank, world, N_BATCHES, **kw)
    try:
        rep = sched.run(work)
    except RuntimeError as e:
        rep = str(e)
    with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
        pickle.dump(rep, f)


def _launch(tmp_path, world, fail=None, extra=None):
    kw = dict(FAST, **(extra or {}))
    ctx = mp.get_context("spawn")
    port = _free_port()
    started = [r for r in range(world) if not (fail and fail[1] == "never" and fail[0] == r)]
    procs = {r: ctx.Process(target=_rank, args=(r, world, port, fail, str(tmp_path), kw)) for r in started}
    # the store's host first, so the others connect to it
    procs[0].start()
    for r in started[1:]:
        procs[r].start()
    codes = {}
    for r, p in procs.items():
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            p.join()
        codes[r] = p.exitcode
    reps = {}
    for r in started:
        path = tmp_path / f"rank{r}.pkl"
        if path.exists():
            with open(path, "rb") as f:
                reps[r] = pickle.load(f)
    return codes, reps


def _check_results(rep):
    assert sorted(rep.results) == list(range(N_BATCHES))
    for b in range(N_BATCHES):
        assert np.array_equal(rep.results[b], _ids(b)), f"batch {b}"


def test_all_ranks_alive_each_batch_runs_once(tmp_path):
    codes, reps = _launch(tmp_path, 3)
    assert codes == {0: 0, 1: 0, 2: 0}
    ran = []
    for r in range(3):
        _check_results(reps[r])
        assert reps[r].taken_over == [] and reps[r].dead == []
        ran += reps[r].ran
    assert sorted(ran) == list(range(N_BATCHES))


def test_rank_killed_mid_batch_is_requeued(tmp_path):
    codes, reps = _launch(tmp_path, 3, fail=(2, "exit"))
    assert codes[2] == 3 and codes[0] == 0 and codes[1] == 0
    assert 2 not in reps
    taken = reps[0].taken_over + reps[1].taken_over
    assert len(taken) == 1, "the dead rank's batch runs again on exactly one survivor"
    assert any(2 in reps[r].dead for r in (0, 1))
    for r in (0, 1):
        _check_results(reps[r])
    assert sorted(reps[0].ran + reps[1].ran) == list(range(N_BATCHES))


def test_rank_whose_work_raises_is_requeued(tmp_path):
    codes, reps = _launch(tmp_path, 3, fail=(1, "raise"))
    assert all(c == 0 for c in codes.values())
    assert reps[1] == "worker failure"
    assert len(reps[0].taken_over + reps[2].taken_over) == 1
    for r in (0, 2):
        _check_results(reps[r])


def test_rank_that_never_starts(tmp_path):
    codes, reps = _launch(tmp_path, 3, fail=(2, "never"))
    assert codes == {0: 0, 1: 0}
    for r in (0, 1):
        _check_results(reps[r])
        assert reps[r].taken_over == []
    assert 2 in reps[0].dead  # rank 0 stops waiting for it once its heartbeat never moves


def test_stuck_rank_batch_is_run_again(tmp_path):
    """A live rank held in one batch past batch_timeout: a survivor runs that
    batch too; both copies are the same, and the stuck rank still finishes."""
    codes, reps = _launch(tmp_path, 2, fail=(1, "stuck"), extra=dict(batch_timeout=1.0))
    assert codes == {0: 0, 1: 0}
    assert len(reps[0].taken_over) == 1 and reps[0].dead == []
    for r in (0, 1):
        _check_results(reps[r])


def test_single_rank_in_process_store():
    import torch.distributed as dist
    from llamamps_b200.dp import DPScheduler
    rep = DPScheduler(dist.HashStore(), 0, 1, 5, **FAST).run(_ids)
    assert rep.ran == [0, 1, 2, 3, 4]
    _check_results_n(rep, 5)


def _check_results_n(rep, n):
    assert sorted(rep.results) == list(range(n))
    for b in range(n):
        assert np.array_equal(rep.results[b], _ids(b))


def test_argument_checks_and_spans():
    import torch.distributed as dist
    from llamamps_b200.dp import DPScheduler, batch_spans
    assert batch_spans(10, 4) == [(0, 4), (4, 8), (8, 10)]
    assert batch_spans(0, 4) == []
    with pytest.raises(ValueError):
        batch_spans(3, 0)
    s = dist.HashStore()
    with pytest.raises(ValueError):
        DPScheduler(s, 2, 2, 1)
    with pytest.raises(ValueError):
        DPScheduler(s, 0, 1, -1)
    with pytest.raises(ValueError):
        DPScheduler(s, 0, 1, 1, heartbeat=1.0, dead_after=1.5)
    with pytest.raises(ValueError):
        DPScheduler(s, 0, 1, 1, batch_timeout=0)
    assert DPScheduler(s, 0, 1, 0, **FAST).run(_ids).results == {}


class _FakeEngine:
    """Stands in for QwenEngine.generate_batch: ids from the prompts and the seed."""
    max_batch = 3

    def __init__(self):
        self.calls = []

    def generate_batch(self, prompts, n, temperature, top_k, seed):
        self.calls.append((len(prompts), seed))
        p = np.asarray(prompts)
        return (p[:, :1] * 1000 + np.arange(n)[None] + seed * 100).astype(np.int32)


def test_generate_dp_batches_seeds_and_order():
    """Prompts split into engine.max_batch rows per batch, batch b sampled
    with seed + b, the rows put back in prompt order."""
    import torch.distributed as dist
    from llamamps_b200.dp import generate_dp
    eng = _FakeEngine()
    prompts = np.arange(8)[:, None] * np.ones((1, 5), dtype=np.int64)
    got, rep = generate_dp(eng, prompts, 4, dist.HashStore(), 0, 1, seed=7, **FAST)
    assert eng.calls == [(3, 7), (3, 8), (2, 9)]
    want = np.concatenate([_FakeEngine().generate_batch(prompts[lo:hi], 4, 0.0, 0, 7 + b)
                           for b, (lo, hi) in enumerate([(0, 3), (3, 6), (6, 8)])])
    assert np.array_equal(got, want) and got.shape == (8, 4)
    assert rep.ran == [0, 1, 2]
    with pytest.raises(ValueError):
        generate_dp(eng, np.zeros((0, 4)), 4, dist.HashStore(), 0, 1, **FAST)


def test_consecutive_jobs_on_one_store_do_not_mix():
    """Two jobs on the same store (as under one torchrun process group): the
    second gets its own keys, so it runs its own batches instead of finding
    the first job's counter and results."""
    import torch.distributed as dist
    from llamamps_b200.dp import DPScheduler
    store = dist.HashStore()
    a = DPScheduler(store, 0, 1, 3, **FAST).run(_ids)
    b = DPScheduler(store, 0, 1, 4, **FAST).run(lambda i: _ids(i + 10))
    assert a.ran == [0, 1, 2] and b.ran == [0, 1, 2, 3]
    for i in range(4):
        assert np.array_equal(b.results[i], _ids(i + 10))
