"""Two-way tensor-parallel decode on two GPUs (NCCL all-reduce over NVLink):
greedy ids against the oracle and against the single-GPU engine.  Skipped on
boxes with fewer than two GPUs."""
import dataclasses
import os
import socket

import numpy as np
import pytest
import torch

from oracle import mirror as M
from tests._util import greedy_ids_match

pytestmark = pytest.mark.gpu

PROMPT_SEED, STEPS = 41, 6


def _cfg():
    from llamamps_b200.config import QWEN2_5_1_5B
    return dataclasses.replace(QWEN2_5_1_5B, n_layers=2, vocab=8192)


def _env(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")


def _rank(rank, world, port, out, dense, comm):
    _env(rank, world, port)
    import torch.distributed as dist
    from llamamps_b200.tp import TPEngine, init_from_env
    from llamamps_b200.weights import synth_model
    init_from_env("nccl", timeout_s=60)
    try:
        mw = synth_model(_cfg(), seed=17, device=f"cuda:{rank}")
        prompts = np.random.default_rng(PROMPT_SEED).integers(0, 8192, (2, 150 if dense else 9))
        eng = TPEngine(mw, rank, world, max_batch=2, max_seq_len=256, device=f"cuda:{rank}",
                       comm="nccl" if comm == "nccl" else "p2p", fuse_exchange=comm == "p2p_fused")
        try:
            got = eng.generate_batch(prompts, STEPS)
            out[rank] = got.tolist()
        finally:
            eng.close()
    finally:
        dist.destroy_process_group()


def _exchange_rank(rank, world, port, out):
    """Peer-memory all-reduce + residual against NCCL's sum + residual_add:
    several sites, back-to-back calls on one site, 1 to 8 rows; and the fused
    GEMV + exchange at the o_proj (1536 x 768) and down_proj (1536 x 4480)
    shapes of a 2-way split against GEMV, NCCL sum, residual_add; and the
    split-vocabulary argmax exchange against the argmax of the whole rows."""
    _env(rank, world, port)
    import torch.distributed as dist
    from llamamps_b200 import kernels as K
    from llamamps_b200.tp import init_from_env
    init_from_env("nccl", timeout_s=60)
    dev = torch.device(f"cuda:{rank}")
    ex = K.PeerExchange(6, 8 * 1536, dev)
    try:
        handles = [None] * world
        dist.all_gather_object(handles, ex.handle())
        ex.connect(handles[1 - rank])
        dist.barrier()
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        xg = torch.Generator(device=dev).manual_seed(7)       # same residual on both ranks
        mism = 0
        for site, rows in [(0, 1), (1, 8), (0, 1), (0, 8), (0, 8), (2, 3), (1, 1), (0, 1)]:
            part = (torch.randn(rows, 1536, generator=g, device=dev) * 4).half()
            x = torch.randn(rows, 1536, generator=xg, device=dev).half()
            ref = part.clone()
            dist.all_reduce(ref)
            ref = K.residual_add(x.clone(), ref, out=torch.empty_like(x))
            K.tp2_allreduce_residual(part, x, ex, site, err)
            torch.cuda.synchronize(dev)
            mism += int((x.view(torch.int16) != ref.view(torch.int16)).sum().item())
        wg = torch.Generator(device=dev).manual_seed(300 + rank)   # each rank its own K slice
        mats = {k: (torch.randint(0, 256, (1536 * k // 2,), generator=wg, device=dev, dtype=torch.uint8),
                    (torch.rand(1536 * k // 32, generator=wg, device=dev) * 0.04 + 0.005).half())
                for k in (768, 4480)}
        part = torch.empty(8 * 1536, dtype=torch.float16, device=dev)
        for site, k, rows in [(3, 768, 1), (4, 4480, 1), (3, 768, 8), (3, 768, 8), (4, 4480, 5), (3, 768, 2)]:
            packed, scales = mats[k]
            a = torch.randn(rows, k, generator=g, device=dev).half()
            x = torch.randn(rows, 1536, generator=xg, device=dev).half()
            ref = K.gemv_q4(packed, scales, a, 1536, k)
            dist.all_reduce(ref)
            ref = K.residual_add(x.clone(), ref, out=torch.empty_like(x))
            K.gemv_q4_tp2_residual(packed, scales, a, 1536, k, x, part[:rows * 1536].view(rows, 1536), ex, site, err)
            torch.cuda.synchronize(dev)
            mism += int((x.view(torch.int16) != ref.view(torch.int16)).sum().item())
        # split-vocabulary argmax: each rank's half of 3 rows of logits,
        # ties inside a half and across the halves (the lower global row wins)
        vg = torch.Generator(device=dev).manual_seed(11)   # same full rows on both ranks
        full = torch.randn(3, 2000, generator=vg, device=dev).half()
        full[1, 1500] = full[1, 400] = 30.0                 # cross-half tie: 400 wins
        full[2, 1200] = full[2, 1700] = 25.0                # tie inside rank 1's half: 1200 wins
        want = torch.zeros(3, dtype=torch.int32, device=dev)
        K.argmax_rows(full, 2000, want)
        half = full[:, rank * 1000:(rank + 1) * 1000].contiguous()
        local = torch.zeros(3, dtype=torch.int32, device=dev)
        K.argmax_rows(half, 1000, local)
        ids = torch.zeros(3, dtype=torch.int32, device=dev)
        for _ in range(2):                                  # back-to-back calls on the site
            K.tp2_argmax_exchange(half, local, rank * 1000, ids, ex, 5, err)
            torch.cuda.synchronize(dev)
            mism += int((ids != want).sum().item())
        assert want.tolist()[1] == 400 and want.tolist()[2] == 1200
        out[rank] = (mism, int(err.item()))
        torch.cuda.synchronize(dev)
        dist.barrier()
    finally:
        ex.close()
        dist.barrier()
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(target, *args):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, 2, port, out) + args) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    return out


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_peer_allreduce_equals_nccl(cuda):
    out = _spawn(_exchange_rank)
    assert out[0] == (0, 0) and out[1] == (0, 0), dict(out)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("dense,comm", [(False, "p2p"), (True, "p2p"), (False, "p2p_fused"), (False, "nccl")])
def test_tp2_generate_matches_oracle(cuda, dense, comm):
    import torch.multiprocessing as mp
    from llamamps_b200.weights import model_host_arrays, synth_model
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out, dense, comm)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    assert out[0] == out[1], "ranks produced different tokens"
    cfg = _cfg()
    host = model_host_arrays(synth_model(cfg, seed=17, device="cuda:0"))
    prompts = np.random.default_rng(PROMPT_SEED).integers(0, 8192, (2, 150 if dense else 9))
    for b in range(2):
        rec = []
        ref = M.OracleModel(host, M.OracleConfig(n_layers=2, vocab=8192)).generate(prompts[b].tolist(), STEPS,
                                                                                 record=rec)
        assert greedy_ids_match(out[0][b], ref, rec) >= 3, f"sequence {b}"


WAIT_NS = 50_000_000   # 50 ms: the exchange's bounded wait, shortened so a missing peer shows up quickly


def test_tp2_wait_runs_out_without_a_peer(cuda):
    """Failure detection of the peer exchange on one GPU: a second local
    buffer stands in for the peer's, so the flags this rank waits for are
    never written.  Each kernel's bounded wait must run out (no trap, no
    hang): the error word reads 1, x is left as it was, and a later call on
    any site returns at once because the error word is set.  The engine-level
    check then raises.  Same for the fused GEMV exchange."""
    import time
    import types
    from llamamps_b200 import kernels as K
    from llamamps_b200.tp import TPEngine
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(3)
    for kind in ("exchange", "fused", "argmax"):
        fused = kind == "fused"
        ex = K.PeerExchange(4, 8 * 1536, dev, wait_ns=WAIT_NS)
        stand_in = K.PeerExchange(4, 8 * 1536, dev)
        ex.peer = stand_in.comm            # flags this rank publishes land here; nothing answers
        try:
            err = torch.zeros(1, dtype=torch.int32, device=dev)
            x = torch.randn(2, 1536, generator=g, device=dev).half()
            x0 = x.clone()
            part = torch.empty(2, 1536, dtype=torch.float16, device=dev)
            packed = torch.randint(0, 256, (1536 * 768 // 2,), generator=g, device=dev, dtype=torch.uint8)
            scales = (torch.rand(1536 * 768 // 32, generator=g, device=dev) * 0.04 + 0.005).half()
            a = torch.randn(2, 768, generator=g, device=dev).half()

            lg = torch.randn(2, 1000, generator=g, device=dev).half()
            local = torch.tensor([3, 999], dtype=torch.int32, device=dev)
            ids = torch.full((2,), -7, dtype=torch.int32, device=dev)

            def one(site):
                if kind == "argmax":
                    K.tp2_argmax_exchange(lg, local, 1000, ids, ex, site, err)
                elif fused:
                    K.gemv_q4_tp2_residual(packed, scales, a, 1536, 768, x, part, ex, site, err)
                else:
                    K.tp2_allreduce_residual(torch.randn(2, 1536, generator=g, device=dev).half(), x, ex, site, err)
                torch.cuda.synchronize(dev)

            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            one(0)
            waited = time.perf_counter() - t0
            assert int(err.item()) == 1, "the wait did not report the missing peer"
            assert torch.equal(x, x0), "x changed although the exchange failed"
            assert ids.tolist() == [-7, -7], "ids written although the exchange failed"
            assert 0.04 <= waited < 3.0, f"first call took {waited:.3f} s"
            t0 = time.perf_counter()
            one(1)
            assert time.perf_counter() - t0 < 0.03, "a call after the error still waited"
            assert int(err.item()) == 1 and torch.equal(x, x0)
            if kind == "exchange":
                # the engine-level check raises on the device error word
                stub = types.SimpleNamespace(exchange=ex, comm_err=err)
                with pytest.raises(RuntimeError, match="timed out"):
                    TPEngine.check_comm(stub)
        finally:
            torch.cuda.synchronize(dev)
            ex.peer = None                  # not an IPC mapping: nothing to unmap
            ex.close()
            stand_in.close()


def _skip_rank(rank, world, port, out):
    """Rank 1 skips the second exchange call: rank 0's bounded wait for it
    runs out and reports through its error word; rank 1 saw nothing wrong.
    No kernel of either rank is in flight when the ranks meet again."""
    _env(rank, world, port)
    import torch.distributed as dist
    from llamamps_b200 import kernels as K
    from llamamps_b200.tp import init_from_env
    init_from_env("nccl", timeout_s=60)
    dev = torch.device(f"cuda:{rank}")
    ex = K.PeerExchange(2, 1536, dev, wait_ns=WAIT_NS)
    try:
        handles = [None] * world
        dist.all_gather_object(handles, ex.handle())
        ex.connect(handles[1 - rank])
        dist.barrier()
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        x = torch.ones(1, 1536, dtype=torch.float16, device=dev)
        part = torch.full((1, 1536), 0.5, dtype=torch.float16, device=dev)
        K.tp2_allreduce_residual(part, x, ex, 0, err)        # both ranks: 1 + (0.5 + 0.5)
        torch.cuda.synchronize(dev)
        first = (int(err.item()), float(x[0, 0].item()))
        dist.barrier()
        if rank == 0:
            K.tp2_allreduce_residual(part, x, ex, 0, err)    # the peer never makes this call
            torch.cuda.synchronize(dev)
        out[rank] = first + (int(err.item()), float(x[0, 0].item()))
        dist.barrier()
    finally:
        torch.cuda.synchronize(dev)
        ex.close()
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_missing_peer_call_times_out(cuda):
    out = _spawn(_skip_rank)
    assert out[0] == (0, 2.0, 1, 2.0), dict(out)     # wait ran out, x untouched by the failed call
    assert out[1] == (0, 2.0, 0, 2.0), dict(out)
