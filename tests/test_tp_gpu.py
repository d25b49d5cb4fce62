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
    shapes of a 2-way split against GEMV, NCCL sum, residual_add."""
    _env(rank, world, port)
    import torch.distributed as dist
    from llamamps_b200 import kernels as K
    from llamamps_b200.tp import init_from_env
    init_from_env("nccl", timeout_s=60)
    dev = torch.device(f"cuda:{rank}")
    ex = K.PeerExchange(5, 8 * 1536, dev)
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
