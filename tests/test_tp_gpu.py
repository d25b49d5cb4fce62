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


def _rank(rank, world, port, out, dense):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from llamamps_b200.tp import TPEngine, init_from_env
    from llamamps_b200.weights import synth_model
    init_from_env("nccl", timeout_s=60)
    try:
        mw = synth_model(_cfg(), seed=17, device=f"cuda:{rank}")
        prompts = np.random.default_rng(PROMPT_SEED).integers(0, 8192, (2, 150 if dense else 9))
        eng = TPEngine(mw, rank, world, max_batch=2, max_seq_len=256, device=f"cuda:{rank}")
        got = eng.generate_batch(prompts, STEPS)
        out[rank] = got.tolist()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("dense", [False, True])
def test_tp2_generate_matches_oracle(cuda, dense):
    import torch.multiprocessing as mp
    from llamamps_b200.weights import model_host_arrays, synth_model
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out, dense)) for r in range(2)]
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
