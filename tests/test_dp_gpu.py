"""The data-parallel batch queue (llamamps_b200/dp.py) driving the real
engine on one GPU: one rank over an in-process store claims every batch of
prompts, and the ids equal the engine's own generate_batch on each batch
(greedy, and sampled with seed + batch index).  The failure cases of the
queue are host-side and covered by tests/test_dp_cpu.py."""
import dataclasses

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_generate_dp_one_rank_matches_generate_batch(cuda):
    import torch.distributed as dist
    from llamamps_b200.config import QWEN2_5_1_5B
    from llamamps_b200.dp import batch_spans, generate_dp
    from llamamps_b200.engine import QwenEngine
    from llamamps_b200.weights import synth_model
    cfg = dataclasses.replace(QWEN2_5_1_5B, n_layers=2, vocab=8192)
    eng = QwenEngine(weights=synth_model(cfg, seed=5, device="cuda"), max_batch=4, max_seq_len=64)
    prompts = np.random.default_rng(9).integers(0, cfg.vocab, (10, 7))
    for kw in (dict(), dict(temperature=0.8, top_k=20, seed=3)):
        got, rep = generate_dp(eng, prompts, 6, dist.HashStore(), 0, 1, heartbeat=0.1, dead_after=1.0, **kw)
        assert got.shape == (10, 6) and rep.ran == [0, 1, 2] and rep.dead == []
        for b, (lo, hi) in enumerate(batch_spans(10, 4)):
            want = eng.generate_batch(prompts[lo:hi], 6, kw.get("temperature", 0.0), kw.get("top_k", 0),
                                      kw.get("seed", 0) + b)
            assert np.array_equal(got[lo:hi], want), f"batch {b} {kw}"
