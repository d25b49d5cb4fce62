"""Top-k / temperature sampling (lmps_sample_rows) against its numpy
restatement (oracle.mirror.sample_top_k), and the engine's sampled decode loop
against the oracle model driven by the same draws.  The reference has no
sampling: runners/engine.py:180-181 is greedy; temperature 0 / top_k 1 is that
argmax."""
import dataclasses

import numpy as np
import pytest
import torch

from oracle import mirror as M

pytestmark = pytest.mark.gpu


def _near_boundary(logits, pick_a, pick_b, k, t, seed, offset, row, slack):
    """True when the restatement's draw falls within ``slack`` (relative to the
    total weight) of the cumulative boundary separating pick_a and pick_b."""
    _, target, z, cand, w = M.sample_top_k(logits, k, t, seed, offset, row, detail=True)
    cs = np.cumsum(w.astype(np.float64))
    pos = {int(c): i for i, c in enumerate(cand)}
    if pick_a not in pos or pick_b not in pos:
        return False
    i, j = sorted((pos[pick_a], pos[pick_b]))
    return any(abs(cs[m] - target) <= slack * z for m in range(i, j))


@pytest.mark.parametrize("n,k,t", [(151936, 40, 0.8), (151936, 1024, 1.3), (1000, 2, 1.0), (1000, 1, 0.7),
                                   (5000, 64, 0.0), (777, 777, 2.0)])
def test_sample_rows_matches_restatement(cuda, n, k, t):
    from llamamps_b200 import kernels as K
    rng = np.random.default_rng(n + k)
    rows = 3
    x = rng.normal(0, 2, (rows, n)).astype(np.float16)
    x[1, rng.integers(0, n, 20)] = np.float16(9.0)        # ties at the top of row 1
    x[2, :] = np.round(x[2, :])                             # many ties at every value of row 2
    xd = torch.from_numpy(x).cuda()
    ids = torch.zeros(rows, dtype=torch.int32, device="cuda")
    copy = torch.zeros(rows, dtype=torch.int32, device="cuda")
    mism = 0
    for offset in range(12):
        K.sample_rows(xd, n, k, t, 1234, offset, ids, copy)
        got = ids.cpu().tolist()
        assert copy.cpu().tolist() == got
        for r in range(rows):
            want = M.sample_top_k(x[r], k, t, 1234, offset, row=r)
            if got[r] != want:
                mism += 1
                assert _near_boundary(x[r], got[r], want, k, t, 1234, offset, r, 1e-5), \
                    f"row {r} offset {offset}: {got[r]} != {want}"
    assert mism <= 2


def test_sample_rows_greedy_and_reproducible(cuda):
    from llamamps_b200 import kernels as K
    x = torch.randn(4, 3000, device="cuda").half()
    x[0, 5] = x[0, 900] = 50.0                             # first index on ties
    ids = torch.zeros(4, dtype=torch.int32, device="cuda")
    K.sample_rows(x, 3000, 50, 0.0, 1, 0, ids)            # temperature 0: argmax
    want = torch.zeros(4, dtype=torch.int32, device="cuda")
    K.argmax_rows(x, 3000, want)
    assert torch.equal(ids, want) and int(ids[0]) == 5
    a = torch.zeros(4, dtype=torch.int32, device="cuda")
    b = torch.zeros(4, dtype=torch.int32, device="cuda")
    K.sample_rows(x, 3000, 50, 1.0, 77, 3, a)
    K.sample_rows(x, 3000, 50, 1.0, 77, 3, b)
    assert torch.equal(a, b)
    with pytest.raises(RuntimeError, match="argument"):
        K.sample_rows(x, 3000, 2000, 1.0, 77, 3, a)       # top_k above 1024


@pytest.mark.parametrize("decoder", ["persistent", "kernels"])
def test_sampled_generation_follows_the_oracle(cuda, decoder):
    """generate(temperature, top_k, seed) step by step against the oracle model
    fed the same draws: ids equal until a draw that the logits tolerance can
    flip (within 5e-3 of a boundary); reproducible for a seed."""
    from llamamps_b200.config import QWEN2_5_1_5B
    from llamamps_b200.engine import QwenEngine
    from llamamps_b200.weights import model_host_arrays, synth_model
    cfg = dataclasses.replace(QWEN2_5_1_5B, n_layers=2, vocab=8192)
    mw = synth_model(cfg, seed=31, device="cuda")
    host = model_host_arrays(mw)
    prompt = [11, 4000, 8191, 7]
    k, t, seed, n = 20, 1.5, 2024, 8
    eng = QwenEngine(weights=mw, max_seq_len=64, decoder=decoder)
    got = eng.generate(prompt, n, temperature=t, top_k=k, seed=seed)
    assert eng.generate(prompt, n, temperature=t, top_k=k, seed=seed) == got
    orc = M.OracleModel(host, M.OracleConfig(n_layers=2, vocab=cfg.vocab))
    lg = None
    for tok in prompt:
        lg = orc.step_token(tok)
    matched = 0
    for i in range(n):
        want = M.sample_top_k(lg, k, t, seed, i, row=0)
        if got[i] != want:
            assert _near_boundary(lg, got[i], want, k, t, seed, i, 0, 5e-3), f"step {i}: {got[i]} != {want}"
            break
        matched += 1
        lg = orc.step_token(want)
    assert matched >= 3
    greedy = eng.generate(prompt, n)
    assert greedy != got            # 8 draws among 20 candidates at T = 1.5 all equal to the argmax: vanishing odds
