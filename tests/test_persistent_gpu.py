"""The persistent decode kernel (one cooperative launch per n steps) against
the oracle, and against the per-stage kernel path."""
import dataclasses

import numpy as np
import pytest
import torch

from oracle import mirror as M
from tests._util import assert_close, greedy_ids_match

pytestmark = pytest.mark.gpu


def _engine(mw, **kw):
    from llamamps_b200.engine import QwenEngine
    return QwenEngine(weights=mw, **kw)


def test_persistent_one_layer_decode_step(cuda):
    """One layer, one step, 31 cached positions, new token at position 31:
    logits and the appended k/v against the oracle."""
    from llamamps_b200.config import QWEN2_5_1_5B as cfg
    from llamamps_b200.quant import pack_q4
    from llamamps_b200.weights import ModelWeights, layer_from_parts, parts_host_arrays, synth_one_layer_case
    parts, x, kp, vp = synth_one_layer_case(cfg, seed=0, prefix=31)
    small = dataclasses.replace(cfg, vocab=512, n_layers=1)
    lw = layer_from_parts(small, {k: torch.from_numpy(v) for k, v in parts.items()}, "cuda")
    rng = np.random.default_rng(9)
    embed = torch.from_numpy(rng.normal(0, 0.02, (512, cfg.hidden)).astype(np.float16)).cuda()
    fnorm = torch.from_numpy((1 + rng.normal(0, 0.02, cfg.hidden)).astype(np.float16)).cuda()
    lp, ls = pack_q4(embed.float())
    mw = ModelWeights(small, [lw], fnorm, lp, ls, embed)
    eng = _engine(mw, max_seq_len=128, decoder="persistent")
    eng.reset(1, start_pos=31)
    eng.cache.write_positions(0, 0, 0, torch.from_numpy(kp), torch.from_numpy(vp))
    logits = eng.run_inference(x)

    ocfg = M.OracleConfig(n_layers=1, vocab=512)
    cache = M.KVCache(1, ocfg.kv_dim)
    cache.set_prefix(0, kp, vp)
    tr = {}
    hl = parts_host_arrays(parts)
    x2 = M.decoder_layer(x, hl, cache, 0, 31, ocfg, trace=tr)
    ref = M.final_logits(x2, fnorm.cpu().numpy(), lp.cpu().numpy(), ls.cpu().numpy(), ocfg)
    assert_close(logits, ref, what="one-layer logits")
    kk, vv = eng.cache.read_positions(0, 0, 32)
    assert_close(kk[-1].cpu().numpy(), tr["k"], what="appended k")
    assert_close(vv[-1].cpu().numpy(), tr["v"], what="appended v")
    assert_close(kk[:31].cpu().numpy(), kp, abs_tol=0, what="untouched prefix")
    assert int(eng.pos[0].item()) == 32


@pytest.fixture(scope="module")
def two_layer_small_vocab():
    from llamamps_b200.config import QWEN2_5_1_5B
    from llamamps_b200.weights import model_host_arrays, synth_model
    cfg = dataclasses.replace(QWEN2_5_1_5B, n_layers=2, vocab=8192)
    mw = synth_model(cfg, seed=5, device="cuda")
    return cfg, mw, model_host_arrays(mw)


@pytest.mark.parametrize("prompt_len", [1, 7, 300])
def test_persistent_generate_matches_oracle(cuda, two_layer_small_vocab, prompt_len):
    """prompt_len 300 puts several 64-position splits per KV head in play, so
    the last-arriver log-sum-exp merge runs."""
    cfg, mw, host = two_layer_small_vocab
    prompt = np.random.default_rng(prompt_len).integers(0, cfg.vocab, prompt_len)
    eng = _engine(mw, max_seq_len=512, decoder="persistent")
    got = eng.generate(prompt.tolist(), 6)
    rec = []
    ref = M.OracleModel(host, M.OracleConfig(n_layers=2, vocab=cfg.vocab)).generate(prompt.tolist(), 6, record=rec)
    n = greedy_ids_match(got, ref, rec)
    assert n >= 3


def test_persistent_logits_track_oracle_over_steps(cuda, two_layer_small_vocab):
    cfg, mw, host = two_layer_small_vocab
    eng = _engine(mw, max_seq_len=256, decoder="persistent")
    orc = M.OracleModel(host, M.OracleConfig(n_layers=2, vocab=cfg.vocab))
    for tok in (5, 8191, 17, 17, 4000):
        lg = eng.run_inference(host["embed"][tok])
        ref = orc.step_vector(host["embed"][tok])
        assert_close(lg, ref, what=f"logits at pos {orc.pos - 1}")


def test_persistent_batch_agrees_with_kernel_path(cuda, two_layer_small_vocab):
    cfg, mw, host = two_layer_small_vocab
    prompts = np.random.default_rng(3).integers(0, cfg.vocab, (4, 9))
    pers = _engine(mw, max_batch=4, max_seq_len=128, decoder="persistent").generate_batch(prompts, 6)
    kern = _engine(mw, max_batch=4, max_seq_len=128, decoder="kernels").generate_batch(prompts, 6)
    for b in range(4):
        rec = []
        ref = M.OracleModel(host, M.OracleConfig(n_layers=2, vocab=cfg.vocab)).generate(
            prompts[b].tolist(), 6, record=rec)
        assert greedy_ids_match(pers[b].tolist(), ref, rec) >= 3
        assert greedy_ids_match(kern[b].tolist(), ref, rec) >= 3


def test_persistent_multi_step_launch_equals_single_steps(cuda, two_layer_small_vocab):
    cfg, mw, _ = two_layer_small_vocab
    prompts = np.random.default_rng(4).integers(0, cfg.vocab, (2, 5))
    a = _engine(mw, max_batch=2, max_seq_len=128, decoder="persistent")
    a.reset(2)
    a.prefill(torch.from_numpy(prompts))
    a.decode_steps(6)
    b = _engine(mw, max_batch=2, max_seq_len=128, decoder="persistent")
    b.reset(2)
    b.prefill(torch.from_numpy(prompts))
    for _ in range(6):
        b.decode_steps(1)
    torch.cuda.synchronize()
    assert torch.equal(a.history[:7].flatten()[:14], b.history[:7].flatten()[:14])
    assert torch.equal(a.tokens, b.tokens) and torch.equal(a.pos, b.pos)


def test_persistent_rejects_positions_past_the_cache(cuda, two_layer_small_vocab):
    """The device-side guard: nothing runs, error code 2, workspace reset."""
    cfg, mw, _ = two_layer_small_vocab
    eng = _engine(mw, max_seq_len=64, decoder="persistent")
    eng.reset(1, start_pos=63)
    eng.tokens.fill_(3)
    eng.pdec.run(1, eng.tokens, eng.pos, 2)      # 63 + 2 > 64
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="past the KV cache"):
        eng.pdec.check_error()
    eng.pos.fill_(0)
    eng.pdec.run(1, eng.tokens, eng.pos, 1)       # usable again afterwards
    torch.cuda.synchronize()
    eng.pdec.check_error()
    assert int(eng.pos[0].item()) == 1


@pytest.mark.parametrize("B", [2, 3, 4])
def test_persistent_batch_logits_match_single_sequence(cuda, two_layer_small_vocab, B):
    """Each sequence of a batch must produce (within tolerance) the logits it
    produces alone, and the oracle's, after a short prompt."""
    cfg, mw, host = two_layer_small_vocab
    rng = np.random.default_rng(40 + B)
    prompts = rng.integers(0, cfg.vocab, (B, 5))
    eng = _engine(mw, max_batch=4, max_seq_len=64, decoder="persistent")
    logits = torch.zeros(4, cfg.vocab, dtype=torch.float16, device="cuda")

    def run(ps):
        n = ps.shape[0]
        eng.reset(n)
        eng.tokens[:n].copy_(torch.from_numpy(ps[:, 0]).to(torch.int32))
        forced = torch.from_numpy(ps[:, 1:]).to("cuda", torch.int32).contiguous()
        eng.pdec.run(n, eng.tokens, eng.pos, ps.shape[1], forced=forced, logits=logits[:n])
        torch.cuda.synchronize()
        eng.pdec.check_error()
        return logits[:n].cpu().numpy().copy()

    batched = run(prompts)
    for b in range(B):
        single = run(prompts[b:b + 1])[0]
        assert_close(batched[b], single, what=f"seq {b} batched vs alone")
        orc = M.OracleModel(host, M.OracleConfig(n_layers=2, vocab=cfg.vocab))
        ref = None
        for t in prompts[b]:
            ref = orc.step_token(int(t))
        assert_close(batched[b], ref, what=f"seq {b} vs oracle")


@pytest.mark.parametrize("B,lens,max_seq", [(1, [20000], 32768), (4, [3000, 2500, 3100, 2050], 4096)])
def test_persistent_long_context_matches_oracle(cuda, two_layer_small_vocab, B, lens, max_seq):
    """Cached contexts of thousands of positions (fp16 N(0,1) rows written
    into the paged cache), so the persistent kernel takes its long-cache path:
    positions split across CTAs in chunks, the second per-warp K buffer of the
    flash loop (cache > 2048 positions) and the last-split log-sum-exp merge.
    Logits of five single-step launches and of one three-step launch against
    the oracle holding the same cache prefix (runners/engine.py:157-181,
    kernels/attention.metal:22-40, softmax.metal:23-36, attn_sum.metal:22-33)."""
    cfg, mw, host = two_layer_small_vocab
    eng = _engine(mw, max_batch=4, max_seq_len=max_seq, decoder="persistent")
    eng.reset(B)
    rng = np.random.default_rng(60 + B)
    orcs = []
    for b in range(B):
        orc = M.OracleModel(host, M.OracleConfig(n_layers=2, vocab=cfg.vocab))
        for layer in range(2):
            k = rng.normal(0, 1, (lens[b], cfg.kv_dim)).astype(np.float16)
            v = rng.normal(0, 1, (lens[b], cfg.kv_dim)).astype(np.float16)
            eng.cache.write_positions(b, layer, 0, torch.from_numpy(k), torch.from_numpy(v))
            orc.cache.set_prefix(layer, k, v)
        orc.pos = lens[b]
        orcs.append(orc)
    eng.pos[:B].copy_(torch.tensor(lens, dtype=torch.int32))
    logits = torch.zeros(B, cfg.vocab, dtype=torch.float16, device="cuda")
    toks = rng.integers(0, cfg.vocab, (B, 8))
    for s in range(5):
        eng.tokens[:B].copy_(torch.from_numpy(toks[:, s]).to(torch.int32))
        eng.pdec.run(B, eng.tokens, eng.pos, 1, logits=logits)
        torch.cuda.synchronize()
        eng.pdec.check_error()
        got = logits.cpu().numpy()
        for b in range(B):
            assert_close(got[b], orcs[b].step_token(int(toks[b, s])), what=f"seq {b} step {s}")
    # three steps in one launch, the fed tokens forced: logits of the last one
    eng.tokens[:B].copy_(torch.from_numpy(toks[:, 5]).to(torch.int32))
    forced = torch.from_numpy(toks[:, 6:8]).to("cuda", torch.int32).contiguous()
    eng.pdec.run(B, eng.tokens, eng.pos, 3, forced=forced, logits=logits)
    torch.cuda.synchronize()
    eng.pdec.check_error()
    got = logits.cpu().numpy()
    for b in range(B):
        ref = None
        for s in range(5, 8):
            ref = orcs[b].step_token(int(toks[b, s]))
        assert_close(got[b], ref, what=f"seq {b} after a three-step launch")
    assert eng.pos[:B].cpu().tolist() == [n + 8 for n in lens]
