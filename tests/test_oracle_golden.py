"""The oracle against the reference's own outputs (tests/golden/*.npz, made by
tests/golden/make_golden.py from utils/pack_weights.py, utils/verify_attention.py
and utils/verify_swiglu.py), plus the oracle's reductions to the reference at
position 0 / one cached token."""
import os

import numpy as np
import pytest
import torch

from oracle import mirror as M
from tests._util import assert_close, f16_bits_equal

GOLD = os.path.join(os.path.dirname(__file__), "golden")
PACK_CASES = ["normal_64x96", "odd_7x33", "kproj_64x1536", "edge_4x32"]


@pytest.fixture(scope="module")
def pack_gold():
    return np.load(os.path.join(GOLD, "pack_cases.npz"))


@pytest.fixture(scope="module")
def verify_gold():
    return np.load(os.path.join(GOLD, "verify_cases.npz"))


@pytest.mark.parametrize("name", PACK_CASES)
def test_oracle_pack_matches_reference_bit_exact(pack_gold, name):
    p, s = M.q4_pack(pack_gold[name + "__w"])
    assert np.array_equal(p, pack_gold[name + "__packed"])
    assert f16_bits_equal(s, pack_gold[name + "__scales"])


@pytest.mark.parametrize("name", PACK_CASES)
def test_host_packer_matches_reference_bit_exact(pack_gold, name):
    from llamamps_b200.quant import pack_q4_host
    p, s = pack_q4_host(torch.from_numpy(pack_gold[name + "__w"]))
    assert np.array_equal(p.numpy(), pack_gold[name + "__packed"])
    assert f16_bits_equal(s.numpy(), pack_gold[name + "__scales"])


def test_unpack_roundtrip_codes(pack_gold):
    w = pack_gold["edge_4x32__w"]
    p, s = M.q4_pack(w)
    codes = M.q4_codes(p)
    # ties group: scale 1.0, half-way values round to even
    assert list(codes[:16]) == [7, 0, 2, 2, 0, -2, -2, 4, -4, 4, 6, 6, -6, 0, 0, 7]
    assert np.all(codes[32:64] == 0) and s[1] == np.float16(1.0)     # dead group
    assert codes.min() >= -8 and codes.max() <= 7


@pytest.mark.parametrize("i", range(3))
def test_oracle_scores_match_verify_attention(verify_gold, i):
    s = M.attention_scores(verify_gold[f"attn{i}__q"], verify_gold[f"attn{i}__k"][None])[:, 0]
    np.testing.assert_allclose(s, verify_gold[f"attn{i}__scores"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("i", range(2))
def test_oracle_swiglu_matches_verify_swiglu(verify_gold, i):
    o = M.swiglu(verify_gold[f"swiglu{i}__gate"], verify_gold[f"swiglu{i}__up"])
    assert f16_bits_equal(o, verify_gold[f"swiglu{i}__out"])


def test_rope_is_identity_at_position_zero():
    rng = np.random.default_rng(1)
    v = rng.normal(0, 1, 1536).astype(np.float16)
    for theta in (1e4, 1e6):
        for style in ("interleaved", "neox"):
            assert f16_bits_equal(M.rope(v, 0, 128, theta, style), v)


def test_single_position_attention_broadcasts_v():
    """engine.py:64 seq_len=1: softmax of one score is 1, output = V per group."""
    rng = np.random.default_rng(2)
    q = rng.normal(0, 1, 1536).astype(np.float16)
    k = rng.normal(0, 1, (1, 256)).astype(np.float16)
    v = rng.normal(0, 1, (1, 256)).astype(np.float16)
    p = M.softmax(M.attention_scores(q, k))
    assert np.all(p == 1.0)
    o = M.attn_weighted_sum(p, v)
    assert f16_bits_equal(o, np.concatenate([v[0, :128]] * 6 + [v[0, 128:]] * 6))


def test_rms_norm_matches_definition():
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, (2, 1536)).astype(np.float16)
    g = (1 + rng.normal(0, 0.02, 1536)).astype(np.float16)
    out = M.rms_norm(x, g)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt((x64 ** 2).mean(-1, keepdims=True) + 1e-6) * g.astype(np.float64)
    np.testing.assert_allclose(out.astype(np.float64), ref, rtol=2e-3, atol=2e-3)


def test_gemv_dequant_semantics():
    rng = np.random.default_rng(4)
    w = rng.normal(0, 0.02, (40, 96)).astype(np.float32)
    p, s = M.q4_pack(w)
    wd = M.q4_dequant(p, s, 40, 96)
    # dequantised weights are within half a step of the originals, plus the
    # fp16 rounding of the stored scale (codes use the fp32 scale, :53 vs :70)
    step = np.repeat(s.astype(np.float32), 32).reshape(40, 96)
    assert np.all(np.abs(wd - w) <= 0.5 * step + 8 * step * 2.0 ** -11 + 1e-7)
    x = rng.normal(0, 1, 96).astype(np.float16)
    y = M.gemv_q4(p, s, x, 40, 96)
    np.testing.assert_allclose(y.astype(np.float32), (wd @ x.astype(np.float32)), rtol=2e-3, atol=2e-3)


def test_oracle_layer_one_token_is_reference_layer():
    """At pos 0 with an empty cache and zero biases the layer is exactly the
    reference's 17-dispatch block (engine.py:187-243) restated stage by stage."""
    from llamamps_b200.config import ModelConfig
    from llamamps_b200.weights import parts_host_arrays, synth_layer_numpy
    cfg = M.OracleConfig()
    parts = synth_layer_numpy(np.random.default_rng(5), ModelConfig(), with_bias=False)
    lw = parts_host_arrays(parts)
    x = np.random.default_rng(6).normal(0, 1, 1536).astype(np.float16)
    cache = M.KVCache(1, cfg.kv_dim)
    tr = {}
    out = M.decoder_layer(x, lw, cache, 0, 0, cfg, trace=tr)
    # step by step with the reference's kernels
    xn = M.rms_norm(x, lw["in_norm"])
    q = M.gemv_q4(lw["q"], lw["qs"], xn, 1536, 1536)
    k = M.gemv_q4(lw["k"], lw["ks"], xn, 256, 1536)
    v = M.gemv_q4(lw["v"], lw["vs"], xn, 256, 1536)
    attn = M.attn_weighted_sum(M.softmax(M.attention_scores(q, k[None])), v[None])
    x1 = M.residual_add(x, M.gemv_q4(lw["o"], lw["os"], attn, 1536, 1536))
    hn = M.rms_norm(x1, lw["post_norm"])
    a = M.swiglu(M.gemv_q4(lw["gt"], lw["gts"], hn, 8960, 1536), M.gemv_q4(lw["up"], lw["ups"], hn, 8960, 1536))
    x2 = M.residual_add(x1, M.gemv_q4(lw["dn"], lw["dns"], a, 1536, 8960))
    assert f16_bits_equal(out, x2)


def _tiny_weights(rng, cfg, n_layers):
    def mat(rows, k):
        return M.q4_pack(rng.normal(0, 0.05, (rows, k)).astype(np.float32))
    layers = []
    for _ in range(n_layers):
        lw = {}
        for name, (r, k) in {"q": (cfg.q_dim, cfg.hidden), "k": (cfg.kv_dim, cfg.hidden), "v": (cfg.kv_dim, cfg.hidden),
                             "o": (cfg.hidden, cfg.q_dim), "gt": (cfg.intermediate, cfg.hidden),
                             "up": (cfg.intermediate, cfg.hidden), "dn": (cfg.hidden, cfg.intermediate)}.items():
            lw[name], lw[name + "s"] = mat(r, k)
        lw["bq"] = rng.normal(0, 0.02, cfg.q_dim).astype(np.float16)
        lw["bk"] = rng.normal(0, 0.02, cfg.kv_dim).astype(np.float16)
        lw["bv"] = rng.normal(0, 0.02, cfg.kv_dim).astype(np.float16)
        lw["in_norm"] = (1 + rng.normal(0, 0.02, cfg.hidden)).astype(np.float16)
        lw["post_norm"] = (1 + rng.normal(0, 0.02, cfg.hidden)).astype(np.float16)
        layers.append(lw)
    embed = rng.normal(0, 0.5, (cfg.vocab, cfg.hidden)).astype(np.float16)
    lp, ls = M.q4_pack(embed.astype(np.float32))
    return {"layers": layers, "final_norm": (1 + rng.normal(0, 0.02, cfg.hidden)).astype(np.float16),
            "lm_packed": lp, "lm_scales": ls, "embed": embed}


def test_batched_oracle_rows_equal_single_sequence_oracle():
    """OracleBatch (used by the full-batch GPU tests) is the per-sequence
    oracle row by row: same greedy ids, logits equal up to fp16 rounding of
    sums taken in another order (GEMM vs GEMV)."""
    cfg = M.OracleConfig(hidden=128, intermediate=256, vocab=300, n_layers=2, n_q_heads=4, n_kv_heads=2,
                         head_dim=32)
    w = _tiny_weights(np.random.default_rng(5), cfg, 2)
    prompts = np.random.default_rng(6).integers(0, cfg.vocab, (3, 5))
    rec_b = []
    ids_b = M.OracleBatch(w, cfg, 3).generate(prompts, 4, record=rec_b)
    for b in range(3):
        rec = []
        ids = M.OracleModel(w, cfg).generate(prompts[b].tolist(), 4, record=rec)
        for i in range(4):
            assert_close(rec_b[i][b], rec[i], what=f"row {b} step {i}")
            if ids[i] != ids_b[b, i]:
                assert M.top2_margin(rec[i]) < 2e-2
                break


def test_philox_known_answers():
    """The Philox4x32-10 restatement against the published known-answer
    vectors of its authors' Random123 distribution (counter, key -> output)."""
    assert M.philox4x32_10((0, 0, 0, 0), (0, 0)) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert M.philox4x32_10((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6,
                                                                        0x6D5451FD]
    assert M.philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0)) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_sampling_restatement_properties():
    """top-k = 1 is the first-index argmax; draws stay inside the top k;
    temperature -> 0 concentrates on the maximum; the empirical frequencies
    of many draws follow the softmax of the top k."""
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, 500).astype(np.float16)
    x[[10, 200]] = np.float16(4.0)                           # tie at the maximum
    assert M.sample_top_k(x, 1, 1.0, 5, 0) == 10
    assert M.sample_top_k(x, 8, 0.0, 5, 0) == 10             # temperature 0: greedy
    top8 = set(np.argsort(-x.astype(np.float32), kind="stable")[:8].tolist())
    draws = [M.sample_top_k(x, 8, 1.0, 99, i) for i in range(3000)]
    assert set(draws) <= top8
    cand = sorted(top8)
    p = np.exp(x[cand].astype(np.float64) - x[cand].max())
    p /= p.sum()
    freq = np.array([draws.count(c) for c in cand]) / len(draws)
    assert np.max(np.abs(freq - p)) < 0.04
    nan_x = x.copy()
    nan_x[3] = np.float16(np.nan)
    assert M.sample_top_k(nan_x, 5, 1.0, 1, 0) != 3
