"""Batched decode in one cooperative launch (csrc/decode_batched.cu): every
layer of a decode step for up to 64 sequences, the projections on tcgen05.
Checked byte for byte on its tile-major weight copy, step by step against
the per-stage kernel path on the same weights and tokens, against the
oracle's greedy loop at the batched-decode configuration's shape, and
against the oracle over long cached contexts (attention split over CTAs,
then merged)."""
import dataclasses

import numpy as np
import pytest
import torch

from oracle import mirror as M
from tests._util import assert_close, greedy_ids_match

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small_model():
    from llamamps_b200.config import QWEN2_5_1_5B
    from llamamps_b200.weights import model_host_arrays, synth_model
    cfg = dataclasses.replace(QWEN2_5_1_5B, n_layers=2, vocab=8192)
    mw = synth_model(cfg, seed=12, device="cuda")
    return cfg, mw, model_host_arrays(mw)


def _engine(mw, **kw):
    from llamamps_b200.engine import QwenEngine
    return QwenEngine(weights=mw, **kw)


def test_tile_blocks_layout(cuda):
    """Block (tile i, step j): the rows' 32 packed bytes of K step j (halves
    swapped when (row >> 2) & 1), then their two group scales."""
    from llamamps_b200.batched import tile_blocks
    n, k = 256, 1536
    rng = np.random.default_rng(3)
    packed = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    scales = rng.normal(0, 0.02, (n, k // 32)).astype(np.float16)
    got = tile_blocks(torch.from_numpy(packed).cuda(), torch.from_numpy(scales).cuda(), n, k).cpu().numpy()
    ks = k // 64
    want = np.zeros((n // 128, ks, 4608), np.uint8)
    for i in range(n // 128):
        for j in range(ks):
            rows = packed[128 * i:128 * (i + 1), 32 * j:32 * (j + 1)].copy()
            swap = ((np.arange(128) >> 2) & 1).astype(bool)
            rows[swap] = np.concatenate([rows[swap, 16:], rows[swap, :16]], axis=1)
            want[i, j, :4096] = rows.reshape(-1)
            want[i, j, 4096:] = scales[128 * i:128 * (i + 1), 2 * j:2 * j + 2].copy().view(np.uint8).reshape(-1)
    assert np.array_equal(got, want.reshape(-1))


def _compare_logits_steps(ref, eng, B, P, N, seed):
    """Prefill the same prompts token by token on both engines, then N
    logits steps with the same fed tokens; the batched engine's fp16 logits
    within the decode tolerance of the reference engine's."""
    cfg = ref.cfg
    prompts = torch.as_tensor(np.random.default_rng(seed).integers(0, cfg.vocab, (B, P)), dtype=torch.int32)
    for e in (ref, eng):
        e.reset(B)
        e.prefill(prompts, dense=False)
    torch.cuda.synchronize()
    eng.bdec.check_error()
    eng.tokens[:B].copy_(ref.tokens[:B])
    for s in range(N):
        ref._logits_step(B)
        eng._logits_step(B)
        torch.cuda.synchronize()
        eng.bdec.check_error()
        a = ref.buf_logits[:B].float().cpu().numpy()
        b = eng.buf_logits[:B].float().cpu().numpy()
        for i in range(B):
            assert_close(b[i], a[i], what=f"B={B} step {s} sequence {i}")
        eng.tokens[:B].copy_(ref.tokens[:B])
    assert eng.pos[:B].cpu().tolist() == [P + N] * B


@pytest.mark.parametrize("B", [5, 16, 64])
def test_batched_decoder_matches_kernel_path(cuda, small_model, B):
    """Same prompts and fed tokens through both decoders (the split-K sums
    are added in a different order)."""
    cfg, mw, host = small_model
    ref = _engine(mw, max_batch=B, max_seq_len=64, decoder="kernels")
    eng = _engine(mw, max_batch=B, max_seq_len=64, decoder="batched")
    _compare_logits_steps(ref, eng, B, 5, 4, B)


def test_batched_decoder_batch_size_changes(cuda, small_model):
    """One engine (and workspace) driven at 16 sequences, then 5, then 16
    again: the split-K accumulators are zero at every launch."""
    cfg, mw, host = small_model
    ref = _engine(mw, max_batch=16, max_seq_len=64, decoder="kernels")
    eng = _engine(mw, max_batch=16, max_seq_len=64, decoder="batched")
    for i, B in enumerate((16, 5, 16)):
        _compare_logits_steps(ref, eng, B, 3, 2, 100 + i)


def test_batched_decoder_c2_shape_matches_oracle(cuda, small_model):
    """64 sequences with 128-id prompts (dense prefill), then greedy decode
    with every layer of a step in one launch: each sequence follows the
    oracle (runners/engine.py:157-181 per row, stepped as one batch), and
    where all its ids matched, the last step's logits are within tolerance."""
    cfg, mw, host = small_model
    B, P, N = 64, 128, 4
    prompts = np.random.default_rng(2).integers(0, cfg.vocab, (B, P))
    eng = _engine(mw, max_batch=B, max_seq_len=P + N + 8, decoder="batched")
    got = eng.generate_batch(prompts, N)
    last = eng.buf_logits[:B].cpu().numpy()
    rec = []
    ref = M.OracleBatch(host, M.OracleConfig(n_layers=2, vocab=cfg.vocab), B).generate(prompts, N, record=rec)
    full = 0
    for b in range(B):
        n = greedy_ids_match(got[b].tolist(), ref[b].tolist(), [r[b] for r in rec])
        if n == N:
            full += 1
            assert_close(last[b], rec[N - 1][b], what=f"sequence {b} last-step logits")
    assert full >= B // 2, f"only {full} of {B} sequences matched every step"


def test_batched_decoder_long_context_matches_oracle(cuda, small_model):
    """Five sequences over 700..2000 cached positions (fp16 N(0,1) rows
    written into the paged cache): the attention phase splits each
    (sequence, KV head) over 5 CTAs and merges the splits.  Three logits
    steps against the oracle holding the same cache prefix
    (kernels/attention.metal:22-40, softmax.metal:23-36, attn_sum.metal:22-33)."""
    cfg, mw, host = small_model
    B, lens, max_seq = 5, [1500, 900, 2000, 1200, 700], 2048 + 64
    eng = _engine(mw, max_batch=B, max_seq_len=max_seq, decoder="batched")
    eng.reset(B)
    rng = np.random.default_rng(77)
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
    eng.seq_lens[:B].copy_(torch.tensor(lens, dtype=torch.int32) + 1)
    toks = rng.integers(0, cfg.vocab, (B, 3))
    for s in range(3):
        eng.tokens[:B].copy_(torch.from_numpy(toks[:, s]).to(torch.int32))
        eng._logits_step(B)
        torch.cuda.synchronize()
        eng.bdec.check_error()
        got = eng.buf_logits[:B].cpu().numpy()
        for b in range(B):
            assert_close(got[b], orcs[b].step_token(int(toks[b, s])), what=f"seq {b} step {s}")
    assert eng.pos[:B].cpu().tolist() == [n + 3 for n in lens]


def test_batched_decoder_rejects_positions_past_the_cache(cuda, small_model):
    """A position outside the cache: the launch returns before any work and
    the error word says so (no write past the block table)."""
    cfg, mw, host = small_model
    eng = _engine(mw, max_batch=8, max_seq_len=64, decoder="batched")
    eng.reset(8)
    eng.pos[:8].fill_(eng.cache.block_table.shape[1] * eng.cache.page_size)
    eng.seq_lens[:8].copy_(eng.pos[:8] + 1)
    eng.bdec.run(8, eng.buf_residual[:8], eng.pos[:8], eng.seq_lens[:8])
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="outside the KV cache"):
        eng.bdec.check_error()
    assert int(eng.bdec.error.item()) == 0  # cleared with the workspace
