"""Large-batch decode (more sequences than the GEMV's 8): the projections and
the LM head run through the tcgen05 W4A16 GEMM, the argmax through the
row-argmax kernel; every sequence must still follow the oracle's greedy loop
and agree with the same sequence decoded in a small batch."""
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


def test_batch16_gemm_path_matches_oracle_and_small_batch(cuda, small_model):
    from llamamps_b200.engine import QwenEngine, GEMV_MAX_BATCH
    cfg, mw, host = small_model
    B = 16
    assert B > GEMV_MAX_BATCH
    prompts = np.random.default_rng(21).integers(0, cfg.vocab, (B, 6))
    big = QwenEngine(weights=mw, max_batch=B, max_seq_len=64, decoder="kernels")
    got = big.generate_batch(prompts, 5)
    assert int(big.gemm_err.item()) == 0
    small = QwenEngine(weights=mw, max_batch=4, max_seq_len=64, decoder="kernels")
    for b in range(B):
        rec = []
        ref = M.OracleModel(host, M.OracleConfig(n_layers=2, vocab=cfg.vocab)).generate(
            prompts[b].tolist(), 5, record=rec)
        assert greedy_ids_match(got[b].tolist(), ref, rec) >= 3, f"sequence {b}"
    alone = small.generate_batch(prompts[:4], 5)
    for b in range(4):  # GEMM (fp16-rounded weights) and GEMV paths agree except near ties
        rec = []
        M.OracleModel(host, M.OracleConfig(n_layers=2, vocab=cfg.vocab)).generate(prompts[b].tolist(), 5, record=rec)
        assert greedy_ids_match(got[b].tolist(), alone[b].tolist(), rec) >= 3


def test_batch64_c2_shape_matches_oracle(cuda, small_model):
    """The batched-decode configuration's shape on two layers: 64 sequences
    with 128-id prompts prefilled densely (tensor-core GEMMs over 8192 token
    rows, causal prefill attention), then greedy decode on the GEMM path.
    Every sequence follows the oracle (runners/engine.py:157-181 per row,
    stepped as one batch), and where all its ids matched, the logits of the
    last step are within the 2e-2 / 1e-2 tolerance."""
    from llamamps_b200.engine import QwenEngine
    cfg, mw, host = small_model
    B, P, N = 64, 128, 4
    prompts = np.random.default_rng(2).integers(0, cfg.vocab, (B, P))
    eng = QwenEngine(weights=mw, max_batch=B, max_seq_len=P + N + 8, decoder="kernels")
    got = eng.generate_batch(prompts, N)
    assert int(eng.gemm_err.item()) == 0
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


def test_argmax_rows_first_index(cuda):
    from llamamps_b200 import kernels as K
    x = torch.full((3, 1000), -1.0, dtype=torch.float16, device="cuda")
    x[0, 5] = 2.0
    x[1, 7] = 3.0
    x[1, 900] = 3.0          # tie: first index wins
    x[2, 999] = 0.5
    ids = torch.zeros(3, dtype=torch.int32, device="cuda")
    K.argmax_rows(x, 1000, ids)
    assert ids.tolist() == [5, 7, 999]


def test_argmax_rows_cluster_path_and_ties_across_slices(cuda):
    """Vocabulary-sized rows take the cluster path (8 CTAs per row, one
    slice each): ties across slices resolve to the first index and the
    ragged tail is scanned."""
    from llamamps_b200 import kernels as K
    V = 151936 + 8 * 3 + 5            # not a multiple of the slice alignment
    x = torch.randn(6, V, generator=torch.Generator(device="cuda").manual_seed(4), device="cuda").half()
    x[0, 100] = 9.0
    x[0, V - 3] = 9.0                 # tie in the last slice: first index wins
    x[1, V - 1] = 11.0                # the ragged tail
    x[2, 50000] = 8.0
    x[2, 19000] = 8.0                 # tie across slices
    ids = torch.zeros(6, dtype=torch.int32, device="cuda")
    K.argmax_rows(x, V, ids)
    ref = [int(torch.argmax(x[r].float()).item()) for r in range(6)]
    assert ids.tolist()[:3] == [100, V - 1, 19000]
    assert ids.tolist() == ref


def test_swiglu_rows_matches_two_input_swiglu(cuda):
    from llamamps_b200 import kernels as K
    g = torch.Generator(device="cuda").manual_seed(2)
    gu = torch.randn(5, 2 * 300, generator=g, device="cuda").half()
    out = torch.empty(5, 300, dtype=torch.float16, device="cuda")
    K.swiglu_rows(gu, 300, out)
    ref = K.swiglu(gu[:, :300].contiguous(), gu[:, 300:].contiguous())
    assert torch.equal(out, ref)


@pytest.mark.parametrize("B,P,ps", [(1, 2048, 64), (3, 700, 128), (2, 129, 64)])
def test_prefill_attention_tcgen05_matches_mma_sync_kernel(cuda, B, P, ps):
    """The tcgen05 prefill attention against the mma.sync kernel on longer
    prompts (many key tiles, the O rescale, several query tiles, pages of
    128 positions, permuted page order)."""
    from llamamps_b200 import kernels as K
    Hq, Hkv, hd = 12, 2, 128
    g = torch.Generator(device="cuda").manual_seed(B * P + ps)
    pages = (P + ps - 1) // ps
    kp = torch.randn(B * pages + 3, Hkv, ps, hd, generator=g, device="cuda").half()
    vp = torch.randn(B * pages + 3, Hkv, ps, hd, generator=g, device="cuda").half()
    bt = (torch.randperm(B * pages, generator=g, device="cuda") + 3).to(torch.int32).reshape(B, pages)
    q = (torch.randn(B * P, Hq * hd, generator=g, device="cuda") * 2).half()
    a, b = torch.empty_like(q), torch.empty_like(q)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.prefill_attention(q, kp, vp, bt, a, B, P, ps, Hq, Hkv, hd, error=err, tcgen05=True)
    K.prefill_attention(q, kp, vp, bt, b, B, P, ps, Hq, Hkv, hd, tcgen05=False)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and bool(torch.isfinite(a.float()).all())
    assert torch.allclose(a.float(), b.float(), atol=4e-3, rtol=1e-2), float((a.float() - b.float()).abs().max())


@pytest.mark.parametrize("m", [1, 5, 64, 127, 128, 300])
def test_gemm_swiglu_epilogue_equals_gemm_then_swiglu(cuda, m):
    """The GEMM's SwiGLU epilogue over row-interleaved gate/up weights, bit for
    bit the GEMM over [gate; up] followed by swiglu_rows, on both tile shapes
    (decode tiles with split K below 128 tokens, prefill tiles above)."""
    from llamamps_b200 import kernels as K
    from llamamps_b200.quant import pack_q4
    from llamamps_b200.weights import interleave_rows
    n, k = 640, 1536
    g = torch.Generator(device="cuda").manual_seed(m)
    gate = torch.randn(n, k, generator=g, device="cuda") * 0.02
    up = torch.randn(n, k, generator=g, device="cuda") * 0.02
    gp, gs = pack_q4(gate)
    upk, us = pack_q4(up)
    x = torch.randn(m, k, generator=g, device="cuda").half()
    cat = K.w4a16_gemm(x, torch.cat([gp, upk]), torch.cat([gs, us]), 2 * n, k)
    ref = torch.empty(m, n, dtype=torch.float16, device="cuda")
    K.swiglu_rows(cat, n, ref)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = K.w4a16_gemm(x, interleave_rows(gp, upk, n), interleave_rows(gs, us, n), 2 * n, k, swiglu=True,
                       error=err)
    assert got.shape == (m, n) and int(err.item()) == 0
    assert torch.equal(got, ref)


@pytest.mark.parametrize("decoder", ["kernels", "persistent"])
def test_dense_prefill_matches_oracle(cuda, small_model, decoder):
    """Prompts prefilled all at once on the GEMM path (3 x 100 tokens), then
    greedy decode; against the oracle's token-by-token loop."""
    from llamamps_b200.engine import QwenEngine
    cfg, mw, host = small_model
    prompts = np.random.default_rng(33).integers(0, cfg.vocab, (3, 100))
    eng = QwenEngine(weights=mw, max_batch=4, max_seq_len=160, decoder=decoder)
    got = eng.generate_batch(prompts, 5)
    assert int(eng.gemm_err.item()) == 0
    for b in range(3):
        rec = []
        ref = M.OracleModel(host, M.OracleConfig(n_layers=2, vocab=cfg.vocab)).generate(
            prompts[b].tolist(), 5, record=rec)
        assert greedy_ids_match(got[b].tolist(), ref, rec) >= 3, f"sequence {b}"


def test_dense_and_stepwise_prefill_fill_the_same_cache(cuda, small_model):
    from llamamps_b200.engine import QwenEngine
    cfg, mw, _ = small_model
    prompts = torch.from_numpy(np.random.default_rng(34).integers(0, cfg.vocab, (2, 40)))
    a = QwenEngine(weights=mw, max_batch=2, max_seq_len=64, decoder="kernels")
    b = QwenEngine(weights=mw, max_batch=2, max_seq_len=64, decoder="kernels")
    a.reset(2)
    a.prefill(prompts, dense=True)
    b.reset(2)
    b.prefill(prompts, dense=False)
    torch.cuda.synchronize()
    for li in (0, 1):
        for s in (0, 1):
            ka, va = a.cache.read_positions(s, li, 40)
            kb, vb = b.cache.read_positions(s, li, 40)
            # GEMM (fp16-rounded weights) vs GEMV (exact dequant) projections
            assert torch.allclose(ka.float(), kb.float(), atol=2e-2, rtol=1e-2)
            assert torch.allclose(va.float(), vb.float(), atol=2e-2, rtol=1e-2)
    assert torch.equal(a.pos[:2], b.pos[:2])


@pytest.mark.parametrize("tcgen05", [True, False])
@pytest.mark.parametrize("P", [1, 37, 130, 300])
def test_prefill_attention_matches_per_row_decode_attention(cuda, P, tcgen05):
    """The causal prefill kernels (tcgen05 / TMEM and mma.sync) against the
    decode attention kernel run with one query row per position (seq_len =
    p + 1) on the same paged cache."""
    from llamamps_b200 import kernels as K
    B, Hq, Hkv, hd, ps = 2, 12, 2, 128, 64
    g = torch.Generator(device="cuda").manual_seed(P)
    pages = (P + ps - 1) // ps
    kp = torch.randn(B * pages, Hkv, ps, hd, generator=g, device="cuda").half()
    vp = torch.randn(B * pages, Hkv, ps, hd, generator=g, device="cuda").half()
    bt = torch.randperm(B * pages, generator=g, device="cuda").to(torch.int32).reshape(B, pages)
    q = torch.randn(B * P, Hq * hd, generator=g, device="cuda").half()
    out = torch.empty_like(q)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.prefill_attention(q, kp, vp, bt, out, B, P, ps, Hq, Hkv, hd, error=err, tcgen05=tcgen05)
    assert int(err.item()) == 0
    rows_bt = bt.repeat_interleave(P, dim=0).contiguous()
    lens = (torch.arange(P, device="cuda", dtype=torch.int32) + 1).repeat(B)
    ref = torch.empty_like(q)
    splits = K.attention_splits(B * P, Hkv, P, ps)
    ws = torch.zeros(max(K.attention_workspace_size(B * P, Hq, hd, splits), 16), dtype=torch.uint8, device="cuda")
    K.gqa_decode_attention(q, kp, vp, rows_bt, lens, ref, ws, ps, Hq, Hkv, hd, P, splits)
    torch.cuda.synchronize()
    assert torch.allclose(out.float(), ref.float(), atol=4e-3, rtol=1e-2), float((out.float() - ref.float()).abs().max())
