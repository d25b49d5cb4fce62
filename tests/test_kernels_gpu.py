"""Kernel-by-kernel parity of the sm_100a C ABI against the numpy oracle.

Every call goes through libllamamps_b200.so (llamamps_b200.kernels is a thin
ctypes front end).  Outputs carry canary padding that must survive the call.
"""
import numpy as np
import pytest
import torch

from oracle import mirror as M
from tests._util import assert_close, f16_bits_equal

pytestmark = pytest.mark.gpu

CANARY = 1234.0


def _padded(n, dtype=torch.float16, dev="cuda", pad=64):
    buf = torch.full((n + 2 * pad,), CANARY, dtype=dtype, device=dev)
    return buf, buf[pad:pad + n]


def _canary_ok(buf, pad=64):
    b = buf.float().cpu().numpy()
    return np.all(b[:pad] == CANARY) and np.all(b[-pad:] == CANARY)


def _q4(rng, rows, k, std=0.02):
    w = rng.normal(0, std, (rows, k)).astype(np.float32)
    return M.q4_pack(w)


def _t(a, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


GEMV_SHAPES = [(1536, 1536), (256, 1536), (2048, 1536), (8960, 1536), (1536, 8960),
               (1, 32), (7, 96), (33, 160), (100, 1024), (5, 64 * 35)]


@pytest.mark.parametrize("rows,k", GEMV_SHAPES)
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_gemv_q4_0(cuda, rows, k, batch):
    from llamamps_b200 import kernels as K
    rng = np.random.default_rng(rows * 7 + k + batch)
    p, s = _q4(rng, rows, k)
    x = rng.normal(0, 1, (batch, k)).astype(np.float16)
    ref = M.gemv_q4(p, s, x, rows, k)
    buf, y = _padded(batch * rows)
    K.gemv_q4(_t(p), _t(s), _t(x), rows, k, out=y.view(batch, rows))
    assert _canary_ok(buf)
    assert_close(y.view(batch, rows).cpu().numpy(), ref, what=f"gemv {rows}x{k} b{batch}")


def test_gemv_lm_head_rows(cuda):
    from llamamps_b200 import kernels as K
    rng = np.random.default_rng(11)
    rows, k = 151936, 1536
    p, s = _q4(rng, rows, k)
    x = rng.normal(0, 1, (1, k)).astype(np.float16)
    ref = M.gemv_q4(p, s, x, rows, k)
    y = K.gemv_q4(_t(p), _t(s), _t(x), rows, k)
    assert_close(y.cpu().numpy(), ref, what="lm head gemv")


@pytest.mark.parametrize("batch", [1, 2, 5])
def test_gemv_bias_residual_swiglu(cuda, batch):
    from llamamps_b200 import kernels as K
    rng = np.random.default_rng(21 + batch)
    rows, k = 2048, 1536
    p, s = _q4(rng, rows, k)
    bias = rng.normal(0, 0.02, rows).astype(np.float16)
    x = rng.normal(0, 1, (batch, k)).astype(np.float16)
    acc = x.astype(np.float32) @ M.q4_dequant(p, s, rows, k).T
    ref = (acc + bias.astype(np.float32)).astype(np.float16)
    y = K.gemv_q4_bias(_t(p), _t(s), _t(bias), _t(x), rows, k)
    assert_close(y.cpu().numpy(), ref, what="bias")

    res = rng.normal(0, 1, (batch, rows)).astype(np.float16)
    ref_r = M.residual_add(res, acc.astype(np.float16))
    r_t = _t(res)
    K.gemv_q4_residual(_t(p), _t(s), _t(x), r_t, rows, k, out=r_t)   # in place, as the engine does
    assert_close(r_t.cpu().numpy(), ref_r, what="residual")

    pg, sg = _q4(rng, 8960, k)
    pu, su = _q4(rng, 8960, k)
    g = M.gemv_q4(pg, sg, x, 8960, k)
    u = M.gemv_q4(pu, su, x, 8960, k)
    ref_a = M.swiglu(g, u)
    a = K.gemv_q4_swiglu(_t(pg), _t(sg), _t(pu), _t(su), _t(x), 8960, k)
    assert_close(a.cpu().numpy(), ref_a, what="swiglu")


@pytest.mark.parametrize("batch", [1, 4])
def test_lm_head_argmax_first_index_ties(cuda, batch):
    """Rows 17, 2500, 3000 and 3999 carry identical codes and the largest
    scale, so their logits tie at the maximum: numpy's first-index rule
    (runners/engine.py:181) must pick 17."""
    from llamamps_b200 import kernels as K
    rng = np.random.default_rng(31)
    rows, k = 4096, 64
    packed = rng.integers(0, 256, rows * k // 2, dtype=np.uint8)
    scales = np.full(rows * k // 32, 0.001, np.float16)
    x = np.abs(rng.normal(0, 1, (batch, k))).astype(np.float16)
    hot = packed[17 * 32:18 * 32].copy()
    hot[:] = 0xFF                                   # every code +7
    for r in (17, 2500, 3000, 3999):
        packed[r * 32:(r + 1) * 32] = hot
        scales[r * 2:r * 2 + 2] = np.float16(0.05)
    ref_logits = M.gemv_q4(packed, scales, x, rows, k)
    keys = torch.zeros(batch, dtype=torch.int64, device="cuda")
    ids = torch.zeros(batch, dtype=torch.int32, device="cuda")
    logits = torch.zeros(batch, rows, dtype=torch.float16, device="cuda")
    K.lm_head_argmax(_t(packed), _t(scales), _t(x), rows, k, keys, ids, logits=logits)
    got = ids.cpu().numpy()
    assert np.all(got == 17)
    assert all(M.predict_next_token(ref_logits[b]) == 17 for b in range(batch))
    assert_close(logits.cpu().numpy(), ref_logits, what="lm head logits")
    assert torch.all(keys == 0), "argmax workspace must be left zeroed"
    K.lm_head_argmax(_t(packed), _t(scales), _t(x), rows, k, keys, ids, logits=None)
    assert np.all(ids.cpu().numpy() == 17)


@pytest.mark.parametrize("dim,batch", [(1536, 1), (1536, 4), (1536, 300), (2048, 263), (8960, 2), (96, 257), (100, 2)])
def test_rms_norm(cuda, dim, batch):
    from llamamps_b200 import kernels as K
    rng = np.random.default_rng(dim + batch)
    x = rng.normal(0, 1, (batch, dim)).astype(np.float16)
    g = (1 + rng.normal(0, 0.02, dim)).astype(np.float16)
    ref = M.rms_norm(x, g)
    y = K.rms_norm(_t(x), _t(g))
    out = y.cpu().numpy()
    assert_close(out, ref, abs_tol=4e-3, what="rmsnorm")
    # the scale differs from numpy's by at most an ulp: nearly all bits match
    assert np.mean(out.view(np.uint16) == ref.view(np.uint16)) > 0.99


@pytest.mark.parametrize("style", ["interleaved", "neox"])
@pytest.mark.parametrize("theta", [1e4, 1e6])
def test_rope(cuda, style, theta):
    from llamamps_b200 import kernels as K
    from llamamps_b200.engine import rope_inv_freq
    rng = np.random.default_rng(41)
    B = 4
    pos = np.array([0, 1, 31, 32767], np.int32)
    v = rng.normal(0, 1, (B, 1536)).astype(np.float16)
    ref = np.stack([M.rope(v[b], int(pos[b]), 128, theta, style) for b in range(B)])
    vt = _t(v)
    K.rope_(vt, _t(pos), _t(rope_inv_freq(128, theta)), 12, 128, 0 if style == "interleaved" else 1)
    out = vt.cpu().numpy()
    assert f16_bits_equal(out[0], v[0])        # m = 0 is the identity (rope.metal:23)
    assert_close(out, ref, abs_tol=1e-2, what="rope")


def test_residual_and_swiglu_elementwise(cuda):
    from llamamps_b200 import kernels as K
    rng = np.random.default_rng(51)
    a = rng.normal(0, 1, 8960).astype(np.float16)
    b = rng.normal(0, 3, 8960).astype(np.float16)
    assert f16_bits_equal(K.residual_add(_t(a), _t(b)).cpu().numpy(), M.residual_add(a, b))
    got = K.swiglu(_t(b), _t(a)).cpu().numpy()
    ref = M.swiglu(b, a)
    assert np.mean(got.view(np.uint16) == ref.view(np.uint16)) > 0.99
    assert_close(got, ref, abs_tol=1e-2, what="swiglu")


def test_embed_gather_and_bad_ids(cuda):
    from llamamps_b200 import kernels as K
    rng = np.random.default_rng(61)
    table = rng.normal(0, 0.02, (1000, 1536)).astype(np.float16)
    ids = np.array([0, 999, 17], np.int32)
    out = torch.zeros(3, 1536, dtype=torch.float16, device="cuda")
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.embed_gather(_t(table), _t(ids), out, bad)
    assert f16_bits_equal(out.cpu().numpy(), table[ids]) and bad.item() == 0
    K.embed_gather(_t(table), _t(np.array([5, 1000, -1], np.int32)), out, bad)
    o = out.cpu().numpy()
    assert bad.item() == 1 and np.all(o[1:] == 0) and f16_bits_equal(o[0], table[5])


@pytest.mark.parametrize("T", [1, 7, 32, 300])
def test_reference_three_stage_attention(cuda, T):
    from llamamps_b200 import kernels as K
    rng = np.random.default_rng(T)
    q = rng.normal(0, 1, 1536).astype(np.float16)
    kc = rng.normal(0, 1, (T, 256)).astype(np.float16)
    vc = rng.normal(0, 1, (T, 256)).astype(np.float16)
    s_ref = M.attention_scores(q, kc)
    s = K.attention_scores(_t(q), _t(kc), T, 12, 2, 128)
    np.testing.assert_allclose(s.cpu().numpy(), s_ref, rtol=1e-4, atol=1e-4)
    K.softmax_(s, T, 12)
    p_ref = M.softmax(s_ref)
    np.testing.assert_allclose(s.cpu().numpy(), p_ref, rtol=1e-4, atol=1e-6)
    o = K.attn_weighted_sum(s, _t(vc), T, 12, 2, 128)
    assert_close(o.cpu().numpy(), M.attn_weighted_sum(p_ref, vc), abs_tol=5e-3, what="attn_sum")


def _paged_setup(rng, B, T_list, page_size, max_seq, n_layers=1, permute=True):
    from llamamps_b200.config import QWEN2_5_1_5B
    from llamamps_b200.kv_cache import PagedKVCache
    pps = (max_seq + page_size - 1) // page_size
    order = list(rng.permutation(B * pps)) if permute else None
    kv = PagedKVCache(QWEN2_5_1_5B, n_layers, B, max_seq, page_size, "cuda", page_order=order)
    rows = []
    for b, T in enumerate(T_list):
        kv.reserve(b, max_seq)
        k = rng.normal(0, 1, (T, 256)).astype(np.float16)
        v = rng.normal(0, 1, (T, 256)).astype(np.float16)
        kv.write_positions(b, 0, 0, _t(k), _t(v))
        rows.append((k, v))
    return kv, rows


@pytest.mark.parametrize("T_list,page_size,max_seq", [
    ([1], 64, 64), ([31], 64, 128), ([32], 16, 64), ([33], 64, 160), ([64], 64, 64),
    ([65, 1, 200], 64, 256), ([4097], 64, 4160), ([129, 384, 130, 200], 64, 384),
])
def test_gqa_decode_attention(cuda, T_list, page_size, max_seq):
    from llamamps_b200 import kernels as K
    rng = np.random.default_rng(sum(T_list) + page_size)
    B = len(T_list)
    kv, rows = _paged_setup(rng, B, T_list, page_size, max_seq)
    q = rng.normal(0, 1, (B, 1536)).astype(np.float16)
    seq_lens = _t(np.array(T_list, np.int32))
    kp, vp = kv.layer(0)
    # 2..8 splits merge inside a thread-block cluster (empty splits included:
    # 5 splits of a 64-position cache), more through the combine kernel
    splits = {1, K.attention_splits(B, 2, kv.max_seq_len, page_size), 2, 3, 5}
    if kv.max_seq_len >= 9 * 64:
        splits |= {8, 9}
    for n_splits in sorted(splits):
        ws = torch.zeros(max(16, K.attention_workspace_size(B, 12, 128, n_splits)), dtype=torch.uint8, device="cuda")
        buf, out = _padded(B * 1536)
        K.gqa_decode_attention(_t(q), kp, vp, kv.block_table, seq_lens, out.view(B, 1536), ws,
                               page_size, 12, 2, 128, kv.max_seq_len, n_splits)
        assert _canary_ok(buf)
        o = out.view(B, 1536).cpu().numpy()
        for b, (k, v) in enumerate(rows):
            ref = M.attn_weighted_sum(M.softmax(M.attention_scores(q[b], k)), v)
            assert_close(o[b], ref, abs_tol=5e-3, what=f"attn T={T_list[b]} splits={n_splits}")


@pytest.mark.parametrize("style", [0, 1])
def test_rope_kv_append_matches_oracle(cuda, style):
    """RoPE on q and k of the fused q|k|v rows and the paged-cache append
    (both pair layouts) against the oracle; the 16-byte kernel (one cos/sin
    table per row) bit-equal to the element-wise one, which a misaligned
    output selects."""
    from llamamps_b200 import kernels as K
    from llamamps_b200.engine import rope_inv_freq
    rng = np.random.default_rng(71 + style)
    B, page_size, max_seq = 3, 16, 64
    kv, _ = _paged_setup(rng, B, [5, 16, 40], page_size, max_seq)
    kv2, _ = _paged_setup(np.random.default_rng(71 + style), B, [5, 16, 40], page_size, max_seq)
    pos = np.array([5, 16, 40], np.int32)
    qkv = rng.normal(0, 1, (B, 2048)).astype(np.float16)
    q_out = torch.zeros(B, 1536, dtype=torch.float16, device="cuda")
    kp, vp = kv.layer(0)
    inv = _t(rope_inv_freq(128, 1e6))
    K.rope_kv_append(_t(qkv), _t(pos), inv, q_out, kp, vp, kv.block_table, page_size, 12, 2, 128, style)
    name = "neox" if style else "interleaved"
    for b in range(B):
        qr = M.rope(qkv[b, :1536], int(pos[b]), 128, 1e6, name)
        kr = M.rope(qkv[b, 1536:1792], int(pos[b]), 128, 1e6, name)
        assert_close(q_out[b].cpu().numpy(), qr, abs_tol=2e-3, what="q rope")
        kk, vv = kv.read_positions(b, 0, int(pos[b]) + 1)
        assert_close(kk[-1].cpu().numpy(), kr, abs_tol=2e-3, what="k append")
        assert f16_bits_equal(vv[-1].cpu().numpy(), qkv[b, 1792:])
    buf = torch.zeros(B * 1536 + 8, dtype=torch.float16, device="cuda")
    q_mis = buf[1:1 + B * 1536].view(B, 1536)  # 2-byte aligned: the element-wise kernel
    kp2, vp2 = kv2.layer(0)
    K.rope_kv_append(_t(qkv), _t(pos), inv, q_mis, kp2, vp2, kv2.block_table, page_size, 12, 2, 128, style)
    torch.cuda.synchronize()
    assert torch.equal(q_mis.view(torch.int16), q_out.view(torch.int16))
    assert torch.equal(kp2.view(torch.int16), kp.view(torch.int16))
    assert torch.equal(vp2.view(torch.int16), vp.view(torch.int16))


def test_q4_pack_device_bit_exact(cuda):
    import os
    from llamamps_b200 import kernels as K
    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", "pack_cases.npz"))
    for name in ["normal_64x96", "odd_7x33", "kproj_64x1536", "edge_4x32"]:
        p, s = K.q4_pack_device(_t(gold[name + "__w"].reshape(-1)))
        assert np.array_equal(p.cpu().numpy(), gold[name + "__packed"]), name
        assert f16_bits_equal(s.cpu().numpy(), gold[name + "__scales"]), name
    rng = np.random.default_rng(81)
    w = rng.normal(0, 0.02, (8960, 1536)).astype(np.float32)
    p, s = K.q4_pack_device(_t(w.reshape(-1)))
    rp, rs = M.q4_pack(w)
    assert np.array_equal(p.cpu().numpy(), rp) and f16_bits_equal(s.cpu().numpy(), rs)


@pytest.mark.parametrize("T_list,max_seq,n_splits", [([5, 16, 40], 64, 1), ([65, 1, 200], 256, 3), ([130, 7], 192, 2)])
def test_attention_rope_equals_rope_append_then_attention(cuda, T_list, max_seq, n_splits):
    """The one-launch RoPE + KV append + attention against lmps_rope_kv_append
    followed by lmps_gqa_decode_attention: same output and same cache, bit for
    bit (the new position is the last one of each sequence)."""
    from llamamps_b200 import kernels as K
    from llamamps_b200.engine import rope_inv_freq
    rng = np.random.default_rng(sum(T_list) + n_splits)
    B, ps = len(T_list), 64
    pos_np = np.array([t - 1 for t in T_list], np.int32)
    kv_a, _ = _paged_setup(rng, B, [max(t - 1, 1) for t in T_list], ps, max_seq)
    kv_b, _ = _paged_setup(np.random.default_rng(sum(T_list) + n_splits), B, [max(t - 1, 1) for t in T_list], ps,
                           max_seq)
    qkv = _t(rng.normal(0, 1, (B, 2048)).astype(np.float16))
    pos, seq_lens = _t(pos_np), _t(pos_np + 1)
    inv = torch.from_numpy(rope_inv_freq(128, 1e6)).cuda()
    ws = torch.zeros(max(16, K.attention_workspace_size(B, 12, 128, n_splits)), dtype=torch.uint8, device="cuda")
    ka, va = kv_a.layer(0)
    q = torch.empty(B, 1536, dtype=torch.float16, device="cuda")
    K.rope_kv_append(qkv, pos, inv, q, ka, va, kv_a.block_table, ps, 12, 2, 128)
    ref = torch.empty(B, 1536, dtype=torch.float16, device="cuda")
    K.gqa_decode_attention(q, ka, va, kv_a.block_table, seq_lens, ref, ws, ps, 12, 2, 128, kv_a.max_seq_len, n_splits)
    kb, vb = kv_b.layer(0)
    got = torch.empty(B, 1536, dtype=torch.float16, device="cuda")
    K.gqa_decode_attention_rope(qkv, pos, inv, kb, vb, kv_b.block_table, seq_lens, got, ws, ps, 12, 2, 128,
                                kv_b.max_seq_len, n_splits)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    assert torch.equal(kb.view(torch.int16), ka.view(torch.int16))
    assert torch.equal(vb.view(torch.int16), va.view(torch.int16))
