"""lmps_gqa_decode_attention_noalloc against lmps_gqa_decode_attention.

The no-allocation entry point exists for callers that cannot allocate device
memory where they call the attention (a binding that only receives device
pointers from another runtime, code under a global-mode stream capture, a
serving loop that bans allocation after warm-up).  It keeps the split
partials in a fixed 4 MiB array inside the library instead of a workspace
the caller passes.  Both entry points are called here through the C ABI on
the same inputs; the outputs must agree within the attention tolerance of the
other parity tests, on two consecutive calls with different inputs (the
array keeps the first call's partials when the second one starts).

This file sorts last so that a run stopping at its first failure has already
run every other test.
"""
import numpy as np
import pytest
import torch

from tests._util import assert_close

pytestmark = pytest.mark.gpu

ATTN_TOL = 5e-3   # the tolerance test_kernels_gpu.py uses for attention outputs
HQ, HKV, HD = 12, 2, 128


def _cache(rng, lens, page_size, max_seq):
    from llamamps_b200.config import QWEN2_5_1_5B
    from llamamps_b200.kv_cache import PagedKVCache
    B = len(lens)
    pps = (max_seq + page_size - 1) // page_size
    kv = PagedKVCache(QWEN2_5_1_5B, 1, B, max_seq, page_size, "cuda",
                      page_order=list(rng.permutation(B * pps)))
    for b, T in enumerate(lens):
        kv.reserve(b, max_seq)
        k = torch.from_numpy(rng.normal(0, 1, (T, HKV * HD)).astype(np.float16))
        v = torch.from_numpy(rng.normal(0, 1, (T, HKV * HD)).astype(np.float16))
        kv.write_positions(b, 0, 0, k, v)
    return kv


def _both(L, kv, q, seq_lens, n_splits):
    B = q.shape[0]
    kp, vp = kv.layer(0)
    stream = torch.cuda.current_stream().cuda_stream
    ws_bytes = L.lmps_gqa_attention_workspace_size(B, HQ, HD, n_splits)
    ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
    ref = torch.zeros(B, HQ * HD, dtype=torch.float16, device="cuda")
    st = L.lmps_gqa_decode_attention(q.data_ptr(), kp.data_ptr(), vp.data_ptr(), kv.block_table.data_ptr(),
                                     seq_lens.data_ptr(), ref.data_ptr(), ws.data_ptr(), ws_bytes,
                                     kv.block_table.shape[1], kv.page_size, HQ, HKV, HD, B,
                                     kv.max_seq_len, n_splits, stream)
    assert st == 0
    got = torch.full((B, HQ * HD), 7.0, dtype=torch.float16, device="cuda")
    st = L.lmps_gqa_decode_attention_noalloc(q.data_ptr(), kp.data_ptr(), vp.data_ptr(),
                                             kv.block_table.data_ptr(), seq_lens.data_ptr(),
                                             got.data_ptr(), kv.block_table.shape[1], kv.page_size,
                                             HQ, HKV, HD, B, kv.max_seq_len, n_splits, stream)
    assert st == 0
    torch.cuda.synchronize()
    return got.cpu().numpy(), ref.cpu().numpy()


def test_noalloc_attention_matches_workspace_entry_point_twice(cuda):
    from llamamps_b200._lib import lib
    L = lib()
    rng = np.random.default_rng(2024)
    # call 1: three sequences, several splits per sequence
    kv1 = _cache(rng, [300, 77, 129], 64, 384)
    q1 = torch.from_numpy(rng.normal(0, 1, (3, HQ * HD)).astype(np.float16)).cuda()
    sl1 = torch.tensor([300, 77, 129], dtype=torch.int32, device="cuda")
    splits1 = L.lmps_gqa_attention_splits(3, HKV, kv1.max_seq_len, 64)
    assert splits1 > 1
    got, ref = _both(L, kv1, q1, sl1, splits1)
    assert_close(got, ref, abs_tol=ATTN_TOL, what="no-alloc attention, call 1")
    # call 2 right after: different batch, lengths and split count
    kv2 = _cache(rng, [1, 4097], 64, 4160)
    q2 = torch.from_numpy(rng.normal(0, 1, (2, HQ * HD)).astype(np.float16)).cuda()
    sl2 = torch.tensor([1, 4097], dtype=torch.int32, device="cuda")
    splits2 = L.lmps_gqa_attention_splits(2, HKV, kv2.max_seq_len, 64)
    assert splits2 > 1 and splits2 != splits1
    got, ref = _both(L, kv2, q2, sl2, splits2)
    assert_close(got, ref, abs_tol=ATTN_TOL, what="no-alloc attention, call 2")


def test_noalloc_attention_rejects_requests_beyond_its_scratch(cuda):
    from llamamps_b200._lib import lib
    L = lib()
    limit = 4 * 1024 * 1024
    # 8 sequences x 12 heads x 1024 splits of 520-byte partials is ~51 MB
    assert L.lmps_gqa_attention_workspace_size(8, HQ, HD, 1024) > limit
    dummy = torch.zeros(16, dtype=torch.float16, device="cuda")
    p = dummy.data_ptr()
    st = L.lmps_gqa_decode_attention_noalloc(p, p, p, p, p, p, 1024, 64, HQ, HKV, HD, 8, 65536, 1024,
                                             torch.cuda.current_stream().cuda_stream)
    assert st == -3  # LMPS_ERR_WORKSPACE: nothing launched
    assert "workspace" in L.lmps_status_string(st).decode()
