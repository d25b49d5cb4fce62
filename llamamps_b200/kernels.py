"""Torch-tensor front end of the C ABI: shape/dtype checks, then one call.

Each function mirrors one reference kernel (named in its docstring) and
launches on torch's current CUDA stream, so the calls compose with torch
streams and can be captured into CUDA graphs.  Outputs may be passed in
(``out=``) so that a decode step allocates nothing.
"""
from __future__ import annotations

from typing import Optional

import torch

from ._lib import call, lib

FP16 = torch.float16


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dev(t: torch.Tensor, name: str, dtype=None):
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the decode path has no CPU fallback)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name}: expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.data_ptr()


def _x2d(x: torch.Tensor):
    x2 = x if x.dim() == 2 else x.reshape(1, -1)
    return x2, x2.shape[0]


def gemv_q4(packed, scales, x, rows: int, k: int, out: Optional[torch.Tensor] = None):
    """kernels/quant_matmul.metal `gemv_q4_0`: y[b] = W x[b] (fp32 accumulate)."""
    x2, B = _x2d(x)
    y = out if out is not None else torch.empty(B, rows, dtype=FP16, device=x.device)
    call("lmps_gemv_q4_0", _dev(packed, "packed", torch.uint8), _dev(scales, "scales", FP16),
         _dev(x2, "x", FP16), k, _dev(y, "y", FP16), rows, rows, k, B, _stream())
    return y if x.dim() == 2 else y.reshape(-1)


def gemv_q4_bias(packed, scales, bias, x, rows: int, k: int, out=None):
    x2, B = _x2d(x)
    y = out if out is not None else torch.empty(B, rows, dtype=FP16, device=x.device)
    call("lmps_gemv_q4_bias", _dev(packed, "packed", torch.uint8), _dev(scales, "scales", FP16),
         _dev(bias, "bias", FP16), _dev(x2, "x", FP16), k, _dev(y, "y", FP16), rows, rows, k, B,
         _stream())
    return y if x.dim() == 2 else y.reshape(-1)


def gemv_q4_residual(packed, scales, x, residual, rows: int, k: int, out=None):
    """GEMV + kernels/residual.metal: out = residual + fp16(W x).  out may be residual."""
    x2, B = _x2d(x)
    r2 = residual if residual.dim() == 2 else residual.reshape(1, -1)
    y = out if out is not None else torch.empty(B, rows, dtype=FP16, device=x.device)
    call("lmps_gemv_q4_residual", _dev(packed, "packed", torch.uint8), _dev(scales, "scales", FP16),
         _dev(x2, "x", FP16), k, _dev(r2, "residual", FP16), _dev(y, "y", FP16), rows, rows, k, B,
         _stream())
    return y if x.dim() == 2 else y.reshape(-1)


def gemv_q4_swiglu(gate_packed, gate_scales, up_packed, up_scales, x, rows: int, k: int, out=None):
    """gate/up GEMVs + kernels/swiglu.metal in one pass."""
    x2, B = _x2d(x)
    y = out if out is not None else torch.empty(B, rows, dtype=FP16, device=x.device)
    call("lmps_gemv_q4_swiglu", _dev(gate_packed, "gate_packed", torch.uint8),
         _dev(gate_scales, "gate_scales", FP16), _dev(up_packed, "up_packed", torch.uint8),
         _dev(up_scales, "up_scales", FP16), _dev(x2, "x", FP16), k, _dev(y, "y", FP16), rows,
         rows, k, B, _stream())
    return y if x.dim() == 2 else y.reshape(-1)


def lm_head_argmax(packed, scales, x, rows: int, k: int, keys: torch.Tensor, ids: torch.Tensor,
                   logits: Optional[torch.Tensor] = None):
    """runners/engine.py:171-181 on the device: Q4 LM head + first-index argmax."""
    x2, B = _x2d(x)
    call("lmps_lm_head_argmax", _dev(packed, "packed", torch.uint8), _dev(scales, "scales", FP16),
         _dev(x2, "x", FP16), k, _dev(logits, "logits", FP16) if logits is not None else None,
         _dev(keys, "keys", torch.int64), _dev(ids, "ids", torch.int32), rows, k, B, _stream())
    return ids


def rms_norm(x, gamma, eps: float = 1e-6, out=None):
    """kernels/rms_norm.metal `rms_norm_q4` (full-vector reduction)."""
    x2, B = _x2d(x)
    y = out if out is not None else torch.empty_like(x2)
    call("lmps_rms_norm", _dev(x2, "x", FP16), _dev(gamma, "gamma", FP16), _dev(y, "out", FP16),
         x2.shape[1], B, float(eps), _stream())
    return y if x.dim() == 2 else y.reshape(-1)


def rope_(vec, pos, inv_freq, n_heads: int, head_dim: int, style: int = 0):
    """kernels/rope.metal `apply_rope_q4`, in place, per-row position."""
    v2, B = _x2d(vec)
    call("lmps_rope", _dev(v2, "vec", FP16), _dev(pos, "pos", torch.int32),
         _dev(inv_freq, "inv_freq", torch.float32), n_heads, head_dim, B, style, _stream())
    return vec


def residual_add(x, y, out=None):
    o = out if out is not None else torch.empty_like(x)
    call("lmps_residual_add", _dev(x, "x", FP16), _dev(y, "y", FP16), _dev(o, "out", FP16),
         x.numel(), _stream())
    return o


def swiglu(gate, up, out=None):
    o = out if out is not None else torch.empty_like(gate)
    call("lmps_swiglu", _dev(gate, "gate", FP16), _dev(up, "up", FP16), _dev(o, "out", FP16),
         gate.numel(), _stream())
    return o


def swiglu_rows(gate_up, n: int, out):
    """out[r] = silu(gate_up[r, :n]) * gate_up[r, n:2n] (a fused gate|up GEMM output)."""
    call("lmps_swiglu_rows", _dev(gate_up, "gate_up", FP16), gate_up.shape[-1], gate_up.shape[0], n,
         _dev(out, "out", FP16), out.shape[-1], _stream())
    return out


def embed_gather(table, ids, out, bad: Optional[torch.Tensor] = None):
    V, D = table.shape
    call("lmps_embed_gather", _dev(table, "table", FP16), _dev(ids, "ids", torch.int32),
         _dev(out, "out", FP16), D, V, ids.numel(),
         _dev(bad, "bad", torch.int32) if bad is not None else None, _stream())
    return out


def attention_scores(q, k_cache, seq_len: int, n_q_heads: int, n_kv_heads: int, head_dim: int, out=None):
    s = out if out is not None else torch.empty(n_q_heads, seq_len, dtype=torch.float32, device=q.device)
    call("lmps_attention_scores", _dev(q, "q", FP16), _dev(k_cache, "k_cache", FP16),
         _dev(s, "scores", torch.float32), seq_len, n_q_heads, n_kv_heads, head_dim, _stream())
    return s


def softmax_(scores, seq_len: int, n_heads: int):
    call("lmps_softmax", _dev(scores, "scores", torch.float32), seq_len, n_heads, _stream())
    return scores


def attn_weighted_sum(scores, v_cache, seq_len: int, n_q_heads: int, n_kv_heads: int, head_dim: int, out=None):
    o = out if out is not None else torch.empty(n_q_heads * head_dim, dtype=FP16, device=scores.device)
    call("lmps_attn_weighted_sum", _dev(scores, "scores", torch.float32), _dev(v_cache, "v_cache", FP16),
         _dev(o, "out", FP16), seq_len, n_q_heads, n_kv_heads, head_dim, _stream())
    return o


def rope_kv_append(qkv, pos, inv_freq, q_out, k_pool, v_pool, block_table, page_size: int,
                   n_q_heads: int, n_kv_heads: int, head_dim: int, style: int = 0):
    B = qkv.shape[0]
    call("lmps_rope_kv_append", _dev(qkv, "qkv", FP16), _dev(pos, "pos", torch.int32),
         _dev(inv_freq, "inv_freq", torch.float32), _dev(q_out, "q_out", FP16),
         _dev(k_pool, "k_pool", FP16), _dev(v_pool, "v_pool", FP16),
         _dev(block_table, "block_table", torch.int32), block_table.shape[1], page_size,
         n_q_heads, n_kv_heads, head_dim, B, style, _stream())
    return q_out


def gqa_decode_attention_rope(qkv, pos, inv_freq, k_pool, v_pool, block_table, seq_lens, out, workspace,
                              page_size: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
                              max_seq_len: int, n_splits: int, style: int = 0):
    """rope_kv_append + gqa_decode_attention in one launch (seq_lens = pos + 1)."""
    B = qkv.shape[0]
    ws_ptr = workspace.data_ptr() if workspace is not None and workspace.numel() else None
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    call("lmps_gqa_decode_attention_rope", _dev(qkv, "qkv", FP16), _dev(pos, "pos", torch.int32),
         _dev(inv_freq, "inv_freq", torch.float32), style, _dev(k_pool, "k_pool", FP16),
         _dev(v_pool, "v_pool", FP16), _dev(block_table, "block_table", torch.int32),
         _dev(seq_lens, "seq_lens", torch.int32), _dev(out, "out", FP16), ws_ptr, ws_bytes,
         block_table.shape[1], page_size, n_q_heads, n_kv_heads, head_dim, B, max_seq_len, n_splits, _stream())
    return out


def attention_splits(batch: int, n_kv_heads: int, max_seq_len: int, page_size: int) -> int:
    return int(lib().lmps_gqa_attention_splits(batch, n_kv_heads, max_seq_len, page_size))


def attention_workspace_size(batch: int, n_q_heads: int, head_dim: int, n_splits: int) -> int:
    return int(lib().lmps_gqa_attention_workspace_size(batch, n_q_heads, head_dim, n_splits))


def gqa_decode_attention(q, k_pool, v_pool, block_table, seq_lens, out, workspace,
                         page_size: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
                         max_seq_len: int, n_splits: int):
    """Fused attention.metal + softmax.metal + attn_sum.metal over the paged cache."""
    B = q.shape[0]
    ws_ptr = workspace.data_ptr() if workspace is not None and workspace.numel() else None
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    call("lmps_gqa_decode_attention", _dev(q, "q", FP16), _dev(k_pool, "k_pool", FP16),
         _dev(v_pool, "v_pool", FP16), _dev(block_table, "block_table", torch.int32),
         _dev(seq_lens, "seq_lens", torch.int32), _dev(out, "out", FP16), ws_ptr, ws_bytes,
         block_table.shape[1], page_size, n_q_heads, n_kv_heads, head_dim, B, max_seq_len,
         n_splits, _stream())
    return out


def q4_pack_device(w: torch.Tensor):
    """utils/pack_weights.py `pack_tensor_4bit` on the device (bit-exact)."""
    n = w.numel()
    groups = (n + 31) // 32
    packed = torch.empty(groups * 16, dtype=torch.uint8, device=w.device)
    scales = torch.empty(groups, dtype=FP16, device=w.device)
    call("lmps_q4_pack", _dev(w, "w", torch.float32), n, packed.data_ptr(), scales.data_ptr(), _stream())
    return packed, scales


def decode_advance(next_ids, tokens, pos, seq_lens, history=None, step=None):
    B = tokens.numel()
    max_steps = history.shape[0] if history is not None else 0
    call("lmps_decode_advance", _dev(next_ids, "next", torch.int32), _dev(tokens, "tokens", torch.int32),
         _dev(pos, "pos", torch.int32), _dev(seq_lens, "seq_lens", torch.int32),
         _dev(history, "history", torch.int32) if history is not None else None,
         _dev(step, "step", torch.int32) if step is not None else None, max_steps, B, _stream())


EPI_NONE, EPI_BIAS, EPI_RESIDUAL, EPI_SWIGLU = 0, 1, 2, 3


def w4a16_gemm_workspace_size(m: int, n: int) -> int:
    return int(lib().lmps_w4a16_gemm_workspace_size(m, n))


def w4a16_gemm(x, packed, scales, n: int, k: int, *, bias=None, residual=None, swiglu: bool = False, out=None,
               error: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None):
    """tcgen05 W4A16 GEMM: out[m] = x[m] . W^T (+ bias | residual + fp16(.)).

    x is fp16 [m, k] (token-major); W the Q4 [n, k] layout.  Used where the
    projections of many tokens at once are dense contractions (prefill, large
    batches).  ``swiglu``: W's rows interleave gate and up rows and out[m, t] =
    SwiGLU(gate row t, up row t), n / 2 columns (interleave_rows builds W).
    Calls with m < 128 split K inside a thread-block cluster; ``workspace`` is
    accepted for API stability and unused."""
    x2, m = _x2d(x)
    y = out if out is not None else torch.empty(m, n // 2 if swiglu else n, dtype=FP16, device=x.device)
    epi, b_ptr, r_ptr, ldr = (EPI_SWIGLU if swiglu else EPI_NONE), None, None, 0
    if swiglu and (bias is not None or residual is not None):
        raise ValueError("the SwiGLU epilogue takes no bias or residual")
    if bias is not None:
        epi, b_ptr = EPI_BIAS, _dev(bias, "bias", FP16)
    if residual is not None:
        if bias is not None:
            raise ValueError("bias and residual epilogues are exclusive")
        r2 = residual if residual.dim() == 2 else residual.reshape(1, -1)
        epi, r_ptr, ldr = EPI_RESIDUAL, _dev(r2, "residual", FP16), r2.shape[1]
    err = error if error is not None else torch.zeros(1, dtype=torch.int32, device=x.device)
    ws_ptr, ws_bytes = None, 0
    if workspace is not None and workspace.numel() > 0:
        ws_ptr, ws_bytes = _dev(workspace, "workspace", torch.uint8), workspace.numel()
    call("lmps_w4a16_gemm", _dev(x2, "x", FP16), x2.shape[1], _dev(packed, "packed", torch.uint8),
         _dev(scales, "scales", FP16), b_ptr, r_ptr, ldr, _dev(y, "y", FP16), y.shape[-1], m, n, k, epi,
         _dev(err, "error", torch.int32), ws_ptr, ws_bytes, _stream())
    return y


def argmax_rows(logits, n: int, ids):
    """First-index argmax of each fp16 row of logits[:, :n] into int32 ids."""
    call("lmps_argmax_rows", _dev(logits, "logits", FP16), logits.shape[-1], logits.shape[0], n,
         _dev(ids, "ids", torch.int32), _stream())
    return ids


def sample_rows(logits, n: int, top_k: int, temperature: float, seed: int, offset: int, ids, ids2=None):
    """Top-k / temperature sample of each fp16 row of logits[:, :n] into int32
    ids (and ids2): seeded Philox draw, reproducible (see include/llamamps_b200.h)."""
    call("lmps_sample_rows", _dev(logits, "logits", FP16), logits.shape[-1], logits.shape[0], n, int(top_k),
         float(temperature), int(seed) & 0xFFFFFFFFFFFFFFFF, int(offset) & 0xFFFFFFFFFFFFFFFF,
         _dev(ids, "ids", torch.int32), _dev(ids2, "ids2", torch.int32) if ids2 is not None else None,
         _stream())
    return ids


def prefill_attention(q, k_pool, v_pool, block_table, out, batch: int, seq_len: int, page_size: int,
                      n_q_heads: int, n_kv_heads: int, head_dim: int, *, error: Optional[torch.Tensor] = None,
                      tcgen05: Optional[bool] = None):
    """Causal attention of every prompt position (q rows b*seq_len + p) over the paged cache.

    On the tcgen05 kernel (S and O in tensor memory, TMA-loaded K/V) where it
    takes the shape -- head_dim 128, page_size a multiple of 64, an even
    query-head group -- else on the mma.sync kernel; ``tcgen05`` forces one.
    ``error`` (int32 [1]) receives the tcgen05 kernel's wait-timeout flag."""
    fits = head_dim == 128 and page_size % 64 == 0 and (n_q_heads // n_kv_heads) % 2 == 0
    if tcgen05 is None:
        tcgen05 = fits
    if tcgen05:
        n_pages = k_pool.numel() // (n_kv_heads * page_size * head_dim)
        err = error if error is not None else torch.zeros(1, dtype=torch.int32, device=q.device)
        call("lmps_prefill_attention_tcgen05", _dev(q, "q", FP16), q.shape[-1], _dev(k_pool, "k_pool", FP16),
             _dev(v_pool, "v_pool", FP16), n_pages, _dev(block_table, "block_table", torch.int32),
             block_table.shape[1], page_size, _dev(out, "out", FP16), out.shape[-1], batch, seq_len, n_q_heads,
             n_kv_heads, head_dim, _dev(err, "error", torch.int32), _stream())
        return out
    call("lmps_prefill_attention", _dev(q, "q", FP16), q.shape[-1], _dev(k_pool, "k_pool", FP16),
         _dev(v_pool, "v_pool", FP16), _dev(block_table, "block_table", torch.int32), block_table.shape[1],
         page_size, _dev(out, "out", FP16), out.shape[-1], batch, seq_len, n_q_heads, n_kv_heads, head_dim,
         _stream())
    return out



# -- two-way tensor parallelism over peer memory ----------------------------
class PeerExchange:
    """This rank's exchange buffer and the peer's, mapped through CUDA IPC,
    for :func:`tp2_allreduce_residual` (``n_sites`` call sites of at most
    ``max_n`` fp16 elements).  ``handle()`` gives the 64 bytes to send to the
    peer, ``connect(peer_handle)`` maps the peer's buffer.  ``close()``
    unmaps and frees; call it on both ranks after a barrier, with no call in
    flight on either GPU."""

    def __init__(self, n_sites: int, max_n: int, device, wait_ns: int = 0):
        import ctypes
        self.n_sites, self.max_n, self.device = n_sites, max_n, torch.device(device)
        # limit of every wait for the peer, in GPU global-timer nanoseconds (0: 5 s)
        self.wait_ns = int(wait_ns)
        nbytes = lib().lmps_tp2_comm_bytes(n_sites, max_n)
        if nbytes == 0:
            raise ValueError("max_n must be a positive multiple of 8")
        with torch.cuda.device(self.device):
            p = ctypes.c_void_p()
            call("lmps_comm_alloc", nbytes, ctypes.byref(p))
            self.comm = p.value
            self.seen = torch.zeros(n_sites * 64, dtype=torch.int32, device=self.device)
        self.peer = None

    def handle(self) -> bytes:
        import ctypes
        buf = ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            call("lmps_ipc_handle", self.comm, buf)
        return buf.raw

    def connect(self, peer_handle: bytes) -> None:
        import ctypes
        if len(peer_handle) != 64:
            raise ValueError("an IPC handle is 64 bytes")
        p = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            call("lmps_ipc_open", ctypes.create_string_buffer(peer_handle, 64), ctypes.byref(p))
        self.peer = p.value

    def close(self) -> None:
        with torch.cuda.device(self.device):
            if self.peer is not None:
                call("lmps_ipc_close", self.peer)
                self.peer = None
            if self.comm is not None:
                call("lmps_comm_free", self.comm)
                self.comm = None


def tp2_allreduce_residual(part, x, ex: PeerExchange, site: int, error):
    """x <- x + (part + the peer's part) through the peer's mapped buffer.
    A wait for the peer longer than ``ex.wait_ns`` sets ``error``."""
    if ex.peer is None:
        raise RuntimeError("the peer exchange is not connected")
    call("lmps_tp2_allreduce_residual", _dev(part, "part", FP16), _dev(x, "x", FP16), part.numel(), ex.comm,
         ex.peer, _dev(ex.seen, "seen", torch.int32), site, ex.n_sites, ex.max_n,
         _dev(error, "error", torch.int32), ex.wait_ns, _stream())
    return x


def tp2_argmax_exchange(logits, local_ids, row_offset: int, ids, ex: PeerExchange, site: int, error):
    """The global first-index argmax of a vocabulary split between two ranks:
    this rank's fp16 logits [B, ld] and local argmax ids in, the winner over
    both ranks' rows (global row numbers) out, on both ranks."""
    if ex.peer is None:
        raise RuntimeError("the peer exchange is not connected")
    B = local_ids.numel()
    call("lmps_tp2_argmax_exchange", _dev(logits, "logits", FP16), logits.shape[-1],
         _dev(local_ids, "local_ids", torch.int32), B, int(row_offset), _dev(ids, "ids", torch.int32), ex.comm,
         ex.peer, _dev(ex.seen, "seen", torch.int32), site, ex.n_sites, ex.max_n, _dev(error, "error", torch.int32),
         ex.wait_ns, _stream())
    return ids


def gemv_q4_tp2_residual(packed, scales, a, rows: int, k: int, x, part, ex: PeerExchange, site: int, error):
    """One kernel: part = W a (this rank's K slice, fp16), stored into the
    peer's receive slot over NVLink, then x <- x + (part + the peer's part)
    after a per-CTA hand-off with the peer's same CTA."""
    if ex.peer is None:
        raise RuntimeError("the peer exchange is not connected")
    a2, B = _x2d(a)
    call("lmps_gemv_q4_tp2_residual", _dev(packed, "packed", torch.uint8), _dev(scales, "scales", FP16),
         _dev(a2, "a", FP16), a2.shape[1], _dev(x, "x", FP16), _dev(part, "part", FP16), rows, k, B, ex.comm,
         ex.peer, _dev(ex.seen, "seen", torch.int32), site, ex.n_sites, ex.max_n,
         _dev(error, "error", torch.int32), ex.wait_ns, _stream())
    return x

