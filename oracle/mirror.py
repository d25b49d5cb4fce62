"""numpy fp32 restatement of the LlamaMPS decode path (the oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  Imported by tests,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``; never by
the product package.

Every function cites the reference file:line it restates (paths relative to
the LlamaMPS project root).  Rounding follows the reference's buffer
boundaries: the engine's intermediate buffers are fp16
(``runners/engine.py:86-100``) except the attention scores, which are fp32
(``runners/engine.py:92``), so every stage output that lands in one of those
buffers is rounded to fp16 here, and all arithmetic in between is fp32.

Deliberate, documented departures from the literal Metal code (each is what
the reference intends or what the decode-loop specification requires):

* GEMV accumulates in fp32 (``quant_matmul.metal:34,46-50`` accumulates in
  fp16); the decode specification asks for fp32 accumulation.
* RMSNorm reduces over the whole vector (``rms_norm.metal:23-39`` is launched
  as two threadgroups and reads ``shared_sums[0..47]`` of a 32-entry array, so
  the Metal result is undefined; the intended math is the full-vector RMS).
* RoPE takes the position ``m`` and the base ``theta`` as parameters
  (``rope.metal:23,28`` hard-code m=0, base 1e4); at m=0 it is the identity,
  exactly as the reference.
* Attention reads a KV cache of ``T`` positions (``runners/engine.py:64`` fixes
  seq_len=1); q/k/v may carry a bias (Qwen2.5 has one; the reference does not
  load it, ``runners/engine.py:124-141``).  With a zero bias and T=1 these
  reduce to the reference.
"""
from __future__ import annotations

import dataclasses
from typing import Dict, List, Optional, Sequence

import numpy as np

F16 = np.float16
F32 = np.float32

# utils/pack_weights.py:9 -- BLOCK_SIZE
Q4_GROUP = 32
# kernels/attention.metal:40 -- the reference's literal 1/sqrt(128)
ATTN_SCALE = F32(0.088388)


@dataclasses.dataclass(frozen=True)
class OracleConfig:
    """Model constants; defaults are runners/engine.py:7-14 (Qwen2.5-1.5B)."""

    hidden: int = 1536            # engine.py:7 HIDDEN_DIM
    intermediate: int = 8960      # engine.py:8 MLP_INTERMEDIATE
    vocab: int = 151936           # engine.py:9 VOCAB_SIZE
    n_layers: int = 28            # engine.py:10 NUM_LAYERS
    n_q_heads: int = 12           # engine.py:11
    n_kv_heads: int = 2           # engine.py:12
    head_dim: int = 128           # engine.py:13
    eps: float = 1e-6             # rms_norm.metal:35-36
    rope_theta: float = 1e6       # Qwen2.5 (the reference hard-codes 1e4 at m=0)
    rope_style: str = "interleaved"   # rope.metal:19 adjacent pairs; "neox" = half split

    @property
    def kv_dim(self) -> int:      # engine.py:14 K_DIM
        return self.n_kv_heads * self.head_dim

    @property
    def q_dim(self) -> int:
        return self.n_q_heads * self.head_dim


# --------------------------------------------------------------------------
# Q4 format (utils/pack_weights.py)
# --------------------------------------------------------------------------

def q4_pack(w: np.ndarray):
    """Symmetric int4 quantisation, utils/pack_weights.py:18-46.

    The tensor is flattened row-major and zero-padded to a multiple of 32
    (``:18-20``), split into groups of 32 (``:22``); scale = max|w|/7 in fp32
    with 0 replaced by 1.0 (``:25-26``); code = round-half-even(w/scale)
    clamped to [-8, 7] (``:29``); stored +8 as a nibble (``:32``), element 2b
    in the low nibble of byte b and 2b+1 in the high nibble (``:34-36``); the
    scale is saved as fp16 (``:46``).
    Returns (packed uint8[n_pad/2], scales float16[n_pad/32]).
    """
    flat = np.asarray(w, dtype=F32).reshape(-1)
    pad = (Q4_GROUP - flat.size % Q4_GROUP) % Q4_GROUP
    if pad:
        flat = np.concatenate([flat, np.zeros(pad, F32)])
    blocks = flat.reshape(-1, Q4_GROUP)
    scales = (np.abs(blocks).max(axis=1) / F32(7.0)).astype(F32)
    scales[scales == 0] = F32(1.0)
    q = np.clip(np.round(blocks / scales[:, None]), -8, 7).astype(np.int8)
    u = (q.astype(np.int16) + 8).astype(np.uint8).reshape(-1)
    packed = (u[0::2] | (u[1::2] << 4)).astype(np.uint8)
    return packed, scales.astype(F16)


def q4_codes(packed: np.ndarray) -> np.ndarray:
    """Signed codes in element order: quant_matmul.metal:39-41 (low nibble = element 2b)."""
    p = np.asarray(packed, dtype=np.uint8).reshape(-1)
    out = np.empty(p.size * 2, dtype=np.int8)
    out[0::2] = (p & 0x0F).astype(np.int8) - 8
    out[1::2] = (p >> 4).astype(np.int8) - 8
    return out


def q4_dequant(packed: np.ndarray, scales: np.ndarray, rows: int, k: int) -> np.ndarray:
    """fp32 weights W[rows, k]; scale of element j of row r is
    scales[(r*k + j) // 32] (quant_matmul.metal:30-31,43-44)."""
    codes = q4_codes(packed)[: rows * k].astype(F32).reshape(rows, k // Q4_GROUP, Q4_GROUP)
    s = np.asarray(scales, dtype=F16).astype(F32).reshape(rows, k // Q4_GROUP, 1)
    return (codes * s).reshape(rows, k)


def gemv_q4(packed, scales, x, rows: int, k: int, w32: Optional[np.ndarray] = None) -> np.ndarray:
    """y[b, r] = sum_k dequant(W)[r, k] * x[b, k]; quant_matmul.metal:30-67.

    fp32 accumulation (see module docstring), output rounded to fp16 like the
    reference's fp16 output buffer.  ``w32`` may carry a cached dequantised
    matrix.  x: f16[B, k] or f16[k].
    """
    if w32 is None:
        w32 = q4_dequant(packed, scales, rows, k)
    x32 = np.asarray(x, dtype=F16).astype(F32)
    return (x32 @ w32.T).astype(F16)


# --------------------------------------------------------------------------
# Elementwise / normalisation kernels
# --------------------------------------------------------------------------

def rms_norm(x: np.ndarray, gamma: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """rms_norm.metal:20-39 (full-vector reduction, see module docstring):
    out = (half)(x * rsqrt(mean(x^2) + eps)) * gamma, the product in fp16."""
    v = np.asarray(x, dtype=F16).astype(F32)
    d = v.shape[-1]
    ss = np.sum(v * v, axis=-1, keepdims=True, dtype=F32)
    scale = (F32(1.0) / np.sqrt(ss / F32(d) + F32(eps))).astype(F32)
    normed = (v * scale).astype(F16)
    return (normed.astype(F32) * np.asarray(gamma, dtype=F16).astype(F32)).astype(F16)


def rope_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    """Per-pair frequency base^-(2i/head_dim) in fp32; rope.metal:28-30 with
    (idx % 128) = 2i for pair i of a head."""
    i2 = np.arange(0, head_dim, 2, dtype=F32)
    return np.power(F32(theta), -(i2 / F32(head_dim))).astype(F32)


def rope(vec: np.ndarray, pos, head_dim: int, theta: float, style: str = "interleaved") -> np.ndarray:
    """Rotate every head of ``vec`` (f16[..., H*head_dim]) by position ``pos``.

    rope.metal:19-40: pair (x1, x2) -> (x1 cos - x2 sin, x1 sin + x2 cos) in
    fp32, stored fp16.  ``interleaved`` pairs adjacent elements (2i, 2i+1) as
    the reference does; ``neox`` pairs (i, i + head_dim/2) as HF Qwen2 does.
    pos: scalar or one position per leading row.
    """
    v = np.asarray(vec, dtype=F16)
    lead = v.shape[:-1]
    nh = v.shape[-1] // head_dim
    v32 = v.astype(F32).reshape(*lead, nh, head_dim)
    inv = rope_inv_freq(head_dim, theta)
    m = np.asarray(pos, dtype=F32).reshape(*lead, 1, 1) if lead else F32(pos)
    ang = (m * inv).astype(F32)                      # [.., 1, half]
    c = np.cos(ang).astype(F32)
    s = np.sin(ang).astype(F32)
    if style == "interleaved":
        x1 = v32[..., 0::2]
        x2 = v32[..., 1::2]
    elif style == "neox":
        x1 = v32[..., : head_dim // 2]
        x2 = v32[..., head_dim // 2:]
    else:
        raise ValueError(f"unknown rope style {style!r}")
    r1 = (x1 * c - x2 * s).astype(F16)
    r2 = (x1 * s + x2 * c).astype(F16)
    out = np.empty(v32.shape, dtype=F16)
    if style == "interleaved":
        out[..., 0::2] = r1
        out[..., 1::2] = r2
    else:
        out[..., : head_dim // 2] = r1
        out[..., head_dim // 2:] = r2
    return out.reshape(v.shape)


def attention_scores(q: np.ndarray, k_cache: np.ndarray, n_q_heads: int = 12,
                     n_kv_heads: int = 2, head_dim: int = 128) -> np.ndarray:
    """attention.metal:22-40: s[h, i] = (q_h . K[i, h/group]) * 0.088388, fp32.
    q: f16[Hq*hd]; k_cache: f16[T, Hkv*hd] (row i = position i, attention.metal:33)."""
    group = n_q_heads // n_kv_heads
    q32 = np.asarray(q, dtype=F16).astype(F32).reshape(n_q_heads, head_dim)
    k32 = np.asarray(k_cache, dtype=F16).astype(F32).reshape(-1, n_kv_heads, head_dim)
    kh = k32[:, np.arange(n_q_heads) // group, :]            # [T, Hq, hd]
    dots = np.einsum("hd,thd->ht", q32, kh).astype(F32)
    return (dots * ATTN_SCALE).astype(F32)


def softmax(scores: np.ndarray) -> np.ndarray:
    """softmax.metal:23-36: max, exp(s - max), divide by the sum; fp32, per head row."""
    s = np.asarray(scores, dtype=F32)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m).astype(F32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)


def attn_weighted_sum(p: np.ndarray, v_cache: np.ndarray, n_q_heads: int = 12,
                      n_kv_heads: int = 2, head_dim: int = 128) -> np.ndarray:
    """attn_sum.metal:21-33: o[h*hd + d] = sum_i p[h, i] * V[i, h/group, d] -> fp16."""
    group = n_q_heads // n_kv_heads
    v32 = np.asarray(v_cache, dtype=F16).astype(F32).reshape(-1, n_kv_heads, head_dim)
    vh = v32[:, np.arange(n_q_heads) // group, :]            # [T, Hq, hd]
    o = np.einsum("ht,thd->hd", np.asarray(p, dtype=F32), vh).astype(F32)
    return o.reshape(-1).astype(F16)


def residual_add(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    """residual.metal:19: out = x + y in fp16."""
    return (np.asarray(x, F16).astype(F32) + np.asarray(y, F16).astype(F32)).astype(F16)


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """swiglu.metal:19-22: (g / (1 + exp(-g))) * u in fp32, stored fp16."""
    g = np.asarray(gate, F16).astype(F32)
    u = np.asarray(up, F16).astype(F32)
    with np.errstate(over="ignore"):
        silu = (g / (F32(1.0) + np.exp(-g))).astype(F32)
    return (silu * u).astype(F16)


def add_bias(y16: np.ndarray, acc32: np.ndarray, bias) -> np.ndarray:
    """Bias epilogue: f16(acc + b) with one rounding (Qwen2 q/k/v bias)."""
    if bias is None:
        return y16
    return (acc32 + np.asarray(bias, F16).astype(F32)).astype(F16)


# --------------------------------------------------------------------------
# Layer / model (runners/engine.py)
# --------------------------------------------------------------------------

LAYER_KEYS = ("q", "k", "v", "o", "gt", "up", "dn")   # engine.py:124-141 dict keys


class DequantCache:
    """Caches fp32 dequantised matrices so full-model oracle runs stay fast."""

    def __init__(self):
        self._c: Dict[int, np.ndarray] = {}

    def get(self, packed, scales, rows, k):
        key = id(packed)
        w = self._c.get(key)
        if w is None:
            w = q4_dequant(packed, scales, rows, k)
            self._c[key] = w
        return w


def _gemv_acc(lw, name, x16, rows, k, cache: Optional[DequantCache]):
    # scale arrays use the engine.py:124-141 key + "s" ("q"/"qs", "gt"/"gts", ...)
    packed, scales = lw[name], lw[name + "s"]
    w32 =cache.get(packed, scales, rows, k) if cache is not None else q4_dequant(packed, scales, rows, k)
    return np.asarray(x16, F16).astype(F32) @ w32.T


class KVCache:
    """Per-sequence, per-layer contiguous K/V rows f16[T, Hkv*hd]: the layout
    attention.metal:33 / attn_sum.metal:30 index (row i = position i)."""

    def __init__(self, n_layers: int, kv_dim: int):
        self.k: List[List[np.ndarray]] = [[] for _ in range(n_layers)]
        self.v: List[List[np.ndarray]] = [[] for _ in range(n_layers)]
        self.kv_dim = kv_dim

    def length(self, layer: int = 0) -> int:
        return len(self.k[layer])

    def set_prefix(self, layer: int, k_rows: np.ndarray, v_rows: np.ndarray):
        self.k[layer] = [r.astype(F16) for r in np.asarray(k_rows, F16).reshape(-1, self.kv_dim)]
        self.v[layer] = [r.astype(F16) for r in np.asarray(v_rows, F16).reshape(-1, self.kv_dim)]

    def append(self, layer: int, pos: int, k_row: np.ndarray, v_row: np.ndarray):
        if pos != len(self.k[layer]):
            raise ValueError(f"append at {pos} but cache holds {len(self.k[layer])} rows")
        self.k[layer].append(np.asarray(k_row, F16).copy())
        self.v[layer].append(np.asarray(v_row, F16).copy())

    def rows(self, layer: int):
        return np.stack(self.k[layer]), np.stack(self.v[layer])


def decoder_layer(x: np.ndarray, lw: dict, cache: KVCache, layer: int, pos: int,
                  cfg: OracleConfig, dq: Optional[DequantCache] = None,
                  trace: Optional[dict] = None) -> np.ndarray:
    """One decoder layer for one sequence, runners/engine.py:187-243.

    x: f16[D] residual (``buf_residual``).  Appends this token's k/v at
    ``pos`` and attends over positions 0..pos.  Returns the new residual.
    """
    D, hd = cfg.hidden, cfg.head_dim
    # engine.py:188-190 rmsnorm(residual, in_norm) -> attn_normed
    xn = rms_norm(x, lw["in_norm"], cfg.eps)
    # engine.py:192-195 q/k/v GEMVs (+ bias, BASELINE extension)
    accq = _gemv_acc(lw, "q", xn, cfg.q_dim, D, dq)
    acck = _gemv_acc(lw, "k", xn, cfg.kv_dim, D, dq)
    accv = _gemv_acc(lw, "v", xn, cfg.kv_dim, D, dq)
    q = add_bias(accq.astype(F16), accq, lw.get("bq"))
    k = add_bias(acck.astype(F16), acck, lw.get("bk"))
    v = add_bias(accv.astype(F16), accv, lw.get("bv"))
    # engine.py:198-200 RoPE on q and k in place
    q = rope(q, pos, hd, cfg.rope_theta, cfg.rope_style)
    k = rope(k, pos, hd, cfg.rope_theta, cfg.rope_style)
    cache.append(layer, pos, k, v)
    kc, vc = cache.rows(layer)
    # engine.py:202-212 scores -> softmax -> weighted sum
    s = attention_scores(q, kc, cfg.n_q_heads, cfg.n_kv_heads, hd)
    p = softmax(s)
    attn = attn_weighted_sum(p, vc, cfg.n_q_heads, cfg.n_kv_heads, hd)
    # engine.py:215-221 o_proj + residual
    o = _gemv_acc(lw, "o", attn, D, cfg.q_dim, dq).astype(F16)
    x1 = residual_add(x, o)
    # engine.py:224-235 post-norm, gate/up, swiglu
    hn = rms_norm(x1, lw["post_norm"], cfg.eps)
    g = _gemv_acc(lw, "gt", hn, cfg.intermediate, D, dq).astype(F16)
    u = _gemv_acc(lw, "up", hn, cfg.intermediate, D, dq).astype(F16)
    a = swiglu(g, u)
    # engine.py:237-243 down_proj + residual
    d = _gemv_acc(lw, "dn", a, D, cfg.intermediate, dq).astype(F16)
    x2 = residual_add(x1, d)
    if trace is not None:
        trace.update(xn=xn, q=q, k=k, v=v, scores=s, p=p, attn=attn, o=o, x1=x1,
                     hn=hn, g=g, u=u, a=a, d=d, x2=x2)
    return x2


def final_logits(x: np.ndarray, final_norm: np.ndarray, lm_packed, lm_scales,
                 cfg: OracleConfig, dq: Optional[DequantCache] = None) -> np.ndarray:
    """runners/engine.py:164-178: rmsnorm(final gamma) then the Q4 LM-head GEMV -> f16[V]."""
    xf = rms_norm(x, final_norm, cfg.eps)
    w = dq.get(lm_packed, lm_scales, cfg.vocab, cfg.hidden) if dq is not None else \
        q4_dequant(lm_packed, lm_scales, cfg.vocab, cfg.hidden)
    return (np.asarray(xf, F16).astype(F32) @ w.T).astype(F16)


def predict_next_token(logits: np.ndarray) -> int:
    """runners/engine.py:180-181: argmax over fp32(logits); first index on ties."""
    return int(np.argmax(np.asarray(logits).astype(F32)))


def top2_margin(logits: np.ndarray) -> float:
    """Gap between the largest and second-largest logit (greedy-parity gate)."""
    l32 = np.asarray(logits).astype(F32)
    top = np.partition(l32, -2)[-2:]
    return float(top[1] - top[0])


def embed_row(embed: np.ndarray, token_id: int, hidden: int) -> np.ndarray:
    """utils/tokenizer.py:22-26: row ``token_id`` of the fp16 [V, D] table."""
    return np.asarray(embed, F16).reshape(-1, hidden)[int(token_id)].copy()


class OracleModel:
    """The whole decode path for one sequence: runners/engine.py:157-181 with a
    KV cache.  ``weights`` = {"layers": [layer dicts], "final_norm", "lm_packed",
    "lm_scales", "embed"}."""

    def __init__(self, weights: dict, cfg: OracleConfig):
        self.w = weights
        self.cfg = cfg
        self.dq = DequantCache()
        self.cache = KVCache(len(weights["layers"]), cfg.kv_dim)
        self.pos = 0

    def step_vector(self, x: np.ndarray) -> np.ndarray:
        """run_inference (engine.py:157-178) on one embedding vector at self.pos."""
        x = np.asarray(x, F16)
        for li, lw in enumerate(self.w["layers"]):
            x = decoder_layer(x, lw, self.cache, li, self.pos, self.cfg, self.dq)
        self.pos += 1
        return final_logits(x, self.w["final_norm"], self.w["lm_packed"],
                            self.w["lm_scales"], self.cfg, self.dq)

    def step_token(self, token_id: int) -> np.ndarray:
        return self.step_vector(embed_row(self.w["embed"], token_id, self.cfg.hidden))

    def generate(self, prompt_ids: Sequence[int], max_new_tokens: int,
                 record: Optional[list] = None) -> List[int]:
        """Greedy decode loop: prompt tokens one by one (causal), then argmax feedback."""
        logits = None
        for t in prompt_ids:
            logits = self.step_token(int(t))
        out: List[int] = []
        for i in range(max_new_tokens):
            nxt = predict_next_token(logits)
            if record is not None:
                record.append(logits)
            out.append(nxt)
            if i + 1 < max_new_tokens:
                logits = self.step_token(nxt)
        return out


class OracleBatch:
    """``batch`` independent sequences stepped together: row b is exactly the
    computation of :class:`OracleModel` on sequence b alone (every stage is
    row-wise; runners/engine.py:157-181 per row), but the Q4 projections of all
    rows run as one matrix product per matrix, so full-shape batches (64
    sequences, 128-id prompts) stay affordable on the host.  Each sequence has
    its own KV cache and position."""

    def __init__(self, weights: dict, cfg: OracleConfig, batch: int):
        self.w = weights
        self.cfg = cfg
        self.batch = batch
        self.dq = DequantCache()
        self.caches = [KVCache(len(weights["layers"]), cfg.kv_dim) for _ in range(batch)]
        self.pos = np.zeros(batch, dtype=np.int64)

    def _layer(self, x: np.ndarray, lw: dict, li: int) -> np.ndarray:
        cfg, D, hd, dq = self.cfg, self.cfg.hidden, self.cfg.head_dim, self.dq
        xn = rms_norm(x, lw["in_norm"], cfg.eps)                       # engine.py:188-190
        accq = _gemv_acc(lw, "q", xn, cfg.q_dim, D, dq)                # engine.py:192-195
        acck = _gemv_acc(lw, "k", xn, cfg.kv_dim, D, dq)
        accv = _gemv_acc(lw, "v", xn, cfg.kv_dim, D, dq)
        q = add_bias(accq.astype(F16), accq, lw.get("bq"))
        k = add_bias(acck.astype(F16), acck, lw.get("bk"))
        v = add_bias(accv.astype(F16), accv, lw.get("bv"))
        q = rope(q, self.pos, hd, cfg.rope_theta, cfg.rope_style)     # engine.py:198-200
        k = rope(k, self.pos, hd, cfg.rope_theta, cfg.rope_style)
        attn = np.empty((self.batch, cfg.q_dim), dtype=F16)
        for b, cache in enumerate(self.caches):                        # engine.py:202-212
            cache.append(li, int(self.pos[b]), k[b], v[b])
            kc, vc = cache.rows(li)
            p = softmax(attention_scores(q[b], kc, cfg.n_q_heads, cfg.n_kv_heads, hd))
            attn[b] = attn_weighted_sum(p, vc, cfg.n_q_heads, cfg.n_kv_heads, hd)
        o = _gemv_acc(lw, "o", attn, D, cfg.q_dim, dq).astype(F16)    # engine.py:215-221
        x1 = residual_add(x, o)
        hn = rms_norm(x1, lw["post_norm"], cfg.eps)                    # engine.py:224-235
        g = _gemv_acc(lw, "gt", hn, cfg.intermediate, D, dq).astype(F16)
        u = _gemv_acc(lw, "up", hn, cfg.intermediate, D, dq).astype(F16)
        a = swiglu(g, u)
        d = _gemv_acc(lw, "dn", a, D, cfg.intermediate, dq).astype(F16)  # engine.py:237-243
        return residual_add(x1, d)

    def step_tokens(self, ids) -> np.ndarray:
        """One token per sequence at its current position -> fp16 logits [batch, V]."""
        x = np.stack([embed_row(self.w["embed"], int(t), self.cfg.hidden) for t in ids])
        for li, lw in enumerate(self.w["layers"]):
            x = self._layer(x, lw, li)
        self.pos += 1
        return final_logits(x, self.w["final_norm"], self.w["lm_packed"], self.w["lm_scales"], self.cfg, self.dq)

    def generate(self, prompts, max_new_tokens: int, record: Optional[list] = None) -> np.ndarray:
        """Greedy loop of every row (prompts int [batch, P]); returns int [batch, max_new_tokens].
        ``record`` receives the logits [batch, V] behind each generated column."""
        prompts = np.asarray(prompts)
        logits = None
        for t in range(prompts.shape[1]):
            logits = self.step_tokens(prompts[:, t])
        out = np.zeros((self.batch, max_new_tokens), dtype=np.int64)
        for i in range(max_new_tokens):
            nxt = [predict_next_token(logits[b]) for b in range(self.batch)]
            if record is not None:
                record.append(logits)
            out[:, i] = nxt
            if i + 1 < max_new_tokens:
                logits = self.step_tokens(nxt)
        return out


# --------------------------------------------------------------------------
# Sampling (no reference counterpart: runners/engine.py:180-181 is greedy)
# --------------------------------------------------------------------------

PHILOX_M0, PHILOX_M1 = 0xD2511F53, 0xCD9E8D57
PHILOX_W0, PHILOX_W1 = 0x9E3779B9, 0xBB67AE85


def philox4x32_10(counter, key):
    """Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC 2011): 4 x 32-bit counter,
    2 x 32-bit key -> 4 x 32-bit output words."""
    c = [int(v) & 0xFFFFFFFF for v in counter]
    k0, k1 = int(key[0]) & 0xFFFFFFFF, int(key[1]) & 0xFFFFFFFF
    for _ in range(10):
        p0, p1 = PHILOX_M0 * c[0], PHILOX_M1 * c[2]
        hi0, lo0 = p0 >> 32, p0 & 0xFFFFFFFF
        hi1, lo1 = p1 >> 32, p1 & 0xFFFFFFFF
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
        k0 = (k0 + PHILOX_W0) & 0xFFFFFFFF
        k1 = (k1 + PHILOX_W1) & 0xFFFFFFFF
    return c


def f16_order_keys(logits: np.ndarray) -> np.ndarray:
    """Order-preserving 16-bit keys of fp16 values (NaN -> 0, below all numbers)."""
    b = np.asarray(logits, F16).view(np.uint16).astype(np.uint32)
    key = np.where(b & 0x8000, (~b) & 0xFFFF, b | 0x8000)
    nan = ((b & 0x7C00) == 0x7C00) & ((b & 0x03FF) != 0)
    return np.where(nan, 0, key).astype(np.uint32)


def sample_top_k(logits: np.ndarray, top_k: int, temperature: float, seed: int, offset: int, row: int = 0,
                 detail: bool = False):
    """Top-k / temperature sampling as lmps_sample_rows defines it: the k
    largest keys (ties at the threshold: lowest indices) in ascending index
    order, fp32 weights exp((v - vmax) * (1/T)), sums in the kernel's fixed
    order (32 contiguous segments of ceil(k/32) candidates, then the segment
    sums in order), u from Philox4x32-10 (key = seed, counter = (row, offset
    lo, offset hi, 0)).  ``detail`` also returns the target and the running
    sums (to judge ties at a boundary)."""
    x = np.asarray(logits, F16).reshape(-1)
    k = 1 if temperature <= 0 else int(top_k)
    keys = f16_order_keys(x)
    order = np.lexsort((np.arange(x.size), -keys.astype(np.int64)))   # key desc, index asc
    cand = np.sort(order[:k])
    inv_t = F32(1.0) if k == 1 else F32(1.0) / F32(temperature)
    v = x[cand].astype(F32)
    vmax = v.max()
    w = np.exp(((v - vmax) * inv_t).astype(F32)).astype(F32)
    seg = (k + 31) // 32
    lane_sum = []
    for l in range(32):
        s = F32(0.0)
        for i in range(min(k, l * seg), min(k, l * seg + seg)):
            s = F32(s + w[i])
        lane_sum.append(s)
    z = F32(0.0)
    for s in lane_sum:
        z = F32(z + s)
    r = philox4x32_10((row, offset & 0xFFFFFFFF, (offset >> 32) & 0xFFFFFFFF, 0),
                      (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))[0]
    target = F32(F32(F32(r >> 8) * F32(1.0 / 16777216.0)) * z)
    run = F32(0.0)
    l = 0
    while l < 31 and not (F32(run + lane_sum[l]) > target):
        run = F32(run + lane_sum[l])
        l += 1
    pick = -1
    sums = []
    for i in range(min(k, l * seg), min(k, l * seg + seg)):
        run = F32(run + w[i])
        sums.append(float(run))
        if run > target:
            pick = i
            break
    if pick < 0:
        pick = k - 1
        while pick > 0 and w[pick] == 0:
            pick -= 1
    out = int(cand[pick])
    if detail:
        return out, float(target), float(z), cand, w
    return out
