"""QwenEngine on B200: the reference's engine API over the sm_100a kernels.

Mirrors runners/engine.py:25-245:

* ``QwenEngine(weights_dir, device=None)`` loads the reference's flat-.bin
  layout (or takes ``weights=`` already on the device) -- but once, into HBM,
  where the reference re-uploads 26 MB per layer per token (engine.py:145-155);
* ``run_inference(input_vector) -> np.float16[V]`` runs one token through all
  layers, the final norm and the LM head (engine.py:157-178); unlike the
  reference it keeps a KV cache, so consecutive calls are consecutive
  positions of one sequence (the first call is exactly the reference's
  seq_len=1, position-0 forward);
* ``predict_next_token(logits) -> int`` is the host argmax (engine.py:180-181).

Added for the decode loop the reference does not have: ``generate`` (greedy,
batch 1), ``generate_batch`` and ``decode_step`` (B independent sequences),
a paged KV cache, the LM-head argmax on the device, and CUDA-graph replay of
a whole decode step (one graph launch per token instead of 29
command-buffer round trips, engine.py:176,244-245).

A decode step per layer (kernel names from csrc/):
    rms_norm -> gemv_q4_bias(q|k|v) -> rope_kv_append -> gqa_decode_attention
    -> gemv_q4_residual(o) -> rms_norm -> gemv_q4_swiglu(gate, up)
    -> gemv_q4_residual(down)
then rms_norm(final) -> lm_head_argmax -> decode_advance.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import numpy as np
import torch

from . import kernels as K
from ._lib import lib
from .config import QWEN2_5_1_5B, ModelConfig
from .kv_cache import PagedKVCache
from .weights import ModelWeights, load_reference_layout


# The CUDA-core GEMV serves up to 4 sequences; larger batches use the
# tensor-core GEMM (measured at batch 8, 128-position contexts: 1.73 ms per
# step on the GEMM path against 2.88 ms on the batch-8 GEMV, 1 x B200).
GEMV_MAX_BATCH = 4


def argmax_first(logits) -> int:
    """runners/engine.py:180-181, ``np.argmax(logits.astype(np.float32))``:
    the first index of the largest value.

    For a contiguous 1-D fp16 array the fp32 copy is skipped.  Read as int16,
    the fp16 bit patterns of positive values keep their order and lie above
    every negative value and zero, so when the largest int16 is a positive
    number (finite or +inf) its first index is the answer -- unless the
    array holds a NaN, which np.argmax would return: a positive NaN would be
    that largest int16 (above +inf's 31744), a negative NaN is a uint16
    pattern above -inf's 0xFC00.  Otherwise (no positive value, or a NaN) the
    order-preserving keys (negative values: magnitude bits flipped) decide,
    and a NaN or a maximum of zero (-0 and +0 compare equal) takes the fp32
    path.  ~10x faster than the fp32 copy on the 151936 LM-head logits."""
    x = np.asarray(logits)
    if x.dtype == np.float16 and x.ndim == 1 and x.flags.c_contiguous and x.size:
        b = x.view(np.int16)
        i = int(np.argmax(b))
        v = int(b[i])
        if 0 < v <= 31744 and int(x.view(np.uint16).max()) <= 0xFC00:
            return i
        key = b ^ ((b >> 15) & np.int16(0x7FFF))
        i = int(np.argmax(key))
        k = int(key[i])
        # keys of +inf / -inf are 31744 / -31745: anything beyond is a NaN;
        # keys 0 / -1 are +0 / -0
        if k <= 31744 and k != 0 and k != -1 and int(key.min()) >= -31745:
            return i
    return int(np.argmax(x.astype(np.float32)))


DENSE_PREFILL_TOKENS = 256  # prompts with at least this many tokens in total prefill on the GEMM path


def rope_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    """base^-(2i/head_dim) in fp32 (kernels/rope.metal:28-30 with idx % 128 = 2i)."""
    i2 = np.arange(0, head_dim, 2, dtype=np.float32)
    return np.power(np.float32(theta), -(i2 / np.float32(head_dim))).astype(np.float32)


class QwenEngine:
    def __init__(self, weights_dir: Optional[str] = None, device=None, *,
                 weights: Optional[ModelWeights] = None, config: ModelConfig = QWEN2_5_1_5B,
                 max_batch: int = 1, max_seq_len: int = 2048, page_size: int = 64,
                 use_graphs: bool = True, page_order: Optional[List[int]] = None,
                 decoder: Optional[str] = None, gemv_max_batch: int = GEMV_MAX_BATCH):
        if not torch.cuda.is_available():
            raise RuntimeError("QwenEngine needs a CUDA device (B200); there is no CPU path.")
        self.device = torch.device(device if device is not None else "cuda")
        lib()  # fail loudly now if the native library is missing
        if weights is None:
            if weights_dir is None:
                raise ValueError("pass weights_dir (reference .bin layout) or weights=")
            weights = load_reference_layout(weights_dir, config, self.device)
        self.weights = weights
        self.cfg = weights.cfg
        self.weights_dir = weights_dir
        self.layers = len(weights.layers)
        self.hidden_dim = self.cfg.hidden
        self.mlp_intermediate = self.cfg.intermediate
        self.max_batch = max_batch
        # batches above this run the projections and LM head on the tensor-core GEMM
        self.gemv_max_batch = gemv_max_batch
        self.use_graphs = use_graphs
        self.cache = PagedKVCache(self.cfg, self.layers, max_batch, max_seq_len, page_size,
                                  self.device, page_order=page_order)
        self.max_seq_len = self.cache.max_seq_len
        self.n_splits = K.attention_splits(max_batch, self.cfg.n_kv_heads, self.max_seq_len, page_size)
        self._create_buffer_pool()
        self._graphs = {}
        # "persistent": one cooperative kernel per launch runs whole decode
        # steps (csrc/decode_persistent.cu, batch <= 4); "batched": one
        # cooperative kernel runs every layer of a step (csrc/decode_batched.cu,
        # batch <= 64), with the head kernels after it; "kernels": one kernel
        # per stage (any batch).  The last two are replayed as CUDA graphs.
        from .persistent import MAX_BATCH as PERSISTENT_MAX_BATCH
        if decoder is None:
            decoder = "persistent" if max_batch <= PERSISTENT_MAX_BATCH else "kernels"
        if decoder not in ("persistent", "kernels", "batched"):
            raise ValueError(f"unknown decoder {decoder!r}")
        self.decoder = decoder
        self.pdec = None
        self.bdec = None
        if decoder == "persistent":
            from .persistent import PersistentDecoder
            self.pdec = PersistentDecoder(self.weights, self.cache, self.inv_freq, max_batch)
        elif decoder == "batched":
            from .batched import BatchedDecoder
            self.bdec = BatchedDecoder(self.weights, self.cache, self.inv_freq, max_batch)
        self.batch = 1
        self.reset(1)

    # -- buffers (runners/engine.py:84-118, plus decode state) ---------------
    def _create_buffer_pool(self) -> None:
        c, B, dev = self.cfg, self.max_batch, self.device
        h = torch.float16
        self.buf_residual = torch.zeros(B, c.hidden, dtype=h, device=dev)
        self.buf_normed = torch.zeros(B, c.hidden, dtype=h, device=dev)
        self.buf_qkv = torch.zeros(B, c.qkv_rows, dtype=h, device=dev)
        self.buf_q = torch.zeros(B, c.q_dim, dtype=h, device=dev)
        self.buf_attn = torch.zeros(B, c.q_dim, dtype=h, device=dev)
        self.buf_mlp = torch.zeros(B, c.intermediate, dtype=h, device=dev)
        # gate/up outputs of the tensor-core GEMM path (batches past the GEMV's 8)
        # fused gate|up GEMM output (batched path): [B, 2 * intermediate]
        self.buf_up = torch.zeros(B if B > self.gemv_max_batch else 1, 2 * c.intermediate, dtype=h, device=dev)
        self.gemm_err = torch.zeros(1, dtype=torch.int32, device=dev)
        # split-K partial tiles of the small-m GEMMs (zero between calls)
        ws = K.w4a16_gemm_workspace_size(B, c.intermediate) if B > self.gemv_max_batch else 0
        self.gemm_ws = torch.zeros(ws + 256, dtype=torch.uint8, device=dev)
        off = (-self.gemm_ws.data_ptr()) % 256
        self.gemm_ws = self.gemm_ws[off:off + ws] if ws else None
        self.buf_logits = torch.zeros(B, c.vocab, dtype=h, device=dev)
        ws = K.attention_workspace_size(B, c.n_q_heads, c.head_dim, self.n_splits)
        self.attn_ws = torch.zeros(max(ws, 16), dtype=torch.uint8, device=dev)
        self.inv_freq = torch.from_numpy(rope_inv_freq(c.head_dim, c.rope_theta)).to(dev)
        i32 = torch.int32
        self.tokens = torch.zeros(B, dtype=i32, device=dev)
        self.pos = torch.zeros(B, dtype=i32, device=dev)
        self.seq_lens = torch.ones(B, dtype=i32, device=dev)
        self.next_ids = torch.zeros(B, dtype=i32, device=dev)
        self.argmax_keys = torch.zeros(B, dtype=torch.int64, device=dev)
        self.bad_ids = torch.zeros(1, dtype=i32, device=dev)
        self.history = torch.zeros(1, B, dtype=i32, device=dev)
        self.step_counter = torch.zeros(1, dtype=i32, device=dev)
        self._pin_vec = torch.zeros(c.hidden, dtype=h).pin_memory()
        self._pin_logits = torch.zeros(c.vocab, dtype=h).pin_memory()
        self._pin_ids = torch.zeros(B, dtype=i32).pin_memory()
        self._pin_next = torch.zeros(B, dtype=i32).pin_memory()
        self._pin_err = torch.zeros(1, dtype=i32).pin_memory()
        # run_inference's views, made once (it runs once per token)
        self._pin_vec_np, self._pin_logits_np, self._pin_err_np = (
            self._pin_vec.numpy(), self._pin_logits.numpy(), self._pin_err.numpy())
        self._x_row0, self._x_rows1 = self.buf_residual[0], self.buf_residual[:1]
        self._lg_row0, self._lg_rows1 = self.buf_logits[0], self.buf_logits[:1]
        self._ri_warm = False  # run_inference has launched once eagerly (then it replays a graph)

    def reset(self, batch: Optional[int] = None, start_pos: int = 0) -> None:
        """Start ``batch`` fresh sequences (slots 0..batch-1) at ``start_pos``."""
        b = self.batch if batch is None else batch
        if not 1 <= b <= self.max_batch:
            raise ValueError(f"batch {b} outside [1, {self.max_batch}]")
        self.batch = b
        self.cache.release_all()
        for s in range(b):
            self.cache.reserve(s, self.max_seq_len)
        self.pos.fill_(start_pos)
        self.seq_lens.fill_(start_pos + 1)
        self.step_counter.zero_()
        self.host_pos = start_pos

    # -- one forward over the current tokens/pos ----------------------------
    def _layers(self, B: int) -> None:
        c, w = self.cfg, self.weights
        x = self.buf_residual[:B]
        xn = self.buf_normed[:B]
        if self.bdec is not None:  # every layer in one launch
            self.bdec.run(B, x, self.pos[:B], self.seq_lens[:B])
            return
        gemm = B > self.gemv_max_batch   # dense contraction: tcgen05 W4A16 GEMM
        for li, lw in enumerate(w.layers):
            kp, vp = self.cache.layer(li)
            K.rms_norm(x, lw.in_norm, c.eps, out=xn)
            if gemm:
                K.w4a16_gemm(xn, lw.qkv_packed, lw.qkv_scales, c.qkv_rows, c.hidden, bias=lw.qkv_bias,
                             out=self.buf_qkv[:B], error=self.gemm_err, workspace=self.gemm_ws)
            else:
                K.gemv_q4_bias(lw.qkv_packed, lw.qkv_scales, lw.qkv_bias, xn, c.qkv_rows, c.hidden,
                               out=self.buf_qkv[:B])
            # RoPE + KV append + attention in one launch (rope_kv_append's work
            # done by the attention CTAs)
            K.gqa_decode_attention_rope(self.buf_qkv[:B], self.pos, self.inv_freq, kp, vp,
                                        self.cache.block_table, self.seq_lens, self.buf_attn[:B],
                                        self.attn_ws, self.cache.page_size, c.n_q_heads, c.n_kv_heads,
                                        c.head_dim, self.max_seq_len, self.n_splits, c.rope_style_code)
            self._o_proj(lw, self.buf_attn[:B], x, gemm)
            K.rms_norm(x, lw.post_norm, c.eps, out=xn)
            if gemm:
                self._gate_up(lw, xn, self.buf_up[:B], self.buf_mlp[:B])
            else:
                K.gemv_q4_swiglu(lw.gate_packed, lw.gate_scales, lw.up_packed, lw.up_scales, xn,
                                 c.intermediate, c.hidden, out=self.buf_mlp[:B])
            self._down_proj(lw, self.buf_mlp[:B], x, gemm)

    def _gate_up(self, lw, xn, gu, out, ws=None) -> None:
        """a = SwiGLU(W_gate xn, W_up xn) on the GEMM path: one GEMM over the
        interleaved gate/up rows with the SwiGLU epilogue when the layer has
        them, else two GEMMs and the SwiGLU kernel."""
        c = self.cfg
        if lw.gu_packed is not None:
            K.w4a16_gemm(xn, lw.gu_packed, lw.gu_scales, 2 * c.intermediate, c.hidden, swiglu=True, out=out,
                         error=self.gemm_err, workspace=self._ws(ws))
        else:
            up = gu.reshape(-1)[:out.numel()].view(out.shape)  # contiguous [B, intermediate] scratch
            K.w4a16_gemm(xn, lw.gate_packed, lw.gate_scales, c.intermediate, c.hidden, out=out,
                         error=self.gemm_err, workspace=self._ws(ws))
            K.w4a16_gemm(xn, lw.up_packed, lw.up_scales, c.intermediate, c.hidden, out=up,
                         error=self.gemm_err, workspace=self._ws(ws))
            K.swiglu(out, up, out=out)

    # x <- x + fp16(W_o attn) and x <- x + fp16(W_down a) (runners/engine.py:215-221,237-243);
    # the tensor-parallel engine overrides these with partial products and an all-reduce
    def _ws(self, ws):
        """Split-K workspace of a GEMM call: the decode buffer by default,
        none (unsplit) for the token rows of a dense prefill (ws=False)."""
        return None if ws is False else (ws if ws is not None else self.gemm_ws)

    def _o_proj(self, lw, att, x, gemm: bool, ws=None) -> None:
        c = self.cfg
        if gemm:
            K.w4a16_gemm(att, lw.o_packed, lw.o_scales, c.hidden, c.q_dim, residual=x, out=x,
                         error=self.gemm_err, workspace=self._ws(ws))
        else:
            K.gemv_q4_residual(lw.o_packed, lw.o_scales, att, x, c.hidden, c.q_dim, out=x)

    def _down_proj(self, lw, a, x, gemm: bool, ws=None) -> None:
        c = self.cfg
        if gemm:
            K.w4a16_gemm(a, lw.down_packed, lw.down_scales, c.hidden, c.intermediate, residual=x, out=x,
                         error=self.gemm_err, workspace=self._ws(ws))
        else:
            K.gemv_q4_residual(lw.down_packed, lw.down_scales, a, x, c.hidden, c.intermediate, out=x)

    def _head(self, B: int, want_logits: bool) -> None:
        c, w = self.cfg, self.weights
        K.rms_norm(self.buf_residual[:B], w.final_norm, c.eps, out=self.buf_normed[:B])
        if B > self.gemv_max_batch:
            K.w4a16_gemm(self.buf_normed[:B], w.lm_packed, w.lm_scales, c.vocab, c.hidden,
                         out=self.buf_logits[:B], error=self.gemm_err, workspace=self.gemm_ws)
            K.argmax_rows(self.buf_logits[:B], c.vocab, self.next_ids[:B])
        else:
            K.lm_head_argmax(w.lm_packed, w.lm_scales, self.buf_normed[:B], c.vocab, c.hidden,
                             self.argmax_keys[:B], self.next_ids[:B],
                             logits=self.buf_logits[:B] if want_logits else None)

    def _device_step(self, B: int, want_logits: bool = False, record: bool = True) -> None:
        """Embed -> layers -> head -> advance; device-only, graph-capturable."""
        K.embed_gather(self.weights.embed, self.tokens[:B], self.buf_residual[:B], self.bad_ids)
        self._layers(B)
        self._head(B, want_logits)
        K.decode_advance(self.next_ids[:B], self.tokens[:B], self.pos[:B], self.seq_lens[:B],
                         self.history if record else None, self.step_counter if record else None)

    # -- reference API -------------------------------------------------------
    def _vector_step(self) -> None:
        """Layers + head + advance from buf_residual[0] (run_inference's body)."""
        self._layers(1)
        self._head(1, want_logits=True)
        K.decode_advance(self.next_ids[:1], self.tokens[:1], self.pos[:1], self.seq_lens[:1])

    def run_inference(self, input_vector: np.ndarray) -> np.ndarray:
        """engine.py:157-178 for sequence 0: one embedding vector in, fp16 logits out.

        The vector goes through pinned host memory; the whole forward is one
        CUDA-graph replay; the fp16 logits come back through pinned memory."""
        if self.batch != 1:
            self.reset(1)
        if self.host_pos >= self.max_seq_len:
            raise RuntimeError("KV cache full")
        vec = np.ascontiguousarray(input_vector, dtype=np.float16).reshape(-1)
        if vec.size != self.cfg.hidden:
            raise ValueError(f"input vector has {vec.size} elements, expected {self.cfg.hidden}")
        self._pin_vec_np[:] = vec
        if self.pdec is not None and self.use_graphs and self._ri_warm:
            # the whole per-token sequence -- input copy, persistent launch,
            # logits and error word back -- as one graph replay
            self._persistent_token_graph().replay()
        else:
            self._persistent_token_ops()
            self._ri_warm = self.pdec is not None
        torch.cuda.current_stream(self.device).synchronize()
        if self.pdec is not None and self._pin_err_np[0] != 0:
            self.pdec.check_error()
        self.host_pos += 1
        return self._pin_logits_np.copy()

    def _persistent_token_ops(self) -> None:
        """run_inference's device work: pinned input row in, one decode step
        (persistent launch, graph replay or per-stage kernels), logits (and
        the persistent kernel's error word) out to pinned memory."""
        self._x_row0.copy_(self._pin_vec, non_blocking=True)
        if self.pdec is not None:
            self.pdec.run(1, self.tokens, self.pos, 1, x_in=self._x_rows1, logits=self._lg_rows1)
        elif self.use_graphs:
            self._graph_for(1, record=False, vector=True).replay()
        else:
            self._vector_step()
        self._pin_logits.copy_(self._lg_row0, non_blocking=True)
        if self.pdec is not None:  # the device error word rides along with the logits
            self._pin_err.copy_(self.pdec.error, non_blocking=True)

    def _persistent_token_graph(self):
        """The persistent per-token sequence captured once (after one eager
        call has set the kernel's launch configuration); the launch reads
        tokens, positions and its tag epoch from device memory, so every
        replay decodes the next position."""
        g = self._graphs.get("token")
        if g is None:
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    self._persistent_token_ops()
            torch.cuda.current_stream(self.device).wait_stream(s)
            self._graphs["token"] = g
        return g

    def predict_next_token(self, logits: np.ndarray) -> int:
        """engine.py:180-181: argmax over fp32(logits), first index on ties."""
        return argmax_first(logits)

    # -- decode loop ---------------------------------------------------------
    def _graph_for(self, B: int, record: bool, vector: bool = False):
        key = (B, record, vector)
        g = self._graphs.get(key)
        if g is None:
            def body():
                if vector:
                    self._vector_step()
                else:
                    self._device_step(B, record=record)
            # Warm every launch path once outside capture (kernel attributes,
            # lazy module loading), then restore the state the warm-up touched.
            state = (self.tokens, self.pos, self.seq_lens, self.step_counter, self.buf_residual)
            saved = [t.clone() for t in state]
            body()
            torch.cuda.synchronize(self.device)
            for t, sv in zip(state, saved):
                t.copy_(sv)
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    body()
            torch.cuda.current_stream(self.device).wait_stream(s)
            for t, sv in zip(state, saved):
                t.copy_(sv)
            torch.cuda.synchronize(self.device)
            self._graphs[key] = g
        return g

    def launches_per_step(self) -> int:
        """Kernels one decode step launches (what a graph replay runs); the
        persistent decoder runs any number of steps in one launch."""
        if self.pdec is not None:
            return 1
        if self.bdec is not None:  # embed, the layers, final norm, LM head + argmax, advance
            return 1 + 1 + 1 + 2 + 1
        # norm, q|k|v, RoPE + append + attention (+ split combine), o, norm,
        # gate/up (+ SwiGLU on the GEMM path), down; then embed, final norm, the
        # LM head with its argmax (two launches on either path), advance
        gemm = self.batch > self.gemv_max_batch
        per_layer = 7 + (1 if self.n_splits > 1 else 0) + (1 if gemm else 0)
        return 1 + self.layers * per_layer + 1 + 2 + 1

    def step_tokens(self, token_ids) -> np.ndarray:
        """Public streaming step: host ids [batch] in (pinned H2D), one graph
        replay, the next ids [batch] out (pinned D2H)."""
        B = self.batch
        ids = np.ascontiguousarray(token_ids, dtype=np.int32).reshape(-1)
        if ids.size != B:
            raise ValueError(f"expected {B} token ids")
        self._pin_ids.numpy()[:B] = ids
        self.tokens[:B].copy_(self._pin_ids[:B], non_blocking=True)
        self.decode_step(record=False)
        self._pin_next.copy_(self.tokens, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        if self.pdec is not None:
            self.pdec.check_error()
        if self.bdec is not None:
            self.bdec.check_error()
        return self._pin_next.numpy()[:B].copy()

    def decode_step(self, record: bool = True) -> None:
        """Advance every active sequence by one token (device-resident state)."""
        self.decode_steps(1, record)

    def decode_steps(self, n: int, record: bool = True) -> None:
        """Advance every active sequence by ``n`` tokens: one persistent launch,
        or ``n`` graph replays of the per-stage kernels."""
        B = self.batch
        if n <= 0:
            return
        if self.host_pos + n > self.max_seq_len:
            raise RuntimeError("KV cache full")
        if self.pdec is not None:
            self.pdec.run(B, self.tokens, self.pos, n,
                          history=self.history if record else None,
                          step_counter=self.step_counter if record else None)
        else:
            for _ in range(n):
                if self.use_graphs:
                    self._graph_for(B, record).replay()
                else:
                    self._device_step(B, record=record)
        self.host_pos += n

    def _ensure_history(self, steps: int) -> None:
        if self.history.shape[0] < steps or self.history.shape[1] != self.max_batch:
            self.history = torch.zeros(steps, self.max_batch, dtype=torch.int32, device=self.device)
            self._graphs.clear()  # graphs captured the old history pointer

    def prefill(self, prompts: torch.Tensor, dense: Optional[bool] = None) -> None:
        """Feed prompt tokens [B, P] (causal); afterwards ``tokens`` holds each
        sequence's first generated token (also history row 0).

        ``dense`` (default: B*P >= DENSE_PREFILL_TOKENS) runs every prompt
        token of every sequence through each layer at once on the tensor-core
        GEMM (:meth:`prefill_dense`); otherwise the tokens go through the
        decode path one position at a time."""
        B, P = prompts.shape
        if P + 1 > self.max_seq_len:
            raise ValueError("prompt longer than the KV cache")
        prompts = prompts.to(self.device, torch.int32)
        if dense is None:
            dense = B * P >= DENSE_PREFILL_TOKENS
        if dense:
            self.prefill_dense(prompts)
            return
        if self.pdec is not None:
            # tokens <- prompt[:, 0]; steps 0..P-2 feed prompt[:, 1:]; the last
            # step's argmax (the first generated token) lands in history row 0.
            self.tokens[:B].copy_(prompts[:, 0])
            forced = prompts[:, 1:].contiguous() if P > 1 else None
            self.step_counter.fill_(-(P - 1))
            if self.host_pos + P > self.max_seq_len:
                raise RuntimeError("KV cache full")
            self.pdec.run(B, self.tokens, self.pos, P, forced=forced, history=self.history,
                          step_counter=self.step_counter)
            self.host_pos += P
            return
        for t in range(P):
            self.tokens[:B].copy_(prompts[:, t])
            if t == P - 1:
                self.step_counter.zero_()
            self.decode_step(record=True)

    def prefill_dense(self, prompts: torch.Tensor) -> None:
        """All B*P prompt tokens through every layer at once: the projections
        are W4A16 tensor-core GEMMs over M = B*P token rows, RoPE and the KV
        append run on every (sequence, position) row, and the causal
        attention of all rows is one flash-attention launch over the paged
        cache.  The LM head runs on each sequence's last row only."""
        c, w, dev = self.cfg, self.weights, self.device
        B, P = prompts.shape
        if self.host_pos != 0:
            raise RuntimeError("dense prefill starts fresh sequences (call reset first)")
        Mt = B * P
        h, i32 = torch.float16, torch.int32
        ids = prompts.reshape(-1).contiguous()
        rows_pos = torch.arange(P, dtype=i32, device=dev).repeat(B)
        rows_bt = self.cache.block_table[:B].repeat_interleave(P, dim=0).contiguous()
        x = torch.empty(Mt, c.hidden, dtype=h, device=dev)
        xn = torch.empty_like(x)
        qkv = torch.empty(Mt, c.qkv_rows, dtype=h, device=dev)
        q = torch.empty(Mt, c.q_dim, dtype=h, device=dev)
        att = torch.empty(Mt, c.q_dim, dtype=h, device=dev)
        gate = torch.empty(Mt, c.intermediate, dtype=h, device=dev)
        gu = torch.empty(Mt, 2 * c.intermediate, dtype=h, device=dev)
        err = self.gemm_err
        K.embed_gather(w.embed, ids, x, self.bad_ids)
        for li, lw in enumerate(w.layers):
            kp, vp = self.cache.layer(li)
            K.rms_norm(x, lw.in_norm, c.eps, out=xn)
            K.w4a16_gemm(xn, lw.qkv_packed, lw.qkv_scales, c.qkv_rows, c.hidden, bias=lw.qkv_bias,
                         out=qkv, error=err)
            K.rope_kv_append(qkv, rows_pos, self.inv_freq, q, kp, vp, rows_bt, self.cache.page_size,
                             c.n_q_heads, c.n_kv_heads, c.head_dim, c.rope_style_code)
            K.prefill_attention(q, kp, vp, self.cache.block_table[:B], att, B, P, self.cache.page_size,
                                c.n_q_heads, c.n_kv_heads, c.head_dim, error=err)
            self._o_proj(lw, att, x, True, ws=False)
            K.rms_norm(x, lw.post_norm, c.eps, out=xn)
            self._gate_up(lw, xn, gu, gate, ws=False)
            self._down_proj(lw, gate, x, True, ws=False)
        # last position of every sequence -> final norm, LM head, argmax
        self.buf_residual[:B].copy_(x.view(B, P, c.hidden)[:, P - 1])
        self._head(B, want_logits=False)
        self.tokens[:B].copy_(self.next_ids[:B])
        self.pos[:B].fill_(P)
        self.seq_lens[:B].fill_(P + 1)
        self.history[0, :B].copy_(self.next_ids[:B])
        self.step_counter.fill_(1)
        self.host_pos += P

    def _logits_step(self, B: int) -> None:
        """One decode step of every sequence that leaves the fp16 logits of
        the step in buf_logits (tokens/pos advance as in decode_step)."""
        if self.host_pos + 1 > self.max_seq_len:
            raise RuntimeError("KV cache full")
        if self.pdec is not None:
            self.pdec.run(B, self.tokens, self.pos, 1, logits=self.buf_logits[:B])
        else:
            K.embed_gather(self.weights.embed, self.tokens[:B], self.buf_residual[:B], self.bad_ids)
            self._layers(B)
            self._head(B, want_logits=True)
            K.decode_advance(self.next_ids[:B], self.tokens[:B], self.pos[:B], self.seq_lens[:B])
        self.host_pos += 1

    def _sample_generate(self, p: torch.Tensor, n: int, top_k: int, temperature: float, seed: int) -> None:
        """generate_batch with sampling: the prompt fed token by token, then
        every next token drawn by lmps_sample_rows from the step's logits
        (Philox offset = the generated token's index, so a run is
        reproducible from its seed); history rows 0..n-1 get the draws."""
        B, P = p.shape
        dev_p = p.to(self.device)
        for t in range(P):
            self.tokens[:B].copy_(dev_p[:, t])
            self._logits_step(B)
        hist = self.history.view(-1)  # [step, B] rows with the active batch as stride (as decode_advance)
        for i in range(n):
            K.sample_rows(self.buf_logits[:B], self.cfg.vocab, top_k, temperature, seed, i,
                          self.tokens[:B], hist[i * B:(i + 1) * B])
            if i + 1 < n:
                self._logits_step(B)

    def generate_batch(self, prompts, max_new_tokens: int, temperature: float = 0.0, top_k: int = 0,
                       seed: int = 0) -> np.ndarray:
        """Decode of B equal-length prompts; returns int32 [B, max_new_tokens].
        Greedy (the reference's argmax, runners/engine.py:180-181) unless
        temperature > 0 and top_k > 1: then each token is sampled among the
        top_k logits at that temperature (lmps_sample_rows, seeded)."""
        p = torch.as_tensor(np.asarray(prompts), dtype=torch.int32)
        if p.dim() == 1:
            p = p[None]
        B, P = p.shape
        if P + max_new_tokens > self.max_seq_len:
            raise ValueError("prompt + generation exceed the KV cache")
        self._ensure_history(max_new_tokens)
        if int(p.min()) < 0 or int(p.max()) >= self.cfg.vocab:
            raise ValueError("token id outside the vocabulary")
        self.reset(B)
        if temperature > 0 and top_k > 1:
            self._sample_generate(p, max_new_tokens, top_k, temperature, seed)
        else:
            self.prefill(p)
            self.decode_steps(max_new_tokens - 1, record=True)
        torch.cuda.synchronize(self.device)
        if self.pdec is not None:
            self.pdec.check_error()
        if self.bdec is not None:
            self.bdec.check_error()
        if int(self.bad_ids.item()) != 0:
            self.bad_ids.zero_()
            raise ValueError("token id outside the vocabulary")
        # decode_advance writes row-major [step, B] with the active batch as stride
        hist = self.history.reshape(-1)[: max_new_tokens * B].reshape(max_new_tokens, B)
        return hist.t().cpu().numpy()

    def generate(self, token_ids: Sequence[int], max_new_tokens: int, temperature: float = 0.0, top_k: int = 0,
                 seed: int = 0) -> List[int]:
        """Continuation of one prompt (the demo.py flow with a real prompt):
        greedy, or top-k / temperature sampling (see generate_batch)."""
        return [int(t) for t in self.generate_batch(np.asarray(token_ids)[None], max_new_tokens, temperature,
                                                    top_k, seed)[0]]
