"""Host side of the persistent decode kernel (csrc/decode_persistent.cu).

Builds the plain-C descriptors of include/llamamps_b200.h (lmps_layer_desc,
lmps_model_desc, lmps_decode_state) from the engine's device tensors and
launches ``lmps_decode_persistent``: n decode steps of the whole model in one
cooperative launch.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from ._lib import check, lib

c_vp, c_int, c_float, c_size = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t


class LayerDesc(ctypes.Structure):
    _fields_ = [(n, c_vp) for n in (
        "qkv_packed", "qkv_scales", "qkv_bias", "o_packed", "o_scales", "gate_packed",
        "gate_scales", "up_packed", "up_scales", "down_packed", "down_scales", "in_norm",
        "post_norm", "k_pool", "v_pool")]


class ModelDesc(ctypes.Structure):
    _fields_ = [("n_layers", c_int), ("hidden", c_int), ("intermediate", c_int), ("vocab", c_int),
                ("n_q_heads", c_int), ("n_kv_heads", c_int), ("head_dim", c_int), ("eps", c_float),
                ("rope_style", c_int), ("layers", c_vp), ("final_norm", c_vp), ("lm_packed", c_vp),
                ("lm_scales", c_vp), ("embed", c_vp), ("inv_freq", c_vp)]


class DecodeState(ctypes.Structure):
    _fields_ = [("batch", c_int), ("page_size", c_int), ("max_pages", c_int), ("max_seq_len", c_int),
                ("block_table", c_vp), ("rope_table", c_vp), ("tokens", c_vp), ("pos", c_vp), ("forced", c_vp),
                ("forced_stride", c_int), ("n_forced", c_int), ("x_in", c_vp), ("logits", c_vp),
                ("history", c_vp), ("step_counter", c_vp), ("history_rows", c_int),
                ("workspace", c_vp), ("workspace_bytes", c_size), ("error", c_vp),
                ("trace", c_vp), ("trace_events", c_int), ("trace_rows", c_int)]


_SIGS = {
    "lmps_decode_persistent_workspace_size": (c_size, [ctypes.POINTER(ModelDesc), c_int, c_int]),
    "lmps_decode_persistent": (c_int, [ctypes.POINTER(ModelDesc), ctypes.POINTER(DecodeState), c_int, c_vp]),
}

MAX_BATCH = 4


def _declare():
    L = lib()
    for name, (res, args) in _SIGS.items():
        fn = getattr(L, name)
        fn.restype, fn.argtypes = res, args
    return L


def _p(t: Optional[torch.Tensor]):
    if t is None:
        return None
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError("persistent decode needs contiguous CUDA tensors")
    if t.data_ptr() % 16:
        raise ValueError("persistent decode needs 16-byte aligned tensors")
    return t.data_ptr()


def rope_table(inv_freq: torch.Tensor, positions: int) -> torch.Tensor:
    """fp32 [positions, head_dim/2, 2]: cos and sin of the fp32 angle
    p * inv_freq[j] (rope.metal:28-33 computes the angle in fp32), each
    correctly rounded from a float64 evaluation."""
    inv = inv_freq.detach().to("cpu", torch.float32).numpy()
    ang = (np.arange(positions, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    ang64 = ang.astype(np.float64)
    tab = np.stack([np.cos(ang64), np.sin(ang64)], axis=-1).astype(np.float32)
    return torch.from_numpy(np.ascontiguousarray(tab))


class PersistentDecoder:
    """Descriptors + workspace for one engine (weights, cache, max batch)."""

    def __init__(self, weights, cache, inv_freq: torch.Tensor, max_batch: int):
        if max_batch > MAX_BATCH:
            raise ValueError(f"persistent decode handles at most {MAX_BATCH} sequences")
        self.L = _declare()
        c = weights.cfg
        self.cfg = c
        self.cache = cache
        descs = (LayerDesc * len(weights.layers))()
        for i, lw in enumerate(weights.layers):
            kp, vp = cache.layer(i)
            descs[i] = LayerDesc(_p(lw.qkv_packed), _p(lw.qkv_scales), _p(lw.qkv_bias), _p(lw.o_packed),
                                 _p(lw.o_scales), _p(lw.gate_packed), _p(lw.gate_scales),
                                 _p(lw.up_packed), _p(lw.up_scales), _p(lw.down_packed),
                                 _p(lw.down_scales), _p(lw.in_norm), _p(lw.post_norm), _p(kp), _p(vp))
        raw = bytes(descs)
        self.layer_table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(weights.device)
        self.keep = (weights, inv_freq)  # descriptors point into these
        self.model = ModelDesc(len(weights.layers), c.hidden, c.intermediate, c.vocab, c.n_q_heads,
                               c.n_kv_heads, c.head_dim, float(c.eps), c.rope_style_code,
                               self.layer_table.data_ptr(), _p(weights.final_norm), _p(weights.lm_packed),
                               _p(weights.lm_scales), _p(weights.embed), _p(inv_freq))
        self.max_batch = max_batch
        self.rope_table = rope_table(inv_freq, cache.max_seq_len).to(weights.device)
        ws = self.L.lmps_decode_persistent_workspace_size(ctypes.byref(self.model), max_batch, cache.max_seq_len)
        self.workspace = torch.zeros(ws + 256, dtype=torch.uint8, device=weights.device)
        off = (-self.workspace.data_ptr()) % 256
        self.ws_view = self.workspace[off:off + ws]
        self.error = torch.zeros(1, dtype=torch.int32, device=weights.device)
        self._states = {}  # launch state by argument pointers (the per-token path reuses one)

    def reset_workspace(self):
        """Zero the workspace (needed once, and after a launch that reported an error)."""
        self.workspace.zero_()
        self.error.zero_()

    def run(self, batch: int, tokens: torch.Tensor, pos: torch.Tensor, n_steps: int, *,
            forced: Optional[torch.Tensor] = None, x_in: Optional[torch.Tensor] = None,
            logits: Optional[torch.Tensor] = None, history: Optional[torch.Tensor] = None,
            step_counter: Optional[torch.Tensor] = None,
            trace: Optional[torch.Tensor] = None) -> None:
        if not 1 <= batch <= self.max_batch:
            raise ValueError(f"batch {batch} outside [1, {self.max_batch}]")
        if forced is None and history is None and trace is None:
            # the per-token path: the state of (batch, tokens, pos, x_in, logits) is built once
            key = (batch, tokens.data_ptr(), pos.data_ptr(), x_in.data_ptr() if x_in is not None else 0,
                   logits.data_ptr() if logits is not None else 0, self.cache.block_table.data_ptr())
            st = self._states.get(key)
            if st is None:
                st = self._state(batch, tokens, pos, None, x_in, logits, None, None, None)
                if len(self._states) < 64:
                    self._states[key] = st
        else:
            st = self._state(batch, tokens, pos, forced, x_in, logits, history, step_counter, trace)
        check(self.L.lmps_decode_persistent(ctypes.byref(self.model), ctypes.byref(st), int(n_steps),
                                            torch.cuda.current_stream().cuda_stream),
              "lmps_decode_persistent")

    def _state(self, batch, tokens, pos, forced, x_in, logits, history, step_counter, trace):
        cache = self.cache
        st = DecodeState()
        st.batch = batch
        st.page_size = cache.page_size
        st.max_pages = cache.pages_per_seq
        st.max_seq_len = cache.max_seq_len
        st.block_table = cache.block_table.data_ptr()
        st.rope_table = _p(self.rope_table)
        st.tokens = _p(tokens)
        st.pos = _p(pos)
        if forced is not None:
            st.forced = forced.data_ptr()
            st.forced_stride = forced.shape[1]
            st.n_forced = forced.shape[1]
        st.x_in = _p(x_in)
        st.logits = logits.data_ptr() if logits is not None else None
        if history is not None:
            st.history = history.data_ptr()
            st.step_counter = step_counter.data_ptr()
            st.history_rows = history.numel() // batch
        st.workspace = self.ws_view.data_ptr()
        st.workspace_bytes = self.ws_view.numel()
        st.error = self.error.data_ptr()
        if trace is not None:
            sms = torch.cuda.get_device_properties(trace.device).multi_processor_count
            if trace.dtype != torch.int64 or trace.dim() != 2 or trace.shape[0] < 3 * sms:
                raise ValueError("trace must be int64 [>= 3 * n_SMs, events]")
            st.trace = trace.data_ptr()
            st.trace_events = trace.shape[1]
            st.trace_rows = trace.shape[0]
        return st

    def check_error(self) -> None:
        e = int(self.error.item())
        if e:
            self.reset_workspace()
            msg = {1: "a bounded device-side wait timed out",
                   2: "position past the KV cache or token id outside the vocabulary",
                   3: "no finite logit (argmax undefined)"}.get(e, f"code {e}")
            raise RuntimeError(f"persistent decode failed: {msg}")
