"""Host side of the batched decode kernel (csrc/decode_batched.cu).

Builds the tile-major copies of every layer's Q4 matrices
(``lmps_q4_tile_blocks``), the plain-C descriptors of include/llamamps_b200.h
(lmps_batched_layer, lmps_batched_desc) and the workspace, and launches
``lmps_decode_batched``: all layers of one decode step for up to 64
sequences in one cooperative launch.  The final norm, LM head and argmax stay
with the caller (the engine's head).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from ._lib import check, lib
from .weights import interleave_rows

c_vp, c_int, c_float, c_size = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t

MAX_BATCH = 64


class BatchedLayer(ctypes.Structure):
    _fields_ = [(n, c_vp) for n in (
        "qkv_blocks", "o_blocks", "gu_blocks", "down_blocks", "qkv_bias", "in_norm", "post_norm",
        "k_pool", "v_pool")]


class BatchedDesc(ctypes.Structure):
    _fields_ = [("layers", c_vp), ("n_layers", c_int), ("hidden", c_int), ("intermediate", c_int),
                ("n_q_heads", c_int), ("n_kv_heads", c_int), ("head_dim", c_int), ("eps", c_float),
                ("rope_style", c_int), ("inv_freq", c_vp)]


_SIGS = {
    "lmps_q4_tile_blocks_size": (c_size, [c_int, c_int]),
    "lmps_q4_tile_blocks": (c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp]),
    "lmps_decode_batched_workspace_size": (c_size, [ctypes.POINTER(BatchedDesc), c_int, c_int]),
    "lmps_decode_batched_barriers": (c_int, [ctypes.POINTER(BatchedDesc), c_int, c_int]),
    "lmps_decode_batched": (c_int, [ctypes.POINTER(BatchedDesc), c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                                    c_int, c_vp, c_size, c_vp, c_vp, c_vp]),
}


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
        raise ValueError("batched decode needs contiguous CUDA tensors")
    if t.data_ptr() % 16:
        raise ValueError("batched decode needs 16-byte aligned tensors")
    return t.data_ptr()


def tile_blocks(packed: torch.Tensor, scales: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """Tile-major copy of a Q4 [n, k] matrix (q4_tile.cuh), on the device."""
    L = _declare()
    size = L.lmps_q4_tile_blocks_size(n, k)
    if size == 0:
        raise ValueError(f"tile blocks need n % 128 == 0 and k % 64 == 0 (got {n} x {k})")
    out = torch.empty(size, dtype=torch.uint8, device=packed.device)
    check(L.lmps_q4_tile_blocks(_p(packed), _p(scales), n, k, _p(out), torch.cuda.current_stream().cuda_stream),
          "lmps_q4_tile_blocks")
    return out


def supported(cfg) -> bool:
    """The batched kernel's shape limits (the C side checks them again)."""
    qkv = (cfg.n_q_heads + 2 * cfg.n_kv_heads) * cfg.head_dim
    return (cfg.head_dim == 128 and cfg.hidden % 512 == 0 and cfg.hidden <= 2048 and qkv % 128 == 0
            and (2 * cfg.intermediate) % 128 == 0 and cfg.intermediate % 64 == 0
            and cfg.n_q_heads // cfg.n_kv_heads <= 8)


class BatchedDecoder:
    """Tile-major weights, descriptors and workspace for one engine."""

    def __init__(self, weights, cache, inv_freq: torch.Tensor, max_batch: int):
        if not 1 <= max_batch <= MAX_BATCH:
            raise ValueError(f"batched decode handles 1..{MAX_BATCH} sequences")
        self.L = _declare()
        c = weights.cfg
        self.cfg, self.cache = c, cache
        qkv_rows = (c.n_q_heads + 2 * c.n_kv_heads) * c.head_dim
        self.blocks = []
        descs = (BatchedLayer * len(weights.layers))()
        for i, lw in enumerate(weights.layers):
            gp, gs = lw.gu_packed, lw.gu_scales
            if gp is None:
                gp = interleave_rows(lw.gate_packed, lw.up_packed, c.intermediate)
                gs = interleave_rows(lw.gate_scales, lw.up_scales, c.intermediate)
            blk = (tile_blocks(lw.qkv_packed, lw.qkv_scales, qkv_rows, c.hidden),
                   tile_blocks(lw.o_packed, lw.o_scales, c.hidden, c.q_dim),
                   tile_blocks(gp, gs, 2 * c.intermediate, c.hidden),
                   tile_blocks(lw.down_packed, lw.down_scales, c.hidden, c.intermediate))
            self.blocks.append(blk)
            kp, vp = cache.layer(i)
            descs[i] = BatchedLayer(*(_p(b) for b in blk), _p(lw.qkv_bias), _p(lw.in_norm), _p(lw.post_norm),
                                    _p(kp), _p(vp))
        self.layer_table = torch.frombuffer(bytearray(bytes(descs)), dtype=torch.uint8).to(weights.device)
        self.keep = (weights, inv_freq)  # the descriptors point into these
        self.desc = BatchedDesc(self.layer_table.data_ptr(), len(weights.layers), c.hidden, c.intermediate,
                                c.n_q_heads, c.n_kv_heads, c.head_dim, float(c.eps), c.rope_style_code,
                                _p(inv_freq))
        self.max_batch = max_batch
        ws = max(self.L.lmps_decode_batched_workspace_size(ctypes.byref(self.desc), b, cache.max_seq_len)
                 for b in range(1, max_batch + 1))
        if ws == 0:
            raise ValueError("model shape not supported by the batched decode kernel")
        self.workspace = torch.zeros(ws + 256, dtype=torch.uint8, device=weights.device)
        off = (-self.workspace.data_ptr()) % 256
        self.ws_view = self.workspace[off:off + ws]
        self.error = torch.zeros(1, dtype=torch.int32, device=weights.device)

    def reset_workspace(self):
        """Zero the workspace (its grid-barrier counter) and the error word:
        needed after a launch that reported an error."""
        self.workspace.zero_()
        self.error.zero_()

    def barriers(self, batch: int) -> int:
        """Grid barriers of one launch for ``batch`` sequences (trace rows per CTA)."""
        return self.L.lmps_decode_batched_barriers(ctypes.byref(self.desc), batch, self.cache.max_seq_len)

    def check_error(self) -> None:
        e = int(self.error.item())
        if e:
            self.reset_workspace()
            msg = {1: "a bounded device-side wait timed out",
                   2: "a position outside the KV cache"}.get(e, f"code {e}")
            raise RuntimeError(f"batched decode failed: {msg}")

    def run(self, batch: int, x: torch.Tensor, pos: torch.Tensor, seq_lens: torch.Tensor,
            trace: Optional[torch.Tensor] = None) -> None:
        """All layers for sequences 0..batch-1: x [batch, hidden] (embedded
        tokens) becomes the residual after the last layer; the new K/V rows
        go into the cache at pos.  trace: optional int64 [grid, barriers, 4]
        timeline (%globaltimer ns; see include/llamamps_b200.h)."""
        cache = self.cache
        if trace is not None:
            want = (torch.cuda.get_device_properties(x.device).multi_processor_count,
                    self.barriers(batch), 4)
            if tuple(trace.shape) != want or trace.dtype != torch.int64:
                raise ValueError(f"trace must be int64 {want}")
        check(self.L.lmps_decode_batched(ctypes.byref(self.desc), _p(x), _p(pos), _p(seq_lens),
                                         _p(cache.block_table), cache.block_table.shape[1], cache.page_size, batch,
                                         cache.max_seq_len, self.ws_view.data_ptr(), self.ws_view.numel(),
                                         _p(self.error), _p(trace), torch.cuda.current_stream().cuda_stream),
              "lmps_decode_batched")
