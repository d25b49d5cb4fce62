"""Tensor-parallel decode: the layers split across ``world`` GPUs (2 for
Qwen2.5-1.5B, one KV head per rank), one process per GPU.

Rank r owns
  * q|k|v output rows of its query heads [r*Hq/W, (r+1)*Hq/W) and KV heads
    [r*Hkv/W, (r+1)*Hkv/W) (a head-aligned row split; its KV cache holds only
    those heads),
  * o_proj input columns of its query heads (K = q_dim / W),
  * gate/up output rows [r*I/W, (r+1)*I/W) and down_proj input columns of the
    same slice (K = I / W),
all at multiples of the 32-element Q4 group, so the packed rows and scales of
runners/engine.py:120-143's layout split without re-quantising.  Each rank
computes partial o_proj / down_proj outputs; one all-reduce (sum, fp16) of
[B, hidden] after each restores the full residual stream, 2 per layer
(runners/engine.py:215-221,237-243 with the sum distributed).  Norms, the
embedding and the LM head are replicated, so every rank derives the same
next token.  The collectives run on the process group handed in (NCCL over
NVLink between GPUs; gloo for the host-side tests).

With the peer exchange (two ranks) the LM head is split by vocabulary rows
as well: each rank runs the Q4 head (GEMV + first-index argmax, or GEMM +
row argmax for larger batches) over its half of the rows only (the cut at a
multiple of 128 rows near V/2), and one exchange of (logit, global row) per
sequence picks the winner on both ranks (lmps_tp2_argmax_exchange), so the
131 MB head is read once per step across the pair instead of on both GPUs
(runners/engine.py:171-181 with the rows divided).
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import torch
import torch.distributed as dist

from . import kernels as K
from .config import ModelConfig
from .engine import QwenEngine
from .weights import LayerWeights, ModelWeights, interleave_rows


def local_config(cfg: ModelConfig, world: int) -> ModelConfig:
    """The per-rank model shape of a ``world``-way split."""
    if cfg.n_kv_heads % world or cfg.n_q_heads % world or cfg.intermediate % world:
        raise ValueError(f"{world}-way split needs heads and intermediate divisible by {world}")
    if (cfg.intermediate // world) % 32 or (cfg.q_dim // world) % 32:
        raise ValueError("a split must keep whole 32-element Q4 groups")
    return dataclasses.replace(cfg, n_q_heads=cfg.n_q_heads // world, n_kv_heads=cfg.n_kv_heads // world,
                               intermediate=cfg.intermediate // world)


def _rows(packed: torch.Tensor, scales: torch.Tensor, k: int, spans):
    """Output rows [a, b) of each span of a Q4 [rows, k] matrix."""
    p2, s2 = packed.reshape(-1, k // 2), scales.reshape(-1, k // 32)
    p = torch.cat([p2[a:b] for a, b in spans]).reshape(-1).contiguous()
    s = torch.cat([s2[a:b] for a, b in spans]).reshape(-1).contiguous()
    return p, s


def _cols(packed: torch.Tensor, scales: torch.Tensor, k: int, k0: int, k1: int):
    """Input columns [k0, k1) (multiples of 32) of a Q4 [rows, k] matrix."""
    p2, s2 = packed.reshape(-1, k // 2), scales.reshape(-1, k // 32)
    return (p2[:, k0 // 2:k1 // 2].reshape(-1).contiguous(),
            s2[:, k0 // 32:k1 // 32].reshape(-1).contiguous())


def shard_layer(lw: LayerWeights, cfg: ModelConfig, rank: int, world: int) -> LayerWeights:
    """Rank ``rank``'s slice of one layer (weights stay on their device)."""
    loc = local_config(cfg, world)
    D, hd = cfg.hidden, cfg.head_dim
    q0 = rank * loc.q_dim
    k0 = cfg.q_dim + rank * loc.kv_dim
    v0 = cfg.q_dim + cfg.kv_dim + rank * loc.kv_dim
    spans = [(q0, q0 + loc.q_dim), (k0, k0 + loc.kv_dim), (v0, v0 + loc.kv_dim)]
    qkv_p, qkv_s = _rows(lw.qkv_packed, lw.qkv_scales, D, spans)
    bias = torch.cat([lw.qkv_bias[a:b] for a, b in spans]).contiguous()
    o_p, o_s = _cols(lw.o_packed, lw.o_scales, cfg.q_dim, q0, q0 + loc.q_dim)
    i0, i1 = rank * loc.intermediate, (rank + 1) * loc.intermediate
    g_p, g_s = _rows(lw.gate_packed, lw.gate_scales, D, [(i0, i1)])
    u_p, u_s = _rows(lw.up_packed, lw.up_scales, D, [(i0, i1)])
    d_p, d_s = _cols(lw.down_packed, lw.down_scales, cfg.intermediate, i0, i1)
    del hd
    n = loc.intermediate
    return LayerWeights(in_norm=lw.in_norm, post_norm=lw.post_norm, qkv_packed=qkv_p, qkv_scales=qkv_s,
                        qkv_bias=bias, o_packed=o_p, o_scales=o_s, gate_packed=g_p, gate_scales=g_s,
                        up_packed=u_p, up_scales=u_s, down_packed=d_p, down_scales=d_s,
                        gu_packed=interleave_rows(g_p, u_p, n), gu_scales=interleave_rows(g_s, u_s, n))


def shard_model(mw: ModelWeights, rank: int, world: int) -> ModelWeights:
    """Rank ``rank``'s weights: sliced layers, replicated norms / embedding / LM head."""
    layers = [shard_layer(lw, mw.cfg, rank, world) for lw in mw.layers]
    return dataclasses.replace(mw, cfg=local_config(mw.cfg, world), layers=layers)


class TPEngine(QwenEngine):
    """QwenEngine on one rank of a tensor-parallel group: the per-stage
    kernels on the rank's slice, an all-reduce after o_proj and down_proj.

    ``comm="p2p"`` (two ranks): decode steps exchange the partial products
    through the peer's memory, so a step has no host-side collective and runs
    as a CUDA graph: the exchange kernel (:func:`kernels.tp2_allreduce_residual`)
    follows the o / down projection; with ``fuse_exchange=True`` the GEMV path
    (batch <= gemv_max_batch) instead does projection, NVLink stores into the peer's
    buffer and residual add in one kernel (:func:`kernels.gemv_q4_tp2_residual`,
    its own call sites).  Dense prefill, whose partials are
    [tokens, hidden], keeps NCCL.  ``comm="nccl"``: every all-reduce is
    NCCL's and steps launch eagerly.

    Every rank must make the same calls in the same order (the exchanges pair
    up by order).  Call :meth:`close` on every rank before the process group
    is destroyed."""

    def __init__(self, weights: ModelWeights, rank: int, world: int, group=None, comm: str = "p2p",
                 fuse_exchange: bool = False, **kw):
        kw.setdefault("decoder", "kernels")
        if kw["decoder"] != "kernels":
            raise ValueError("the tensor-parallel engine runs the per-stage kernels")
        if comm not in ("p2p", "nccl"):
            raise ValueError("comm is 'p2p' or 'nccl'")
        self.rank, self.world, self.group = rank, world, group
        self.full_cfg = weights.cfg
        super().__init__(weights=shard_model(weights, rank, world), **kw)
        self._part = torch.zeros(self.max_batch, self.cfg.hidden, dtype=torch.float16, device=self.device)
        self._site = {id(lw): 2 * li for li, lw in enumerate(self.weights.layers)}
        self.comm_err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.exchange = None
        self.fuse_exchange = fuse_exchange
        if comm == "p2p" and world == 2 and self.device.type == "cuda":
            # sites [0, 2L): exchanges after a GEMM; [2L, 4L): fused GEMV
            # exchanges; 4L: the split LM head's argmax
            self.exchange = K.PeerExchange(4 * self.cfg.n_layers + 1, self.max_batch * self.cfg.hidden, self.device)
            handles = [None] * world
            dist.all_gather_object(handles, self.exchange.handle(), group=group)
            self.exchange.connect(handles[1 - rank])
            dist.barrier(group=group)
        self.use_graphs = self.exchange is not None
        self.split_head = self.exchange is not None
        if self.split_head:  # this rank's vocabulary rows of the tied Q4 head (views, no copy)
            c, w = self.cfg, self.weights
            # split at a multiple of 128 rows: the GEMM path's row tiles
            cut = (c.vocab // 2 + 64) // 128 * 128
            v0, v1 = (0, cut) if rank == 0 else (cut, c.vocab)
            self._head_rows = (v0, v1)
            self._head_p = w.lm_packed[v0 * c.hidden // 2:v1 * c.hidden // 2]
            self._head_s = w.lm_scales[v0 * c.hidden // 32:v1 * c.hidden // 32]
            self._head_logits = torch.zeros(self.max_batch, v1 - v0, dtype=torch.float16, device=self.device)
            self._head_local = torch.zeros(self.max_batch, dtype=torch.int32, device=self.device)

    def close(self) -> None:
        """Unmap and free the peer exchange (collective: every rank calls it)."""
        if self.exchange is not None:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self._graphs.clear()
            self.exchange.close()
            self.exchange = None
            dist.barrier(group=self.group)

    def check_comm(self) -> None:
        if self.exchange is not None and int(self.comm_err.item()) != 0:
            raise RuntimeError("tensor-parallel exchange: a wait for the peer GPU timed out")

    def generate_batch(self, prompts, max_new_tokens: int):
        out = super().generate_batch(prompts, max_new_tokens)
        self.check_comm()
        return out

    def _head(self, B: int, want_logits: bool) -> None:
        """Final norm, LM head and argmax: split by vocabulary rows over the two
        ranks when only the next ids are wanted (each rank's rows through the
        GEMV + argmax, or for larger batches the GEMM + row argmax); the
        replicated head when the full logits are wanted."""
        if not (self.split_head and not want_logits):
            super()._head(B, want_logits)
            return
        c, w = self.cfg, self.weights
        v0, v1 = self._head_rows
        K.rms_norm(self.buf_residual[:B], w.final_norm, c.eps, out=self.buf_normed[:B])
        if B > self.gemv_max_batch:
            K.w4a16_gemm(self.buf_normed[:B], self._head_p, self._head_s, v1 - v0, c.hidden,
                         out=self._head_logits[:B], error=self.gemm_err, workspace=self.gemm_ws)
            K.argmax_rows(self._head_logits[:B], v1 - v0, self._head_local[:B])
        else:
            K.lm_head_argmax(self._head_p, self._head_s, self.buf_normed[:B], v1 - v0, c.hidden,
                             self.argmax_keys[:B], self._head_local[:B], logits=self._head_logits[:B])
        K.tp2_argmax_exchange(self._head_logits[:B], self._head_local[:B], v0, self.next_ids[:B], self.exchange,
                              4 * c.n_layers, self.comm_err)

    def _reduce_add(self, part: torch.Tensor, x: torch.Tensor, site: int = -1) -> None:
        if self.exchange is not None and site >= 0 and part.numel() <= self.exchange.max_n:
            K.tp2_allreduce_residual(part, x, self.exchange, site, self.comm_err)
            return
        dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
        K.residual_add(x, part, out=x)

    def _fused(self, x: torch.Tensor) -> bool:
        return self.fuse_exchange and self.exchange is not None and x.numel() <= self.exchange.max_n

    def _partial(self, rows: int) -> torch.Tensor:
        return self._part[:rows] if rows <= self._part.shape[0] else torch.empty(
            rows, self.cfg.hidden, dtype=torch.float16, device=self.device)

    def _o_proj(self, lw, att, x, gemm: bool, ws=None) -> None:
        c, part = self.cfg, self._partial(x.shape[0])
        if gemm:
            K.w4a16_gemm(att, lw.o_packed, lw.o_scales, c.hidden, c.q_dim, out=part, error=self.gemm_err,
                         workspace=self._ws(ws))
        elif self._fused(x):
            K.gemv_q4_tp2_residual(lw.o_packed, lw.o_scales, att, c.hidden, c.q_dim, x, part, self.exchange,
                                   2 * c.n_layers + self._site[id(lw)], self.comm_err)
            return
        else:
            K.gemv_q4(lw.o_packed, lw.o_scales, att, c.hidden, c.q_dim, out=part)
        self._reduce_add(part, x, self._site[id(lw)])

    def _down_proj(self, lw, a, x, gemm: bool, ws=None) -> None:
        c, part = self.cfg, self._partial(x.shape[0])
        if gemm:
            K.w4a16_gemm(a, lw.down_packed, lw.down_scales, c.hidden, c.intermediate, out=part,
                         error=self.gemm_err, workspace=self._ws(ws))
        elif self._fused(x):
            K.gemv_q4_tp2_residual(lw.down_packed, lw.down_scales, a, c.hidden, c.intermediate, x, part,
                                   self.exchange, 2 * c.n_layers + self._site[id(lw)] + 1, self.comm_err)
            return
        else:
            K.gemv_q4(lw.down_packed, lw.down_scales, a, c.hidden, c.intermediate, out=part)
        self._reduce_add(part, x, self._site[id(lw)] + 1)


def init_from_env(backend: str = "nccl", timeout_s: Optional[float] = 60.0):
    """Join the process group described by RANK / WORLD_SIZE / MASTER_* (torchrun)."""
    import datetime
    import os
    if not dist.is_initialized():
        kw = {"timeout": datetime.timedelta(seconds=timeout_s)} if timeout_s else {}
        if backend == "nccl":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group(backend=backend, **kw)
    return dist.get_rank(), dist.get_world_size()
