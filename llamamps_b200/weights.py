"""Device-resident Q4 weights: the reference's on-disk layout, synthetic models.

HBM layout.  Per layer the seven Q4 matrices stay in the reference format
(row-major packed nibbles + one fp16 scale per 32 elements) but q|k|v are
concatenated row-wise into one [2048, 1536] matrix (with a [2048] bias) so a
single GEMV produces all three, and gate/up are kept as two matrices read by
the same fused SwiGLU GEMV.  Everything is loaded once and stays resident:
the reference instead memcpys every layer into shared buffers on every token
(runners/engine.py:145-155).

On-disk layout read and written here (runners/engine.py:40-46, :120-143;
utils/tokenizer.py:8; scripts/extract_all.py:20-49):

    <dir>/layer{i}/layer{i}_norm.bin, layer{i}_post_attn_norm.bin     fp16 [D]
    <dir>/layer{i}/{q,k,v,o,gate,up,down}_proj_4bit.bin                 uint8
    <dir>/layer{i}/{q,k,v,o,gate,up,down}_proj_scales.bin               fp16
    <dir>/layer{i}/{q,k,v}_proj_bias.bin      fp16, optional (Qwen2 biases; the reference has none)
    <dir>/global/final_norm.bin                                          fp16 [D]
    <dir>/global/embed_tokens.bin                                        fp16 [V, D]
    <dir>/embed_tokens_4bit.bin, <dir>/embed_tokens_scales.bin           Q4 tied LM head
"""
from __future__ import annotations

import dataclasses
import os
from typing import Dict, List, Optional

import numpy as np
import torch

from .config import ModelConfig
from .quant import pack_q4, pack_q4_host

_MATS = ("q", "k", "v", "o", "gate", "up", "down")


@dataclasses.dataclass
class LayerWeights:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    qkv_packed: torch.Tensor
    qkv_scales: torch.Tensor
    qkv_bias: torch.Tensor
    o_packed: torch.Tensor
    o_scales: torch.Tensor
    gate_packed: torch.Tensor
    gate_scales: torch.Tensor
    up_packed: torch.Tensor
    up_scales: torch.Tensor
    down_packed: torch.Tensor
    down_scales: torch.Tensor
    # gate and up rows interleaved (row 2t = gate row t, 2t + 1 = up row t),
    # a copy for the batched path: one GEMM with the SwiGLU epilogue.  None
    # when absent (two GEMMs and a SwiGLU kernel instead).
    gu_packed: Optional[torch.Tensor] = None
    gu_scales: Optional[torch.Tensor] = None

    def q4_bytes(self) -> int:
        ts = [self.qkv_packed, self.qkv_scales, self.o_packed, self.o_scales, self.gate_packed,
              self.gate_scales, self.up_packed, self.up_scales, self.down_packed, self.down_scales]
        return sum(t.numel() * t.element_size() for t in ts)


@dataclasses.dataclass
class ModelWeights:
    cfg: ModelConfig
    layers: List[LayerWeights]
    final_norm: torch.Tensor
    lm_packed: torch.Tensor
    lm_scales: torch.Tensor
    embed: torch.Tensor

    @property
    def device(self) -> torch.device:
        return self.final_norm.device


def _mat_shape(cfg: ModelConfig, name: str):
    d, i = cfg.hidden, cfg.intermediate
    return {"q": (cfg.q_dim, d), "k": (cfg.kv_dim, d), "v": (cfg.kv_dim, d), "o": (d, cfg.q_dim),
            "gate": (i, d), "up": (i, d), "down": (d, i)}[name]


def interleave_rows(a: torch.Tensor, b: torch.Tensor, rows: int) -> torch.Tensor:
    """Row-interleave two [rows, w] matrices given flat: row 2t of the result
    is a's row t, row 2t + 1 is b's (the gate/up layout of the GEMM's SwiGLU
    epilogue)."""
    return torch.stack([a.reshape(rows, -1), b.reshape(rows, -1)], dim=1).reshape(-1).contiguous()


def layer_from_parts(cfg: ModelConfig, parts: Dict[str, torch.Tensor], device) -> LayerWeights:
    """Assemble the device layout from per-matrix packed/scales (+ optional bias)."""
    dev = torch.device(device)

    def t(x, dtype):
        return torch.as_tensor(x).to(device=dev, dtype=dtype).contiguous()

    bias = []
    for n, rows in (("q", cfg.q_dim), ("k", cfg.kv_dim), ("v", cfg.kv_dim)):
        b = parts.get(f"{n}_bias")
        bias.append(t(b, torch.float16) if b is not None else torch.zeros(rows, dtype=torch.float16, device=dev))
    gp, gs = t(parts["gate_packed"], torch.uint8), t(parts["gate_scales"], torch.float16)
    up, us = t(parts["up_packed"], torch.uint8), t(parts["up_scales"], torch.float16)
    return LayerWeights(
        in_norm=t(parts["in_norm"], torch.float16),
        post_norm=t(parts["post_norm"], torch.float16),
        qkv_packed=torch.cat([t(parts[f"{n}_packed"], torch.uint8) for n in "qkv"]),
        qkv_scales=torch.cat([t(parts[f"{n}_scales"], torch.float16) for n in "qkv"]),
        qkv_bias=torch.cat(bias),
        o_packed=t(parts["o_packed"], torch.uint8), o_scales=t(parts["o_scales"], torch.float16),
        gate_packed=gp, gate_scales=gs, up_packed=up, up_scales=us,
        down_packed=t(parts["down_packed"], torch.uint8), down_scales=t(parts["down_scales"], torch.float16),
        gu_packed=interleave_rows(gp, up, cfg.intermediate), gu_scales=interleave_rows(gs, us, cfg.intermediate),
    )


# ---------------------------------------------------------------------------
# Reference on-disk layout
# ---------------------------------------------------------------------------

def _load_bin(path: str, dtype) -> np.ndarray:
    """runners/engine.py:20-23 `load_bin`."""
    if not os.path.exists(path):
        raise FileNotFoundError(f"Missing weight file: {path}")
    return np.fromfile(path, dtype=dtype)


def load_reference_layout(weights_dir: str, cfg: ModelConfig, device="cuda",
                          n_layers: Optional[int] = None) -> ModelWeights:
    """Read the flat-.bin layout written by the reference's extract scripts."""
    layers = []
    for i in range(cfg.n_layers if n_layers is None else n_layers):
        d = os.path.join(weights_dir, f"layer{i}")
        parts = {"in_norm": _load_bin(os.path.join(d, f"layer{i}_norm.bin"), np.float16),
                 "post_norm": _load_bin(os.path.join(d, f"layer{i}_post_attn_norm.bin"), np.float16)}
        for m in _MATS:
            parts[f"{m}_packed"] = _load_bin(os.path.join(d, f"{m}_proj_4bit.bin"), np.uint8)
            parts[f"{m}_scales"] = _load_bin(os.path.join(d, f"{m}_proj_scales.bin"), np.float16)
        for m in "qkv":
            bp = os.path.join(d, f"{m}_proj_bias.bin")
            if os.path.exists(bp):
                parts[f"{m}_bias"] = np.fromfile(bp, np.float16)
        _check_layer_sizes(cfg, parts, i)
        layers.append(layer_from_parts(cfg, {k: torch.from_numpy(v) for k, v in parts.items()}, device))
    g = os.path.join(weights_dir, "global")
    final_norm = torch.from_numpy(_load_bin(os.path.join(g, "final_norm.bin"), np.float16))
    lm_packed = torch.from_numpy(_load_bin(os.path.join(weights_dir, "embed_tokens_4bit.bin"), np.uint8))
    lm_scales = torch.from_numpy(_load_bin(os.path.join(weights_dir, "embed_tokens_scales.bin"), np.float16))
    embed = torch.from_numpy(_load_bin(os.path.join(g, "embed_tokens.bin"), np.float16)).reshape(-1, cfg.hidden)
    dev = torch.device(device)
    return ModelWeights(cfg, layers, final_norm.to(dev), lm_packed.to(dev), lm_scales.to(dev), embed.to(dev))


def _check_layer_sizes(cfg: ModelConfig, parts, layer):
    for m in _MATS:
        rows, k = _mat_shape(cfg, m)
        if parts[f"{m}_packed"].size != rows * k // 2 or parts[f"{m}_scales"].size != rows * k // 32:
            raise ValueError(f"layer{layer} {m}_proj: expected {rows}x{k} Q4 data, got "
                             f"{parts[f'{m}_packed'].size} bytes / {parts[f'{m}_scales'].size} scales")


def save_reference_layout(mw: ModelWeights, weights_dir: str) -> None:
    """Write ``mw`` in the reference's flat-.bin layout (see module docstring)."""
    cfg = mw.cfg

    def dump(t: torch.Tensor, path: str):
        t.detach().cpu().contiguous().numpy().tofile(path)

    for i, lw in enumerate(mw.layers):
        d = os.path.join(weights_dir, f"layer{i}")
        os.makedirs(d, exist_ok=True)
        dump(lw.in_norm, os.path.join(d, f"layer{i}_norm.bin"))
        dump(lw.post_norm, os.path.join(d, f"layer{i}_post_attn_norm.bin"))
        qb = cfg.q_dim * cfg.hidden // 2
        kb = cfg.kv_dim * cfg.hidden // 2
        for m, lo, hi in (("q", 0, qb), ("k", qb, qb + kb), ("v", qb + kb, qb + 2 * kb)):
            dump(lw.qkv_packed[lo:hi], os.path.join(d, f"{m}_proj_4bit.bin"))
            dump(lw.qkv_scales[lo // 16:hi // 16], os.path.join(d, f"{m}_proj_scales.bin"))
        qr, kr = cfg.q_dim, cfg.kv_dim
        for m, lo, hi in (("q", 0, qr), ("k", qr, qr + kr), ("v", qr + kr, qr + 2 * kr)):
            dump(lw.qkv_bias[lo:hi], os.path.join(d, f"{m}_proj_bias.bin"))
        for m in ("o", "gate", "up", "down"):
            dump(getattr(lw, f"{m}_packed"), os.path.join(d, f"{m}_proj_4bit.bin"))
            dump(getattr(lw, f"{m}_scales"), os.path.join(d, f"{m}_proj_scales.bin"))
    g = os.path.join(weights_dir, "global")
    os.makedirs(g, exist_ok=True)
    dump(mw.final_norm, os.path.join(g, "final_norm.bin"))
    dump(mw.embed, os.path.join(g, "embed_tokens.bin"))
    dump(mw.lm_packed, os.path.join(weights_dir, "embed_tokens_4bit.bin"))
    dump(mw.lm_scales, os.path.join(weights_dir, "embed_tokens_scales.bin"))


# ---------------------------------------------------------------------------
# Synthetic weights (seeded)
# ---------------------------------------------------------------------------

def synth_layer_numpy(rng: np.random.Generator, cfg: ModelConfig, with_bias: bool = True):
    """One layer drawn with numpy: each of q, k, v, o, gate, up, down ~ N(0, 0.02)
    fp32 [out, in] (in that order) packed to Q4; then q/k/v biases fp16
    N(0, 0.02); then the two RMSNorm gammas 1 + N(0, 0.02) in fp16."""
    parts = {}
    for m in _MATS:
        w = rng.normal(0.0, 0.02, _mat_shape(cfg, m)).astype(np.float32)
        p, s = pack_q4_host(torch.from_numpy(w))
        parts[f"{m}_packed"], parts[f"{m}_scales"] = p.numpy(), s.numpy()
    if with_bias:
        for m, rows in (("q", cfg.q_dim), ("k", cfg.kv_dim), ("v", cfg.kv_dim)):
            parts[f"{m}_bias"] = rng.normal(0.0, 0.02, rows).astype(np.float16)
    parts["in_norm"] = (1.0 + rng.normal(0.0, 0.02, cfg.hidden)).astype(np.float16)
    parts["post_norm"] = (1.0 + rng.normal(0.0, 0.02, cfg.hidden)).astype(np.float16)
    return parts


def synth_one_layer_case(cfg: ModelConfig, seed: int = 0, prefix: int = 31):
    """One decoder layer, one decode step, batch 1, from one numpy seed: the
    layer's weights (synth_layer_numpy), then the fp16 N(0,1) input hidden
    state, then a K cache and a V cache of ``prefix`` positions fp16 N(0,1);
    the new token sits at position ``prefix``."""
    rng = np.random.default_rng(seed)
    parts = synth_layer_numpy(rng, cfg)
    x = rng.normal(0.0, 1.0, cfg.hidden).astype(np.float16)
    k_prefix = rng.normal(0.0, 1.0, (prefix, cfg.kv_dim)).astype(np.float16)
    v_prefix = rng.normal(0.0, 1.0, (prefix, cfg.kv_dim)).astype(np.float16)
    return parts, x, k_prefix, v_prefix


def synth_model(cfg: ModelConfig, seed: int, device="cuda", n_layers: Optional[int] = None,
                with_bias: bool = True) -> ModelWeights:
    """A random-init model drawn by torch's generator on ``device`` (seeded):
    per layer q, k, v, o, gate, up, down ~ N(0, 0.02) fp32 packed to Q4 on the
    device, q/k/v biases fp16 N(0, 0.02), gammas 1 + N(0, 0.02); then the tied
    fp16 embedding N(0, 0.02) [V, D] (its Q4 packing is the LM head) and the
    final gamma."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(int(seed))
    layers = []
    for _ in range(cfg.n_layers if n_layers is None else n_layers):
        parts = {}
        for m in _MATS:
            rows, k = _mat_shape(cfg, m)
            w = torch.randn(rows, k, generator=g, device=dev, dtype=torch.float32).mul_(0.02)
            parts[f"{m}_packed"], parts[f"{m}_scales"] = pack_q4(w)
            del w
        if with_bias:
            for m, rows in (("q", cfg.q_dim), ("k", cfg.kv_dim), ("v", cfg.kv_dim)):
                parts[f"{m}_bias"] = (torch.randn(rows, generator=g, device=dev) * 0.02).half()
        parts["in_norm"] = (1.0 + 0.02 * torch.randn(cfg.hidden, generator=g, device=dev)).half()
        parts["post_norm"] = (1.0 + 0.02 * torch.randn(cfg.hidden, generator=g, device=dev)).half()
        layers.append(layer_from_parts(cfg, parts, dev))
    embed = (torch.randn(cfg.vocab, cfg.hidden, generator=g, device=dev) * 0.02).half()
    lm_packed, lm_scales = pack_q4(embed.float())
    final_norm = (1.0 + 0.02 * torch.randn(cfg.hidden, generator=g, device=dev)).half()
    return ModelWeights(cfg, layers, final_norm, lm_packed, lm_scales, embed)


def layer_host_arrays(lw: LayerWeights, cfg: ModelConfig) -> dict:
    """Host numpy copy of a layer in the reference's key naming (engine.py:124-141)."""
    qb, kb = cfg.q_dim * cfg.hidden // 2, cfg.kv_dim * cfg.hidden // 2
    qkv_p = lw.qkv_packed.cpu().numpy()
    qkv_s = lw.qkv_scales.cpu().numpy()
    bias = lw.qkv_bias.cpu().numpy()
    qr, kr = cfg.q_dim, cfg.kv_dim
    return {
        "in_norm": lw.in_norm.cpu().numpy(), "post_norm": lw.post_norm.cpu().numpy(),
        "q": qkv_p[:qb], "qs": qkv_s[:qb // 16],
        "k": qkv_p[qb:qb + kb], "ks": qkv_s[qb // 16:(qb + kb) // 16],
        "v": qkv_p[qb + kb:], "vs": qkv_s[(qb + kb) // 16:],
        "bq": bias[:qr], "bk": bias[qr:qr + kr], "bv": bias[qr + kr:],
        "o": lw.o_packed.cpu().numpy(), "os": lw.o_scales.cpu().numpy(),
        "gt": lw.gate_packed.cpu().numpy(), "gts": lw.gate_scales.cpu().numpy(),
        "up": lw.up_packed.cpu().numpy(), "ups": lw.up_scales.cpu().numpy(),
        "dn": lw.down_packed.cpu().numpy(), "dns": lw.down_scales.cpu().numpy(),
    }


def parts_host_arrays(parts: dict) -> dict:
    """numpy parts (synth_layer_numpy) -> the reference's key naming."""
    return {
        "in_norm": parts["in_norm"], "post_norm": parts["post_norm"],
        "q": parts["q_packed"], "qs": parts["q_scales"], "k": parts["k_packed"], "ks": parts["k_scales"],
        "v": parts["v_packed"], "vs": parts["v_scales"], "o": parts["o_packed"], "os": parts["o_scales"],
        "gt": parts["gate_packed"], "gts": parts["gate_scales"], "up": parts["up_packed"],
        "ups": parts["up_scales"], "dn": parts["down_packed"], "dns": parts["down_scales"],
        "bq": parts.get("q_bias"), "bk": parts.get("k_bias"), "bv": parts.get("v_bias"),
    }


def model_host_arrays(mw: ModelWeights) -> dict:
    return {"layers": [layer_host_arrays(lw, mw.cfg) for lw in mw.layers],
            "final_norm": mw.final_norm.cpu().numpy(), "lm_packed": mw.lm_packed.cpu().numpy(),
            "lm_scales": mw.lm_scales.cpu().numpy(), "embed": mw.embed.cpu().numpy()}
