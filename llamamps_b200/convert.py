"""Offline converter: a Qwen2 safetensors checkpoint -> the reference's flat-.bin layout.

Restates the reference's extraction pipeline over one in-memory state dict:

* ``scripts/extract_layernorm.py:11-27`` / ``extract_postnorm.py:8-21``: the
  two RMSNorm gammas of layer i, cast to fp16, as ``layer{i}_norm.bin`` and
  ``layer{i}_post_attn_norm.bin``;
* ``scripts/extract_attn.py:15-26`` / ``extract_mlp.py:14-23``: every
  ``self_attn.{q,k,v,o,c}_proj`` and ``mlp.{down,up,gate}_proj`` weight packed
  by ``pack_tensor_4bit`` (``utils/pack_weights.py:11-47``: fp32, groups of
  32, scale max|w|/7, round-half-even, +8, two nibbles per byte, fp16
  scales) as ``{name}_4bit.bin`` / ``{name}_scales.bin``; a tensor the
  checkpoint lacks (Qwen2 has no ``c_proj``) is skipped, as the packer's
  KeyError branch does (``utils/pack_weights.py:13-17``);
* ``scripts/extract_all.py:20-60``: those files land in ``layer{i}/``;
* ``scripts/extract_global.py:17-34``: ``global/embed_tokens.bin`` and
  ``global/final_norm.bin`` in fp16, and the tied embedding packed as the LM
  head, ``embed_tokens_4bit.bin`` / ``embed_tokens_scales.bin`` at the top of
  the output directory (where ``pack_tensor_4bit`` writes them).

Qwen2's q/k/v biases, which the reference neither extracts nor applies
(``scripts/extract_attn.py:17-23``, ``runners/engine.py:124-141``), are
written as ``layer{i}/{q,k,v}_proj_bias.bin`` (fp16) unless
``with_bias=False``; ``weights.load_reference_layout`` reads them when present.

``write_synthetic_checkpoint`` writes a seeded random-init checkpoint with the
tensor names and bf16 storage of a Hugging Face Qwen2 ``model.safetensors``
(no real checkpoint is available offline).
"""
from __future__ import annotations

import os
import re
from typing import Dict, Optional

import numpy as np
import torch

from .config import ModelConfig
from .quant import pack_q4_host

_ATTN = ("q_proj", "k_proj", "v_proj", "o_proj", "c_proj")   # scripts/extract_attn.py:17-23
_MLP = ("down_proj", "up_proj", "gate_proj")                 # scripts/extract_mlp.py:16-20


def _n_layers(state: Dict[str, torch.Tensor]) -> int:
    idx = [int(m.group(1)) for k in state for m in [re.match(r"model\.layers\.(\d+)\.", k)] if m]
    if not idx:
        raise ValueError("no model.layers.<i>. tensors in the checkpoint")
    return max(idx) + 1


def _dump_f16(t: torch.Tensor, path: str) -> None:
    t.detach().to(torch.float16).contiguous().numpy().tofile(path)


def _dump_q4(t: torch.Tensor, stem: str) -> None:
    packed, scales = pack_q4_host(t.to(torch.float32))
    packed.numpy().tofile(stem + "_4bit.bin")
    scales.numpy().tofile(stem + "_scales.bin")


def convert_state_dict(state: Dict[str, torch.Tensor], out_dir: str, n_layers: Optional[int] = None,
                       with_bias: bool = True) -> int:
    """Write ``state`` (HF Qwen2 tensor names) in the reference layout under
    ``out_dir``; returns the number of layers written."""
    n = _n_layers(state) if n_layers is None else n_layers
    os.makedirs(out_dir, exist_ok=True)
    for i in range(n):
        d = os.path.join(out_dir, f"layer{i}")
        os.makedirs(d, exist_ok=True)
        pre = f"model.layers.{i}."
        for key, name in ((pre + "input_layernorm.weight", f"layer{i}_norm.bin"),
                          (pre + "post_attention_layernorm.weight", f"layer{i}_post_attn_norm.bin")):
            if key not in state:
                raise KeyError(f"checkpoint lacks {key}")
            _dump_f16(state[key], os.path.join(d, name))
        for part, names in (("self_attn", _ATTN), ("mlp", _MLP)):
            for name in names:
                key = f"{pre}{part}.{name}.weight"
                if key in state:
                    _dump_q4(state[key], os.path.join(d, name))
        if with_bias:
            for name in ("q_proj", "k_proj", "v_proj"):
                key = f"{pre}self_attn.{name}.bias"
                if key in state:
                    _dump_f16(state[key], os.path.join(d, f"{name}_bias.bin"))
    g = os.path.join(out_dir, "global")
    os.makedirs(g, exist_ok=True)
    _dump_f16(state["model.embed_tokens.weight"], os.path.join(g, "embed_tokens.bin"))
    _dump_f16(state["model.norm.weight"], os.path.join(g, "final_norm.bin"))
    _dump_q4(state["model.embed_tokens.weight"], os.path.join(out_dir, "embed_tokens"))
    return n


def convert_safetensors(model_path: str, out_dir: str, n_layers: Optional[int] = None,
                        with_bias: bool = True) -> int:
    """``model.safetensors`` -> reference layout (see the module docstring)."""
    from safetensors.torch import load_file
    return convert_state_dict(load_file(model_path), out_dir, n_layers, with_bias)


def synthetic_state_dict(cfg: ModelConfig, seed: int, dtype=torch.bfloat16) -> Dict[str, torch.Tensor]:
    """Seeded random-init Qwen2 tensors (numpy default_rng(seed), drawn in the
    order below, stored as ``dtype``): per layer q/k/v/o/gate/up/down weights
    N(0, 0.02), q/k/v biases N(0, 0.02), the two gammas 1 + N(0, 0.02); then
    the tied embedding N(0, 0.02) and the final gamma."""
    rng = np.random.default_rng(seed)
    d, i = cfg.hidden, cfg.intermediate
    shapes = (("self_attn.q_proj", (cfg.q_dim, d)), ("self_attn.k_proj", (cfg.kv_dim, d)),
              ("self_attn.v_proj", (cfg.kv_dim, d)), ("self_attn.o_proj", (d, cfg.q_dim)),
              ("mlp.gate_proj", (i, d)), ("mlp.up_proj", (i, d)), ("mlp.down_proj", (d, i)))

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dtype)
    st: Dict[str, torch.Tensor] = {}
    for li in range(cfg.n_layers):
        pre = f"model.layers.{li}."
        for name, shape in shapes:
            st[pre + name + ".weight"] = t(rng.normal(0.0, 0.02, shape))
        for name, rows in (("q_proj", cfg.q_dim), ("k_proj", cfg.kv_dim), ("v_proj", cfg.kv_dim)):
            st[pre + f"self_attn.{name}.bias"] = t(rng.normal(0.0, 0.02, rows))
        st[pre + "input_layernorm.weight"] = t(1.0 + rng.normal(0.0, 0.02, d))
        st[pre + "post_attention_layernorm.weight"] = t(1.0 + rng.normal(0.0, 0.02, d))
    st["model.embed_tokens.weight"] = t(rng.normal(0.0, 0.02, (cfg.vocab, d)))
    st["model.norm.weight"] = t(1.0 + rng.normal(0.0, 0.02, d))
    return st


def write_synthetic_checkpoint(path: str, cfg: ModelConfig, seed: int) -> None:
    """``synthetic_state_dict`` saved as a safetensors file at ``path``."""
    from safetensors.torch import save_file
    save_file(synthetic_state_dict(cfg, seed), path)
