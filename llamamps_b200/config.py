"""Model constants of the decode path.

Defaults are the reference's module constants (runners/engine.py:7-18,
Qwen2.5-1.5B) plus what the reference hard-codes inside kernels: RMSNorm eps
1e-6 (kernels/rms_norm.metal:35-36), head_dim 128 and the GQA group of 6
(kernels/attention.metal:23,26).  ``rope_theta`` and ``rope_style`` are
parameters here because the reference fixes them at m=0 / base 1e4
(kernels/rope.metal:23,28), where any base gives the identity rotation.
"""
from __future__ import annotations

import dataclasses


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    hidden: int = 1536
    intermediate: int = 8960
    vocab: int = 151936
    n_layers: int = 28
    n_q_heads: int = 12
    n_kv_heads: int = 2
    head_dim: int = 128
    eps: float = 1e-6
    rope_theta: float = 1e6
    rope_style: str = "interleaved"   # kernels/rope.metal adjacent pairs; "neox" = HF half split

    @property
    def q_dim(self) -> int:
        return self.n_q_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_rows(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    @property
    def rope_style_code(self) -> int:
        return {"interleaved": 0, "neox": 1}[self.rope_style]

    def layer_q4_bytes(self) -> int:
        """Packed + scale bytes of one layer's seven Q4 matrices."""
        d, i = self.hidden, self.intermediate
        elems = (self.qkv_rows + self.q_dim) * d + 3 * i * d
        return elems // 2 + elems // 32 * 2

    def step_weight_bytes(self) -> int:
        """Algorithmic weight bytes one decode step reads: Q4 layers, the Q4
        LM head, norms, biases, the final norm and one embedding row."""
        d = self.hidden
        lm = self.vocab * d // 2 + self.vocab * d // 32 * 2
        norms = self.n_layers * 2 * d * 2
        biases = self.n_layers * self.qkv_rows * 2
        return self.n_layers * self.layer_q4_bytes() + lm + norms + biases + d * 2 + d * 2

    def kv_bytes_per_position(self) -> int:
        """K + V bytes read per attended position over all layers."""
        return self.n_layers * 2 * self.kv_dim * 2


QWEN2_5_1_5B = ModelConfig()
