"""LlamaMPS decode path on NVIDIA B200 (sm_100a).

Host side in Python (the reference's ``QwenEngine`` API), device side in
hand-written CUDA behind the C ABI of ``include/llamamps_b200.h``.
"""
from .config import QWEN2_5_1_5B, ModelConfig

__all__ = ["ModelConfig", "QWEN2_5_1_5B", "QwenEngine"]


def __getattr__(name):
    if name == "QwenEngine":
        from .engine import QwenEngine
        return QwenEngine
    raise AttributeError(name)
