"""ctypes binding of ``libllamamps_b200.so`` (the C ABI in include/llamamps_b200.h).

This is the B200 counterpart of the reference's pyobjc Metal binding
(runners/engine.py:49-58, where kernels are looked up by name and fed
positional device buffers).  Every entry point takes raw device pointers, an
int status comes back, and :func:`check` turns a non-zero status into a
``RuntimeError`` naming the call.  There is no CPU fallback: if the library
is missing, importing a kernel raises.
"""
from __future__ import annotations

import ctypes
import os
import re
from typing import List

from .build import INCLUDE, LIB_PATH

c_int, c_float, c_ll, c_size = ctypes.c_int, ctypes.c_float, ctypes.c_longlong, ctypes.c_size_t
c_vp = ctypes.c_void_p

# name -> (restype, argtypes); pointers are passed as integers (tensor.data_ptr()).
_SIGS = {
    "lmps_version": (c_int, []),
    "lmps_status_string": (ctypes.c_char_p, [c_int]),
    "lmps_gemv_q4_0": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp, c_int, c_int, c_int, c_int, c_vp]),
    "lmps_gemv_q4_bias": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_int, c_int, c_int, c_int, c_vp]),
    "lmps_gemv_q4_residual": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp]),
    "lmps_gemv_q4_swiglu": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_int, c_int, c_int, c_int, c_vp]),
    "lmps_lm_head_argmax": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp]),
    "lmps_rms_norm": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_float, c_vp]),
    "lmps_rope": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp]),
    "lmps_residual_add": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp]),
    "lmps_swiglu": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp]),
    "lmps_embed_gather": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp]),
    "lmps_attention_scores": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp]),
    "lmps_softmax": (c_int, [c_vp, c_int, c_int, c_vp]),
    "lmps_attn_weighted_sum": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp]),
    "lmps_rope_kv_append": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                                    c_int, c_int, c_int, c_int, c_vp]),
    "lmps_gqa_attention_splits": (c_int, [c_int, c_int, c_int, c_int]),
    "lmps_gqa_attention_workspace_size": (c_size, [c_int, c_int, c_int, c_int]),
    "lmps_gqa_decode_attention": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_size, c_int,
                                          c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_vp]),
    "lmps_gqa_decode_attention_noalloc": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int,
                                                  c_int, c_int, c_int, c_int, c_int, c_int, c_vp]),
    "lmps_q4_pack": (c_int, [c_vp, c_ll, c_vp, c_vp, c_vp]),
    "lmps_decode_advance": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_vp]),
    "lmps_prefill_attention": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_vp, c_int, c_int, c_int,
                                       c_int, c_int, c_int, c_vp]),
    "lmps_prefill_attention_tcgen05": (c_int, [c_vp, c_int, c_vp, c_vp, c_int, c_vp, c_int, c_int, c_vp, c_int,
                                               c_int, c_int, c_int, c_int, c_int, c_vp, c_vp]),
    "lmps_swiglu_rows": (c_int, [c_vp, c_int, c_int, c_int, c_vp, c_int, c_vp]),
    "lmps_gqa_decode_attention_rope": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                               c_size, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                               c_vp]),
    "lmps_comm_alloc": (c_int, [c_size, ctypes.POINTER(c_vp)]),
    "lmps_comm_free": (c_int, [c_vp]),
    "lmps_ipc_handle": (c_int, [c_vp, c_vp]),
    "lmps_ipc_open": (c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "lmps_ipc_close": (c_int, [c_vp]),
    "lmps_tp2_comm_bytes": (c_size, [c_int, c_int]),
    "lmps_tp2_allreduce_residual": (c_int, [c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp,
                                            ctypes.c_ulonglong, c_vp]),
    "lmps_gemv_q4_tp2_residual": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp,
                                          c_vp, c_int, c_int, c_int, c_vp, ctypes.c_ulonglong, c_vp]),
    "lmps_argmax_rows": (c_int, [c_vp, c_int, c_int, c_int, c_vp, c_vp]),
    "lmps_tp2_argmax_exchange": (c_int, [c_vp, c_int, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_int, c_int,
                                         c_int, c_vp, ctypes.c_ulonglong, c_vp]),
    "lmps_sample_rows": (c_int, [c_vp, c_int, c_int, c_int, c_int, c_float, ctypes.c_ulonglong,
                                 ctypes.c_ulonglong, c_vp, c_vp, c_vp]),
    "lmps_w4a16_gemm_workspace_size": (c_size, [c_int, c_int]),
    "lmps_w4a16_gemm": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_int, c_int, c_int, c_int,
                                c_int, c_vp, c_vp, c_size, c_vp]),
}

_LIB = None


def header_symbols() -> List[str]:
    """Function names declared in include/llamamps_b200.h."""
    with open(os.path.join(INCLUDE, "llamamps_b200.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(lmps_[a-z0-9_]+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    """Load the shared library (once) and declare every signature."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m llamamps_b200.build` "
                "(the decode path has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def status_string(status: int) -> str:
    return lib().lmps_status_string(int(status)).decode()


def check(status: int, name: str) -> None:
    if status != 0:
        raise RuntimeError(f"{name} failed: {status_string(status)} (status {status})")


def call(name: str, *args) -> None:
    """Invoke entry point ``name`` and raise on a non-zero status."""
    check(getattr(lib(), name)(*args), name)
