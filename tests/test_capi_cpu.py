"""The C-ABI library loads and exports every symbol include/llamamps_b200.h
declares; argument validation rejects bad calls before any device work.
No kernel runs here (no GPU)."""
import ctypes
import subprocess

import pytest

from llamamps_b200 import _lib
from llamamps_b200.build import LIB_PATH


def test_library_exports_every_header_symbol():
    L = _lib.lib()
    syms = _lib.header_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, f"not exported: {missing}"
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert set(syms) <= exported


def test_every_header_symbol_has_a_python_signature():
    from llamamps_b200 import batched, persistent
    assert set(_lib.header_symbols()) == set(_lib._SIGS) | set(persistent._SIGS) | set(batched._SIGS)


def test_batched_descriptor_layouts_match_the_header():
    """ctypes mirrors of lmps_batched_layer / lmps_batched_desc; argument
    validation of the batched decode and the tile-major repack."""
    import ctypes
    from llamamps_b200 import batched as Bd
    assert ctypes.sizeof(Bd.BatchedLayer) == 9 * 8
    assert Bd.BatchedDesc.n_layers.offset == 8 and Bd.BatchedDesc.inv_freq.offset == 40
    assert ctypes.sizeof(Bd.BatchedDesc) == 48
    L = Bd._declare()
    assert L.lmps_q4_tile_blocks_size(2048, 1536) == 16 * 24 * 4608
    assert L.lmps_q4_tile_blocks_size(100, 1536) == 0 and L.lmps_q4_tile_blocks_size(128, 100) == 0
    assert L.lmps_q4_tile_blocks(None, None, 128, 64, None, None) == -1
    assert L.lmps_q4_tile_blocks(16, 16, 100, 64, 16, None) == -1
    m = Bd.BatchedDesc(None, 28, 1536, 8960, 12, 2, 128, 1e-6, 0, None)
    assert L.lmps_decode_batched(ctypes.byref(m), 16, 16, 16, 16, 1, 64, 8, 64, 256, 1 << 20, 16, None, None) == -1
    m = Bd.BatchedDesc(16, 28, 1536, 8960, 12, 2, 64, 1e-6, 0, 16)  # head_dim 64
    assert L.lmps_decode_batched(ctypes.byref(m), 16, 16, 16, 16, 1, 64, 8, 64, 256, 1 << 20, 16, None, None) == -2
    m = Bd.BatchedDesc(16, 28, 1536, 8960, 12, 2, 128, 1e-6, 0, 16)
    assert L.lmps_decode_batched(ctypes.byref(m), 16, 16, 16, 16, 1, 64, 65, 64, 256, 1 << 20, 16, None, None) == -2


def test_persistent_descriptor_layouts_match_the_header():
    """ctypes mirrors of lmps_layer_desc / lmps_model_desc / lmps_decode_state."""
    import ctypes
    from llamamps_b200 import persistent as P
    assert ctypes.sizeof(P.LayerDesc) == 15 * 8
    assert P.ModelDesc.layers.offset == 40 and ctypes.sizeof(P.ModelDesc) == 40 + 6 * 8
    assert P.DecodeState.block_table.offset == 16 and P.DecodeState.rope_table.offset == 24
    assert P.DecodeState.error.offset == 120
    L = _lib.lib()
    P._declare()
    m = P.ModelDesc(28, 1536, 8960, 151936, 12, 2, 128, 1e-6, 0, None, None, None, None, None, None)
    ws = L.lmps_decode_persistent_workspace_size(ctypes.byref(m), 1, 4096)
    assert ws > 0 and ws % 256 == 0
    # argument validation happens before any device work
    st = P.DecodeState()
    assert L.lmps_decode_persistent(ctypes.byref(m), ctypes.byref(st), 1, None) == -1


def test_status_strings():
    assert _lib.status_string(0) == "ok"
    assert "argument" in _lib.status_string(-1)
    assert "workspace" in _lib.status_string(-3)
    assert "timed out" in _lib.status_string(-4)
    assert _lib.lib().lmps_version() >= 100


@pytest.mark.parametrize("call", [
    lambda L: L.lmps_gemv_q4_0(None, None, None, 1536, None, 1536, 1536, 1536, 1, None),
    lambda L: L.lmps_gemv_q4_0(16, 16, 16, 1536, 16, 1536, 1536, 1500, 1, None),   # k % 32
    lambda L: L.lmps_gemv_q4_0(16, 16, 16, 1536, 16, 1536, 1536, 1536, 9, None),   # batch > 8
    lambda L: L.lmps_gemv_q4_0(17, 16, 16, 1536, 16, 1536, 1536, 1536, 1, None),   # misaligned
    lambda L: L.lmps_rms_norm(16, 16, 16, 0, 1, 1e-6, None),
    lambda L: L.lmps_rope(16, 16, 16, 12, 127, 1, 0, None),                        # odd head_dim
    lambda L: L.lmps_rope(16, 16, 16, 12, 128, 1, 7, None),                        # bad style
    lambda L: L.lmps_gqa_decode_attention(16, 16, 16, 16, 16, 16, None, 0, 1, 64, 12, 5, 128, 1, 64, 1, None),
    lambda L: L.lmps_q4_pack(16, 0, 16, 16, None),
])
def test_invalid_arguments_rejected(call):
    assert call(_lib.lib()) == -1


def test_attention_unsupported_head_dim_and_workspace():
    L = _lib.lib()
    assert L.lmps_gqa_decode_attention(16, 16, 16, 16, 16, 16, None, 0, 1, 64, 12, 2, 64, 1, 64, 1, None) == -2
    need = L.lmps_gqa_attention_workspace_size(1, 12, 128, 4)
    assert need == 12 * 4 * (128 * 4 + 8)
    assert L.lmps_gqa_decode_attention(16, 16, 16, 16, 16, 16, 16, need - 1, 1, 64, 12, 2, 128, 1, 64, 4, None) == -3


def test_split_heuristic():
    L = _lib.lib()
    assert L.lmps_gqa_attention_splits(1, 2, 160, 64) == 3        # bounded by 64-position tiles
    assert L.lmps_gqa_attention_splits(4, 2, 32768 + 128, 64) == 52    # 514 tiles, <= 444 CTAs: 10 tiles each
    assert L.lmps_gqa_attention_splits(64, 2, 384, 64) == 3         # 6 tiles, at most 3 splits: 2 each
    assert L.lmps_gqa_attention_splits(64, 2, 416, 64) == 3         # 7 tiles: 3, 3, 1
    assert L.lmps_gqa_attention_splits(16, 2, 1024, 64) == 8        # two tiles per split
    assert L.lmps_gqa_attention_splits(128, 2, 4096, 64) == 1       # 256 items: the grid is full
    assert L.lmps_gqa_attention_splits(256, 2, 4096, 64) == 1


def test_tensor_parallel_exchange_validation():
    """Buffer size of the peer exchange and the checks of both exchange entry
    points, all before any device work (fake, aligned addresses)."""
    L = _lib.lib()
    assert L.lmps_tp2_comm_bytes(56, 8 * 1536) == 56 * (2 * 8 * 1536 * 2 + 64 * 4)
    assert L.lmps_tp2_comm_bytes(0, 8) == 0 and L.lmps_tp2_comm_bytes(1, 12) == 0
    a = 1 << 20                                                   # 16-byte aligned, never dereferenced
    ok = dict(part=a, x=a, n=1536, comm=a, peer=a, seen=a, site=0, n_sites=4, max_n=1536, err=a)

    def ar(**kw):
        v = {**ok, **kw}
        return L.lmps_tp2_allreduce_residual(v["part"], v["x"], v["n"], v["comm"], v["peer"], v["seen"], v["site"],
                                             v["n_sites"], v["max_n"], v["err"], 0, None)
    assert ar(peer=None) == -1
    assert ar(site=4) == -1                                       # site outside n_sites
    assert ar(n=1544, max_n=1536) == -1                           # more than a slot holds
    assert ar(n=1537) == -1                                       # not a multiple of 8
    assert ar(part=a + 8) == -1                                   # misaligned
    # fused GEMV exchange: rows x batch beyond the slot, and a grid beyond 64 CTAs
    g = L.lmps_gemv_q4_tp2_residual
    assert g(a, a, a, 768, None, a, 1536, 768, 1, a, a, a, 0, 4, 1536, a, 0, None) == -1
    assert g(a, a, a, 768, a, a, 1536, 768, 2, a, a, a, 0, 4, 1536, a, 0, None) == -1
    assert g(a, a, a, 768, a, a, 4096, 768, 1, a, a, a, 0, 4, 4096, a, 0, None) == -2   # 128 CTAs


def test_attention_rope_validation():
    L = _lib.lib()
    a = 1 << 20
    bad_style = L.lmps_gqa_decode_attention_rope(a, a, a, 5, a, a, a, a, a, None, 0, 1, 64, 12, 2, 128, 1, 64, 1,
                                                 None)
    assert bad_style == -1
    no_pos = L.lmps_gqa_decode_attention_rope(a, None, a, 0, a, a, a, a, a, None, 0, 1, 64, 12, 2, 128, 1, 64, 1,
                                              None)
    assert no_pos == -1
