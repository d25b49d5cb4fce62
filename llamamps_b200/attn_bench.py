"""Timing of the split-KV decode attention (``lmps_gqa_decode_attention``,
attention + combine) over a paged fp16 cache for a range of split counts,
as a CUDA graph of 20 calls (CUDA events, us per call).  The count that
``lmps_gqa_attention_splits`` picks is marked ``*``.

    python -m llamamps_b200.attn_bench                       # the shapes of the decode configurations
    python -m llamamps_b200.attn_bench --shape 64,400,416    # batch, attended positions, cache positions
"""
from __future__ import annotations

import argparse

import torch

from . import kernels as K

SHAPES = [(64, 400, 416), (64, 1000, 1024), (8, 2100, 2144), (4, 300, 320), (16, 1000, 1024), (64, 140, 155)]
HQ, HKV, HD, PAGE = 12, 2, 128, 64


def time_shape(B: int, T: int, maxlen: int, calls: int = 20):
    dev = torch.device("cuda")
    pages = (maxlen + PAGE - 1) // PAGE
    g = torch.Generator(device=dev).manual_seed(1)
    kp = torch.randn(B * pages, HKV, PAGE, HD, generator=g, device=dev).half()
    vp = torch.randn(B * pages, HKV, PAGE, HD, generator=g, device=dev).half()
    bt = torch.randperm(B * pages, generator=g, device=dev).to(torch.int32).reshape(B, pages)
    q = torch.randn(B, HQ * HD, generator=g, device=dev).half()
    lens = torch.full((B,), min(T, maxlen), dtype=torch.int32, device=dev)
    auto = K.attention_splits(B, HKV, maxlen, PAGE)
    tiles = (maxlen + 63) // 64
    res = []
    for sp in sorted({1, 2, 3, 4, 6, 8, 12, 16, 24, 32, auto}):
        if sp > tiles:
            continue
        ws = torch.zeros(max(K.attention_workspace_size(B, HQ, HD, sp), 16), dtype=torch.uint8, device=dev)
        out = torch.empty_like(q)

        def call():
            K.gqa_decode_attention(q, kp, vp, bt, lens, out, ws, PAGE, HQ, HKV, HD, maxlen, sp)
        for _ in range(3):
            call()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(calls):
                call()
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        res.append((sp, sp == auto, e0.elapsed_time(e1) / calls * 1e3))
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", action="append", help="batch,attended,cache (repeatable)")
    a = ap.parse_args()
    shapes = [tuple(int(v) for v in s.split(",")) for s in a.shape] if a.shape else SHAPES
    for B, T, maxlen in shapes:
        res = time_shape(B, T, maxlen)
        print(f"B={B} T={T} maxlen={maxlen}  " +
              "  ".join(f"{sp}{'*' if auto else ''}:{us:.1f}" for sp, auto, us in res))


if __name__ == "__main__":
    main()
