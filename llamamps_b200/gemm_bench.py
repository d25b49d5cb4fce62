"""Timing of the tcgen05 W4A16 GEMM on its own (CUDA events, random Q4
weights, fp16 activations).

    python -m llamamps_b200.gemm_bench                 # the prefill and bs64 shapes of Qwen2.5-1.5B
    python -m llamamps_b200.gemm_bench --shape 16384,8960,1536 --iters 1 --warmup 3
"""
from __future__ import annotations

import argparse
import json

import torch

from . import kernels as K

SHAPES = [(16384, 2048, 1536), (16384, 8960, 1536), (16384, 1536, 8960), (16384, 1536, 1536),
          (64, 2048, 1536), (64, 8960, 1536), (64, 1536, 8960), (64, 151936, 1536)]


def time_gemm(m: int, n: int, k: int, iters: int = 20, warmup: int = 3) -> dict:
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(m, k, dtype=torch.float16, device="cuda", generator=g)
    pk = torch.randint(0, 256, (n * k // 2,), dtype=torch.uint8, device="cuda", generator=g)
    sc = (torch.rand(n * k // 32, device="cuda", generator=g) * 0.01).half()
    y = torch.empty(m, n, dtype=torch.float16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    wsb = K.w4a16_gemm_workspace_size(m, n)
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda") if m <= 128 and wsb < (1 << 28) else None
    for _ in range(warmup):
        K.w4a16_gemm(x, pk, sc, n, k, out=y, error=err, workspace=ws)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        K.w4a16_gemm(x, pk, sc, n, k, out=y, error=err, workspace=ws)
    b.record()
    torch.cuda.synchronize()
    t = a.elapsed_time(b) / iters / 1e3
    return {"m": m, "n": n, "k": k, "us": round(t * 1e6, 2), "tflops": round(2.0 * m * n * k / t / 1e12, 1),
            "weight_gbs": round((n * k / 2 + n * k / 16) / t / 1e9, 1), "split_k": ws is not None,
            "error": int(err.item())}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", action="append", help="m,n,k (repeatable); default: the model's shapes")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    shapes = [tuple(int(v) for v in s.split(",")) for s in a.shape] if a.shape else SHAPES
    for m, n, k in shapes:
        print(json.dumps(time_gemm(m, n, k, a.iters, a.warmup)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
