"""Decode-throughput benchmark of the B200 LlamaMPS engine (one JSON line).

Workload (per GPU): the full Qwen2.5-1.5B shape (28 layers, hidden 1536,
12/2 heads, intermediate 8960, vocab 151936) with random-init Q4 weights
(torch generator seed 1 on the device, replicated on every GPU), batch 1, a
32-id prompt (numpy seed 1, offset by rank) fed through the decode path, then
greedy decode.  A step is one decode token per sequence.  Weights (868.6 MB
per step) are larger than L2 (126 MB), so no L2 flush is needed between
steps.  N GPUs run N independent copies of that workload (data-parallel
requests, no collective): ``value`` is the sum over GPUs of tokens/s, timed
as the max over ranks of CUDA-event time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the reference's decode math on the host cores
(the numpy restatement under oracle/, a bounded sample per step: one of the
28 layers plus 1/28 of the LM head, i.e. 1/28 of a token).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Qwen2.5-1.5B-Q4 decode tok/s (bs1, bs64); Q4 GEMV GB/s vs HBM peak"
PROMPT_LEN = 32
# DRAM bytes per algorithmic byte of the persistent decode kernel, from one
# ncu capture of a 4-layer, one-step launch (`bench.py --layers 4 --steps 1`):
# dram__bytes_read.sum + dram__bytes_write.sum = 236.9 MB + 4.7 MB against
# 236.8 MB of algorithmic bytes.  Every layer's weights are read once, so the
# ratio carries over to the 28-layer launch.
PERSISTENT_TRAFFIC_PER_ALGO_BYTE = (236.9 + 4.7) / 236.8


def _dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled through NVML from a
    background thread about once a millisecond while the timed region runs
    (read-only queries).  ``mark(True/False)`` brackets the timed region; only
    samples taken inside it are summarised."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self.inside = False
        self.stop = False
        self.thread = None
        self.nvml = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None
            return self
        import threading
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        return self

    def _run(self):
        nv = self.nvml
        while not self.stop:
            if self.inside:
                try:
                    mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    self.samples.append((mhz, rs))
                except Exception:
                    pass
            time.sleep(0.001)

    def mark(self, inside: bool):
        self.inside = inside

    def __exit__(self, *a):
        self.stop = True
        if self.thread is not None:
            self.thread.join(timeout=5)
        if self.nvml is not None:
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        if self.nvml is None or not self.samples:
            return None
        reasons = set()
        for _, rs in self.samples:
            for name, attr in self.REASONS:
                if rs & getattr(self.nvml, attr, 0):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "nvml"}


def cpu_baseline_sample(seconds: float = 15.0):
    """The oracle decode forward (numpy, fp32 with on-the-fly Q4 dequant, as
    the reference re-reads packed weights every token) on a bounded sample:
    whole decoder layers of the full-size model until ``seconds`` pass, plus
    the LM head once; tokens/s = 1 / (28 * t_layer + t_head)."""
    import numpy as np
    from oracle import mirror as M
    from llamamps_b200.config import QWEN2_5_1_5B as cfg
    from llamamps_b200.weights import parts_host_arrays, synth_layer_numpy
    rng = np.random.default_rng(1)
    lw = parts_host_arrays(synth_layer_numpy(rng, cfg))
    ocfg = M.OracleConfig()
    x = rng.normal(0, 1, cfg.hidden).astype(np.float16)
    kv = M.KVCache(1, ocfg.kv_dim)
    kv.set_prefix(0, rng.normal(0, 1, (PROMPT_LEN, ocfg.kv_dim)).astype(np.float16),
                  rng.normal(0, 1, (PROMPT_LEN, ocfg.kv_dim)).astype(np.float16))
    times = []
    t_end = time.perf_counter() + seconds
    pos = PROMPT_LEN
    while time.perf_counter() < t_end or not times:
        t0 = time.perf_counter()
        x = M.decoder_layer(x, lw, kv, 0, pos, ocfg)      # dq=None: dequantise every call
        times.append(time.perf_counter() - t0)
        pos += 1
    rows = 151936 // 8
    lm_p, lm_s = M.q4_pack(rng.normal(0, 0.02, (rows, cfg.hidden)).astype(np.float32))
    t0 = time.perf_counter()
    M.gemv_q4(lm_p, lm_s, x, rows, cfg.hidden)
    t_head = (time.perf_counter() - t0) * 8
    t_layer = statistics.median(times)
    tok_s = 1.0 / (cfg.n_layers * t_layer + t_head)
    return {"value": tok_s, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{len(times)} oracle decoder layers (full Qwen2.5-1.5B layer shape, T={PROMPT_LEN + 1}..) "
                      f"+ 1/8 of the LM head, scaled to one token of 28 layers + head"}


def run_reference(args):
    """--impl reference: the reference's decode math on the host (oracle port)."""
    rank, world, _ = _dist_env()
    if rank != 0:
        return 0
    import numpy as np
    from oracle import mirror as M
    from llamamps_b200.config import QWEN2_5_1_5B as cfg
    from llamamps_b200.weights import parts_host_arrays, synth_layer_numpy
    rng = np.random.default_rng(1)
    layers = [parts_host_arrays(synth_layer_numpy(rng, cfg)) for _ in range(2)]
    ocfg = M.OracleConfig()
    lm_rows = cfg.vocab // cfg.n_layers
    lm_p, lm_s = M.q4_pack(rng.normal(0, 0.02, (lm_rows, cfg.hidden)).astype(np.float32))
    kv = M.KVCache(1, ocfg.kv_dim)
    kv.set_prefix(0, rng.normal(0, 1, (PROMPT_LEN, ocfg.kv_dim)).astype(np.float16),
                  rng.normal(0, 1, (PROMPT_LEN, ocfg.kv_dim)).astype(np.float16))
    x = rng.normal(0, 1, cfg.hidden).astype(np.float16)
    pos = PROMPT_LEN

    def one_step():
        nonlocal x, pos
        x = M.decoder_layer(x, layers[pos % 2], kv, 0, pos, ocfg)
        M.gemv_q4(lm_p, lm_s, x, lm_rows, cfg.hidden)
        pos += 1

    for _ in range(args.warmup):
        one_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    dt = time.perf_counter() - t0
    # one step = 1/28 of a token's work
    tok_s = args.steps / cfg.n_layers / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "Qwen2.5-1.5B-Q4 decode bs1 on host cores: per step one decoder layer "
                               "(full layer shape) + 1/28 of the LM head = 1/28 token",
                   "batch_per_gpu": 1, "prompt_len": PROMPT_LEN},
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": "oracle (numpy fp32 restatement) decoder layer + LM-head slice per step"},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("one host process (rank 0) at every n_gpus: the value is one CPU sequence's rate and does "
                 "not grow with n_gpus, so at n_gpus > 1 a GPU/CPU ratio divides N GPUs' tokens by one "
                 "process's"),
    }
    print(json.dumps(line))
    return 0


def gemv_roofline(eng, peak_gbs, peak_kind, reps: int = 3):
    """Time the dominant kernel (fused gate/up SwiGLU Q4 GEMV, 59% of a
    step's bytes) with CUDA events on its launch stream, cycling through all
    layers so every launch streams its 15.5 MB from HBM."""
    import torch
    from llamamps_b200 import kernels as K
    c = eng.cfg
    xn = eng.buf_normed[:1]
    out = eng.buf_mlp[:1]
    lws = eng.weights.layers
    for lw in lws:   # warm
        K.gemv_q4_swiglu(lw.gate_packed, lw.gate_scales, lw.up_packed, lw.up_scales, xn,
                         c.intermediate, c.hidden, out=out)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    n = 0
    for _ in range(reps):
        for lw in lws:
            K.gemv_q4_swiglu(lw.gate_packed, lw.gate_scales, lw.up_packed, lw.up_scales, xn,
                             c.intermediate, c.hidden, out=out)
            n += 1
    e1.record(st)
    torch.cuda.synchronize()
    per_launch_s = e0.elapsed_time(e1) / 1e3 / n
    bytes_per_launch = 2 * (c.intermediate * c.hidden // 2 + c.intermediate * c.hidden // 32 * 2) \
        + c.hidden * 2 + c.intermediate * 2
    achieved = bytes_per_launch / per_launch_s / 1e9
    return {"kernel": "q4_gemv_kernel<LPR=16,NB=1,SWIGLU> (gate+up 17920x1536)", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": peak_gbs, "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(achieved / peak_gbs, 4), "traffic": None,
            "bytes_per_launch": bytes_per_launch, "us_per_launch": round(per_launch_s * 1e6, 3)}


def _busy_stream(ms: float = 3.0):
    """Keep the current stream busy for about ``ms`` with a device-side spin
    (clock64 cycles at the 1965 MHz SM clock), so that the start event and
    the launches after it are already queued when the GPU reaches them: the
    host's time to enqueue them (and anything that delays the host thread,
    such as the clock sampler's NVML queries) stays out of the device time.
    The end-to-end measurement keeps every host cost."""
    import torch
    torch.cuda._sleep(int(ms * 1e-3 * 1.965e9))


def _timed(fn, world, dist):
    """Device time of fn() bracketed by a barrier and synchronizes, max over ranks."""
    import torch
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _busy_stream()
    e0.record(st)
    fn()
    e1.record(st)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / 1e3], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def extra_configs(mw, cfg, args, rank, world, dist, peak):
    """The other configurations of the headline metric, each measured on the
    device (CUDA events, max over ranks) after the bs1 line:
      c2  batched decode, 64 sequences over the job (64/N per GPU), 128-id prompts;
      c3  prefill of 8 x 2048 ids on the tensor-core GEMM path, then decode (1 GPU);
      c4  long-context decode, 4 sequences per GPU over a 32768-position KV cache."""
    import numpy as np
    import torch
    from llamamps_b200.engine import QwenEngine
    out = {}
    steps = max(4, min(args.steps, 16))

    def want(name):
        return args.only is None or args.only == name
    # -- c2
    if want("c2"):
        try:
            B = max(1, 64 // world)
            eng = QwenEngine(weights=mw, device=torch.device("cuda"), max_batch=B,
                             max_seq_len=128 + args.warmup + steps + 8, decoder="kernels")
            prompt = np.random.default_rng(2 + rank).integers(0, cfg.vocab, (B, 128))
            eng.reset(B)
            eng.prefill(torch.from_numpy(prompt))
            eng.decode_steps(args.warmup, record=False)
            t = _timed(lambda: eng.decode_steps(steps, record=False), world, dist)
            mean_T = 128 + args.warmup + (steps + 1) / 2
            step_bytes = cfg.step_weight_bytes() + B * cfg.kv_bytes_per_position() * mean_T
            out["c2_batched_decode"] = {
                "value": round(world * B * steps / t, 1), "unit": "tok/s", "batch_per_gpu": B,
                "global_batch": B * world, "ms_per_step": round(t / steps * 1e3, 3),
                "hbm_frac_of_measured": round(step_bytes / (t / steps) / 1e9 / peak, 4),
                "path": "per-stage kernels; projections and LM head on the tcgen05 W4A16 GEMM (split-K)"}
            del eng
        except Exception as e:  # a sub-measurement never hides the headline line
            out["c2_batched_decode"] = {"error": repr(e)[:200]}
    # -- c3 (one GPU)
    if world == 1 and want("c3"):
        try:
            B, P = 8, 2048
            eng = QwenEngine(weights=mw, device=torch.device("cuda"), max_batch=B, max_seq_len=P + 32,
                             decoder="kernels")
            prompt = torch.from_numpy(np.random.default_rng(3).integers(0, cfg.vocab, (B, P)))
            eng.reset(B)
            eng.prefill(prompt, dense=True)  # warm-up
            eng.reset(B)
            t = _timed(lambda: eng.prefill(prompt, dense=True), world, dist)
            lin_flops = 2.0 * B * P * (cfg.n_layers * (cfg.qkv_rows + cfg.q_dim + 3 * cfg.intermediate)
                                       * cfg.hidden)
            att_flops = 2.0 * 2 * cfg.n_layers * B * cfg.n_q_heads * cfg.head_dim * P * (P + 1) / 2
            eng.decode_steps(2, record=False)   # graph capture outside the timed region
            td = _timed(lambda: eng.decode_steps(16, record=False), world, dist)
            out["c3_prefill"] = {
                "value": round(B * P / t, 1), "unit": "prompt tok/s", "ms": round(t * 1e3, 2),
                "tflops": round((lin_flops + att_flops) / t / 1e12, 1),
                "decode_after_prefill_tok_s": round(B * 16 / td, 1),
                "path": "dense prefill: W4A16 tcgen05 GEMMs over 16384 token rows, causal flash "
                        "attention over the paged cache; then bs8 decode on the per-stage kernels"}
            del eng
        except Exception as e:
            out["c3_prefill"] = {"error": repr(e)[:200]}
    # -- c3 in 2-way tensor-parallel mode (both ranks run the same 8 prompts)
    if world == 2 and want("c3_tp2"):
        try:
            from llamamps_b200.tp import TPEngine
            B, P = 8, 2048
            prompt = torch.from_numpy(np.random.default_rng(3).integers(0, cfg.vocab, (B, P)))
            res = {}
            # parity: greedy ids of every variant against the single-GPU engine
            # on the same prompts (64-id prefix of each prompt, 12 new tokens)
            n_new = 12
            one = QwenEngine(weights=mw, device=torch.device("cuda"), max_batch=B, max_seq_len=P + 32,
                             decoder="kernels")
            ref_ids = one.generate_batch(prompt[:, :64].numpy(), n_new)
            del one
            solo = QwenEngine(weights=mw, device=torch.device("cuda"), max_batch=1, max_seq_len=128,
                              decoder="kernels")

            def margin_at(b, step):
                """Top-2 logit gap of the single-GPU engine where sequence b's
                ids first differ: fp16 rounding of the split sums may flip the
                pick only where this is within the logits tolerance."""
                solo.reset(1)
                for t in list(prompt[b, :64].tolist()) + list(ref_ids[b, :step]):
                    solo.tokens[0] = int(t)
                    solo._logits_step(1)
                top = torch.topk(solo.buf_logits[0].float(), 2).values
                return float(top[0] - top[1])
            parity = {}
            for comm, fuse in (("p2p", False), ("p2p", True), ("nccl", False)):
                # the fused GEMV exchange belongs to the GEMV path: keep batch 8 on it there
                eng = TPEngine(mw, rank, world, device=torch.device("cuda"), max_batch=B, max_seq_len=P + 32,
                               comm=comm, fuse_exchange=fuse, **({"gemv_max_batch": B} if fuse else {}))
                name = comm + ("_fused" if fuse else "")
                try:
                    eng.reset(B)
                    eng.prefill(prompt, dense=True)  # warm-up
                    eng.reset(B)
                    t = _timed(lambda: eng.prefill(prompt, dense=True), world, dist)
                    eng.decode_steps(2, record=False)  # graph capture outside the timed region
                    td = _timed(lambda: eng.decode_steps(16, record=False), world, dist)
                    eng.check_comm()
                    res[name] = (t, td)
                    ids = eng.generate_batch(prompt[:, :64].numpy(), n_new)
                    eng.check_comm()
                    # ids up to each sequence's first difference (after it the sequences differ)
                    same = [int(np.argmax(np.append(ids[b] != ref_ids[b], True))) for b in range(B)]
                    diffs = [(b, x) for b, x in enumerate(same) if x < n_new]
                    parity[name] = {"sequences_identical": B - len(diffs), "sequences": B,
                                    "first_difference_steps": [x for _, x in diffs],
                                    "top2_margin_at_difference": [round(margin_at(b, x), 5) for b, x in diffs]}
                finally:
                    eng.close()
                del eng
            t, td = res["p2p"]
            out["c3_prefill_tp2"] = {
                "value": round(B * P / t, 1), "unit": "prompt tok/s", "ms": round(t * 1e3, 2),
                "decode_after_prefill_tok_s": round(B * 16 / td, 1),
                "decode_fused_gemv_exchange_tok_s": round(B * 16 / res["p2p_fused"][1], 1),
                "decode_nccl_tok_s": round(B * 16 / res["nccl"][1], 1),
                # ids equal to the single-GPU engine's wherever its top-2 margin exceeds the
                # logits tolerance (2e-2), the greedy-parity rule of the tests
                "tp_parity": all(m <= 2e-2 for v in parity.values() for m in v["top2_margin_at_difference"]),
                "tp_parity_detail": {"against": "greedy ids of the single-GPU engine, same weights and prompts "
                                                "(8 x 64-id prompts, 12 new tokens); a difference counts only "
                                                "where that engine's top-2 logit margin exceeds 2e-2", **parity},
                "path": "tp2: KV head r and its query heads on rank r; dense GEMM prefill with NCCL "
                        "all-reduces (sum, fp16) after o_proj and down_proj, then bs8 decode as a CUDA graph "
                        "with the all-reduces over peer memory (NVLink stores + flags, fused with the "
                        "residual add); decode_fused_gemv_exchange_tok_s: GEMV and exchange in one kernel; "
                        "decode_nccl_tok_s: the same decode with NCCL all-reduces, eager"}
        except Exception as e:
            out["c3_prefill_tp2"] = {"error": repr(e)[:200]}
    # -- c4
    if want("c4"):
        try:
            B, T = 4, 32768
            eng = QwenEngine(weights=mw, device=torch.device("cuda"), max_batch=B,
                             max_seq_len=T + args.warmup + steps + 8, decoder="persistent")
            eng.reset(B, start_pos=T)
            g = torch.Generator(device="cuda").manual_seed(4 + rank)
            for layer in range(cfg.n_layers):   # the KV cache of T positions, fp16 N(0,1)
                eng.cache.k[layer].normal_(generator=g)
                eng.cache.v[layer].normal_(generator=g)
            eng.tokens[:B].copy_(torch.from_numpy(np.random.default_rng(4).integers(0, cfg.vocab, B)))
            eng.decode_steps(args.warmup, record=False)
            t = _timed(lambda: eng.decode_steps(steps, record=False), world, dist)
            eng.pdec.check_error()
            kv = B * cfg.kv_bytes_per_position() * (T + args.warmup + steps / 2)
            out["c4_long_context"] = {
                "value": round(world * B * steps / t, 1), "unit": "tok/s", "batch_per_gpu": B, "kv_positions": T,
                "ms_per_step": round(t / steps * 1e3, 3),
                "hbm_frac_of_measured": round((cfg.step_weight_bytes() + kv) / (t / steps) / 1e9 / peak, 4),
                "path": "persistent decode kernel"}
            del eng
        except Exception as e:
            out["c4_long_context"] = {"error": repr(e)[:200]}
    return out


# -- per-kernel timing tables (the commands behind the profiles/ summaries) --
GEMM_SHAPES = [(16384, 2048, 1536), (16384, 8960, 1536), (16384, 1536, 8960), (16384, 1536, 1536),
               (64, 2048, 1536), (64, 8960, 1536), (64, 1536, 8960), (64, 151936, 1536)]
ATTN_SHAPES = [(64, 400, 416), (64, 1000, 1024), (8, 2100, 2144), (4, 300, 320), (16, 1000, 1024), (64, 140, 155)]


def time_gemm(m: int, n: int, k: int, iters: int = 20, warmup: int = 3) -> dict:
    """The tcgen05 W4A16 GEMM alone: random Q4 weights, fp16 activations,
    CUDA events around ``iters`` back-to-back calls."""
    import torch
    from llamamps_b200 import kernels as K
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
    return {"kernel": "w4a16_gemm", "m": m, "n": n, "k": k, "us": round(t * 1e6, 2),
            "tflops": round(2.0 * m * n * k / t / 1e12, 1),
            "weight_gbs": round((n * k / 2 + n * k / 16) / t / 1e9, 1), "split_k": ws is not None,
            "error": int(err.item())}


def time_attention(B: int, T: int, maxlen: int, calls: int = 20, auto_only: bool = False) -> dict:
    """The split-KV decode attention (attention + combine) over a paged fp16
    cache of ``maxlen`` positions, ``T`` attended, for a range of split
    counts: a CUDA graph of ``calls`` calls, us per call; ``auto`` is the
    count lmps_gqa_attention_splits picks."""
    import torch
    from llamamps_b200 import kernels as K
    hq, hkv, hd, page = 12, 2, 128, 64
    dev = torch.device("cuda")
    pages = (maxlen + page - 1) // page
    g = torch.Generator(device=dev).manual_seed(1)
    kp = torch.randn(B * pages, hkv, page, hd, generator=g, device=dev).half()
    vp = torch.randn(B * pages, hkv, page, hd, generator=g, device=dev).half()
    bt = torch.randperm(B * pages, generator=g, device=dev).to(torch.int32).reshape(B, pages)
    q = torch.randn(B, hq * hd, generator=g, device=dev).half()
    lens = torch.full((B,), min(T, maxlen), dtype=torch.int32, device=dev)
    auto = K.attention_splits(B, hkv, maxlen, page)
    tiles = (maxlen + 63) // 64
    us = {}
    for sp in ([auto] if auto_only else sorted({1, 2, 3, 4, 6, 8, 12, 16, 24, 32, auto})):
        if sp > tiles:
            continue
        ws = torch.zeros(max(K.attention_workspace_size(B, hq, hd, sp), 16), dtype=torch.uint8, device=dev)
        out = torch.empty_like(q)

        def call():
            K.gqa_decode_attention(q, kp, vp, bt, lens, out, ws, page, hq, hkv, hd, maxlen, sp)
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
        us[sp] = round(e0.elapsed_time(e1) / calls * 1e3, 2)
    return {"kernel": "gqa_decode_attention", "batch": B, "attended": T, "cache": maxlen, "auto_splits": auto,
            "us_by_splits": us}


def time_prefill_attention(B: int, P: int, iters: int = 5) -> dict:
    """The causal prefill attention alone over a paged fp16 cache: B
    sequences of P positions, 12 query / 2 KV heads of 128 dims (the dense
    prefill of the 8 x 2048 configuration); FLOP = 4 * 128 * P (P + 1) / 2
    per (sequence, query head)."""
    import torch
    from llamamps_b200 import kernels as K
    hq, hkv, hd, ps = 12, 2, 128, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    pages = (P + ps - 1) // ps
    kp = torch.randn(B * pages, hkv, ps, hd, generator=g, device="cuda").half()
    vp = torch.randn(B * pages, hkv, ps, hd, generator=g, device="cuda").half()
    bt = torch.randperm(B * pages, generator=g, device="cuda").to(torch.int32).reshape(B, pages)
    q = torch.randn(B * P, hq * hd, generator=g, device="cuda").half()
    out = torch.empty_like(q)
    flops = 4.0 * hd * P * (P + 1) / 2 * B * hq
    res = {"batch": B, "seq_len": P}
    for name, tc in (("prefill_attn_tc_kernel", True), ("prefill_attn_kernel", False)):
        for _ in range(2):
            K.prefill_attention(q, kp, vp, bt, out, B, P, ps, hq, hkv, hd, tcgen05=tc)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            K.prefill_attention(q, kp, vp, bt, out, B, P, ps, hq, hkv, hd, tcgen05=tc)
        b.record()
        torch.cuda.synchronize()
        t = a.elapsed_time(b) / iters / 1e3
        res[name] = {"us": round(t * 1e6, 1), "tflops": round(flops / t / 1e12, 1)}
    return res


def time_gemv(rows: int, k: int, batch: int, iters: int = 20) -> dict:
    """The CUDA-core Q4 GEMV alone (lmps_gemv_q4_swiglu when rows is a
    gate|up pair count, i.e. the call reads 2 x rows x k weights; CUDA events
    around ``iters`` calls that cycle over matrices larger than L2 together)."""
    import torch
    from llamamps_b200 import kernels as K
    g = torch.Generator(device="cuda").manual_seed(2)
    n_mats = max(2, (256 << 20) // (rows * k))   # > 126 MB of weights in rotation
    mats = [(torch.randint(0, 256, (2 * rows * k // 2,), dtype=torch.uint8, device="cuda", generator=g),
             (torch.rand(2 * rows * k // 32, device="cuda", generator=g) * 0.01).half()) for _ in range(n_mats)]
    x = torch.randn(batch, k, generator=g, device="cuda").half()
    out = torch.empty(batch, rows, dtype=torch.float16, device="cuda")

    def call(i):
        p, sc = mats[i % n_mats]
        K.gemv_q4_swiglu(p[:rows * k // 2], sc[:rows * k // 32], p[rows * k // 2:], sc[rows * k // 32:], x, rows, k,
                         out=out)
    for i in range(3):
        call(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()   # the launches back to back, without the host in between
    with torch.cuda.graph(graph):
        for i in range(iters):
            call(i)
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    torch.cuda.synchronize()
    t = a.elapsed_time(b) / iters / 1e3
    nbytes = 2 * (rows * k // 2 + rows * k // 32 * 2) + 2 * k * batch + 2 * rows * batch
    return {"kernel": "q4_gemv_kernel (SwiGLU)", "rows": rows, "k": k, "batch": batch, "us": round(t * 1e6, 2),
            "gbs": round(nbytes / t / 1e9, 1), "bytes_per_launch": nbytes}


def time_decode(B: int, T: int, n_layers: int, steps: int, launches: int = 3, timeline=None) -> dict:
    """The persistent decoder alone: ``B`` sequences over a ``T``-position
    fp16 N(0,1) KV cache (c4's shape at B=4, T=32768), ``n_layers`` decoder
    layers, ``steps`` decode steps per launch; CUDA events around each of
    ``launches`` launches after three warm-up launches (weights and KV > L2)."""
    import dataclasses
    import numpy as np
    import torch
    from llamamps_b200.config import QWEN2_5_1_5B
    from llamamps_b200.engine import QwenEngine
    from llamamps_b200.weights import synth_model
    cfg = dataclasses.replace(QWEN2_5_1_5B, n_layers=n_layers)
    mw = synth_model(cfg, seed=1, device="cuda")
    eng = QwenEngine(weights=mw, max_batch=B, max_seq_len=T + (launches + 4) * steps + 8, decoder="persistent")
    eng.reset(B, start_pos=T)
    g = torch.Generator(device="cuda").manual_seed(4)
    for layer in range(cfg.n_layers):
        eng.cache.k[layer].normal_(generator=g)
        eng.cache.v[layer].normal_(generator=g)
    eng.tokens[:B].copy_(torch.from_numpy(np.random.default_rng(4).integers(0, cfg.vocab, B)))
    for _ in range(3):
        eng.decode_steps(steps, record=False)
    torch.cuda.synchronize()
    times = []
    for _ in range(launches):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        eng.decode_steps(steps, record=False)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3 / steps)
    eng.pdec.check_error()
    kv = B * cfg.kv_bytes_per_position() * (T + 3 * steps + steps * launches / 2)
    us = float(np.median(times))
    out = {"kernel": f"decode_persistent_kernel (batch {B})", "batch": B, "kv_positions": T, "layers": n_layers,
           "steps_per_launch": steps, "us_per_step": round(us, 1),
           "bytes_per_step": int(cfg.step_weight_bytes() + kv),
           "gbs": round((cfg.step_weight_bytes() + kv) / us / 1e3, 1)}
    if timeline:
        from llamamps_b200.timeline import capture
        with open(timeline, "w") as f:
            json.dump(capture(eng, 4), f)
    return out


def time_batched(B: int, steps: int, timeline: bool) -> dict:
    """Decode steps of ``B`` sequences after 128-id prompts (the batched
    configuration's prompt length), full model: the per-stage kernel path
    against the one-launch batched decode kernel (csrc/decode_batched.cu),
    CUDA events over ``steps`` graph replays.  With ``timeline``, the
    batched kernel's grid-barrier timeline of one launch: per stage, the
    median over layers of (last arrival - previous stage's last arrival),
    and for the projection stages when the CTAs' weight tiles were
    dequantised and their accumulators ready (medians over CTAs, us after
    the gate barrier)."""
    import numpy as np
    import torch
    from llamamps_b200 import kernels as K
    from llamamps_b200.config import QWEN2_5_1_5B as cfg
    from llamamps_b200.engine import QwenEngine
    from llamamps_b200.weights import synth_model
    mw = synth_model(cfg, seed=0, device="cuda")
    out = {"kernel": "decode_batched_kernel vs per-stage kernels", "batch": B, "prompt": 128, "layers": cfg.n_layers}
    for dec in ("kernels", "batched"):
        eng = QwenEngine(weights=mw, max_batch=B, max_seq_len=128 + steps + 16, decoder=dec)
        prompt = np.random.default_rng(2).integers(0, cfg.vocab, (B, 128))
        eng.reset(B)
        eng.prefill(torch.from_numpy(prompt))
        eng.decode_steps(3, record=False)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        eng.decode_steps(steps, record=False)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        out[f"{dec}_ms_per_step"] = round(ms, 3)
        out[f"{dec}_tok_s"] = round(B / ms * 1e3, 1)
        if dec == "batched":
            eng.bdec.check_error()
        if dec == "batched" and timeline:
            G = torch.cuda.get_device_properties(0).multi_processor_count
            L = cfg.n_layers
            nb = eng.bdec.barriers(B)
            per = (nb - 1) // L
            names = ["qkv", "attention"] + (["merge"] if per == 8 else []) + ["o", "reduce_o", "gate_up", "down",
                                                                                  "reduce_down"]
            tr = torch.zeros(G, nb, 4, dtype=torch.int64, device="cuda")
            K.embed_gather(eng.weights.embed, eng.tokens[:B], eng.buf_residual[:B], eng.bad_ids)
            eng.bdec.run(B, eng.buf_residual[:B], eng.pos[:B], eng.seq_lens[:B], trace=tr)
            torch.cuda.synchronize()
            t = tr.cpu().numpy().astype(np.float64)
            last = t[:, :, 0].max(axis=0)
            stage = {}
            for j, nm in enumerate(names):
                ks = [1 + l * per + j for l in range(L)]
                d = {"us": round(float(np.median([(last[k] - last[k - 1]) / 1e3 for k in ks])), 2)}
                if nm in ("qkv", "o", "gate_up", "down"):
                    dq, ac = [], []
                    for k in ks:
                        m = t[:, k, 2] > 0
                        dq.append((np.median(t[m, k, 2]) - last[k - 1]) / 1e3)
                        ac.append((np.median(t[m, k, 3]) - last[k - 1]) / 1e3)
                    d["dequantised_us"] = round(float(np.median(dq)), 2)
                    d["accumulated_us"] = round(float(np.median(ac)), 2)
                stage[nm] = d
            obs = t[:, :, 1]
            lat = [float(np.min(obs[obs[:, k] > 0, k]) - last[k]) / 1e3 for k in range(1, nb) if np.any(obs[:, k] > 0)]
            out["timeline"] = {"per_layer_us": round(float((last[-1] - last[0]) / 1e3 / L), 2), "stages": stage,
                               "barrier_latency_us": round(float(np.median(lat)), 2)}
        del eng
        torch.cuda.empty_cache()
    return out


def run_kernel_timing(args) -> int:
    """--time gemm|attention|prefill_attention|gemv|decode: one JSON line per shape (not a benchmark line)."""
    if args.time == "batched":
        for b in ([int(s) for s in args.shape] if args.shape else [8, 64]):
            print(json.dumps(time_batched(b, args.iters, bool(args.timeline))))
        return 0
    if args.time == "decode":
        shapes = [tuple(int(v) for v in s.split(",")) for s in args.shape] if args.shape else [(4, 32768)]
        for b, t in shapes:
            print(json.dumps(time_decode(b, t, args.layers or 28, args.iters, timeline=args.timeline)))
        return 0
    if args.time == "gemv":
        shapes = [tuple(int(v) for v in s.split(",")) for s in args.shape] if args.shape else [(8960, 1536, 1)]
        for r, k, b in shapes:
            print(json.dumps(time_gemv(r, k, b, args.iters)))
        return 0
    if args.time == "prefill_attention":
        shapes = [tuple(int(v) for v in s.split(",")) for s in args.shape] if args.shape else [(8, 2048)]
        for b, p in shapes:
            print(json.dumps(time_prefill_attention(b, p)))
        return 0
    if args.time == "gemm":
        shapes = [tuple(int(v) for v in s.split(",")) for s in args.shape] if args.shape else GEMM_SHAPES
        for m, n, k in shapes:
            print(json.dumps(time_gemm(m, n, k, args.iters, args.warmup)))
    else:
        shapes = [tuple(int(v) for v in s.split(",")) for s in args.shape] if args.shape else ATTN_SHAPES
        for b, t, c in shapes:
            print(json.dumps(time_attention(b, t, c, auto_only=args.auto_splits)))
    return 0


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    rank, world, local = _dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    from llamamps_b200.config import QWEN2_5_1_5B as cfg
    from llamamps_b200.engine import QwenEngine
    from llamamps_b200.weights import synth_model

    B = 1
    if args.layers is not None:
        import dataclasses
        cfg = dataclasses.replace(cfg, n_layers=args.layers)
    mw = synth_model(cfg, seed=1, device=dev)
    max_seq = PROMPT_LEN + args.warmup + 2 * args.steps + 16
    eng = QwenEngine(weights=mw, device=dev, max_batch=B, max_seq_len=max_seq, decoder=args.decoder)
    prompt = np.random.default_rng(1 + rank).integers(0, cfg.vocab, (B, PROMPT_LEN))
    eng.reset(B)
    eng.prefill(torch.from_numpy(prompt))
    for _ in range(max(args.warmup, 1)):
        eng.decode_step(record=False)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    # -- device-resident timed region ---------------------------------------
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        _busy_stream()
        clk.mark(True)
        e0.record(st)
        eng.decode_steps(args.steps, record=False)   # persistent: one launch for all K steps
        e1.record(st)
        torch.cuda.synchronize()
        clk.mark(False)
    if eng.pdec is not None:
        eng.pdec.check_error()
    barrier()
    t_local = e0.elapsed_time(e1) / 1e3
    t = torch.tensor([t_local], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t_max = float(t.item())
    value = world * B * args.steps / t_max

    if args.timeline and eng.pdec is not None and rank == 0:
        from llamamps_b200.timeline import capture
        with open(args.timeline, "w") as f:
            json.dump(capture(eng, 4), f, indent=1)

    # -- end to end through the reference-facing API ------------------------
    # run_inference(vector) -> fp16 logits on the host -> predict_next_token,
    # the reference's per-token flow (runners/engine.py:157-181): per step the
    # 3 KB embedding row goes host->device and the 304 KB logits come back.
    embed_host = mw.embed.cpu().numpy()
    eng.reset(1)
    tok = int(prompt[0, 0])
    for _ in range(max(args.warmup, 1)):
        tok = eng.predict_next_token(eng.run_inference(embed_host[tok]))
    barrier()
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    for _ in range(args.steps):
        tok = eng.predict_next_token(eng.run_inference(embed_host[tok]))
    torch.cuda.synchronize()
    e2e_local = time.perf_counter() - w0
    barrier()
    te = torch.tensor([e2e_local], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * args.steps / float(te.item())

    peak, peak_kind = _peaks()
    # algorithmic bytes of one decode step: all Q4 weights + norms + biases +
    # one embedding row, plus K and V of every attended position
    mean_T = PROMPT_LEN + args.warmup + (args.steps + 1) / 2
    step_bytes = cfg.step_weight_bytes() + cfg.kv_bytes_per_position() * mean_T
    step_gbs = step_bytes / (t_max / args.steps) / 1e9
    if eng.pdec is not None:
        roof = {"kernel": "decode_persistent_kernel<1> (one launch = all timed steps)", "bound": "hbm",
                "achieved": round(step_gbs, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                "frac": round(step_gbs / peak, 4),
                "traffic": int(step_bytes * PERSISTENT_TRAFFIC_PER_ALGO_BYTE * args.steps),
                "traffic_unit": "DRAM bytes per launch",
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of a 4-layer one-step "
                                  "launch, scaled to this launch by its algorithmic bytes",
                "bytes_per_step": int(step_bytes), "steps_per_launch": args.steps,
                "us_per_step": round(t_max / args.steps * 1e6, 2)}
        gemv = None
    else:
        roof = gemv_roofline(eng, peak, peak_kind)
        gemv = roof
    clocks = clk.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_max / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 act / int4 weights, f32 accumulate",
            "data": "synthetic (random-init Q4 weights, random token ids)",
            "config": {"workload": ("c1: Qwen2.5-1.5B-Q4 (28 layers, vocab 151936) bs1 per GPU, 32-id "
                                    "prompt then greedy decode; weights 868.6 MB/step > L2, no flush")
                       if args.layers is None else
                       f"PROFILING ONLY: {cfg.n_layers}-layer reduction of c1 (not a benchmark)",
                       "model": "Qwen2.5-1.5B", "batch_per_gpu": B, "global_batch": B * world,
                       "prompt_len": PROMPT_LEN, "parallelism": f"dp{world} (independent requests)",
                       "l2": "inputs larger than L2"},
            "roofline": roof,
            "step_roofline": {"bytes_per_step": int(step_bytes), "achieved_gbs": round(step_gbs, 1),
                              "peak": peak, "frac": round(step_gbs / peak, 4), "unit": "GB/s",
                              "frac_of_8TBs": round(step_gbs / 8000.0, 4)},
            "decoder": eng.decoder,
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": cfg.hidden * 2,
                    "d2h_bytes_per_step": cfg.vocab * 2,
                    "api": "QwenEngine.run_inference + predict_next_token"},
            "gpu_launches": 1 if eng.pdec is not None else eng.launches_per_step() * args.steps,
            "clocks": clocks,
        }
    extras = None
    if not args.no_extra and args.layers is None:
        extras = extra_configs(mw, cfg, args, rank, world, dist, peak)
    if rank == 0:
        if extras is not None:
            line["configs"] = extras
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample()
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the c2/c3/c4 sub-measurements (batch 64, 8x2048 prefill, 32K context)")
    ap.add_argument("--only", choices=["c2", "c3", "c3_tp2", "c4"], default=None,
                    help="run only this sub-measurement after the headline line (for profiling)")
    ap.add_argument("--decoder", choices=["persistent", "kernels"], default=None)
    ap.add_argument("--timeline", default=None,
                    help="after the timed region, write the persistent kernel's stage timeline "
                         "(4 traced steps) as JSON to this path")
    ap.add_argument("--layers", type=int, default=None,
                    help="profiling only: build a model with fewer decoder layers (the JSON line "
                         "then names the reduced workload and is not a measurement of it)")
    ap.add_argument("--time", choices=["gemm", "attention", "prefill_attention", "gemv", "decode", "batched"],
                    default=None,
                    help="kernel timing tables instead of the benchmark: the tcgen05 W4A16 GEMM, the "
                         "split-KV decode attention, the causal prefill attention, the gate/up SwiGLU Q4 "
                         "GEMV, the persistent decoder (--layers, --iters steps per launch) or the batched "
                         "decode kernel against the per-stage path (--iters steps; --timeline any value: "
                         "its barrier timeline), per --shape (m,n,k / batch,attended,cache / "
                         "batch,seq_len / rows,k,batch / batch,cached / batch)")
    ap.add_argument("--shape", action="append", default=None, help="shape for --time (repeatable)")
    ap.add_argument("--iters", type=int, default=20,
                    help="calls per timing for --time gemm / gemv; steps per launch for --time decode")
    ap.add_argument("--auto-splits", action="store_true",
                    help="--time attention: only the split count the library picks")
    args = ap.parse_args()
    if args.time is not None:
        return run_kernel_timing(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
