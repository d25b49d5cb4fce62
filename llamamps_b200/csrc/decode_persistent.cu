// Persistent decode kernel: one cooperative launch runs n decode steps of the
// whole model (runners/engine.py:157-181 repeated), one CTA per SM.
//
// Why: a bs1 decode step reads 868.6 MB of Q4 weights in ~230 dependent
// pieces (28 x 5 stages + head); as separate kernels each piece pays launch
// latency and a cold start of its memory stream (the fused gate/up GEMV alone
// reaches ~23% of HBM bandwidth).  Here the weight stream never stops:
//
//  * warp 8 of every CTA (the producer) walks the same static schedule as the
//    compute warps and issues TMA bulk copies (cp.async.bulk, L2 evict-first)
//    of the CTA's row slice of every matrix, layer after layer, into a ring of
//    shared-memory slots guarded by full/empty mbarriers.  Weights do not
//    depend on activations, so the producer runs up to a ring (~160 KB, about
//    one layer per SM) ahead of the compute;
//  * warps 0-7 (the consumers) wait for a stage's input activation, stage it
//    in shared memory (RMSNorm'd where the reference normalises), consume
//    their slots (unpack nibbles -> fp16 codes, sm_100 mixed-precision FMA
//    into fp32, scale per group, warp-shuffle reduction) and write the stage
//    output with the fused epilogue;
//  * stages hand data across CTAs through global memory and one monotonic
//    arrival counter (fence + atomic add; a CTA waits with ld.acquire.gpu for
//    all CTAs to have finished the previous stage).  Every wait is bounded
//    (2 s of %globaltimer): on expiry the CTA raises state.error, stops the
//    producer, drains its in-flight copies and returns.
//
// Stages per layer (rows split evenly over the CTAs):
//   QKV  rmsnorm(x, in_norm) -> q|k|v = Wqkv x + b              (engine.py:188-195)
//   ATT  per (seq, kv head, position split): RoPE q/k, KV append at pos, GQA
//        scores/softmax/weighted sum over the paged cache; the last split to
//        finish merges the partials (log-sum-exp)                (engine.py:198-212)
//   O    x1 = x + fp16(Wo attn)                                  (engine.py:215-221)
//   GU   a = swiglu(Wg n, Wu n), n = rmsnorm(x1, post_norm)      (engine.py:224-235)
//   DN   x = x1 + fp16(Wd a)                                     (engine.py:237-243)
// then HEAD: logits = Wlm rmsnorm(x, final_norm) with the first-index argmax
// (engine.py:163-181), and every CTA derives the next token from the argmax.
#include <cmath>

#include "common.cuh"

namespace lmps {
namespace pk {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * kWarp;        // 256
constexpr int kThreads = kConsumers + kWarp;              // + producer warp
constexpr int kSlotBytes = 20480;
constexpr int kRows1536 = 16;     // rows per ring chunk when k = hidden
constexpr int kPairsGU = 8;       // gate/up row pairs per chunk
constexpr int kRowsDown = 4;      // rows per chunk when k = intermediate
constexpr int kAttnTile = 64;
constexpr int kHD = 128;
constexpr int kMaxG = 8;
constexpr int kKStride = kHD + 8;
constexpr unsigned long long kTimeoutNs = 2000000000ull;
constexpr int kMaxB = 4;

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// Plain (non-multicast) TMA bulk copy global -> this CTA's shared memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ float fma_hhf(uint16_t a, uint16_t b, float c) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint16_t lo16(uint32_t v) { return static_cast<uint16_t>(v & 0xFFFFu); }
__device__ __forceinline__ uint16_t hi16(uint32_t v) { return static_cast<uint16_t>(v >> 16); }

// 8 nibbles of w (elements e0..e7) times 8 fp16 activations, fp32 accumulate.
__device__ __forceinline__ float dot8(uint32_t w, const uint4& xv, float acc) {
  const uint32_t kMask = 0x000F000Fu, kMagic = 0x64006400u;
  const __half2 kBias = __halves2half2(__ushort_as_half(0xE408u), __ushort_as_half(0xE408u));
  uint32_t t0 = (w & kMask) | kMagic, t1 = ((w >> 4) & kMask) | kMagic;
  uint32_t t2 = ((w >> 8) & kMask) | kMagic, t3 = ((w >> 12) & kMask) | kMagic;
  __half2 h0 = __hadd2(*reinterpret_cast<__half2*>(&t0), kBias);
  __half2 h1 = __hadd2(*reinterpret_cast<__half2*>(&t1), kBias);
  __half2 h2 = __hadd2(*reinterpret_cast<__half2*>(&t2), kBias);
  __half2 h3 = __hadd2(*reinterpret_cast<__half2*>(&t3), kBias);
  const uint32_t c0 = *reinterpret_cast<uint32_t*>(&h0), c1 = *reinterpret_cast<uint32_t*>(&h1);
  const uint32_t c2 = *reinterpret_cast<uint32_t*>(&h2), c3 = *reinterpret_cast<uint32_t*>(&h3);
  acc = fma_hhf(lo16(c0), lo16(xv.x), acc);
  acc = fma_hhf(lo16(c1), hi16(xv.x), acc);
  acc = fma_hhf(lo16(c2), lo16(xv.y), acc);
  acc = fma_hhf(lo16(c3), hi16(xv.y), acc);
  acc = fma_hhf(hi16(c0), lo16(xv.z), acc);
  acc = fma_hhf(hi16(c1), hi16(xv.z), acc);
  acc = fma_hhf(hi16(c2), lo16(xv.w), acc);
  acc = fma_hhf(hi16(c3), hi16(xv.w), acc);
  return acc;
}
__device__ __forceinline__ int xswz(int vi) { return (vi & ~7) | ((vi & 7) ^ ((vi >> 3) & 7)); }
__device__ __forceinline__ float group_dot(const uint4& wv, const uint4* xrow, int g) {
  const int v0 = g * 4;
  const uint4 x0 = xrow[xswz(v0)], x1 = xrow[xswz(v0 + 1)];
  const uint4 x2 = xrow[xswz(v0 + 2)], x3 = xrow[xswz(v0 + 3)];
  float a0 = dot8(wv.x, x0, 0.0f), a1 = dot8(wv.y, x1, 0.0f);
  a0 = dot8(wv.z, x2, a0);
  a1 = dot8(wv.w, x3, a1);
  return a0 + a1;
}

struct Params {
  lmps_model_desc m;
  lmps_decode_state s;
  int n_steps;
  int slots;       // ring slots
  int act_bytes;   // activation / attention staging bytes
  // workspace carve-up
  __half* x;        // [B, hidden] residual after a layer
  __half* x1;       // [B, hidden] residual after attention
  __half* qkv;      // [B, qkv_rows]
  __half* attn;     // [B, q_dim]
  __half* a;        // [B, intermediate]
  float* part_o;    // [B, Hq, max_splits, 128]
  float2* part_ml;  // [B, Hq, max_splits]
  uint32_t* att_cnt;  // [B, Hkv]
  unsigned long long* keys;  // [2, B]
  uint32_t* arrive;          // [1]
  int max_splits;
};

enum StageKind { ST_QKV = 0, ST_O = 1, ST_GU = 2, ST_DN = 3, ST_HEAD = 4 };

struct Smem {
  unsigned char* ring;
  unsigned char* act;
  uint64_t* full;
  uint64_t* empty;
  float* red;        // [2][8 warps][4 rows][kMaxB]
  float* red8;       // [8 * kMaxB] block-reduction scratch
  unsigned long long* best;  // [8 warps][kMaxB]
  int* misc;         // [0] abort, [1] is_last, [2..] tok[kMaxB], pos[kMaxB]
};

__device__ __forceinline__ void row_range(int rows, int cta, int ctas, int& r0, int& r1) {
  r0 = static_cast<int>((static_cast<long long>(rows) * cta) / ctas);
  r1 = static_cast<int>((static_cast<long long>(rows) * (cta + 1)) / ctas);
}

// Weight chunk geometry of a stage for this CTA.
struct Chunking {
  const uint8_t* w;
  const __half* s;
  const uint8_t* w2;
  const __half* s2;
  int k, r0, r1, rows_per_chunk;
};

__device__ __forceinline__ Chunking stage_chunks(const Params& P, int kind, int layer) {
  Chunking c{};
  const lmps_model_desc& m = P.m;
  int rows = 0;
  if (kind == ST_HEAD) {
    c.w = m.lm_packed; c.s = reinterpret_cast<const __half*>(m.lm_scales);
    c.k = m.hidden; rows = m.vocab; c.rows_per_chunk = kRows1536;
  } else {
    const lmps_layer_desc& L = m.layers[layer];
    if (kind == ST_QKV) {
      c.w = L.qkv_packed; c.s = reinterpret_cast<const __half*>(L.qkv_scales);
      c.k = m.hidden; rows = (m.n_q_heads + 2 * m.n_kv_heads) * m.head_dim; c.rows_per_chunk = kRows1536;
    } else if (kind == ST_O) {
      c.w = L.o_packed; c.s = reinterpret_cast<const __half*>(L.o_scales);
      c.k = m.n_q_heads * m.head_dim; rows = m.hidden; c.rows_per_chunk = kRows1536;
    } else if (kind == ST_GU) {
      c.w = L.gate_packed; c.s = reinterpret_cast<const __half*>(L.gate_scales);
      c.w2 = L.up_packed; c.s2 = reinterpret_cast<const __half*>(L.up_scales);
      c.k = m.hidden; rows = m.intermediate; c.rows_per_chunk = kPairsGU;
    } else {
      c.w = L.down_packed; c.s = reinterpret_cast<const __half*>(L.down_scales);
      c.k = m.intermediate; rows = m.hidden; c.rows_per_chunk = kRowsDown;
    }
  }
  row_range(rows, blockIdx.x, gridDim.x, c.r0, c.r1);
  return c;
}

// ---------------------------------------------------------------------------
// Producer: one lane streams every chunk of every stage into the ring.
// ---------------------------------------------------------------------------
__device__ void producer(const Params& P, Smem& S) {
  const uint64_t policy = evict_first_policy();
  uint32_t chunk = 0;
  bool ok = true;
  const int kinds[4] = {ST_QKV, ST_O, ST_GU, ST_DN};
  for (int step = 0; step < P.n_steps && ok; ++step) {
    for (int l = 0; l <= P.m.n_layers && ok; ++l) {
      const int nk = (l < P.m.n_layers) ? 4 : 1;
      for (int ki = 0; ki < nk && ok; ++ki) {
        const int kind = (l < P.m.n_layers) ? kinds[ki] : ST_HEAD;
        const Chunking c = stage_chunks(P, kind, l);
        const size_t row_bytes = static_cast<size_t>(c.k) / 2;
        const size_t row_scales = static_cast<size_t>(c.k) / 32;
        for (int r = c.r0; r < c.r1 && ok; r += c.rows_per_chunk, ++chunk) {
          const int n = min(c.rows_per_chunk, c.r1 - r);
          const int slot = chunk % P.slots;
          const uint32_t phase = (chunk / P.slots) & 1u;
          // wait until the consumers released this slot's previous contents
          if (chunk >= static_cast<uint32_t>(P.slots)) {
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(&S.empty[slot], phase ^ 1u)) {
              if (*reinterpret_cast<volatile int*>(&S.misc[0]) || globaltimer() - t0 > kTimeoutNs) {
                ok = false;
                break;
              }
            }
            if (!ok) break;
          }
          unsigned char* dst = S.ring + static_cast<size_t>(slot) * kSlotBytes;
          const uint32_t pbytes = static_cast<uint32_t>(n * row_bytes);
          const uint32_t sbytes = static_cast<uint32_t>(n * row_scales * 2);
          const uint32_t total = (kind == ST_GU) ? 2 * (pbytes + sbytes) : pbytes + sbytes;
          mbar_expect_tx(&S.full[slot], total);
          if (kind == ST_GU) {
            bulk_g2s(dst, c.w + r * row_bytes, pbytes, &S.full[slot], policy);
            bulk_g2s(dst + pbytes, c.w2 + r * row_bytes, pbytes, &S.full[slot], policy);
            bulk_g2s(dst + 2 * pbytes, c.s + r * row_scales, sbytes, &S.full[slot], policy);
            bulk_g2s(dst + 2 * pbytes + sbytes, c.s2 + r * row_scales, sbytes, &S.full[slot], policy);
          } else {
            bulk_g2s(dst, c.w + r * row_bytes, pbytes, &S.full[slot], policy);
            bulk_g2s(dst + pbytes, c.s + r * row_scales, sbytes, &S.full[slot], policy);
          }
        }
      }
    }
  }
  // Drain: every issued copy must land before this CTA may exit.
  const uint32_t issued = chunk;
  const uint32_t first = issued > static_cast<uint32_t>(P.slots) ? issued - P.slots : 0u;
  for (uint32_t c = first; c < issued; ++c) {
    const int slot = c % P.slots;
    const uint32_t phase = (c / P.slots) & 1u;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(&S.full[slot], phase)) {
      if (globaltimer() - t0 > kTimeoutNs) break;
    }
  }
}

// ---------------------------------------------------------------------------
// Consumer helpers
// ---------------------------------------------------------------------------
struct CState {
  uint32_t chunk;     // ring chunk counter (same sequence as the producer)
  uint32_t arrivals;  // grid arrivals expected so far
  bool ok;
};

// All CTAs finished the previous stage?  Thread 0 polls, then the consumers sync.
__device__ bool grid_wait(const Params& P, Smem& S, CState& cs) {
  if (threadIdx.x == 0 && *reinterpret_cast<volatile int*>(&S.misc[0]) == 0) {
    const uint32_t target = cs.arrivals;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_u32(P.arrive) < target) {
      if (globaltimer() - t0 > kTimeoutNs) {
        atomicExch(P.s.error, 1);
        *reinterpret_cast<volatile int*>(&S.misc[0]) = 1;
        break;
      }
    }
  }
  consumer_sync();
  cs.ok = *reinterpret_cast<volatile int*>(&S.misc[0]) == 0;
  return cs.ok;
}

// This CTA finished a stage: publish its writes, then count it.
__device__ void grid_arrive(const Params& P, CState& cs) {
  __threadfence();
  consumer_sync();
  if (threadIdx.x == 0) atomicAdd(P.arrive, 1u);
  cs.arrivals += gridDim.x;
}

// Wait for the next ring chunk.  Control flow stays uniform across the
// consumers: a thread that gives up (timeout, or the CTA already aborting)
// raises the abort flag and carries on with the slot's stale contents -- all
// reads stay inside shared memory and all writes inside the stage's outputs --
// and the CTA leaves together at its next grid_wait.
__device__ void slot_wait(Smem& S, const Params& P, CState& cs, int& slot) {
  slot = cs.chunk % P.slots;
  const uint32_t phase = (cs.chunk / P.slots) & 1u;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(&S.misc[0]);
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(&S.full[slot], phase)) {
    if (*abort_flag) return;
    if (globaltimer() - t0 > kTimeoutNs) {
      atomicExch(P.s.error, 1);
      *abort_flag = 1;
      return;
    }
  }
}

__device__ __forceinline__ void slot_release(Smem& S, CState& cs, int slot) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&S.empty[slot]);
}

// Block (consumer) sum of one float per thread; every consumer gets the total.
__device__ __forceinline__ float consumer_sum(float v, float* red8) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red8[warp] = v;
  consumer_sync();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) t += red8[w];
  consumer_sync();
  return t;
}

// act[b] <- fp16(fp16(x*scale) * gamma) with x = rows[b] (k elements, swizzled
// 16-byte chunks) -- rms_norm.metal:20-39 over the full vector.
template <int NB>
__device__ void stage_norm(const Params& P, Smem& S, const __half* const* rows, bool rows_nc,
                           const __half* gamma, int k) {
  const int vpr = k / 8;  // 16-byte chunks per row (multiple of 8)
  uint4* act = reinterpret_cast<uint4*>(S.act);
  constexpr int kMaxV = 2;  // k <= 2 * 8 * 256 = 4096
  for (int b = 0; b < NB; ++b) {
    if (b >= P.s.batch) break;
    uint4 v[kMaxV];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxV; ++i) {
      const int c = threadIdx.x + i * kConsumers;
      v[i] = make_uint4(0u, 0u, 0u, 0u);
      if (c < vpr) {
        const uint4* src = reinterpret_cast<const uint4*>(rows[b]) + c;
        v[i] = rows_nc ? __ldg(src) : __ldcg(src);
        const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(h[e]);
          ss = fmaf(f.x, f.x, ss);
          ss = fmaf(f.y, f.y, ss);
        }
      }
    }
    ss = consumer_sum(ss, S.red8);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(k) + P.m.eps);
#pragma unroll
    for (int i = 0; i < kMaxV; ++i) {
      const int c = threadIdx.x + i * kConsumers;
      if (c < vpr) {
        const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gamma) + c);
        const __half* xh = reinterpret_cast<const __half*>(&v[i]);
        const __half* gh = reinterpret_cast<const __half*>(&gv);
        uint4 o;
        __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const __half nrm = __float2half_rn(__half2float(xh[e]) * scale);
          oh[e] = __float2half_rn(__half2float(nrm) * __half2float(gh[e]));
        }
        act[b * vpr + xswz(c)] = o;
      }
    }
  }
  consumer_sync();
}

// act[b] <- src[b] (k elements) for every sequence.
template <int NB>
__device__ void stage_copy(const Params& P, Smem& S, const __half* src, int ld, int k) {
  const int vpr = k / 8;
  uint4* act = reinterpret_cast<uint4*>(S.act);
  for (int i = threadIdx.x; i < NB * vpr; i += kConsumers) {
    const int b = i / vpr, c = i - b * vpr;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (b < P.s.batch) v = __ldcg(reinterpret_cast<const uint4*>(src + static_cast<size_t>(b) * ld) + c);
    act[b * vpr + xswz(c)] = v;
  }
  consumer_sync();
}

// ---------------------------------------------------------------------------
// GEMV stages over ring chunks
// ---------------------------------------------------------------------------
// k = hidden stages (QKV, O, HEAD): chunk of <= 16 rows; warp w owns rows
// 2w (lanes 0-15) and 2w+1 (lanes 16-31); lane sub walks groups sub, sub+16, ...
template <int NB, int KIND>
__device__ void gemv_hidden(const Params& P, Smem& S, CState& cs, const Chunking& c,
                            const __half* bias, const __half* const* res_rows, __half* out, int ldo,
                            unsigned long long* best) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = c.k / 32;
  const int vpr = c.k / 8;
  const uint4* act = reinterpret_cast<const uint4*>(S.act);
  for (int r = c.r0; r < c.r1; r += c.rows_per_chunk) {
    const int n = min(c.rows_per_chunk, c.r1 - r);
    int slot;
    slot_wait(S, P, cs, slot);
    const unsigned char* base = S.ring + static_cast<size_t>(slot) * kSlotBytes;
    const int lrow = 2 * warp + (lane >> 4);
    const int sub = lane & 15;
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
    if (lrow < n) {
      const unsigned char* wrow = base + static_cast<size_t>(lrow) * (c.k / 2);
      const __half* srow = reinterpret_cast<const __half*>(base + static_cast<size_t>(n) * (c.k / 2)) + lrow * G;
      for (int g = sub; g < G; g += 16) {
        const uint4 wv = *reinterpret_cast<const uint4*>(wrow + g * 16);
        const float sc = __half2float(srow[g]);
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[b] = fmaf(sc, group_dot(wv, act + b * vpr, g), acc[b]);
      }
    }
    slot_release(S, cs, slot);
    ++cs.chunk;
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = segment_sum<16>(acc[b]);
    if (sub == 0 && lrow < n) {
      const int row = r + lrow;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b >= P.s.batch) break;
        if constexpr (KIND == ST_QKV) {
          out[static_cast<size_t>(b) * ldo + row] = __float2half_rn(acc[b] + __half2float(bias[row]));
        } else if constexpr (KIND == ST_O) {
          const __half o = __float2half_rn(acc[b]);
          out[static_cast<size_t>(b) * ldo + row] = __hadd(__ldcg(res_rows[b] + row), o);
        } else {  // ST_HEAD
          const __half v = __float2half_rn(acc[b]);
          if (out) out[static_cast<size_t>(b) * ldo + row] = v;
          best[b] = u64_max(best[b], argmax_key(__half2float(v), static_cast<uint32_t>(row)));
        }
      }
    }
  }
}

// Gate/up: chunk of <= 8 row pairs; warp w: gate row w on lanes 0-15, up row w
// on lanes 16-31; lane 0 applies SwiGLU (swiglu.metal:19-22).
template <int NB>
__device__ void gemv_gateup(const Params& P, Smem& S, CState& cs, const Chunking& c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = c.k / 32, vpr = c.k / 8;
  const uint4* act = reinterpret_cast<const uint4*>(S.act);
  const int inter = P.m.intermediate;
  for (int r = c.r0; r < c.r1; r += c.rows_per_chunk) {
    const int n = min(c.rows_per_chunk, c.r1 - r);
    int slot;
    slot_wait(S, P, cs, slot);
    const unsigned char* base = S.ring + static_cast<size_t>(slot) * kSlotBytes;
    const size_t pbytes = static_cast<size_t>(n) * (c.k / 2);
    const size_t sbytes = static_cast<size_t>(n) * G * 2;
    const int up = lane >> 4, sub = lane & 15;
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
    if (warp < n) {
      const unsigned char* wrow = base + up * pbytes + static_cast<size_t>(warp) * (c.k / 2);
      const __half* srow = reinterpret_cast<const __half*>(base + 2 * pbytes + up * sbytes) + warp * G;
      for (int g = sub; g < G; g += 16) {
        const uint4 wv = *reinterpret_cast<const uint4*>(wrow + g * 16);
        const float sc = __half2float(srow[g]);
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[b] = fmaf(sc, group_dot(wv, act + b * vpr, g), acc[b]);
      }
    }
    slot_release(S, cs, slot);
    ++cs.chunk;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      acc[b] = segment_sum<16>(acc[b]);
      const float u = __shfl_sync(0xffffffffu, acc[b], 16);
      if (lane == 0 && warp < n && b < P.s.batch) {
        const float gf = __half2float(__float2half_rn(acc[b]));
        const float uf = __half2float(__float2half_rn(u));
        P.a[static_cast<size_t>(b) * inter + r + warp] = __float2half_rn(silu_mul(gf, uf));
      }
    }
  }
}

// Down projection (k = intermediate): chunk of <= 4 rows; warp w sums groups
// [G*w/8, G*(w+1)/8) of every row (lane = row*8 + sub), partials meet in
// shared memory and warp 0 finishes: x = x1 + fp16(acc).
template <int NB>
__device__ void gemv_down(const Params& P, Smem& S, CState& cs, const Chunking& c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = c.k / 32, vpr = c.k / 8;
  const int g0 = G * warp / kConsumerWarps, g1 = G * (warp + 1) / kConsumerWarps;
  const uint4* act = reinterpret_cast<const uint4*>(S.act);
  const int hidden = P.m.hidden;
  int par = 0;
  for (int r = c.r0; r < c.r1; r += c.rows_per_chunk, par ^= 1) {
    const int n = min(c.rows_per_chunk, c.r1 - r);
    int slot;
    slot_wait(S, P, cs, slot);
    const unsigned char* base = S.ring + static_cast<size_t>(slot) * kSlotBytes;
    const int lrow = lane >> 3, sub = lane & 7;
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
    if (lrow < n) {
      const unsigned char* wrow = base + static_cast<size_t>(lrow) * (c.k / 2);
      const __half* srow = reinterpret_cast<const __half*>(base + static_cast<size_t>(n) * (c.k / 2)) + lrow * G;
      for (int g = g0 + sub; g < g1; g += 8) {
        const uint4 wv = *reinterpret_cast<const uint4*>(wrow + g * 16);
        const float sc = __half2float(srow[g]);
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[b] = fmaf(sc, group_dot(wv, act + b * vpr, g), acc[b]);
      }
    }
    slot_release(S, cs, slot);
    ++cs.chunk;
    float* red = S.red + par * (kConsumerWarps * kRowsDown * kMaxB);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      acc[b] = segment_sum<8>(acc[b]);
      if (sub == 0) red[(warp * kRowsDown + lrow) * kMaxB + b] = acc[b];
    }
    consumer_sync();
    if (threadIdx.x < n * NB) {
      const int lr = threadIdx.x / NB, b = threadIdx.x % NB;
      if (b < P.s.batch) {
        float t = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) t += red[(w * kRowsDown + lr) * kMaxB + b];
        const int row = r + lr;
        const __half d = __float2half_rn(t);
        P.x[static_cast<size_t>(b) * hidden + row] = __hadd(__ldcg(P.x1 + static_cast<size_t>(b) * hidden + row), d);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Attention stage: one work item = (sequence b, kv head, split of positions)
// ---------------------------------------------------------------------------
struct AttnSmemP {
  float q[kMaxG][kHD];
  __half k[kAttnTile][kKStride];
  __half v[kAttnTile][kHD];
  float p[kMaxG][kAttnTile];
  float m[kMaxG];
  float l[kMaxG];
  float alpha[kMaxG];
  int is_last;
};

__device__ __forceinline__ void rope_pair(int j, int style, int& i1, int& i2) {
  if (style == LMPS_ROPE_INTERLEAVED) {
    i1 = 2 * j;
    i2 = i1 + 1;
  } else {
    i1 = j;
    i2 = j + kHD / 2;
  }
}

__device__ void attn_item(const Params& P, Smem& S, const lmps_layer_desc& L, int b, int kvh,
                          int split, int n_splits, int chunk, int pos) {
  AttnSmemP& A = *reinterpret_cast<AttnSmemP*>(S.act);
  const lmps_model_desc& m = P.m;
  const int tid = threadIdx.x;
  const int Hq = m.n_q_heads, Hkv = m.n_kv_heads, G = Hq / Hkv;
  const int qkv_rows = (Hq + 2 * Hkv) * kHD;
  const int T = pos + 1;
  const int start = split * chunk, end = min(T, start + chunk);
  const __half* row = P.qkv + static_cast<size_t>(b) * qkv_rows;
  const float fpos = static_cast<float>(pos);
  const int ps = P.s.page_size;
  const int32_t* bt = P.s.block_table + static_cast<size_t>(b) * P.s.max_pages;
  __half* kpool = reinterpret_cast<__half*>(L.k_pool);
  __half* vpool = reinterpret_cast<__half*>(L.v_pool);

  // RoPE'd q of the G heads sharing this KV head (rope.metal:19-40), fp16-rounded.
  for (int i = tid; i < G * (kHD / 2); i += kConsumers) {
    const int h = i / (kHD / 2), j = i - h * (kHD / 2);
    int i1, i2;
    rope_pair(j, m.rope_style, i1, i2);
    const __half* qh = row + (kvh * G + h) * kHD;
    const float x1 = __half2float(__ldcg(qh + i1)), x2 = __half2float(__ldcg(qh + i2));
    float sn, cs;
    sincosf(fpos * __ldg(m.inv_freq + j), &sn, &cs);
    A.q[h][i1] = __half2float(__float2half_rn(x1 * cs - x2 * sn));
    A.q[h][i2] = __half2float(__float2half_rn(x1 * sn + x2 * cs));
  }
  // The split holding the new position appends its rotated k and raw v.
  if (pos >= start && pos < end) {
    const int page = bt[pos / ps], off = pos % ps;
    const size_t base = ((static_cast<size_t>(page) * Hkv + kvh) * ps + off) * kHD;
    const __half* kh = row + (Hq + kvh) * kHD;
    const __half* vh = row + (Hq + Hkv + kvh) * kHD;
    if (tid < kHD / 2) {
      int i1, i2;
      rope_pair(tid, m.rope_style, i1, i2);
      const float x1 = __half2float(__ldcg(kh + i1)), x2 = __half2float(__ldcg(kh + i2));
      float sn, cs;
      sincosf(fpos * __ldg(m.inv_freq + tid), &sn, &cs);
      kpool[base + i1] = __float2half_rn(x1 * cs - x2 * sn);
      kpool[base + i2] = __float2half_rn(x1 * sn + x2 * cs);
    } else if (tid < kHD / 2 + kHD) {
      const int d = tid - kHD / 2;
      vpool[base + d] = __ldcg(vh + d);
    }
  }
  if (tid < kMaxG) {
    A.m[tid] = -INFINITY;
    A.l[tid] = 0.0f;
  }
  float acc[kMaxG / 2];
#pragma unroll
  for (int j = 0; j < kMaxG / 2; ++j) acc[j] = 0.0f;
  consumer_sync();

  for (int t0 = start; t0 < end; t0 += kAttnTile) {
    const int n = min(kAttnTile, end - t0);
    for (int i = tid; i < kAttnTile * (kHD / 8); i += kConsumers) {
      const int r = i / (kHD / 8), c = i - r * (kHD / 8);
      uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = make_uint4(0u, 0u, 0u, 0u);
      if (r < n) {
        const int p = t0 + r;
        const size_t off = ((static_cast<size_t>(bt[p / ps]) * Hkv + kvh) * ps + p % ps) * kHD + c * 8;
        kv = __ldcg(reinterpret_cast<const uint4*>(kpool + off));
        vv = __ldcg(reinterpret_cast<const uint4*>(vpool + off));
      }
      *reinterpret_cast<uint4*>(&A.k[r][c * 8]) = kv;
      *reinterpret_cast<uint4*>(&A.v[r][c * 8]) = vv;
    }
    consumer_sync();
    {  // scores: thread -> (position r, heads hq, hq+4)
      const int r = tid & (kAttnTile - 1), hq = tid >> 6;
      float dots[2] = {0.0f, 0.0f};
#pragma unroll 4
      for (int c = 0; c < kHD / 8; ++c) {
        const uint4 kk = *reinterpret_cast<const uint4*>(&A.k[r][c * 8]);
        const __half2* k2 = reinterpret_cast<const __half2*>(&kk);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(k2[e]);
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int h = hq + 4 * j;
          if (h < G) {
#pragma unroll
            for (int e = 0; e < 8; ++e) dots[j] = fmaf(A.q[h][c * 8 + e], kf[e], dots[j]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int h = hq + 4 * j;
        if (h < G) A.p[h][r] = (r < n) ? dots[j] * kAttnScale : -INFINITY;
      }
    }
    consumer_sync();
    {  // online softmax, one warp per head (softmax.metal:23-36)
      const int warp = tid >> 5, lane = tid & 31;
      if (warp < G) {
        const int h = warp;
        const float s0 = A.p[h][lane], s1 = A.p[h][lane + 32];
        const float m_old = A.m[h];
        const float m_new = fmaxf(m_old, warp_max(fmaxf(s0, s1)));
        float e0 = 0.0f, e1 = 0.0f, alpha = 1.0f;
        if (m_new != -INFINITY) {
          e0 = expf(s0 - m_new);
          e1 = expf(s1 - m_new);
          alpha = expf(m_old - m_new);
        }
        const float sum = warp_sum(e0 + e1);
        A.p[h][lane] = e0;
        A.p[h][lane + 32] = e1;
        __syncwarp();
        if (lane == 0) {
          A.alpha[h] = alpha;
          A.m[h] = m_new;
          A.l[h] = A.l[h] * alpha + sum;
        }
      }
    }
    consumer_sync();
    {  // P.V (attn_sum.metal:26-32): thread -> (dim d, heads hh, hh+2, ...)
      const int d = tid & (kHD - 1), hh = tid >> 7;
#pragma unroll
      for (int j = 0; j < kMaxG / 2; ++j) {
        const int h = hh + 2 * j;
        if (h < G) acc[j] *= A.alpha[h];
      }
      for (int r = 0; r < n; ++r) {
        const float v = __half2float(A.v[r][d]);
#pragma unroll
        for (int j = 0; j < kMaxG / 2; ++j) {
          const int h = hh + 2 * j;
          if (h < G) acc[j] = fmaf(A.p[h][r], v, acc[j]);
        }
      }
    }
    consumer_sync();
  }

  const int d = tid & (kHD - 1), hh = tid >> 7;
  if (n_splits == 1) {
#pragma unroll
    for (int j = 0; j < kMaxG / 2; ++j) {
      const int h = hh + 2 * j;
      if (h < G) {
        const float l = A.l[h];
        P.attn[static_cast<size_t>(b) * Hq * kHD + (kvh * G + h) * kHD + d] =
            __float2half_rn(l > 0.0f ? acc[j] / l : 0.0f);
      }
    }
    consumer_sync();
    return;
  }
  const size_t ms = P.max_splits;
#pragma unroll
  for (int j = 0; j < kMaxG / 2; ++j) {
    const int h = hh + 2 * j;
    if (h < G) {
      const size_t prow = (static_cast<size_t>(b) * Hq + kvh * G + h) * ms + split;
      P.part_o[prow * kHD + d] = acc[j];
      if (d == 0) P.part_ml[prow] = make_float2(A.m[h], A.l[h]);
    }
  }
  __threadfence();
  consumer_sync();
  if (tid == 0) {
    const uint32_t old = atomicAdd(P.att_cnt + b * Hkv + kvh, 1u);
    A.is_last = (old == static_cast<uint32_t>(n_splits - 1)) ? 1 : 0;
  }
  consumer_sync();
  if (A.is_last) {  // the last split merges all partials of (b, kvh)
    __threadfence();
#pragma unroll
    for (int j = 0; j < kMaxG / 2; ++j) {
      const int h = hh + 2 * j;
      if (h < G) {
        const size_t prow0 = (static_cast<size_t>(b) * Hq + kvh * G + h) * ms;
        float M = -INFINITY;
        for (int sp = 0; sp < n_splits; ++sp) M = fmaxf(M, __ldcg(&P.part_ml[prow0 + sp].x));
        float num = 0.0f, den = 0.0f;
        for (int sp = 0; sp < n_splits; ++sp) {
          const float2 ml = __ldcg(&P.part_ml[prow0 + sp]);
          if (ml.y > 0.0f) {
            const float w = expf(ml.x - M);
            num = fmaf(w, __ldcg(&P.part_o[(prow0 + sp) * kHD + d]), num);
            den = fmaf(w, ml.y, den);
          }
        }
        P.attn[static_cast<size_t>(b) * Hq * kHD + (kvh * G + h) * kHD + d] =
            __float2half_rn(den > 0.0f ? num / den : 0.0f);
      }
    }
    if (tid == 0) P.att_cnt[b * Hkv + kvh] = 0u;
  }
  consumer_sync();
}

// Positions per attention split this step (all CTAs compute the same value):
// at least one 64-position tile, and about two work items per CTA overall.
__device__ __forceinline__ int attn_chunk_len(const int* pos, int batch, int n_kv) {
  long long total = 0;
  for (int b = 0; b < batch; ++b) total += pos[b] + 1;
  long long c = (total * n_kv + 2 * gridDim.x - 1) / (2 * gridDim.x);
  c = (c + kAttnTile - 1) / kAttnTile * kAttnTile;
  return static_cast<int>(c < kAttnTile ? kAttnTile : c);
}

// ---------------------------------------------------------------------------
// Consumers: the decode loop
// ---------------------------------------------------------------------------
template <int NB>
__device__ void consumer(const Params& P, Smem& S) {
  CState cs{0u, 0u, true};
  const lmps_model_desc& m = P.m;
  const int B = P.s.batch;
  const int hidden = m.hidden, Hq = m.n_q_heads, Hkv = m.n_kv_heads;
  const int q_dim = Hq * kHD, qkv_rows = (Hq + 2 * Hkv) * kHD;
  int tok[NB], pos[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    tok[b] = b < B ? P.s.tokens[b] : 0;
    pos[b] = b < B ? P.s.pos[b] : 0;
  }
  const int hist0 = (P.s.history && P.s.step_counter) ? P.s.step_counter[0] : 0;
  bool first_stage = true;

  for (int step = 0; step < P.n_steps; ++step) {
    const int par = step & 1;
    if (!first_stage) {
      // previous step's HEAD finished everywhere: next tokens from its argmax
      if (!grid_wait(P, S, cs)) return;
      const int pp = par ^ 1;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b < B) {
          const unsigned long long key = __ldcg(P.keys + pp * B + b);
          int nxt = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
          if (nxt < 0 || nxt >= m.vocab) {  // no logit won (non-finite head output)
            if (threadIdx.x == 0) atomicExch(P.s.error, 3);
            nxt = 0;
          }
          if (blockIdx.x == 0 && threadIdx.x == 0 && P.s.history && hist0 + step - 1 >= 0 &&
              hist0 + step - 1 < P.s.history_rows)
            P.s.history[static_cast<size_t>(hist0 + step - 1) * B + b] = nxt;
          tok[b] = (step - 1 < P.s.n_forced && P.s.forced) ? P.s.forced[static_cast<size_t>(b) * P.s.forced_stride + step - 1] : nxt;
          pos[b] += 1;
        }
      }
    }
    const __half* xin[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int bb = b < B ? b : 0;
      xin[b] = (step == 0 && P.s.x_in) ? reinterpret_cast<const __half*>(P.s.x_in) + static_cast<size_t>(bb) * hidden
                                       : reinterpret_cast<const __half*>(m.embed) + static_cast<size_t>(tok[bb]) * hidden;
    }
    const __half* xres[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) xres[b] = P.x + static_cast<size_t>(b < B ? b : 0) * hidden;
    const __half* x1rows[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) x1rows[b] = P.x1 + static_cast<size_t>(b < B ? b : 0) * hidden;

    for (int l = 0; l < m.n_layers; ++l) {
      const lmps_layer_desc& L = m.layers[l];
      // ---- QKV
      if (!first_stage && l > 0) {
        if (!grid_wait(P, S, cs)) return;
      }
      first_stage = false;
      stage_norm<NB>(P, S, l == 0 ? xin : xres, l == 0, reinterpret_cast<const __half*>(L.in_norm), hidden);
      {
        const Chunking c = stage_chunks(P, ST_QKV, l);
        gemv_hidden<NB, ST_QKV>(P, S, cs, c, reinterpret_cast<const __half*>(L.qkv_bias), nullptr, P.qkv,
                                qkv_rows, nullptr);
      }
      grid_arrive(P, cs);
      // ---- ATT
      if (!grid_wait(P, S, cs)) return;
      if (l == 0 && step > 0 && blockIdx.x == 0 && threadIdx.x < B)
        P.keys[(par ^ 1) * B + threadIdx.x] = 0ull;  // everyone has read the previous argmax
      {
        const int chunk = attn_chunk_len(pos, B, Hkv);
        int n_items = 0;
#pragma unroll
        for (int b = 0; b < NB; ++b)
          if (b < B) n_items += Hkv * ((pos[b] + chunk) / chunk);
        for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
          int rem = it, bsel = 0, nsp = 1;
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            if (b < B && bsel == b) {
              nsp = (pos[b] + chunk) / chunk;
              if (rem >= Hkv * nsp) {
                rem -= Hkv * nsp;
                ++bsel;
              }
            }
          }
          const int kvh = rem / nsp, sp = rem - kvh * nsp;
          int pb = pos[0];
#pragma unroll
          for (int b = 0; b < NB; ++b)
            if (b == bsel) pb = pos[b];
          attn_item(P, S, L, bsel, kvh, sp, nsp, chunk, pb);
        }
      }
      grid_arrive(P, cs);
      // ---- O
      if (!grid_wait(P, S, cs)) return;
      stage_copy<NB>(P, S, P.attn, q_dim, q_dim);
      {
        const Chunking c = stage_chunks(P, ST_O, l);
        gemv_hidden<NB, ST_O>(P, S, cs, c, nullptr, l == 0 ? xin : xres, P.x1, hidden, nullptr);
      }
      grid_arrive(P, cs);
      // ---- GU
      if (!grid_wait(P, S, cs)) return;
      stage_norm<NB>(P, S, x1rows, false, reinterpret_cast<const __half*>(L.post_norm), hidden);
      {
        const Chunking c = stage_chunks(P, ST_GU, l);
        gemv_gateup<NB>(P, S, cs, c);
      }
      grid_arrive(P, cs);
      // ---- DN
      if (!grid_wait(P, S, cs)) return;
      stage_copy<NB>(P, S, P.a, m.intermediate, m.intermediate);
      {
        const Chunking c = stage_chunks(P, ST_DN, l);
        gemv_down<NB>(P, S, cs, c);
      }
      grid_arrive(P, cs);
    }
    // ---- HEAD
    if (!grid_wait(P, S, cs)) return;
    stage_norm<NB>(P, S, xres, false, reinterpret_cast<const __half*>(m.final_norm), hidden);
    {
      unsigned long long best[NB];
#pragma unroll
      for (int b = 0; b < NB; ++b) best[b] = 0ull;
      const Chunking c = stage_chunks(P, ST_HEAD, 0);
      __half* lg = (step == P.n_steps - 1 && P.s.logits) ? reinterpret_cast<__half*>(P.s.logits) : nullptr;
      gemv_hidden<NB, ST_HEAD>(P, S, cs, c, nullptr, nullptr, lg, m.vocab, best);
      const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const unsigned long long w = warp_max_u64(best[b]);
        if (lane == 0) S.best[warp * kMaxB + b] = w;
      }
      consumer_sync();
      if (threadIdx.x < B) {
        unsigned long long v = 0ull;
        for (int w = 0; w < kConsumerWarps; ++w) v = u64_max(v, S.best[w * kMaxB + threadIdx.x]);
        if (v) atomicMax(P.keys + par * B + threadIdx.x, v);
      }
    }
    grid_arrive(P, cs);
  }
  // ---- final tokens, state write-back, exit barrier
  if (!grid_wait(P, S, cs)) return;
  {
    const int last = P.n_steps - 1, pp = last & 1;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      for (int b = 0; b < B; ++b) {
        const unsigned long long key = __ldcg(P.keys + pp * B + b);
        const int nxt = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
        if (P.s.history && hist0 + last >= 0 && hist0 + last < P.s.history_rows)
          P.s.history[static_cast<size_t>(hist0 + last) * B + b] = nxt;
        int p_fin = 0;
#pragma unroll
        for (int bb = 0; bb < NB; ++bb)
          if (bb == b) p_fin = pos[bb];
        P.s.tokens[b] = (last < P.s.n_forced && P.s.forced) ? P.s.forced[static_cast<size_t>(b) * P.s.forced_stride + last] : nxt;
        P.s.pos[b] = p_fin + 1;
      }
      if (P.s.history && P.s.step_counter) P.s.step_counter[0] = hist0 + P.n_steps;
    }
  }
  grid_arrive(P, cs);
  if (blockIdx.x == 0) {
    if (!grid_wait(P, S, cs)) return;
    if (threadIdx.x < 2 * B) P.keys[threadIdx.x] = 0ull;
    if (threadIdx.x == 0) *P.arrive = 0u;
  }
}

template <int NB>
__global__ void __launch_bounds__(kThreads, 1) decode_persistent_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(128) unsigned char smem[];
  Smem S;
  S.ring = smem;
  S.act = smem + static_cast<size_t>(P.slots) * kSlotBytes;
  unsigned char* tail = S.act + P.act_bytes;
  S.full = reinterpret_cast<uint64_t*>(tail);
  S.empty = S.full + 16;
  S.red = reinterpret_cast<float*>(S.empty + 16);
  S.red8 = S.red + 2 * kConsumerWarps * kRowsDown * kMaxB;
  S.best = reinterpret_cast<unsigned long long*>(S.red8 + 8 * kMaxB);
  S.misc = reinterpret_cast<int*>(S.best + kConsumerWarps * kMaxB);
  // Every position this launch touches must be inside the cache and every fed
  // token inside the vocabulary; all CTAs read the same values, so all leave
  // together (nothing has been issued yet).
  {
    bool bad = false;
    for (int b = 0; b < P.s.batch; ++b) {
      const int p0 = P.s.pos[b], t0 = P.s.tokens[b];
      if (p0 < 0 || p0 + P.n_steps > P.s.max_seq_len) bad = true;
      if (!P.s.x_in && (t0 < 0 || t0 >= P.m.vocab)) bad = true;
      for (int i = 0; P.s.forced && i < P.s.n_forced && i < P.n_steps; ++i) {
        const int f = P.s.forced[static_cast<size_t>(b) * P.s.forced_stride + i];
        if (f < 0 || f >= P.m.vocab) bad = true;
      }
    }
    if (bad) {
      if (threadIdx.x == 0) atomicExch(P.s.error, 2);
      return;
    }
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < P.slots; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.empty[i], kConsumerWarps);
    }
    S.misc[0] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x >= kConsumers) {
    if (threadIdx.x == kConsumers) producer(P, S);
    return;
  }
  consumer<NB>(P, S);
}

constexpr int kTailBytes = 4096;

struct WsLayout {
  size_t x, x1, qkv, attn, a, part_o, part_ml, att_cnt, keys, arrive, total;
  int max_splits;
};

static size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

static WsLayout ws_layout(const lmps_model_desc& m, int B, int max_seq_len) {
  WsLayout w{};
  const size_t qkv_rows = static_cast<size_t>(m.n_q_heads + 2 * m.n_kv_heads) * m.head_dim;
  const size_t q_dim = static_cast<size_t>(m.n_q_heads) * m.head_dim;
  w.max_splits = (max_seq_len + kAttnTile - 1) / kAttnTile;
  size_t off = 0;
  w.x = off; off = align256(off + sizeof(__half) * B * m.hidden);
  w.x1 = off; off = align256(off + sizeof(__half) * B * m.hidden);
  w.qkv = off; off = align256(off + sizeof(__half) * B * qkv_rows);
  w.attn = off; off = align256(off + sizeof(__half) * B * q_dim);
  w.a = off; off = align256(off + sizeof(__half) * B * m.intermediate);
  w.part_o = off; off = align256(off + sizeof(float) * B * m.n_q_heads * w.max_splits * m.head_dim);
  w.part_ml = off; off = align256(off + sizeof(float2) * B * m.n_q_heads * w.max_splits);
  w.att_cnt = off; off = align256(off + sizeof(uint32_t) * B * m.n_kv_heads);
  w.keys = off; off = align256(off + sizeof(unsigned long long) * 2 * B);
  w.arrive = off; off = align256(off + sizeof(uint32_t));
  w.total = off;
  return w;
}

static int act_bytes_for(const lmps_model_desc& m, int nb) {
  size_t a = sizeof(AttnSmemP);
  const size_t stage = static_cast<size_t>(nb) * (m.intermediate > m.hidden ? m.intermediate : m.hidden) * 2;
  if (stage > a) a = stage;
  return static_cast<int>((a + 127) & ~static_cast<size_t>(127));
}

template <int NB>
static int launch(const Params& P0, const lmps_model_desc& m, cudaStream_t st) {
  Params P = P0;
  int dev = 0, sms = 0, max_smem = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  P.act_bytes = act_bytes_for(m, NB);
  int slots = (max_smem - P.act_bytes - kTailBytes) / kSlotBytes;
  if (slots > 16) slots = 16;
  if (slots < 3) return LMPS_ERR_UNSUPPORTED;
  P.slots = slots;
  const size_t smem = static_cast<size_t>(slots) * kSlotBytes + P.act_bytes + kTailBytes;
  auto kern = decode_persistent_kernel<NB>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return static_cast<int>(e);
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (per_sm < 1) return LMPS_ERR_UNSUPPORTED;
  void* args[] = {&P};
  e = cudaLaunchCooperativeKernel(reinterpret_cast<void*>(kern), dim3(sms), dim3(kThreads), args, smem, st);
  return e == cudaSuccess ? LMPS_OK : static_cast<int>(e);
}

}  // namespace pk
}  // namespace lmps

using namespace lmps;

extern "C" size_t lmps_decode_persistent_workspace_size(const lmps_model_desc* model, int batch,
                                                        int max_seq_len) {
  if (!model || batch <= 0 || max_seq_len <= 0) return 0;
  return pk::ws_layout(*model, batch, max_seq_len).total;
}

extern "C" int lmps_decode_persistent(const lmps_model_desc* model, const lmps_decode_state* state,
                                      int n_steps, void* stream) {
  LMPS_CHECK_ARG(model && state && n_steps >= 1);
  const lmps_model_desc& m = *model;
  const lmps_decode_state& s = *state;
  LMPS_CHECK_ARG(m.layers && m.final_norm && m.lm_packed && m.lm_scales && m.embed && m.inv_freq);
  LMPS_CHECK_ARG(m.n_layers >= 1 && m.n_kv_heads >= 1 && m.n_q_heads % m.n_kv_heads == 0);
  if (m.head_dim != pk::kHD || m.n_q_heads / m.n_kv_heads > pk::kMaxG) return LMPS_ERR_UNSUPPORTED;
  if (m.hidden % 512 != 0 || m.hidden > 2048 || m.intermediate % 256 != 0 ||
      m.n_q_heads * m.head_dim != m.hidden)
    return LMPS_ERR_UNSUPPORTED;
  // ring chunks must fit a slot
  if (static_cast<size_t>(pk::kRows1536) * (m.hidden / 2 + m.hidden / 16) > pk::kSlotBytes ||
      static_cast<size_t>(pk::kRowsDown) * (m.intermediate / 2 + m.intermediate / 16) > pk::kSlotBytes)
    return LMPS_ERR_UNSUPPORTED;
  LMPS_CHECK_ARG(s.batch >= 1 && s.batch <= pk::kMaxB);
  LMPS_CHECK_ARG(s.block_table && s.tokens && s.pos && s.workspace && s.error);
  LMPS_CHECK_ARG(s.page_size > 0 && s.max_pages > 0 && s.max_seq_len > 0 &&
                 s.max_seq_len <= s.max_pages * s.page_size);
  LMPS_CHECK_ARG(!s.forced || s.forced_stride >= s.n_forced);
  LMPS_CHECK_ARG(!s.history || (s.step_counter && s.history_rows > 0));
  const pk::WsLayout w = pk::ws_layout(m, s.batch, s.max_seq_len);
  if (s.workspace_bytes < w.total) return LMPS_ERR_WORKSPACE;
  LMPS_CHECK_ARG(lmps_aligned(s.workspace, 256) && lmps_aligned(m.lm_packed, 16));
  pk::Params P{};
  P.m = m;
  P.s = s;
  P.n_steps = n_steps;
  char* ws = reinterpret_cast<char*>(s.workspace);
  P.x = reinterpret_cast<__half*>(ws + w.x);
  P.x1 = reinterpret_cast<__half*>(ws + w.x1);
  P.qkv = reinterpret_cast<__half*>(ws + w.qkv);
  P.attn = reinterpret_cast<__half*>(ws + w.attn);
  P.a = reinterpret_cast<__half*>(ws + w.a);
  P.part_o = reinterpret_cast<float*>(ws + w.part_o);
  P.part_ml = reinterpret_cast<float2*>(ws + w.part_ml);
  P.att_cnt = reinterpret_cast<uint32_t*>(ws + w.att_cnt);
  P.keys = reinterpret_cast<unsigned long long*>(ws + w.keys);
  P.arrive = reinterpret_cast<uint32_t*>(ws + w.arrive);
  P.max_splits = w.max_splits;
  cudaStream_t st = lmps_stream(stream);
  switch (s.batch) {
    case 1: return pk::launch<1>(P, m, st);
    case 2: return pk::launch<2>(P, m, st);
    default: return pk::launch<4>(P, m, st);
  }
}
