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

constexpr int kConsumerWarps = 11;   // + 1 producer warp = 12 warps (registers are allocated per 4 warps)
constexpr int kConsumers = kConsumerWarps * kWarp;        // 352
constexpr int kThreads = kConsumers + kWarp;              // + producer warp
constexpr int kSlotBytes = 20160;
constexpr int kRows1536 = 2 * kConsumerWarps;  // rows per ring chunk when k = hidden
constexpr int kPairsGU = kConsumerWarps;    // gate/up row pairs per chunk
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
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }

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
  float* inv_freq;   // [head_dim/2] RoPE frequencies, staged once per launch
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

// Optional timeline: one %globaltimer stamp per event and row (see the header).
__device__ __forceinline__ void trace_event(const Params& P, int row, int& ev,
                                            unsigned long long wait_ns = ~0ull) {
  if (P.s.trace) {
    if (ev < P.s.trace_events) {
      P.s.trace[static_cast<size_t>(row) * P.s.trace_events + ev] = globaltimer();
      if (wait_ns != ~0ull)   // consumer rows: cumulative ring wait in rows [2*grid, 3*grid)
        P.s.trace[(static_cast<size_t>(row) + 2 * gridDim.x) * P.s.trace_events + ev] = wait_ns;
    }
    ++ev;
  }
}

// ---------------------------------------------------------------------------
// Producer: one lane streams every chunk of every stage into the ring.
// ---------------------------------------------------------------------------
__device__ void producer(const Params& P, Smem& S) {
  const uint64_t policy = evict_first_policy();
  uint32_t chunk = 0;
  bool ok = true;
  int pev = 0;
  const int kinds[4] = {ST_QKV, ST_O, ST_GU, ST_DN};
  for (int step = 0; step < P.n_steps && ok; ++step) {
    for (int l = 0; l <= P.m.n_layers && ok; ++l) {
      const int nk = (l < P.m.n_layers) ? 4 : 1;
      for (int ki = 0; ki < nk && ok; ++ki) {
        const int kind = (l < P.m.n_layers) ? kinds[ki] : ST_HEAD;
        const Chunking c = stage_chunks(P, kind, l);
        const size_t row_bytes = static_cast<size_t>(c.k) / 2;
        const size_t row_scales = static_cast<size_t>(c.k) / 32;
        trace_event(P, gridDim.x + blockIdx.x, pev);
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
        trace_event(P, gridDim.x + blockIdx.x, pev);
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
  unsigned long long wait_ns;  // time thread 0 spent waiting for ring chunks (timeline only)
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
  if (mbar_try_wait(&S.full[slot], phase)) return;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(&S.full[slot], phase)) {
    if (*abort_flag) return;
    if (globaltimer() - t0 > kTimeoutNs) {
      atomicExch(P.s.error, 1);
      *abort_flag = 1;
      return;
    }
  }
  if (P.s.trace && threadIdx.x == 0) cs.wait_ns += globaltimer() - t0;
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

// ---------------------------------------------------------------------------
// Activation planes.  A staged activation vector (RMSNorm'd x, attention
// output, SwiGLU output) is kept per 32-element group -- the Q4 group of the
// weights it meets -- as a 16-bit block fixed point X = rint(x * 2^(15-e)),
// with e the smallest exponent such that every |x| of the group is < 2^e,
// split into a signed high byte H and an unsigned low byte L (X = 256 H + L).
// With the weight nibbles n (0..15) as bytes, dp4a gives the group's dot
// product exactly in integers:
//     sum_k (n_k - 8) X_k = 256 * sum n H + sum n L - 8 * sum X,
// and the fp32 accumulation across groups applies scale * 2^(e-15) once per
// group.  The only rounding is x -> X (below 2^-15 of the group's largest
// |x|).  Word layout of one group: He[4] Ho[4] Le[4] Lo[4]; word c of He holds
// H of elements 8c, 8c+2, 8c+4, 8c+6 (the low nibbles of packed bytes
// 4c..4c+3), Ho the odd elements 8c+1, 8c+3, 8c+5, 8c+7.
// ---------------------------------------------------------------------------
struct Planes {
  uint32_t* w;  // [NB][G][16]
  float* scl;   // [NB][G]   2^(e-15)
  int* xs8;     // [NB][G]   8 * sum X
  int G;
};

__device__ __forceinline__ Planes planes_view(Smem& S, int G, int nb) {
  Planes pl;
  pl.w = reinterpret_cast<uint32_t*>(S.act);
  pl.scl = reinterpret_cast<float*>(pl.w + static_cast<size_t>(nb) * G * 16);
  pl.xs8 = reinterpret_cast<int*>(pl.scl + nb * G);
  pl.G = G;
  return pl;
}

// Convert the 8 values v (elements 8c..8c+7 of group g, c = lane & 3; the 4
// lanes of a group are consecutive) into their plane words.  Every lane of the
// warp must call this (shuffles); `active` marks lanes holding real data.
__device__ __forceinline__ void store_planes(const float (&v)[8], bool active, const Planes& pl,
                                             int b, int g) {
  float mx = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(v[e]));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  // frexp exponent: mx = f * 2^e, f in [0.5, 1); e = 0 for mx == 0
  const int ebits = (__float_as_int(mx) >> 23) & 0xFF;
  const int e = (mx > 0.0f) ? ebits - 126 : 0;
  const float q = __int_as_float((127 + 15 - e) << 23);   // 2^(15-e)
  int X[8], sx = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int xi = __float2int_rn(v[i] * q);
    xi = max(-32768, min(32767, xi));
    X[i] = xi;
    sx += xi;
  }
  sx += __shfl_xor_sync(0xffffffffu, sx, 1);
  sx += __shfl_xor_sync(0xffffffffu, sx, 2);
  if (active) {
    uint32_t he = 0, ho = 0, le = 0, lo = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      he |= (static_cast<uint32_t>(X[2 * k] >> 8) & 0xFFu) << (8 * k);
      ho |= (static_cast<uint32_t>(X[2 * k + 1] >> 8) & 0xFFu) << (8 * k);
      le |= (static_cast<uint32_t>(X[2 * k]) & 0xFFu) << (8 * k);
      lo |= (static_cast<uint32_t>(X[2 * k + 1]) & 0xFFu) << (8 * k);
    }
    const int c = threadIdx.x & 3;
    const int sw = (g >> 1) & 3;  // quad swizzle, see load_xgroup
    uint32_t* gw = pl.w + (static_cast<size_t>(b) * pl.G + g) * 16;
    gw[4 * (0 ^ sw) + c] = he;
    gw[4 * (1 ^ sw) + c] = ho;
    gw[4 * (2 ^ sw) + c] = le;
    gw[4 * (3 ^ sw) + c] = lo;
    if (c == 0) {
      pl.scl[b * pl.G + g] = __int_as_float((127 + e - 15) << 23);  // 2^(e-15)
      pl.xs8[b * pl.G + g] = 8 * sx;
    }
  }
}

// Planes of fp16(fp16(x*scale) * gamma), x = rows[b] -- rms_norm.metal:20-39
// over the full vector (k <= 4096).
template <int NB>
__device__ void stage_norm(const Params& P, Smem& S, const __half* const* rows, bool rows_nc,
                           const __half* gamma, int k) {
  const int vpr = k / 8;
  const Planes pl = planes_view(S, k / 32, NB);
  constexpr int kMaxV = 1;  // vpr <= 512 chunks
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
      const bool active = c < vpr;
      float nv[8];
      uint4 gv = make_uint4(0u, 0u, 0u, 0u);
      if (active) gv = __ldg(reinterpret_cast<const uint4*>(gamma) + c);
      const __half* xh = reinterpret_cast<const __half*>(&v[i]);
      const __half* gh = reinterpret_cast<const __half*>(&gv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const __half nrm = __float2half_rn(__half2float(xh[e]) * scale);
        nv[e] = __half2float(__float2half_rn(__half2float(nrm) * __half2float(gh[e])));
      }
      store_planes(nv, active, pl, b, c >> 2);
    }
  }
  consumer_sync();
}

// Planes of src[b] (k fp16 elements, row stride ld) for every sequence.
template <int NB>
__device__ void stage_copy(const Params& P, Smem& S, const __half* src, int ld, int k) {
  const int vpr = k / 8;
  const Planes pl = planes_view(S, k / 32, NB);
  const int total = NB * vpr;
  const int rounds = (total + kConsumers - 1) / kConsumers;
  constexpr int kBatch = 4;  // loads in flight per thread
  for (int r0 = 0; r0 < rounds; r0 += kBatch) {
    uint4 v[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int i = threadIdx.x + (r0 + k) * kConsumers;
      const int b = i / vpr, c = i - b * vpr;
      v[k] = make_uint4(0u, 0u, 0u, 0u);
      if (r0 + k < rounds && i < total && b < P.s.batch)
        v[k] = __ldcg(reinterpret_cast<const uint4*>(src + static_cast<size_t>(b) * ld) + c);
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      if (r0 + k < rounds) {  // uniform across the CTA
        const int i = threadIdx.x + (r0 + k) * kConsumers;
        const int b = i / vpr, c = i - b * vpr;
        const bool active = i < total && b < P.s.batch;
        const __half* h = reinterpret_cast<const __half*>(&v[k]);
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = __half2float(h[e]);
        store_planes(f, active, pl, active ? b : 0, c >> 2);
      }
    }
  }
  consumer_sync();
}

__device__ __forceinline__ void dp4a_us(int& acc, uint32_t a, uint32_t b) {
  asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(a), "r"(b));
}
__device__ __forceinline__ void dp4a_uu(uint32_t& acc, uint32_t a, uint32_t b) {
  asm("dp4a.u32.u32 %0, %1, %2, %0;" : "+r"(acc) : "r"(a), "r"(b));
}

// Exact sum_k (n_k - 8) X_k of one group: wv = 16 packed bytes, x = plane words.
__device__ __forceinline__ int group_idot(const uint4& wv, const uint32_t (&x)[16], int xs8) {
  int sh = 0;
  uint32_t sl = 0u;
  const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t ne = ws[c] & 0x0F0F0F0Fu, no = (ws[c] >> 4) & 0x0F0F0F0Fu;
    dp4a_us(sh, ne, x[c]);
    dp4a_us(sh, no, x[4 + c]);
    dp4a_uu(sl, ne, x[8 + c]);
    dp4a_uu(sl, no, x[12 + c]);
  }
  return sh * 256 + static_cast<int>(sl) - xs8;
}

struct XGroup {
  uint32_t w[16];
  float scl;
  int xs8;
};

// A group's four 16-byte quads (He, Ho, Le, Lo) are stored in the order
// q ^ ((g >> 1) & 3): lanes reading the same quad of 8 consecutive groups then
// touch 8 different 16-byte bank groups (one wavefront) instead of two.
__device__ __forceinline__ void load_xgroup(const Planes& pl, int b, int g, XGroup& x) {
  const uint4* src = reinterpret_cast<const uint4*>(pl.w + (static_cast<size_t>(b) * pl.G + g) * 16);
  const int sw = (g >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 v = src[q ^ sw];
    x.w[4 * q] = v.x;
    x.w[4 * q + 1] = v.y;
    x.w[4 * q + 2] = v.z;
    x.w[4 * q + 3] = v.w;
  }
  x.scl = pl.scl[b * pl.G + g];
  x.xs8 = pl.xs8[b * pl.G + g];
}

constexpr int kMaxJ = 4;  // groups per lane: G / 16 <= 3 (hidden <= 1536); down: ceil(G / warps / 8) <= 4

// ---------------------------------------------------------------------------
// GEMV stages over ring chunks
// ---------------------------------------------------------------------------
// k = hidden stages (QKV, O, HEAD): chunk of <= 2*warps rows; warp w owns
// rows 2w (lanes 0-15) and 2w+1 (lanes 16-31); lane sub takes groups sub,
// sub+16, sub+32 of its row (weights and activation planes from shared memory).
template <int NB, int KIND>
__device__ void gemv_hidden(const Params& P, Smem& S, CState& cs, const Chunking& c,
                            const __half* bias, const __half* const* res_rows, __half* out, int ldo,
                            unsigned long long* best) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = c.k / 32, JG = G / 16;
  const int sub = lane & 15;
  const Planes pl = planes_view(S, G, NB);
  for (int r = c.r0; r < c.r1; r += c.rows_per_chunk) {
    const int n = min(c.rows_per_chunk, c.r1 - r);
    int slot;
    slot_wait(S, P, cs, slot);
    const unsigned char* base = S.ring + static_cast<size_t>(slot) * kSlotBytes;
    const int lrow = 2 * warp + (lane >> 4);
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
    if (lrow < n) {
      const unsigned char* wrow = base + static_cast<size_t>(lrow) * (c.k / 2);
      const __half* srow = reinterpret_cast<const __half*>(base + static_cast<size_t>(n) * (c.k / 2)) + lrow * G;
      uint4 wv[kMaxJ];
      float sc[kMaxJ];
#pragma unroll
      for (int j = 0; j < kMaxJ; ++j) {
        if (j < JG) {
          wv[j] = *reinterpret_cast<const uint4*>(wrow + (sub + 16 * j) * 16);
          sc[j] = __half2float(srow[sub + 16 * j]);
        }
      }
#pragma unroll
      for (int j = 0; j < kMaxJ; ++j) {
        if (j < JG) {
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            XGroup xg;
            load_xgroup(pl, b, sub + 16 * j, xg);
            acc[b] = fmaf(sc[j] * xg.scl, static_cast<float>(group_idot(wv[j], xg.w, xg.xs8)), acc[b]);
          }
        }
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

// Gate/up: chunk of <= 16 row pairs; warp w: gate row w on lanes 0-15, up row
// w on lanes 16-31; lane 0 applies SwiGLU (swiglu.metal:19-22).
template <int NB>
__device__ void gemv_gateup(const Params& P, Smem& S, CState& cs, const Chunking& c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = c.k / 32, JG = G / 16;
  const int up = lane >> 4, sub = lane & 15;
  const int inter = P.m.intermediate;
  const Planes pl = planes_view(S, G, NB);
  for (int r = c.r0; r < c.r1; r += c.rows_per_chunk) {
    const int n = min(c.rows_per_chunk, c.r1 - r);
    int slot;
    slot_wait(S, P, cs, slot);
    const unsigned char* base = S.ring + static_cast<size_t>(slot) * kSlotBytes;
    const size_t pbytes = static_cast<size_t>(n) * (c.k / 2);
    const size_t sbytes = static_cast<size_t>(n) * G * 2;
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
    if (warp < n) {
      const unsigned char* wrow = base + up * pbytes + static_cast<size_t>(warp) * (c.k / 2);
      const __half* srow = reinterpret_cast<const __half*>(base + 2 * pbytes + up * sbytes) + warp * G;
      uint4 wv[kMaxJ];
      float sc[kMaxJ];
#pragma unroll
      for (int j = 0; j < kMaxJ; ++j) {
        if (j < JG) {
          wv[j] = *reinterpret_cast<const uint4*>(wrow + (sub + 16 * j) * 16);
          sc[j] = __half2float(srow[sub + 16 * j]);
        }
      }
#pragma unroll
      for (int j = 0; j < kMaxJ; ++j) {
        if (j < JG) {
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            XGroup xg;
            load_xgroup(pl, b, sub + 16 * j, xg);
            acc[b] = fmaf(sc[j] * xg.scl, static_cast<float>(group_idot(wv[j], xg.w, xg.xs8)), acc[b]);
          }
        }
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
// [G*w/16, G*(w+1)/16) of every row (lane = row*8 + sub, groups g0+sub+8j),
// partials meet in shared memory and one thread per row finishes:
// x = x1 + fp16(acc).
template <int NB>
__device__ void gemv_down(const Params& P, Smem& S, CState& cs, const Chunking& c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = c.k / 32;
  const int g0 = G * warp / kConsumerWarps, g1 = G * (warp + 1) / kConsumerWarps;
  const int lrow = lane >> 3, sub = lane & 7;
  const int hidden = P.m.hidden;
  const Planes pl = planes_view(S, G, NB);
  int par = 0;
  for (int r = c.r0; r < c.r1; r += c.rows_per_chunk, par ^= 1) {
    const int n = min(c.rows_per_chunk, c.r1 - r);
    int slot;
    slot_wait(S, P, cs, slot);
    const unsigned char* base = S.ring + static_cast<size_t>(slot) * kSlotBytes;
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
    if (lrow < n) {
      const unsigned char* wrow = base + static_cast<size_t>(lrow) * (c.k / 2);
      const __half* srow = reinterpret_cast<const __half*>(base + static_cast<size_t>(n) * (c.k / 2)) + lrow * G;
#pragma unroll
      for (int j = 0; j < kMaxJ; ++j) {
        const int g = g0 + sub + 8 * j;
        if (g < g1) {
          const uint4 wv = *reinterpret_cast<const uint4*>(wrow + g * 16);
          const float sc = __half2float(srow[g]);
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            XGroup xg;
            load_xgroup(pl, b, g, xg);
            acc[b] = fmaf(sc * xg.scl, static_cast<float>(group_idot(wv, xg.w, xg.xs8)), acc[b]);
          }
        }
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

// Attention sub-phase stamps of CTA 0 (timeline row 3*grid, when allocated).
__device__ __forceinline__ void attn_stamp(const Params& P, int& aev) {
  if (P.s.trace && P.s.trace_rows > 3 * static_cast<int>(gridDim.x) && blockIdx.x == 0 && threadIdx.x == 0) {
    if (aev < P.s.trace_events)
      P.s.trace[static_cast<size_t>(3 * gridDim.x) * P.s.trace_events + aev] = globaltimer();
    ++aev;
  }
}

// ---------------------------------------------------------------------------
// Attention stage: one work item = (sequence b, kv head, split of positions)
// ---------------------------------------------------------------------------
// Decode-attention tiles go through the tensor cores with mma.sync m16n8k16
// (fp16 in, fp32 accumulate): the G query heads of a KV head are the M rows
// (padded to 16), positions are N for the scores and K for P.V.  At decode
// these tiles are tiny and latency-bound; the MMAs replace 128-long dependent
// FMA chains per (position, head).
struct AttnSmemP {
  __half qh[16][kKStride];            // rotated q (fp16); rows >= G are zero
  __half knew[kHD];                   // this step's rotated k / raw v (position pos)
  __half vnew[kHD];
  __half k[kAttnTile][kKStride];
  __half v[kAttnTile][kKStride];
  float p[kMaxG][kAttnTile];          // scores
  __half ph[16][kAttnTile + 8];       // exp(scores - max) in fp16; rows >= G are zero
  float m[kMaxG];
  float l[kMaxG];
  float alpha[kMaxG];
  int is_last;
};

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(const void* p, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2_trans(const void* p, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

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
                          int split, int n_splits, int chunk, int pos, int& aev) {
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

  // K/V rows of one 64-position tile, loaded straight into registers so the
  // loads of the first tile overlap the q/k/v loads and RoPE below.  The new
  // position `pos` is not read from the cache: it comes from A.knew/A.vnew.
  constexpr int kTileVec = kAttnTile * (kHD / 8);                       // 16-byte chunks per tile
  constexpr int kLd = (kTileVec + kConsumers - 1) / kConsumers;
  uint4 kreg[kLd], vreg[kLd];
  auto load_tile = [&](int t0) {
    const int n = min(kAttnTile, end - t0);
#pragma unroll
    for (int it = 0; it < kLd; ++it) {
      const int i = tid + it * kConsumers;
      const int r = i / (kHD / 8), c = i - r * (kHD / 8);
      kreg[it] = make_uint4(0u, 0u, 0u, 0u);
      vreg[it] = make_uint4(0u, 0u, 0u, 0u);
      const int p = t0 + r;
      if (i < kTileVec && r < n && p != pos) {
        const size_t off = ((static_cast<size_t>(bt[p / ps]) * Hkv + kvh) * ps + p % ps) * kHD + c * 8;
        kreg[it] = __ldcg(reinterpret_cast<const uint4*>(kpool + off));
        vreg[it] = __ldcg(reinterpret_cast<const uint4*>(vpool + off));
      }
    }
  };
  auto store_tile = [&](int t0) {
#pragma unroll
    for (int it = 0; it < kLd; ++it) {
      const int i = tid + it * kConsumers;
      if (i < kTileVec) {
        const int r = i / (kHD / 8), c = i - r * (kHD / 8);
        uint4 kv = kreg[it], vv = vreg[it];
        if (t0 + r == pos) {
          kv = *reinterpret_cast<const uint4*>(&A.knew[c * 8]);
          vv = *reinterpret_cast<const uint4*>(&A.vnew[c * 8]);
        }
        *reinterpret_cast<uint4*>(&A.k[r][c * 8]) = kv;
        *reinterpret_cast<uint4*>(&A.v[r][c * 8]) = vv;
      }
    }
  };
  attn_stamp(P, aev);
  // Every global load of the prologue is issued before any of them is used:
  // the first K/V tile, this group's q pairs, the new k pair and v element.
  if (start < end) load_tile(start);
  constexpr int kQ = (kMaxG * (kHD / 2) + kConsumers - 1) / kConsumers;
  float qa[kQ], qb[kQ];
#pragma unroll
  for (int it = 0; it < kQ; ++it) {
    const int i = tid + it * kConsumers;
    qa[it] = qb[it] = 0.0f;
    if (i < G * (kHD / 2)) {
      const int h = i / (kHD / 2), j = i - h * (kHD / 2);
      int i1, i2;
      rope_pair(j, m.rope_style, i1, i2);
      const __half* qh = row + (kvh * G + h) * kHD;
      qa[it] = __half2float(__ldcg(qh + i1));
      qb[it] = __half2float(__ldcg(qh + i2));
    }
  }
  const bool has_pos = pos >= start && pos < end;
  const __half* kh = row + (Hq + kvh) * kHD;
  const __half* vh = row + (Hq + Hkv + kvh) * kHD;
  float ka = 0.0f, kb = 0.0f;
  __half vnew = __float2half_rn(0.0f);
  int ki1 = 0, ki2 = 0;
  if (has_pos) {
    if (tid < kHD / 2) {
      rope_pair(tid, m.rope_style, ki1, ki2);
      ka = __half2float(__ldcg(kh + ki1));
      kb = __half2float(__ldcg(kh + ki2));
    } else if (tid < kHD / 2 + kHD) {
      vnew = __ldcg(vh + (tid - kHD / 2));
    }
  }
  // RoPE'd q of the G heads sharing this KV head (rope.metal:19-40), fp16-rounded.
#pragma unroll
  for (int it = 0; it < kQ; ++it) {
    const int i = tid + it * kConsumers;
    if (i < G * (kHD / 2)) {
      const int h = i / (kHD / 2), j = i - h * (kHD / 2);
      int i1, i2;
      rope_pair(j, m.rope_style, i1, i2);
      float sn, cs;
      sincosf(fpos * S.inv_freq[j], &sn, &cs);
      A.qh[h][i1] = __float2half_rn(qa[it] * cs - qb[it] * sn);
      A.qh[h][i2] = __float2half_rn(qa[it] * sn + qb[it] * cs);
    }
  }
  // The split holding the new position appends its rotated k and raw v.
  if (has_pos) {
    const int page = bt[pos / ps], off = pos % ps;
    const size_t base = ((static_cast<size_t>(page) * Hkv + kvh) * ps + off) * kHD;
    if (tid < kHD / 2) {
      float sn, cs;
      sincosf(fpos * S.inv_freq[tid], &sn, &cs);
      const __half k1 = __float2half_rn(ka * cs - kb * sn), k2 = __float2half_rn(ka * sn + kb * cs);
      kpool[base + ki1] = k1;
      kpool[base + ki2] = k2;
      A.knew[ki1] = k1;
      A.knew[ki2] = k2;
    } else if (tid < kHD / 2 + kHD) {
      const int d = tid - kHD / 2;
      vpool[base + d] = vnew;
      A.vnew[d] = vnew;
    }
  }
  if (tid < kMaxG) {
    A.m[tid] = -INFINITY;
    A.l[tid] = 0.0f;
  }
  for (int i = tid; i < (16 - G) * kKStride; i += kConsumers)
    A.qh[G + i / kKStride][i % kKStride] = __float2half_rn(0.0f);
  for (int i = tid; i < (16 - G) * (kAttnTile + 8); i += kConsumers)
    A.ph[G + i / (kAttnTile + 8)][i % (kAttnTile + 8)] = __float2half_rn(0.0f);
  constexpr int kHPT = (kMaxG + kConsumers / kHD - 1) / (kConsumers / kHD);   // heads per combine thread
  const int warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;           // mma fragment row / column pair
  const int mi = lane >> 3, r8 = lane & 7;           // ldmatrix lane -> matrix, row
  constexpr int kNT = kHD / 8;                       // P.V output n-tiles (8 dims each)
  constexpr int kNTW = (kNT + kConsumerWarps - 1) / kConsumerWarps;
  float o[kNTW][4];
#pragma unroll
  for (int j = 0; j < kNTW; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  consumer_sync();
  attn_stamp(P, aev);

  for (int t0 = start; t0 < end; t0 += kAttnTile) {
    const int n = min(kAttnTile, end - t0);
    if (t0 != start) load_tile(t0);
    store_tile(t0);
    consumer_sync();
    attn_stamp(P, aev);
    // scores S = Q K^T * 0.088388 (attention.metal:32-40): warp w < 8 owns
    // positions 8w..8w+7, eight k-steps over the 128 dims.
    if (warp < kAttnTile / 8) {
      float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int ks = 0; ks < kHD / 16; ++ks) {
        uint32_t a0, a1, a2, a3, b0, b1;
        ldsm_x4(&A.qh[(mi & 1) * 8 + r8][16 * ks + (mi >> 1) * 8], a0, a1, a2, a3);
        ldsm_x2(&A.k[8 * warp + r8][16 * ks + (mi & 1) * 8], b0, b1);
        mma_16816(d, a0, a1, a2, a3, b0, b1);
      }
      if (g8 < G) {
        const int p0 = 8 * warp + 2 * t4;
        A.p[g8][p0] = (p0 < n) ? d[0] * kAttnScale : -INFINITY;
        A.p[g8][p0 + 1] = (p0 + 1 < n) ? d[1] * kAttnScale : -INFINITY;
      }
    }
    consumer_sync();
    attn_stamp(P, aev);
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
        A.ph[h][lane] = __float2half_rn(e0);
        A.ph[h][lane + 32] = __float2half_rn(e1);
        __syncwarp();
        if (lane == 0) {
          A.alpha[h] = alpha;
          A.m[h] = m_new;
          A.l[h] = A.l[h] * alpha + sum;
        }
      }
    }
    consumer_sync();
    attn_stamp(P, aev);
    // O += P V (attn_sum.metal:26-32): warp w owns output dims 8nt..8nt+7 for
    // nt = w, w + warps; the running sums are rescaled by this tile's alpha.
    {
      const float al0 = (g8 < G) ? A.alpha[g8] : 1.0f;
#pragma unroll
      for (int j = 0; j < kNTW; ++j) {
        o[j][0] *= al0;
        o[j][1] *= al0;
      }
#pragma unroll
      for (int ks = 0; ks < kAttnTile / 16; ++ks) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(&A.ph[(mi & 1) * 8 + r8][16 * ks + (mi >> 1) * 8], a0, a1, a2, a3);
#pragma unroll
        for (int j = 0; j < kNTW; ++j) {
          const int nt = warp + kConsumerWarps * j;
          if (nt < kNT) {
            uint32_t b0, b1;
            ldsm_x2_trans(&A.v[16 * ks + (mi & 1) * 8 + r8][8 * nt], b0, b1);
            mma_16816(o[j], a0, a1, a2, a3, b0, b1);
          }
        }
      }
    }
    consumer_sync();
    attn_stamp(P, aev);
  }

  if (n_splits == 1) {
    if (g8 < G) {
      const float l = A.l[g8];
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
      for (int j = 0; j < kNTW; ++j) {
        const int nt = warp + kConsumerWarps * j;
        if (nt < kNT) {
          __half* dst = P.attn + static_cast<size_t>(b) * Hq * kHD + (kvh * G + g8) * kHD + 8 * nt + 2 * t4;
          dst[0] = __float2half_rn(o[j][0] * inv);
          dst[1] = __float2half_rn(o[j][1] * inv);
        }
      }
    }
    consumer_sync();
    return;
  }
  const size_t ms = P.max_splits;
  if (g8 < G) {
    const size_t prow = (static_cast<size_t>(b) * Hq + kvh * G + g8) * ms + split;
#pragma unroll
    for (int j = 0; j < kNTW; ++j) {
      const int nt = warp + kConsumerWarps * j;
      if (nt < kNT) {
        P.part_o[prow * kHD + 8 * nt + 2 * t4] = o[j][0];
        P.part_o[prow * kHD + 8 * nt + 2 * t4 + 1] = o[j][1];
      }
    }
  }
  if (tid < G) {
    const size_t prow = (static_cast<size_t>(b) * Hq + kvh * G + tid) * ms + split;
    P.part_ml[prow] = make_float2(A.m[tid], A.l[tid]);
  }
  const int d = tid & (kHD - 1), hh = (tid < (kConsumers / kHD) * kHD) ? tid / kHD : kMaxG;
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
    for (int j = 0; j < kHPT; ++j) {
      const int h = hh + (kConsumers / kHD) * j;
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
  CState cs{0u, 0u, true, 0ull};
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
  int ev = 0, aev = 0;
  const bool tr = threadIdx.x == 0;

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
      if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
      stage_norm<NB>(P, S, l == 0 ? xin : xres, l == 0, reinterpret_cast<const __half*>(L.in_norm), hidden);
      {
        const Chunking c = stage_chunks(P, ST_QKV, l);
        gemv_hidden<NB, ST_QKV>(P, S, cs, c, reinterpret_cast<const __half*>(L.qkv_bias), nullptr, P.qkv,
                                qkv_rows, nullptr);
      }
      if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
      grid_arrive(P, cs);
      // ---- ATT
      if (!grid_wait(P, S, cs)) return;
      if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
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
          attn_item(P, S, L, bsel, kvh, sp, nsp, chunk, pb, aev);
        }
      }
      if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
      grid_arrive(P, cs);
      // ---- O
      if (!grid_wait(P, S, cs)) return;
      if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
      stage_copy<NB>(P, S, P.attn, q_dim, q_dim);
      {
        const Chunking c = stage_chunks(P, ST_O, l);
        gemv_hidden<NB, ST_O>(P, S, cs, c, nullptr, l == 0 ? xin : xres, P.x1, hidden, nullptr);
      }
      if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
      grid_arrive(P, cs);
      // ---- GU
      if (!grid_wait(P, S, cs)) return;
      if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
      stage_norm<NB>(P, S, x1rows, false, reinterpret_cast<const __half*>(L.post_norm), hidden);
      {
        const Chunking c = stage_chunks(P, ST_GU, l);
        gemv_gateup<NB>(P, S, cs, c);
      }
      if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
      grid_arrive(P, cs);
      // ---- DN
      if (!grid_wait(P, S, cs)) return;
      if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
      stage_copy<NB>(P, S, P.a, m.intermediate, m.intermediate);
      {
        const Chunking c = stage_chunks(P, ST_DN, l);
        gemv_down<NB>(P, S, cs, c);
      }
      if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
      grid_arrive(P, cs);
    }
    // ---- HEAD
    if (!grid_wait(P, S, cs)) return;
    if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
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
    if (tr) trace_event(P, blockIdx.x, ev, cs.wait_ns);
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
  S.inv_freq = reinterpret_cast<float*>(S.misc + 16);
  for (int i = threadIdx.x; i < kHD / 2; i += blockDim.x) S.inv_freq[i] = P.m.inv_freq[i];
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
  // Counters that persist from one launch to the next come first, at offsets
  // that do not depend on the batch size of the launch.
  w.arrive = off; off = align256(off + sizeof(uint32_t));
  w.keys = off; off = align256(off + sizeof(unsigned long long) * 2 * kMaxB);
  w.att_cnt = off; off = align256(off + sizeof(uint32_t) * kMaxB * m.n_kv_heads);
  w.x = off; off = align256(off + sizeof(__half) * B * m.hidden);
  w.x1 = off; off = align256(off + sizeof(__half) * B * m.hidden);
  w.qkv = off; off = align256(off + sizeof(__half) * B * qkv_rows);
  w.attn = off; off = align256(off + sizeof(__half) * B * q_dim);
  w.a = off; off = align256(off + sizeof(__half) * B * m.intermediate);
  w.part_o = off; off = align256(off + sizeof(float) * B * m.n_q_heads * w.max_splits * m.head_dim);
  w.part_ml = off; off = align256(off + sizeof(float2) * B * m.n_q_heads * w.max_splits);
  w.total = off;
  return w;
}

static int act_bytes_for(const lmps_model_desc& m, int nb) {
  size_t a = sizeof(AttnSmemP);
  const int kmax = m.intermediate > m.hidden ? m.intermediate : m.hidden;
  const size_t planes = static_cast<size_t>(nb) * (kmax / 32) * (16 * 4 + 4 + 4);  // words + scl + xs8
  if (planes > a) a = planes;
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
  auto kern = decode_persistent_kernel<NB>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return static_cast<int>(e);
  // As many ring slots as fit next to one resident CTA per SM.
  int slots = (max_smem - P.act_bytes - kTailBytes) / kSlotBytes;
  if (slots > 16) slots = 16;
  size_t smem = 0;
  for (; slots >= 3; --slots) {
    smem = static_cast<size_t>(slots) * kSlotBytes + P.act_bytes + kTailBytes;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (per_sm >= 1) break;
  }
  if (slots < 3) return LMPS_ERR_UNSUPPORTED;
  P.slots = slots;
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
  // lanes own hidden/512 groups of a row (<= 3) and G_down/16/8 groups of the
  // down projection (<= 3); see gemv_hidden / gemv_down
  if (m.hidden % 512 != 0 || m.hidden > 1536 || m.intermediate % 32 != 0 ||
      (m.intermediate / 32 + pk::kConsumerWarps - 1) / pk::kConsumerWarps > 8 * pk::kMaxJ ||
      m.n_q_heads * m.head_dim != m.hidden)
    return LMPS_ERR_UNSUPPORTED;
  // ring chunks must fit a slot
  if (static_cast<size_t>(pk::kRows1536) * (m.hidden / 2 + m.hidden / 16) > pk::kSlotBytes ||
      static_cast<size_t>(2 * pk::kPairsGU) * (m.hidden / 2 + m.hidden / 16) > pk::kSlotBytes ||
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
