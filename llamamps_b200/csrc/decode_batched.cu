// Batched decode in one cooperative launch: every layer of the model for 5..64
// sequences, the Q4 projections on the 5th-generation tensor cores
// (runners/engine.py:183-245 per layer, for a batch of sequences at once).
//
// The per-stage path spends ~8 us of fixed latency in each of the ~113 GEMM
// launches of a step (prologue, first weight tile landing, split-K
// reduction).  Here one CTA per SM stays resident for the whole step and
// streams the weights of its share of every projection through a ring of
// shared-memory slots that runs ahead across stage boundaries: the weights do
// not depend on the activations, so the loads of the next projection's
// weights and their dequantisation overlap the current stage and the grid
// barrier that ends it.
//
// Per layer, separated by grid barriers (a monotonic counter in the
// workspace; all CTAs are co-resident by the cooperative launch):
//   QKV   tcgen05 GEMM units (128 weight rows x a K range), fp32 partials
//   ATT   split-KV attention items (decode_attention.cuh) fed from the q|k|v
//         partials (+ bias, RoPE); the new K/V row appended to the paged cache
//   [MRG] log-sum-exp merge of the splits (only with more than one split)
//   O     GEMM units -> fp32 partials
//   RED   x += fp16(sum of partials); xn = RMSNorm(x) * post_norm (a CTA per sequence)
//   GU    GEMM units over the interleaved gate/up rows, SwiGLU epilogue -> a
//   DN    GEMM units -> fp32 partials
//   RED   x += fp16(sum); xn = RMSNorm(x) * in_norm of the next layer
// The activations the GEMMs read (xn, the attention output, a) are loaded by
// TMA (128-byte swizzle) after the barrier; the weights come from a
// tile-major copy of the Q4 matrices (lmps_q4_tile_blocks): per 128 rows and
// 64-wide K step one 4608-byte block (packed nibbles, then the group scales),
// fetched with one bulk copy.
//
// Roles of the 192 threads of a CTA (as in the W4A16 GEMM): warp 0 lane 0
// issues the weight and activation loads, warp 1 lane 0 the MMAs
// (A = 128 dequantised weight rows, B = the tokens, N = batch rounded up to
// 16, two TMEM accumulators used alternately), warps 2-5 dequantise, run the
// epilogues and the attention / reduction phases.  Every wait is bounded: a
// timeout sets the error word and a workspace abort flag that every CTA
// polls, and the launch ends without a hang.
#include <cmath>

#include "common.cuh"
#include "decode_attention.cuh"
#include "q4_tile.cuh"
#include "tcgen05.cuh"

namespace lmps {
namespace bd {

using namespace tc;

constexpr int kThreads = 192;
constexpr int kWorkers = 128;                 // warps 2-5
constexpr int kBK = 64;
constexpr int kRows = 128;
constexpr int kBlockBytes = q4t::kBlockBytes; // 4096 packed + 512 scale bytes
constexpr int kMaxNt = 64;                    // tokens per MMA (batch rounded up to 16)
constexpr int kXStages = 4;
constexpr int kDStages = 3;
constexpr int kXSlot = kMaxNt * 128;          // 8 KB: nt rows x 128 bytes, 1024-byte aligned
constexpr int kDSlot = kRows * 128;           // 16 KB dequantised fp16 tile
constexpr int kMaxWSlots = 32;
constexpr int kTmemCols = 2 * kMaxNt;         // two accumulators
constexpr int kMaxLayers = 64;

enum Stage { ST_QKV = 0, ST_O = 1, ST_GU = 2, ST_DN = 3, ST_N = 4 };

struct __align__(64) Params {
  CUtensorMap tx[ST_N];  // activations read by each GEMM stage: xn, attn, xn, a (box {64, nt})
  const lmps_batched_layer* layers;
  int n_layers;
  __half* x;     // residual [B, hidden], in and out
  __half* xn;    // normalised activations [B, hidden]
  __half* attn;  // attention output [B, q_dim]
  __half* a;     // SwiGLU output [B, intermediate]
  float* part[ST_N];  // fp32 split partials of QKV, O, DN: [split][B][rows]
  float* att_o;       // attention split partials
  float2* att_ml;
  unsigned long long* bar;  // grid barrier counter
  int* abort_flag;
  int32_t* error;
  const float* inv_freq;
  const int32_t* pos;
  const int32_t* seq_lens;
  const int32_t* block_table;
  int max_pages, page_size, page_shift, rope_style;
  int B, nt;
  int hidden, inter, n_q, n_kv, qkv_rows;
  float eps;
  int tiles[ST_N], splits[ST_N], ksteps[ST_N];
  int att_splits, att_chunk;
  int wslots;
  unsigned long long* trace;  // optional [grid][barriers][2]: arrival, completion seen (%globaltimer)
  int n_bars;
};

// ---- grid barrier ---------------------------------------------------------
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ bool aborted(const Params& P) {
  return *reinterpret_cast<volatile int*>(P.abort_flag) != 0;
}
__device__ __noinline__ void raise_abort(const Params& P) {
  atomicExch(P.error, 1);
  atomicExch(P.abort_flag, 1);
}
// Bounded wait until the counter reaches `target` (false: aborted / timed out).
__device__ bool counter_wait(const Params& P, unsigned long long target) {
  if (ld_acquire_u64(P.bar) >= target) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_u64(P.bar) < target) {
    if (aborted(P)) return false;
    if (globaltimer() - t0 > kTimeoutNs) {
      raise_abort(P);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void workers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kWorkers) : "memory"); }

// Bounded mbarrier wait that also gives up when another CTA aborted.
__device__ __forceinline__ bool mwait(const Params& P, uint64_t* bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try(bar, parity)) {
    if (aborted(P)) return false;
    if (globaltimer() - t0 > kTimeoutNs) {
      raise_abort(P);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy global -> this CTA's shared memory (no multicast).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

struct RingPos {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int n) {
    if (++slot == n) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// The GEMM unit of CTA c in a stage: weight-row tile and K-step range.
struct Unit {
  bool valid;
  int tile, split, k0, k1;
};
__device__ __forceinline__ Unit unit_of(const Params& P, int s, int c) {
  Unit u{};
  const int ns = P.splits[s];
  u.valid = c < P.tiles[s] * ns;
  if (!u.valid) return u;
  u.tile = c / ns;
  u.split = c - u.tile * ns;
  u.k0 = u.split * P.ksteps[s] / ns;
  u.k1 = (u.split + 1) * P.ksteps[s] / ns;
  return u;
}
__device__ __forceinline__ const unsigned char* stage_blocks(const lmps_batched_layer& L, int s) {
  const void* p = s == ST_QKV ? L.qkv_blocks : s == ST_O ? L.o_blocks : s == ST_GU ? L.gu_blocks : L.down_blocks;
  return static_cast<const unsigned char*>(p);
}

// Barrier indices: 0 after the first norm; layer l's barriers start at
// 1 + l * per_layer, in the order QKV, ATT, [MRG], O, RED, GU, DN, RED.
struct Bars {
  int per_layer, merge;
  __device__ __forceinline__ int first(int l) const { return 1 + l * per_layer; }
  __device__ __forceinline__ int after(int l, int s) const {  // barrier that ends GEMM stage s of layer l
    const int b = first(l);
    return s == ST_QKV ? b : s == ST_O ? b + 2 + merge : s == ST_GU ? b + 4 + merge : b + 5 + merge;
  }
  // barrier whose completion the stage's activation loads wait for
  __device__ __forceinline__ int gate(int l, int s) const {
    const int b = first(l);
    return s == ST_QKV ? b - 1 : s == ST_O ? b + 1 + merge : s == ST_GU ? b + 3 + merge : b + 4 + merge;
  }
};

struct Smem {
  unsigned char* xs;  // [kXStages][kXSlot] activation tiles (128-byte swizzle)
  unsigned char* wd;  // [kDStages][kDSlot] dequantised weight tiles (128-byte swizzle)
  unsigned char* wr;  // [wslots][kBlockBytes] tile-major weight blocks
  uint64_t *fullw, *emptyw, *fullx, *emptyx, *deq, *emptyd, *accf, *acce, *done;
  uint32_t* tmem_slot;
  int* stop;                 // workers' shared stop decision
  unsigned long long* base;  // grid-barrier count at launch start
  float* red;                // [4] per-warp sums
};
constexpr int kFixedSmem = 1024 + kXStages * kXSlot + kDStages * kDSlot + 2048;
static_assert(sizeof(AttnSmem) + (kMaxGroup + 2) * kHeadDim * 2 <= kXStages * kXSlot + kDStages * kDSlot,
              "attention aliases the tile rings");

// Sum over the K splits of a partial value, in split order, with every
// split's load issued before the first add (one L2 round trip, not nsplit).
constexpr int kMaxSplits = 16;
__device__ __forceinline__ float split_sum(const float* p, size_t stride, int nsplit) {
  float v[kMaxSplits];
#pragma unroll
  for (int k = 0; k < kMaxSplits; ++k) v[k] = k < nsplit ? __ldcg(p + k * stride) : 0.0f;
  float s = v[0];
#pragma unroll
  for (int k = 1; k < kMaxSplits; ++k)
    if (k < nsplit) s += v[k];
  return s;
}
__device__ __forceinline__ float4 split_sum4(const float4* p, size_t stride, int nsplit) {
  float4 v[kMaxSplits];
#pragma unroll
  for (int k = 0; k < kMaxSplits; ++k) v[k] = k < nsplit ? __ldcg(p + k * stride) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 s = v[0];
#pragma unroll
  for (int k = 1; k < kMaxSplits; ++k)
    if (k < nsplit) {
      s.x += v[k].x;
      s.y += v[k].y;
      s.z += v[k].z;
      s.w += v[k].w;
    }
  return s;
}

// q|k|v rows of one attention item, staged in shared memory before the item
// runs: value = fp16(sum over the QKV splits (in order) + bias), the W4A16
// GEMM's bias epilogue.  The item's loader reads them back by row index.
struct StagedQkv {
  const __half* vals;  // [(G + 2) * 128]: the G query heads of the KV head, then its k and v rows
  int q0, k0, v0, G;   // row indices where the three runs start; heads per KV head
  __device__ __forceinline__ __half operator()(int, int i) const {
    const int j = i >= v0 ? kHeadDim * (G + 1) + (i - v0) : i >= k0 ? kHeadDim * G + (i - k0) : i - q0;
    return vals[j];
  }
};
struct WorkerSync {
  __device__ __forceinline__ void operator()() const { workers_sync(); }
};

__device__ __forceinline__ __half swiglu_value(float gate, float up) {
  return __float2half_rn(silu_mul(__half2float(__float2half_rn(gate)), __half2float(__float2half_rn(up))));
}

// Walks the CTA's GEMM units in launch order: (layer, stage, K step).
struct Cursor {
  int l = 0, s = 0, k = 0;
  __device__ __forceinline__ void skip(const Unit (&U)[ST_N], int L) {
    while (l < L && !U[s].valid) {
      if (++s == ST_N) {
        s = 0;
        ++l;
      }
    }
    if (l < L) k = U[s].k0;
  }
  __device__ __forceinline__ void next(const Unit (&U)[ST_N], int L) {
    if (++k < U[s].k1) return;
    if (++s == ST_N) {
      s = 0;
      ++l;
    }
    skip(U, L);
  }
};

// ---- warp 0 lane 0: weight blocks run up to wslots steps ahead; the
// activation tiles of a stage wait for the barrier that publishes them.
__device__ void producer(const Params& P, const Smem& S, const Unit (&U)[ST_N], const Bars& bars,
                         unsigned long long bbase) {
  const int R = P.wslots, L = P.n_layers, G = gridDim.x;
  const uint32_t xbytes = static_cast<uint32_t>(P.nt) * 128u;
  Cursor wc, xc;
  wc.skip(U, L);
  xc.skip(U, L);
  RingPos wp, xp;
  int nw = 0, nx = 0;  // copies issued
  int seen = -1;       // highest barrier known complete
  uint64_t t0 = globaltimer();
  while (wc.l < L || xc.l < L) {
    bool progress = false;
    if (wc.l < L) {
      if (mbar_try(&S.emptyw[wp.slot], wp.phase ^ 1u)) {
        const unsigned char* src =
            stage_blocks(P.layers[wc.l], wc.s) +
            (static_cast<size_t>(U[wc.s].tile) * P.ksteps[wc.s] + wc.k) * kBlockBytes;
        mbar_expect_tx(&S.fullw[wp.slot], kBlockBytes);
        bulk_load(S.wr + static_cast<size_t>(wp.slot) * kBlockBytes, src, kBlockBytes, &S.fullw[wp.slot]);
        wp.next(R);
        ++nw;
        wc.next(U, L);
        progress = true;
      }
    }
    if (xc.l < L) {
      const int g = bars.gate(xc.l, xc.s);
      if (g > seen) {
        const unsigned long long cnt = ld_acquire_u64(P.bar);
        const int done_bars = static_cast<int>((cnt - bbase) / static_cast<unsigned long long>(G));
        if (done_bars - 1 > seen) {
          seen = done_bars - 1;
          // the generic-proxy writes published by the barrier -> the TMA reads below
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
      }
      if (g <= seen && mbar_try(&S.emptyx[xp.slot], xp.phase ^ 1u)) {
        mbar_expect_tx(&S.fullx[xp.slot], xbytes);
        tma_load_2d(S.xs + static_cast<size_t>(xp.slot) * kXSlot, &P.tx[xc.s], xc.k * kBK, 0, &S.fullx[xp.slot]);
        xp.next(kXStages);
        ++nx;
        xc.next(U, L);
        progress = true;
      }
    }
    if (progress) {
      t0 = globaltimer();
    } else {
      if (aborted(P)) break;
      if (globaltimer() - t0 > kTimeoutNs) {
        raise_abort(P);
        break;
      }
    }
  }
  // every issued copy lands before the CTA may exit
  for (int n = max(0, nw - R); n < nw; ++n) {
    const uint64_t t1 = globaltimer();
    while (!mbar_try(&S.fullw[n % R], static_cast<uint32_t>(n / R) & 1u))
      if (globaltimer() - t1 > kTimeoutNs) break;
  }
  for (int n = max(0, nx - kXStages); n < nx; ++n) {
    const uint64_t t1 = globaltimer();
    while (!mbar_try(&S.fullx[n % kXStages], static_cast<uint32_t>(n / kXStages) & 1u))
      if (globaltimer() - t1 > kTimeoutNs) break;
  }
}

// ---- warp 1 lane 0: four K = 16 MMAs per step into the unit's accumulator.
__device__ void mma_issuer(const Params& P, const Smem& S, const Unit (&U)[ST_N], uint32_t tmem) {
  const uint32_t idesc = idesc_f16(kRows, P.nt);
  RingPos xp, dp;
  uint32_t uses[2] = {0u, 0u};
  int buf = 0;
  bool ok = true;
  for (int l = 0; ok && l < P.n_layers; ++l) {
    for (int s = 0; ok && s < ST_N; ++s) {
      const Unit& u = U[s];
      if (!u.valid) continue;
      // the epilogue has drained this accumulator's previous unit
      if (!mwait(P, &S.acce[buf], (uses[buf] & 1u) ^ 1u)) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t acc = tmem + static_cast<uint32_t>(buf * kMaxNt);
      for (int k = u.k0; k < u.k1; ++k) {
        if (!mwait(P, &S.fullx[xp.slot], xp.phase) || !mwait(P, &S.deq[dp.slot], dp.phase)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t xd = sw128_desc(smem_u32(S.xs + static_cast<size_t>(xp.slot) * kXSlot));
        const uint64_t wdd = sw128_desc(smem_u32(S.wd + static_cast<size_t>(dp.slot) * kDSlot));
#pragma unroll
        for (int j = 0; j < kBK / 16; ++j)  // K = 16 per MMA: 32 bytes further into the swizzle atom
          mma_f16(acc, wdd + 2 * j, xd + 2 * j, idesc, (k > u.k0 || j > 0) ? 1u : 0u);
        mma_commit(&S.emptyx[xp.slot]);
        mma_commit(&S.emptyd[dp.slot]);
        xp.next(kXStages);
        dp.next(kDStages);
      }
      if (!ok) break;
      mma_commit(&S.accf[buf]);
      ++uses[buf];
      buf ^= 1;
    }
  }
  // every MMA issued above has finished before the CTA frees the tensor memory
  mma_commit(S.done);
  const uint64_t t1 = globaltimer();
  while (!mbar_try(S.done, 0u))
    if (globaltimer() - t1 > kTimeoutNs) break;
}

// ---- warps 2-5 --------------------------------------------------------------
struct Workers {
  const Params& P;
  const Smem& S;
  const Unit (&U)[ST_N];
  uint32_t tmem;
  unsigned long long bbase;
  int t, warp, lane, c, G;
  RingPos wp, dp;
  uint32_t uses[2] = {0u, 0u};
  int buf = 0;
  bool dead = false;  // warp-uniform: a wait of this warp gave up (the launch is aborting)

  __device__ Workers(const Params& P_, const Smem& S_, const Unit (&U_)[ST_N], uint32_t tmem_,
                     unsigned long long bbase_)
      : P(P_), S(S_), U(U_), tmem(tmem_), bbase(bbase_) {
    t = threadIdx.x - 64;
    warp = threadIdx.x >> 5;
    lane = threadIdx.x & 31;
    c = blockIdx.x;
    G = gridDim.x;
  }

  __device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity) {
    const bool ok = !dead && mwait(P, bar, parity);
    dead = !__all_sync(0xffffffffu, ok);
    return !dead;
  }

  // This CTA's outputs of the stage ending at barrier k are written: count
  // it in (after barrier k - 1 completed, which keeps each barrier's
  // arrivals inside one multiple of the grid size).
  __device__ void arrive(int k) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    workers_sync();
    if (t == 0 && P.trace) P.trace[(static_cast<size_t>(c) * P.n_bars + k) * 2] = globaltimer();
    if (t == 0) {
      if (k > 0) counter_wait(P, bbase + static_cast<unsigned long long>(k) * G);
      __threadfence();
      red_release_add(P.bar, 1ull);
    }
  }
  // Wait for barrier k; true when the launch is aborting (same answer in every worker).
  __device__ bool wait(int k) {
    if (t == 0) {
      const bool ok = counter_wait(P, bbase + static_cast<unsigned long long>(k + 1) * G);
      *S.stop = (!ok || aborted(P)) ? 1 : 0;
      if (P.trace) P.trace[(static_cast<size_t>(c) * P.n_bars + k) * 2 + 1] = globaltimer();
    }
    workers_sync();
    const bool stop = *reinterpret_cast<volatile int*>(S.stop) != 0;
    workers_sync();  // *S.stop is read before the next wait rewrites it
    return stop;
  }

  // Dequantise the unit's weight blocks and write its epilogue.
  __device__ void gemm_unit(int s) {
    const Unit& u = U[s];
    if (!u.valid || dead) return;
    const int R = P.wslots, sw = t & 7, hs = q4t::half_swap(t);
    for (int k = u.k0; k < u.k1; ++k) {
      if (!wait_all(&S.fullw[wp.slot], wp.phase)) return;
      const unsigned char* blk = S.wr + static_cast<size_t>(wp.slot) * kBlockBytes;
      const uint4 g0 = *reinterpret_cast<const uint4*>(blk + 32 * t + 16 * hs);
      const uint4 g1 = *reinterpret_cast<const uint4*>(blk + 32 * t + 16 * (hs ^ 1));
      const uint32_t sc = *reinterpret_cast<const uint32_t*>(blk + q4t::kPackedBytes + 4 * t);
      mbar_arrive(&S.emptyw[wp.slot]);
      wp.next(R);
      if (!wait_all(&S.emptyd[dp.slot], dp.phase ^ 1u)) return;  // the MMAs are done with this tile
      const __half2 sc2 = *reinterpret_cast<const __half2*>(&sc);
      const __half2 s0 = __low2half2(sc2), s1 = __high2half2(sc2);
      unsigned char* row = S.wd + static_cast<size_t>(dp.slot) * kDSlot + t * 128;
      *reinterpret_cast<uint4*>(row + ((0 ^ sw) << 4)) = q4t::dequant8(g0.x, s0);
      *reinterpret_cast<uint4*>(row + ((1 ^ sw) << 4)) = q4t::dequant8(g0.y, s0);
      *reinterpret_cast<uint4*>(row + ((2 ^ sw) << 4)) = q4t::dequant8(g0.z, s0);
      *reinterpret_cast<uint4*>(row + ((3 ^ sw) << 4)) = q4t::dequant8(g0.w, s0);
      *reinterpret_cast<uint4*>(row + ((4 ^ sw) << 4)) = q4t::dequant8(g1.x, s1);
      *reinterpret_cast<uint4*>(row + ((5 ^ sw) << 4)) = q4t::dequant8(g1.y, s1);
      *reinterpret_cast<uint4*>(row + ((6 ^ sw) << 4)) = q4t::dequant8(g1.z, s1);
      *reinterpret_cast<uint4*>(row + ((7 ^ sw) << 4)) = q4t::dequant8(g1.w, s1);
      // generic-proxy shared-memory writes -> visible to the tensor core
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&S.deq[dp.slot]);
      dp.next(kDStages);
    }
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. = weight rows of the tile
    if (!wait_all(&S.accf[buf], uses[buf] & 1u)) return;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int q = warp & 3, row = 32 * q + lane;
    const int n0 = u.tile * kRows;
    const uint32_t tl = tmem + static_cast<uint32_t>(buf * kMaxNt) + (static_cast<uint32_t>(32 * q) << 16);
    const int rows = P.tiles[s] * kRows;
    for (int c0 = 0; c0 < P.nt; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tl + c0, r);
      if (s == ST_GU) {  // gate row in the even lane, its up row in the next
        __half* dst = P.a + (n0 + row) / 2;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float up = __shfl_down_sync(0xffffffffu, __uint_as_float(r[j]), 1);
          if ((lane & 1) == 0 && c0 + j < P.B)
            dst[static_cast<size_t>(c0 + j) * P.inter] = swiglu_value(__uint_as_float(r[j]), up);
        }
      } else {
        float* dst = P.part[s] + static_cast<size_t>(u.split) * P.B * rows + n0 + row;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < P.B) dst[static_cast<size_t>(c0 + j) * rows] = __uint_as_float(r[j]);
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    mbar_arrive(&S.acce[buf]);
    ++uses[buf];
    buf ^= 1;
  }

  // Sequence c (a CTA per sequence): x += fp16(sum of the stage's partials)
  // (the residual epilogue, runners/engine.py:215-221, 237-243), then
  // xn = RMSNorm(x) * gamma (rms_norm.metal:14-40) when gamma is given.
  // s < 0: no partials (the norm of the embedded input).
  __device__ void reduce_rows(int s, const __half* gamma) {
    if (c >= P.B) return;
    const int H = P.hidden, per = H / 512;  // 4-element groups per thread
    const int ns = s >= 0 ? P.splits[s] : 0;
    __half* xr = P.x + static_cast<size_t>(c) * H;
    uint2 xv[8];
    float ss = 0.0f;
    for (int i = 0; i < per; ++i) {
      const int g = t + kWorkers * i;
      uint2 xo = __ldcg(reinterpret_cast<const uint2*>(xr) + g);
      if (ns > 0) {
        const float4* pp = reinterpret_cast<const float4*>(P.part[s] + static_cast<size_t>(c) * H) + g;
        const float4 acc = split_sum4(pp, static_cast<size_t>(P.B) * H / 4, ns);
        __half2* h = reinterpret_cast<__half2*>(&xo);
        h[0] = __halves2half2(__hadd(__low2half(h[0]), __float2half_rn(acc.x)),
                              __hadd(__high2half(h[0]), __float2half_rn(acc.y)));
        h[1] = __halves2half2(__hadd(__low2half(h[1]), __float2half_rn(acc.z)),
                              __hadd(__high2half(h[1]), __float2half_rn(acc.w)));
        reinterpret_cast<uint2*>(xr)[g] = xo;
      }
      xv[i] = xo;
      const __half* h = reinterpret_cast<const __half*>(&xo);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float v = __half2float(h[e]);
        ss = fmaf(v, v, ss);
      }
    }
    if (gamma == nullptr) return;  // (uniform)
    ss = warp_sum(ss);
    if (lane == 0) S.red[warp & 3] = ss;
    workers_sync();
    ss = S.red[0] + S.red[1] + S.red[2] + S.red[3];
    workers_sync();  // S.red is read before its next use
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(H) + P.eps);
    __half* xnr = P.xn + static_cast<size_t>(c) * H;
    for (int i = 0; i < per; ++i) {
      const int g = t + kWorkers * i;
      const uint2 gv = __ldg(reinterpret_cast<const uint2*>(gamma) + g);
      const __half* h = reinterpret_cast<const __half*>(&xv[i]);
      const __half* gh = reinterpret_cast<const __half*>(&gv);
      __half o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __half nrm = __float2half_rn(__half2float(h[e]) * scale);
        o[e] = __float2half_rn(__half2float(nrm) * __half2float(gh[e]));
      }
      reinterpret_cast<uint2*>(xnr)[g] = *reinterpret_cast<const uint2*>(o);
    }
  }

  __device__ AttnParams attn_params(int l) const {
    const lmps_batched_layer& L = P.layers[l];
    AttnParams A{};
    A.k_pool = reinterpret_cast<const __half*>(L.k_pool);
    A.v_pool = reinterpret_cast<const __half*>(L.v_pool);
    A.k_new = reinterpret_cast<__half*>(L.k_pool);
    A.v_new = reinterpret_cast<__half*>(L.v_pool);
    A.block_table = P.block_table;
    A.seq_lens = P.seq_lens;
    A.out = P.attn;
    A.part_o = P.att_o;
    A.part_ml = P.att_ml;
    A.max_pages = P.max_pages;
    A.page_size = P.page_size;
    A.page_shift = P.page_shift;
    A.n_q_heads = P.n_q;
    A.n_kv_heads = P.n_kv;
    A.n_splits = P.att_splits;
    A.chunk = P.att_chunk;
    A.pos = P.pos;
    A.inv_freq = P.inv_freq;
    A.rope_style = P.rope_style;
    return A;
  }

  // Split-KV items (sequence, KV head, split) of layer l, round robin over the grid.
  __device__ void attention(int l) {
    const AttnParams A = attn_params(l);
    const __half* bias = reinterpret_cast<const __half*>(P.layers[l].qkv_bias);
    const int Gq = P.n_q / P.n_kv, q_dim = P.n_q * kHeadDim, kv_dim = P.n_kv * kHeadDim;
    const size_t stride = static_cast<size_t>(P.B) * P.qkv_rows;
    const int nsplit = P.splits[ST_QKV];
    AttnSmem& AS = *reinterpret_cast<AttnSmem*>(S.xs);
    __half* staged = reinterpret_cast<__half*>(S.xs + sizeof(AttnSmem));
    const int items = P.B * P.n_kv * P.att_splits;
    for (int it = c; it < items; it += G) {
      const int split = it % P.att_splits, kvh = (it / P.att_splits) % P.n_kv;
      const int b = it / (P.att_splits * P.n_kv);
      // the item's q heads, k and v rows: (Gq + 2) * 128 values, two per thread per round
      const int n = (Gq + 2) * kHeadDim;
      const float* row = P.part[ST_QKV] + static_cast<size_t>(b) * P.qkv_rows;
      for (int j0 = 2 * t; j0 < n; j0 += 2 * kWorkers) {
        const int r = j0 / kHeadDim, d = j0 - r * kHeadDim;
        const int src = r < Gq ? (kvh * Gq + r) * kHeadDim + d
                               : (r == Gq ? q_dim + kvh * kHeadDim + d : q_dim + kv_dim + kvh * kHeadDim + d);
        const float s0 = split_sum(row + src, stride, nsplit), s1 = split_sum(row + src + 1, stride, nsplit);
        staged[j0] = __float2half_rn(s0 + __half2float(__ldg(bias + src)));
        staged[j0 + 1] = __float2half_rn(s1 + __half2float(__ldg(bias + src + 1)));
      }
      workers_sync();
      const StagedQkv ld{staged, (kvh * Gq) * kHeadDim, q_dim + kvh * kHeadDim, q_dim + kv_dim + kvh * kHeadDim, Gq};
      attn_item(A, AS, split, kvh, b, t, true, ld, WorkerSync{});
      workers_sync();  // the item's shared memory is read before the next item stages into it
    }
  }
  __device__ void merge(int l) {
    const AttnParams A = attn_params(l);
    for (int r = c; r < P.B * P.n_q; r += G) attn_combine(A, r % P.n_q, r / P.n_q, t);
  }

  __device__ void run() {
    const int L = P.n_layers;
    const Bars bars{7 + (P.att_splits > 1 ? 1 : 0), P.att_splits > 1 ? 1 : 0};
    reduce_rows(-1, reinterpret_cast<const __half*>(P.layers[0].in_norm));
    arrive(0);
    for (int l = 0; l < L; ++l) {
      const lmps_batched_layer& Ly = P.layers[l];
      const int b0 = bars.first(l);
      gemm_unit(ST_QKV);
      arrive(b0);
      if (wait(b0)) return;
      attention(l);
      arrive(b0 + 1);
      if (bars.merge) {
        if (wait(b0 + 1)) return;
        merge(l);
        arrive(b0 + 2);
      }
      const int bo = bars.after(l, ST_O);
      gemm_unit(ST_O);
      arrive(bo);
      if (wait(bo)) return;
      reduce_rows(ST_O, reinterpret_cast<const __half*>(Ly.post_norm));
      arrive(bo + 1);
      gemm_unit(ST_GU);
      arrive(bo + 2);
      gemm_unit(ST_DN);
      arrive(bo + 3);
      if (wait(bo + 3)) return;
      reduce_rows(ST_DN, l + 1 < L ? reinterpret_cast<const __half*>(P.layers[l + 1].in_norm) : nullptr);
      arrive(bo + 4);
    }
  }
};

__global__ void __launch_bounds__(kThreads, 1) decode_batched_kernel(const __grid_constant__ Params P) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int R = P.wslots;
  Smem S;
  S.xs = base;
  S.wd = S.xs + kXStages * kXSlot;
  S.wr = S.wd + kDStages * kDSlot;
  S.fullw = reinterpret_cast<uint64_t*>(S.wr + static_cast<size_t>(R) * kBlockBytes);
  S.emptyw = S.fullw + R;
  S.fullx = S.emptyw + R;
  S.emptyx = S.fullx + kXStages;
  S.deq = S.emptyx + kXStages;
  S.emptyd = S.deq + kDStages;
  S.accf = S.emptyd + kDStages;
  S.acce = S.accf + 2;
  S.done = S.acce + 2;
  S.base = reinterpret_cast<unsigned long long*>(S.done + 1);
  S.tmem_slot = reinterpret_cast<uint32_t*>(S.base + 1);
  S.stop = reinterpret_cast<int*>(S.tmem_slot + 1);
  S.red = reinterpret_cast<float*>(S.stop + 1);
  const int tid = threadIdx.x, warp = tid >> 5;

  // Every position must lie inside the cache: all CTAs read the same values
  // and leave together before any barrier or copy.
  for (int b = 0; b < P.B; ++b) {
    const int p = P.pos[b];
    if (p < 0 || p >= P.max_pages * P.page_size || P.seq_lens[b] != p + 1) {
      if (tid == 0 && blockIdx.x == 0) atomicExch(P.error, 2);
      return;
    }
  }
  if (tid == 0) {
    for (int i = 0; i < R; ++i) {
      mbar_init(&S.fullw[i], 1);
      mbar_init(&S.emptyw[i], kWorkers);
    }
    for (int i = 0; i < kXStages; ++i) {
      mbar_init(&S.fullx[i], 1);
      mbar_init(&S.emptyx[i], 1);
    }
    for (int i = 0; i < kDStages; ++i) {
      mbar_init(&S.deq[i], kWorkers);
      mbar_init(&S.emptyd[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.accf[i], 1);
      mbar_init(&S.acce[i], kWorkers);
    }
    mbar_init(S.done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // This CTA has not arrived at the launch's first barrier, so the count is
    // below the next multiple of the grid size.
    const unsigned long long cnt = ld_acquire_u64(P.bar);
    *S.base = cnt - cnt % gridDim.x;
    *S.stop = 0;
  }
  if (tid == 32) {
#pragma unroll
    for (int s = 0; s < ST_N; ++s)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&P.tx[s])) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(S.tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *S.tmem_slot;
  const unsigned long long bbase = *S.base;
  Unit U[ST_N];
#pragma unroll
  for (int s = 0; s < ST_N; ++s) U[s] = unit_of(P, s, blockIdx.x);
  const int merge = P.att_splits > 1 ? 1 : 0;
  const Bars bars{7 + merge, merge};

  if (warp == 0) {
    if (tid == 0) producer(P, S, U, bars, bbase);
  } else if (warp == 1) {
    if (tid == 32) mma_issuer(P, S, U, tmem);
  } else {
    Workers w(P, S, U, tmem, bbase);
    w.run();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

}  // namespace bd
}  // namespace lmps

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace lmps {
namespace bd {

// Repack one Q4 matrix into tile-major blocks (q4_tile.cuh): thread = (block, row).
__global__ void q4_tile_blocks_kernel(const uint8_t* __restrict__ packed, const __half* __restrict__ scales, int n,
                                      int k, unsigned char* __restrict__ out) {
  const int ks = k / kBK;
  const size_t total = static_cast<size_t>(n / kRows) * ks * kRows;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i % kRows);
    const size_t blk = i / kRows;
    const int tile = static_cast<int>(blk / ks), j = static_cast<int>(blk % ks);
    const size_t row = static_cast<size_t>(tile) * kRows + r;
    const uint4* src = reinterpret_cast<const uint4*>(packed + row * (k / 2) + static_cast<size_t>(j) * 32);
    unsigned char* dst = out + blk * kBlockBytes;
    const int hs = q4t::half_swap(r);
    reinterpret_cast<uint4*>(dst + 32 * r + 16 * hs)[0] = src[0];
    reinterpret_cast<uint4*>(dst + 32 * r + 16 * (hs ^ 1))[0] = src[1];
    const __half* sp = scales + row * (k / 32) + 2 * j;
    const __half2 s2 = __halves2half2(sp[0], sp[1]);
    reinterpret_cast<__half2*>(dst + q4t::kPackedBytes)[r] = s2;
  }
}

struct Geometry {
  int G, nt;
  int tiles[ST_N], splits[ST_N], ksteps[ST_N];
  int att_splits, att_chunk;
};

static int sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return sms;
}

// Units per stage: the weight-row tiles, each K range split so that the
// tiles x splits units fill the grid (the gate/up stage keeps whole K for
// its SwiGLU epilogue); attention splits likewise.
static bool geometry(const lmps_batched_desc& m, int B, int max_seq_len, int G, Geometry& g) {
  const int qkv_rows = (m.n_q_heads + 2 * m.n_kv_heads) * m.head_dim, q_dim = m.n_q_heads * m.head_dim;
  const int rows[ST_N] = {qkv_rows, m.hidden, 2 * m.intermediate, m.hidden};
  const int kdim[ST_N] = {m.hidden, q_dim, m.hidden, m.intermediate};
  g.G = G;
  g.nt = (B + 15) / 16 * 16;
  for (int s = 0; s < ST_N; ++s) {
    if (rows[s] % kRows || kdim[s] % kBK) return false;
    g.tiles[s] = rows[s] / kRows;
    g.ksteps[s] = kdim[s] / kBK;
    if (g.tiles[s] > G) return false;
    int sp = G / g.tiles[s];
    if (sp > g.ksteps[s]) sp = g.ksteps[s];
    if (sp > kMaxSplits) sp = kMaxSplits;
    if (s == ST_GU || sp < 1) sp = 1;
    g.splits[s] = sp;
  }
  const int ptiles = (max_seq_len + kAttnTile - 1) / kAttnTile;
  int S = G / (B * m.n_kv_heads);
  if (S < 1) S = 1;
  if (S > ptiles) S = ptiles;
  g.att_chunk = attn_chunk(max_seq_len, S);
  g.att_splits = (max_seq_len + g.att_chunk - 1) / g.att_chunk;
  return true;
}

struct WsLayout {
  size_t xn, attn, a, part[ST_N], att_o, att_ml, total;
};
static size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }
static WsLayout ws_layout(const lmps_batched_desc& m, int B, const Geometry& g) {
  const size_t qkv_rows = static_cast<size_t>(m.n_q_heads + 2 * m.n_kv_heads) * m.head_dim;
  const size_t q_dim = static_cast<size_t>(m.n_q_heads) * m.head_dim;
  WsLayout w{};
  size_t off = 256;  // [0, 8): grid-barrier counter, [8, 12): abort flag
  w.xn = off; off = align256(off + 2 * static_cast<size_t>(B) * m.hidden);
  w.attn = off; off = align256(off + 2 * static_cast<size_t>(B) * q_dim);
  w.a = off; off = align256(off + 2 * static_cast<size_t>(B) * m.intermediate);
  const size_t prow[ST_N] = {qkv_rows, static_cast<size_t>(m.hidden), 0, static_cast<size_t>(m.hidden)};
  for (int s = 0; s < ST_N; ++s) {
    w.part[s] = off;
    off = align256(off + 4 * static_cast<size_t>(g.splits[s]) * B * prow[s]);
  }
  const size_t arows = static_cast<size_t>(B) * m.n_q_heads * (g.att_splits > 1 ? g.att_splits : 0);
  w.att_o = off; off = align256(off + 4 * arows * m.head_dim);
  w.att_ml = off; off = align256(off + 8 * arows);
  w.total = off;
  return w;
}

}  // namespace bd
}  // namespace lmps

using namespace lmps;

extern "C" size_t lmps_q4_tile_blocks_size(int n, int k) {
  if (n <= 0 || k <= 0 || n % bd::kRows || k % bd::kBK) return 0;
  return static_cast<size_t>(n / bd::kRows) * (k / bd::kBK) * bd::kBlockBytes;
}

extern "C" int lmps_q4_tile_blocks(const uint8_t* packed, const uint16_t* scales, int n, int k, void* out,
                                   void* stream) {
  LMPS_CHECK_ARG(packed && scales && out);
  LMPS_CHECK_ARG(n > 0 && k > 0 && n % bd::kRows == 0 && k % bd::kBK == 0);
  LMPS_CHECK_ARG(lmps_aligned(packed, 16) && lmps_aligned(out, 16) && lmps_aligned(scales, 4));
  const size_t total = static_cast<size_t>(n) * (k / bd::kBK);
  const int threads = 256;
  const int blocks = static_cast<int>(total / threads < 4096 ? (total + threads - 1) / threads : 4096);
  bd::q4_tile_blocks_kernel<<<blocks, threads, 0, lmps_stream(stream)>>>(
      packed, reinterpret_cast<const __half*>(scales), n, k, static_cast<unsigned char*>(out));
  return lmps_launch_status();
}

static int batched_check(const lmps_batched_desc* model, int batch, int max_seq_len) {
  if (!model || batch < 1 || max_seq_len < 1) return LMPS_ERR_INVALID_ARGUMENT;
  const lmps_batched_desc& m = *model;
  if (!m.layers || m.n_layers < 1 || m.n_kv_heads < 1 || m.n_q_heads % m.n_kv_heads) return LMPS_ERR_INVALID_ARGUMENT;
  if (batch > bd::kMaxNt || m.head_dim != kHeadDim || m.n_q_heads / m.n_kv_heads > kMaxGroup ||
      m.hidden % 512 || m.hidden > 4096 || m.n_layers > bd::kMaxLayers)
    return LMPS_ERR_UNSUPPORTED;
  return LMPS_OK;
}

extern "C" size_t lmps_decode_batched_workspace_size(const lmps_batched_desc* model, int batch, int max_seq_len) {
  if (batched_check(model, batch, max_seq_len) != LMPS_OK) return 0;
  bd::Geometry g{};
  const int G = bd::sm_count();
  if (G < 1 || !bd::geometry(*model, batch, max_seq_len, G, g)) return 0;
  return bd::ws_layout(*model, batch, g).total;
}

extern "C" int lmps_decode_batched(const lmps_batched_desc* model, uint16_t* x, const int32_t* pos,
                                   const int32_t* seq_lens, const int32_t* block_table, int max_pages,
                                   int page_size, int batch, int max_seq_len, void* workspace,
                                   size_t workspace_bytes, int32_t* error, unsigned long long* trace,
                                   void* stream) {
  const int chk = batched_check(model, batch, max_seq_len);
  if (chk != LMPS_OK) return chk;
  LMPS_CHECK_ARG(x && pos && seq_lens && block_table && workspace && error && model->inv_freq);
  LMPS_CHECK_ARG(max_pages > 0 && page_size > 0 && max_seq_len <= max_pages * page_size);
  LMPS_CHECK_ARG(model->rope_style == LMPS_ROPE_INTERLEAVED || model->rope_style == LMPS_ROPE_NEOX);
  LMPS_CHECK_ARG(lmps_aligned(x, 16) && lmps_aligned(workspace, 256));
  const lmps_batched_desc& m = *model;
  const int G = bd::sm_count();
  if (G < 1) return LMPS_ERR_UNSUPPORTED;
  bd::Geometry g{};
  if (!bd::geometry(m, batch, max_seq_len, G, g)) return LMPS_ERR_UNSUPPORTED;
  const bd::WsLayout w = bd::ws_layout(m, batch, g);
  if (workspace_bytes < w.total) return LMPS_ERR_WORKSPACE;
  char* ws = static_cast<char*>(workspace);
  bd::Params P{};
  P.layers = m.layers;
  P.n_layers = m.n_layers;
  P.x = reinterpret_cast<__half*>(x);
  P.xn = reinterpret_cast<__half*>(ws + w.xn);
  P.attn = reinterpret_cast<__half*>(ws + w.attn);
  P.a = reinterpret_cast<__half*>(ws + w.a);
  for (int s = 0; s < bd::ST_N; ++s) P.part[s] = reinterpret_cast<float*>(ws + w.part[s]);
  P.att_o = reinterpret_cast<float*>(ws + w.att_o);
  P.att_ml = reinterpret_cast<float2*>(ws + w.att_ml);
  P.bar = reinterpret_cast<unsigned long long*>(ws);
  P.abort_flag = reinterpret_cast<int*>(ws + 8);
  P.error = error;
  P.inv_freq = m.inv_freq;
  P.pos = pos;
  P.seq_lens = seq_lens;
  P.block_table = block_table;
  P.max_pages = max_pages;
  P.page_size = page_size;
  P.page_shift = (page_size & (page_size - 1)) == 0 ? __builtin_ctz(static_cast<unsigned>(page_size)) : -1;
  P.rope_style = m.rope_style;
  P.B = batch;
  P.nt = g.nt;
  P.hidden = m.hidden;
  P.inter = m.intermediate;
  P.n_q = m.n_q_heads;
  P.n_kv = m.n_kv_heads;
  P.qkv_rows = (m.n_q_heads + 2 * m.n_kv_heads) * m.head_dim;
  P.eps = m.eps;
  for (int s = 0; s < bd::ST_N; ++s) {
    P.tiles[s] = g.tiles[s];
    P.splits[s] = g.splits[s];
    P.ksteps[s] = g.ksteps[s];
  }
  P.att_splits = g.att_splits;
  P.att_chunk = g.att_chunk;
  P.trace = trace;
  P.n_bars = 1 + m.n_layers * (7 + (g.att_splits > 1 ? 1 : 0));
  // activation tiles: box {64 elements, nt tokens}, rows past the batch read as zero
  const int q_dim = m.n_q_heads * m.head_dim;
  const void* xsrc[bd::ST_N] = {P.xn, P.attn, P.xn, P.a};
  const int xk[bd::ST_N] = {m.hidden, q_dim, m.hidden, m.intermediate};
  for (int s = 0; s < bd::ST_N; ++s)
    if (!tc::encode_2d(&P.tx[s], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xsrc[s], static_cast<uint64_t>(xk[s]),
                       static_cast<uint64_t>(batch), static_cast<uint64_t>(xk[s]) * 2, bd::kBK,
                       static_cast<uint32_t>(g.nt), CU_TENSOR_MAP_SWIZZLE_128B))
      return LMPS_ERR_UNSUPPORTED;
  int dev = 0, max_smem = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  int R = (max_smem - bd::kFixedSmem) / bd::kBlockBytes;
  if (R > bd::kMaxWSlots) R = bd::kMaxWSlots;
  if (R < 4) return LMPS_ERR_UNSUPPORTED;
  P.wslots = R;
  const size_t smem = static_cast<size_t>(bd::kFixedSmem) + static_cast<size_t>(R) * bd::kBlockBytes;
  const int st_attr = lmps_max_dyn_smem<bd::decode_batched_kernel>(static_cast<int>(smem));
  if (st_attr != LMPS_OK) return st_attr;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, bd::decode_batched_kernel, bd::kThreads,
                                                                smem);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (per_sm < 1) return LMPS_ERR_UNSUPPORTED;
  void* args[] = {&P};
  e = cudaLaunchCooperativeKernel(reinterpret_cast<void*>(bd::decode_batched_kernel), dim3(G), dim3(bd::kThreads),
                                  args, smem, lmps_stream(stream));
  return e == cudaSuccess ? lmps_launch_status() : static_cast<int>(e);
}
