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
// Roles of the 352 threads of a CTA (as in the W4A16 GEMM): warp 0 lane 0
// issues the weight and activation loads, warp 1 lane 0 the MMAs
// (A = 128 dequantised weight rows, B = the tokens, N = batch rounded up to
// 16, two TMEM accumulators used alternately), warps 2-9 dequantise (half a
// weight row of a K step per thread), warps 2-5 also run the epilogues and
// the attention / reduction phases, warp 10 lane 0 watches the grid barrier
// counter (the only thread of the CTA that polls global memory in a wait;
// everything else waits on shared memory).  Every wait is bounded: a timeout
// sets the error word and a workspace abort flag that the watchers see, and
// the launch ends without a hang.
#include <cmath>

#include "common.cuh"
#include "decode_attention.cuh"
#include "q4_tile.cuh"
#include "tcgen05.cuh"

namespace lmps {
namespace bd {

using namespace tc;

constexpr int kThreads = 352;                 // 11 warps
constexpr int kWorkers = 128;                 // warps 2-5: dequantise, epilogues, attention, reductions
constexpr int kDequant = 256;                 // warps 2-9 dequantise (half a weight row per thread)
constexpr int kWatcherTid = 320;              // warp 10 lane 0
constexpr int kAttnStagesB = 3;               // K/V tiles in flight in the attention phase
constexpr int kTPitch = 36;                   // epilogue transpose: floats per token row (16-byte rows)
constexpr int kBK = 64;
constexpr int kRows = 128;
constexpr int kBlockBytes = q4t::kBlockBytes; // 4096 packed + 512 scale bytes
constexpr int kMaxNt = 64;                    // tokens per MMA (batch rounded up to 16)
constexpr int kXBytes = 48 * 1024;            // activation ring: nt x 128-byte slots (1024-byte multiples)
constexpr int kMaxXStages = 16;
constexpr int kDStages = 5;
constexpr int kDSlot = kRows * 128;           // 16 KB dequantised fp16 tile
constexpr int kMaxWSlots = 32;
constexpr int kTmemCols = 2 * kMaxNt;         // two accumulators
constexpr int kMaxLayers = 64;
constexpr int kAttnMinChunk = 512;
constexpr unsigned kIdleNs = 64;  // pause of a polling thread that found nothing to do

enum Stage { ST_QKV = 0, ST_O = 1, ST_GU = 2, ST_DN = 3, ST_N = 4 };

struct __align__(64) Params {
  CUtensorMap tx[ST_N];  // activations read by each GEMM stage: xn, attn, xn, a (box {64, nt})
  const lmps_batched_layer* layers;
  int n_layers;
  __half* x;     // residual [B, hidden], in and out
  __half* xn;    // normalised activations [B, hidden]
  __half* attn;  // attention output [B, q_dim]
  __half* a;     // SwiGLU output [B, intermediate]
  float* part[ST_N];  // fp32 split-K accumulators of QKV, O, DN: [B][rows], zero between uses
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
  int xstages, xslot;         // activation ring: slots of nt * 128 bytes
  unsigned long long* trace;  // optional [grid][barriers][4] %globaltimer stamps (see lmps_decode_batched)
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
__device__ __forceinline__ int ld_acquire_cta(const int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_cta(int* p, int v) {
  asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ void workers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kWorkers) : "memory"); }

// Non-blocking probe of a phase (try_wait may suspend the thread for a while,
// which the producer, polling two rings, cannot afford).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
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

using AttnSmemB = AttnSmemT<kAttnStagesB>;

struct Smem {
  unsigned char* xs;  // [xstages][xslot] activation tiles (128-byte swizzle)
  unsigned char* wd;  // [kDStages][kDSlot] dequantised weight tiles (128-byte swizzle)
  unsigned char* wr;  // [wslots][kBlockBytes] tile-major weight blocks
  uint64_t *fullw, *emptyw, *fullx, *emptyx, *deq, *emptyd, *accf, *acce, *done, *attn_done;
  uint32_t* tmem_slot;
  int* stop;                 // workers' shared stop decision
  int* sabort;               // this CTA is giving up (mirror of the launch's abort flag)
  int* sseen;                // highest grid barrier seen complete (kept by the watcher)
  unsigned long long* base;  // grid-barrier count at launch start
  float* red;                // [4] per-warp sums
};
constexpr int kFixedSmem = 1024 + kXBytes + kDStages * kDSlot + 2048;

// Every wait polls shared memory only: a timeout (or a give-up seen by the
// watcher) sets the CTA's abort word, and the launch's error and abort words.
__device__ __forceinline__ bool cta_aborting(const Smem& S) { return *reinterpret_cast<volatile int*>(S.sabort) != 0; }
__device__ __noinline__ void raise_abort(const Params& P, const Smem& S) {
  atomicExch(P.error, 1);
  atomicExch(P.abort_flag, 1);
  *reinterpret_cast<volatile int*>(S.sabort) = 1;
}
__device__ __forceinline__ bool mwait(const Params& P, const Smem& S, uint64_t* bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try(bar, parity)) {
    if (cta_aborting(S)) return false;
    if (globaltimer() - t0 > kTimeoutNs) {
      raise_abort(P, S);
      return false;
    }
  }
  return true;
}
// Bounded wait until grid barrier k is complete (as the watcher saw it).
__device__ __forceinline__ bool bar_wait(const Params& P, const Smem& S, int k) {
  if (ld_acquire_cta(S.sseen) >= k) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_cta(S.sseen) < k) {
    __nanosleep(kIdleNs);
    if (cta_aborting(S)) return false;
    if (globaltimer() - t0 > kTimeoutNs) {
      raise_abort(P, S);
      return false;
    }
  }
  return true;
}

// ---- warp 6 lane 0: the only poller of the launch's barrier counter; it
// publishes each completed barrier to the CTA (release / acquire through
// shared memory), and a give-up by another CTA.
__device__ void watcher(const Params& P, const Smem& S, unsigned long long bbase) {
  const unsigned long long G = gridDim.x;
  const int last = P.n_bars - 1;
  int seen = -1;
  uint64_t t0 = globaltimer();
  for (unsigned it = 0; seen < last; ++it) {
    const int now = static_cast<int>((ld_acquire_u64(P.bar) - bbase) / G) - 1;
    if (now > seen) {
      seen = now;
      st_release_cta(S.sseen, seen);
      t0 = globaltimer();
      continue;
    }
    if (cta_aborting(S)) return;
    if ((it & 15u) == 15u && *reinterpret_cast<volatile int*>(P.abort_flag) != 0) {
      *reinterpret_cast<volatile int*>(S.sabort) = 1;
      return;
    }
    if (globaltimer() - t0 > kTimeoutNs) {
      raise_abort(P, S);
      return;
    }
  }
}
static_assert(sizeof(AttnSmemB) + (kMaxGroup + 2) * kHeadDim * 2 <= kXBytes + kDStages * kDSlot,
              "attention aliases the tile rings");

// fp32 add into the L2-resident accumulator of a split-K stage (the splits
// of a tile meet there; the reduction phase reads the sums and zeroes them).
__device__ __forceinline__ void red_add_v4(float* p, float4 v) {  // p 16-byte aligned
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// q|k|v rows of one attention item, staged in shared memory before the item
// runs: value = fp16(sum of the QKV splits + bias), the W4A16 GEMM's bias
// epilogue.  The item's loader reads them back by row index.
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
__device__ void producer(const Params& P, const Smem& S, const Unit (&U)[ST_N], const Bars& bars) {
  const int R = P.wslots, L = P.n_layers;
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
      if (mbar_test(&S.emptyw[wp.slot], wp.phase ^ 1u)) {
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
        const int now = ld_acquire_cta(S.sseen);
        if (now > seen) {
          seen = now;
          // the generic-proxy writes published by the barrier -> the TMA reads below
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
      }
      if (g <= seen && mbar_test(&S.emptyx[xp.slot], xp.phase ^ 1u)) {
        mbar_expect_tx(&S.fullx[xp.slot], xbytes);
        tma_load_2d(S.xs + static_cast<size_t>(xp.slot) * P.xslot, &P.tx[xc.s], xc.k * kBK, 0, &S.fullx[xp.slot]);
        xp.next(P.xstages);
        ++nx;
        xc.next(U, L);
        progress = true;
      }
    }
    if (progress) {
      t0 = globaltimer();
    } else {
      __nanosleep(kIdleNs);  // leave the issue slots to the dequantising warps of this sub-partition
      if (cta_aborting(S)) break;
      if (globaltimer() - t0 > kTimeoutNs) {
        raise_abort(P, S);
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
  for (int n = max(0, nx - P.xstages); n < nx; ++n) {
    const uint64_t t1 = globaltimer();
    while (!mbar_try(&S.fullx[n % P.xstages], static_cast<uint32_t>(n / P.xstages) & 1u))
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
      if (!mwait(P, S, &S.acce[buf], (uses[buf] & 1u) ^ 1u)) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t acc = tmem + static_cast<uint32_t>(buf * kMaxNt);
      for (int k = u.k0; k < u.k1; ++k) {
        if (!mwait(P, S, &S.fullx[xp.slot], xp.phase) || !mwait(P, S, &S.deq[dp.slot], dp.phase)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t xd = sw128_desc(smem_u32(S.xs + static_cast<size_t>(xp.slot) * P.xslot));
        const uint64_t wdd = sw128_desc(smem_u32(S.wd + static_cast<size_t>(dp.slot) * kDSlot));
#pragma unroll
        for (int j = 0; j < kBK / 16; ++j)  // K = 16 per MMA: 32 bytes further into the swizzle atom
          mma_f16(acc, wdd + 2 * j, xd + 2 * j, idesc, (k > u.k0 || j > 0) ? 1u : 0u);
        mma_commit(&S.emptyx[xp.slot]);
        mma_commit(&S.emptyd[dp.slot]);
        xp.next(P.xstages);
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

// ---- dequantisation (warps 2-9): thread d takes half d >> 7 (32 elements) of
// weight row d & 127 of every K step of the CTA's units, in unit order.
struct Dequant {
  const Params& P;
  const Smem& S;
  int r, h;  // weight row in the tile, half of the K step
  RingPos wp, dp;
  bool dead = false;  // warp-uniform: a wait of this warp gave up (the launch is aborting)

  __device__ Dequant(const Params& P_, const Smem& S_, int d) : P(P_), S(S_), r(d & (kRows - 1)), h(d >> 7) {}

  __device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity) {
    const bool ok = !dead && mwait(P, S, bar, parity);
    dead = !__all_sync(0xffffffffu, ok);
    return !dead;
  }
  __device__ void unit(const Unit& u) {
    if (!u.valid || dead) return;
    const int sw = r & 7, hs = q4t::half_swap(r), c0 = 4 * h;
    for (int k = u.k0; k < u.k1; ++k) {
      if (!wait_all(&S.fullw[wp.slot], wp.phase)) return;
      const unsigned char* blk = S.wr + static_cast<size_t>(wp.slot) * kBlockBytes;
      const uint4 g = *reinterpret_cast<const uint4*>(blk + 32 * r + 16 * (h ^ hs));
      const uint32_t sc = *reinterpret_cast<const uint32_t*>(blk + q4t::kPackedBytes + 4 * r);
      mbar_arrive(&S.emptyw[wp.slot]);
      wp.next(P.wslots);
      if (!wait_all(&S.emptyd[dp.slot], dp.phase ^ 1u)) return;  // the MMAs are done with this tile
      const __half2 sc2 = *reinterpret_cast<const __half2*>(&sc);
      const __half2 s2 = h ? __high2half2(sc2) : __low2half2(sc2);
      unsigned char* row = S.wd + static_cast<size_t>(dp.slot) * kDSlot + r * 128;
      *reinterpret_cast<uint4*>(row + (((c0 + 0) ^ sw) << 4)) = q4t::dequant8(g.x, s2);
      *reinterpret_cast<uint4*>(row + (((c0 + 1) ^ sw) << 4)) = q4t::dequant8(g.y, s2);
      *reinterpret_cast<uint4*>(row + (((c0 + 2) ^ sw) << 4)) = q4t::dequant8(g.z, s2);
      *reinterpret_cast<uint4*>(row + (((c0 + 3) ^ sw) << 4)) = q4t::dequant8(g.w, s2);
      // generic-proxy shared-memory writes -> visible to the tensor core
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&S.deq[dp.slot]);
      dp.next(kDStages);
    }
  }
};

// Warps 6-9: the second halves of every K step.  The attention phase of the
// workers uses the dequantisation ring's shared memory, so these warps start
// on a layer's o projection only after that layer's attention.
__device__ void dequant_helper(const Params& P, const Smem& S, const Unit (&U)[ST_N]) {
  Dequant dq(P, S, threadIdx.x - 64);
  for (int l = 0; l < P.n_layers && !dq.dead; ++l) {
    for (int s = 0; s < ST_N && !dq.dead; ++s) {
      if (s == ST_O) dq.wait_all(S.attn_done, static_cast<uint32_t>(l) & 1u);
      dq.unit(U[s]);
    }
  }
}

// ---- warps 2-5 --------------------------------------------------------------
struct Workers {
  const Params& P;
  const Smem& S;
  const Unit (&U)[ST_N];
  uint32_t tmem;
  int t, warp, lane, c, G;
  Dequant dq;
  uint32_t uses[2] = {0u, 0u};
  int buf = 0;

  __device__ Workers(const Params& P_, const Smem& S_, const Unit (&U_)[ST_N], uint32_t tmem_)
      : P(P_), S(S_), U(U_), tmem(tmem_), dq(P_, S_, threadIdx.x - 64) {
    t = threadIdx.x - 64;
    warp = threadIdx.x >> 5;
    lane = threadIdx.x & 31;
    c = blockIdx.x;
    G = gridDim.x;
  }

  // This CTA's outputs of the stage ending at barrier k are written: count
  // it in (after barrier k - 1 completed, which keeps each barrier's
  // arrivals inside one multiple of the grid size).
  __device__ void arrive(int k) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    workers_sync();
    if (t == 0 && P.trace) P.trace[(static_cast<size_t>(c) * P.n_bars + k) * 4] = globaltimer();
    if (t == 0) {
      if (k > 0) bar_wait(P, S, k - 1);
      red_release_add(P.bar, 1ull);  // release: the workers' writes, ordered before it by the named barrier
    }
  }
  // Wait for barrier k; true when the launch is aborting (same answer in every worker).
  __device__ bool wait(int k) {
    if (t == 0) {
      const bool ok = bar_wait(P, S, k);
      *S.stop = (!ok || cta_aborting(S)) ? 1 : 0;
      if (P.trace) P.trace[(static_cast<size_t>(c) * P.n_bars + k) * 4 + 1] = globaltimer();
    }
    workers_sync();
    const bool stop = *reinterpret_cast<volatile int*>(S.stop) != 0;
    workers_sync();  // *S.stop is read before the next wait rewrites it
    return stop;
  }

  // Dequantise the first halves of the unit's weight blocks and write its
  // epilogue: the accumulator tile goes through shared memory (the idle
  // activation ring) so that each lane then adds four consecutive rows of a
  // token at once into the split-K accumulator (vector atomics: a quarter of
  // the L2 atomic operations), or writes eight SwiGLU outputs at once.
  __device__ void gemm_unit(int s, int k_end) {
    const Unit& u = U[s];
    if (!u.valid || dq.dead) return;
    dq.unit(u);
    if (dq.dead) return;
    if (t == 0 && P.trace) P.trace[(static_cast<size_t>(c) * P.n_bars + k_end) * 4 + 2] = globaltimer();
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. = weight rows of the tile
    if (!dq.wait_all(&S.accf[buf], uses[buf] & 1u)) return;
    if (t == 0 && P.trace) P.trace[(static_cast<size_t>(c) * P.n_bars + k_end) * 4 + 3] = globaltimer();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int q = warp & 3;
    const int n0 = u.tile * kRows + 32 * q;  // this warp's first weight row
    const uint32_t tl = tmem + static_cast<uint32_t>(buf * kMaxNt) + (static_cast<uint32_t>(32 * q) << 16);
    const int rows = P.tiles[s] * kRows;
    float* T = reinterpret_cast<float*>(S.xs) + q * (kMaxNt * kTPitch);  // [token][row of the warp]
    for (int c0 = 0; c0 < P.nt; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tl + c0, r);
#pragma unroll
      for (int j = 0; j < 32; ++j) T[j * kTPitch + lane] = __uint_as_float(r[j]);
      __syncwarp();
      if (s == ST_GU) {
        // lane: token (lane >> 1) + 16 it, pairs 8 (lane & 1) .. + 7 (gate row 2p, up row 2p + 1)
#pragma unroll
        for (int it = 0; it < 2; ++it) {
          const int jj = (lane >> 1) + 16 * it, hh = lane & 1, tok = c0 + jj;
          const float4* src = reinterpret_cast<const float4*>(T + jj * kTPitch + 16 * hh);
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 v = src[i];
            const __half2 hv = __halves2half2(swiglu_value(v.x, v.y), swiglu_value(v.z, v.w));
            o[i] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          if (tok < P.B)
            *reinterpret_cast<uint4*>(P.a + static_cast<size_t>(tok) * P.inter + n0 / 2 + 8 * hh) =
                make_uint4(o[0], o[1], o[2], o[3]);
        }
      } else {
        // lane: rows 4 (lane & 7) .. + 3 of token (lane >> 3) + 4 it
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int jj = (lane >> 3) + 4 * it, tok = c0 + jj;
          if (tok < P.B) {
            const float4 v = *reinterpret_cast<const float4*>(T + jj * kTPitch + 4 * (lane & 7));
            red_add_v4(P.part[s] + static_cast<size_t>(tok) * rows + n0 + 4 * (lane & 7), v);
          }
        }
      }
      __syncwarp();  // T is read before the next chunk overwrites it
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    mbar_arrive(&S.acce[buf]);
    ++uses[buf];
    buf ^= 1;
  }

  // Sequence c (a CTA per sequence): x += fp16(the stage's accumulated sum)
  // (the residual epilogue, runners/engine.py:215-221, 237-243), the
  // accumulator row zeroed for its next use, then xn = RMSNorm(x) * gamma
  // (rms_norm.metal:14-40) when gamma is given.  s < 0: no sum (the norm of
  // the embedded input).  zero_qkv: also zero the q|k|v accumulator row
  // (its readers, the attention items, are done).
  __device__ void reduce_rows(int s, const __half* gamma, bool zero_qkv) {
    if (c >= P.B) return;
    constexpr int kMaxPer = 4;              // hidden <= 2048
    const int H = P.hidden, per = H / 512;  // 4-element groups per thread
    __half* xr = P.x + static_cast<size_t>(c) * H;
    float4* pr = s >= 0 ? reinterpret_cast<float4*>(P.part[s] + static_cast<size_t>(c) * H) : nullptr;
    // every load first (one L2 round trip), then the stores
    uint2 xv[kMaxPer], gv[kMaxPer];
    float4 acc[kMaxPer];
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      if (i >= per) break;
      const int g = t + kWorkers * i;
      xv[i] = __ldcg(reinterpret_cast<const uint2*>(xr) + g);
      acc[i] = pr ? __ldcg(pr + g) : make_float4(0.f, 0.f, 0.f, 0.f);
      gv[i] = gamma ? __ldg(reinterpret_cast<const uint2*>(gamma) + g) : make_uint2(0u, 0u);
    }
    if (zero_qkv) {
      float4* q = reinterpret_cast<float4*>(P.part[ST_QKV] + static_cast<size_t>(c) * P.qkv_rows);
      for (int i = t; i < P.qkv_rows / 4; i += kWorkers) q[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      if (i >= per) break;
      const int g = t + kWorkers * i;
      if (pr) {
        pr[g] = make_float4(0.f, 0.f, 0.f, 0.f);
        __half2* h = reinterpret_cast<__half2*>(&xv[i]);
        h[0] = __halves2half2(__hadd(__low2half(h[0]), __float2half_rn(acc[i].x)),
                              __hadd(__high2half(h[0]), __float2half_rn(acc[i].y)));
        h[1] = __halves2half2(__hadd(__low2half(h[1]), __float2half_rn(acc[i].z)),
                              __hadd(__high2half(h[1]), __float2half_rn(acc[i].w)));
        reinterpret_cast<uint2*>(xr)[g] = xv[i];
      }
      const __half* h = reinterpret_cast<const __half*>(&xv[i]);
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
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      if (i >= per) break;
      const int g = t + kWorkers * i;
      const __half* h = reinterpret_cast<const __half*>(&xv[i]);
      const __half* gh = reinterpret_cast<const __half*>(&gv[i]);
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
    AttnSmemB& AS = *reinterpret_cast<AttnSmemB*>(S.xs);
    __half* staged = reinterpret_cast<__half*>(S.xs + sizeof(AttnSmemB));
    const int items = P.B * P.n_kv * P.att_splits;
    for (int it = c; it < items; it += G) {
      const int split = it % P.att_splits, kvh = (it / P.att_splits) % P.n_kv;
      const int b = it / (P.att_splits * P.n_kv);
      // the item's q heads, k and v rows: (Gq + 2) * 128 <= 1280 values, two
      // per thread per round, every round's loads issued before the stores
      constexpr int kRounds = (kMaxGroup + 2) * kHeadDim / (2 * kWorkers);
      const int n = (Gq + 2) * kHeadDim;
      const float* row = P.part[ST_QKV] + static_cast<size_t>(b) * P.qkv_rows;
      float2 v[kRounds];
      __half2 bv[kRounds];
#pragma unroll
      for (int r = 0; r < kRounds; ++r) {
        const int j0 = 2 * t + 2 * kWorkers * r;
        if (j0 >= n) break;
        const int hr = j0 / kHeadDim, d = j0 - hr * kHeadDim;
        const int src = hr < Gq ? (kvh * Gq + hr) * kHeadDim + d
                                : (hr == Gq ? q_dim + kvh * kHeadDim + d : q_dim + kv_dim + kvh * kHeadDim + d);
        v[r] = __ldcg(reinterpret_cast<const float2*>(row + src));
        bv[r] = __ldg(reinterpret_cast<const __half2*>(bias + src));
      }
#pragma unroll
      for (int r = 0; r < kRounds; ++r) {
        const int j0 = 2 * t + 2 * kWorkers * r;
        if (j0 >= n) break;
        staged[j0] = __float2half_rn(v[r].x + __half2float(__low2half(bv[r])));
        staged[j0 + 1] = __float2half_rn(v[r].y + __half2float(__high2half(bv[r])));
      }
      workers_sync();
      const StagedQkv ld{staged, (kvh * Gq) * kHeadDim, q_dim + kvh * kHeadDim, q_dim + kv_dim + kvh * kHeadDim, Gq};
      attn_item<kAttnStagesB>(A, AS, split, kvh, b, t, true, ld, WorkerSync{});
      workers_sync();  // the item's shared memory is read before the next item stages into it
    }
    mbar_arrive(S.attn_done);  // the dequantisation ring's memory is free again
  }
  __device__ void merge(int l) {
    const AttnParams A = attn_params(l);
    for (int r = c; r < P.B * P.n_q; r += G) attn_combine(A, r % P.n_q, r / P.n_q, t);
  }

  __device__ void run() {
    const int L = P.n_layers;
    const Bars bars{7 + (P.att_splits > 1 ? 1 : 0), P.att_splits > 1 ? 1 : 0};
    reduce_rows(-1, reinterpret_cast<const __half*>(P.layers[0].in_norm), false);
    arrive(0);
    for (int l = 0; l < L; ++l) {
      const lmps_batched_layer& Ly = P.layers[l];
      const int b0 = bars.first(l);
      gemm_unit(ST_QKV, b0);
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
      gemm_unit(ST_O, bo);
      arrive(bo);
      if (wait(bo)) return;
      reduce_rows(ST_O, reinterpret_cast<const __half*>(Ly.post_norm), true);
      arrive(bo + 1);
      gemm_unit(ST_GU, bo + 2);
      arrive(bo + 2);
      gemm_unit(ST_DN, bo + 3);
      arrive(bo + 3);
      if (wait(bo + 3)) return;
      reduce_rows(ST_DN, l + 1 < L ? reinterpret_cast<const __half*>(P.layers[l + 1].in_norm) : nullptr, false);
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
  S.wd = S.xs + kXBytes;
  S.wr = S.wd + kDStages * kDSlot;
  S.fullw = reinterpret_cast<uint64_t*>(S.wr + static_cast<size_t>(R) * kBlockBytes);
  S.emptyw = S.fullw + R;
  S.fullx = S.emptyw + R;
  S.emptyx = S.fullx + kMaxXStages;
  S.deq = S.emptyx + kMaxXStages;
  S.emptyd = S.deq + kDStages;
  S.accf = S.emptyd + kDStages;
  S.acce = S.accf + 2;
  S.done = S.acce + 2;
  S.attn_done = S.done + 1;
  S.base = reinterpret_cast<unsigned long long*>(S.attn_done + 1);
  S.tmem_slot = reinterpret_cast<uint32_t*>(S.base + 1);
  S.stop = reinterpret_cast<int*>(S.tmem_slot + 1);
  S.sabort = S.stop + 1;
  S.sseen = S.sabort + 1;
  S.red = reinterpret_cast<float*>(S.sseen + 1);
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
      mbar_init(&S.emptyw[i], kDequant);
    }
    for (int i = 0; i < P.xstages; ++i) {
      mbar_init(&S.fullx[i], 1);
      mbar_init(&S.emptyx[i], 1);
    }
    for (int i = 0; i < kDStages; ++i) {
      mbar_init(&S.deq[i], kDequant);
      mbar_init(&S.emptyd[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.accf[i], 1);
      mbar_init(&S.acce[i], kWorkers);
    }
    mbar_init(S.done, 1);
    mbar_init(S.attn_done, kWorkers);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // This CTA has not arrived at the launch's first barrier, so the count is
    // below the next multiple of the grid size.
    const unsigned long long cnt = ld_acquire_u64(P.bar);
    *S.base = cnt - cnt % gridDim.x;
    *S.stop = 0;
    *S.sabort = 0;
    *S.sseen = -1;
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
    if (tid == 0) producer(P, S, U, bars);
  } else if (warp == 1) {
    if (tid == 32) mma_issuer(P, S, U, tmem);
  } else if (warp == 10) {
    if (tid == kWatcherTid) watcher(P, S, bbase);
  } else if (warp >= 6) {
    dequant_helper(P, S, U);
  } else {
    Workers w(P, S, U, tmem);
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
    if (s == ST_GU || sp < 1) sp = 1;
    g.splits[s] = sp;
  }
  // attention: split a (sequence, KV head) over CTAs only in chunks of at
  // least 512 positions (below that the merge phase costs more than it saves)
  int S = G / (B * m.n_kv_heads);
  const int by_len = (max_seq_len + kAttnMinChunk - 1) / kAttnMinChunk;
  if (S > by_len) S = by_len;
  if (S < 1) S = 1;
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
  const size_t T = kMaxNt;  // token rows of the fixed part: the same offsets for every batch size
  WsLayout w{};
  size_t off = 256;  // [0, 8): grid-barrier counter, [8, 12): abort flag
  // split-K accumulators first: they must be zero when a launch starts, and
  // every launch leaves the rows it used zeroed, whatever its batch size
  const size_t prow[ST_N] = {qkv_rows, static_cast<size_t>(m.hidden), 0, static_cast<size_t>(m.hidden)};
  for (int s = 0; s < ST_N; ++s) {
    w.part[s] = off;
    off = align256(off + 4 * T * prow[s]);
  }
  w.xn = off; off = align256(off + 2 * T * m.hidden);
  w.attn = off; off = align256(off + 2 * T * q_dim);
  w.a = off; off = align256(off + 2 * T * m.intermediate);
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
      m.hidden % 512 || m.hidden > 2048 || m.n_layers > bd::kMaxLayers)
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

extern "C" int lmps_decode_batched_barriers(const lmps_batched_desc* model, int batch, int max_seq_len) {
  if (batched_check(model, batch, max_seq_len) != LMPS_OK) return 0;
  bd::Geometry g{};
  const int G = bd::sm_count();
  if (G < 1 || !bd::geometry(*model, batch, max_seq_len, G, g)) return 0;
  return 1 + model->n_layers * (7 + (g.att_splits > 1 ? 1 : 0));
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
  P.xslot = g.nt * 128;
  P.xstages = bd::kXBytes / P.xslot;
  if (P.xstages > bd::kMaxXStages) P.xstages = bd::kMaxXStages;
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
