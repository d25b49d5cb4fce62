// W4A16 GEMM on the 5th-generation tensor cores: tcgen05.mma with fp32
// accumulators in tensor memory (TMEM), for prefill and large-batch decode
// where the Q4 projections are dense contractions.
//
//   Y[M, N] = X[M, K] . W[N, K]^T  (+ epilogue)
//
// X: fp16 activations, token-major (row m = one token).  W: the Q4 layout of
// utils/pack_weights.py:11-47 -- packed u8 [N, K/2], element 2b in the low
// nibble of byte b, fp16 scales [N, K/32], w = (nibble - 8) * scale
// (quant_matmul.metal:39-47).
//
// One CTA owns 128 weight rows and a tile of tokens, over K in stages of 64
// (one 128-byte swizzle atom of fp16).  Warp-specialised pipeline:
//   * warp 0 (one lane) issues the TMA loads of a stage: the X tile (tokens x
//     64, written by the TMA unit in the 128-byte-swizzled K-major layout the
//     tensor core reads) and the packed W tile (128 rows x 32 bytes);
//   * warps 2-5 dequantise the packed tile (thread t = weight row t) into a
//     swizzled fp16 tile: (nibble | 0x6400) is the fp16 1024 + nibble, minus
//     1032 gives nibble - 8 exactly, times the group scale rounds once;
//   * warp 1 (one lane) issues four tcgen05.mma (K = 16 each) per stage and
//     commits them to the stage's `empty` barrier, which frees the stage for
//     the next TMA load and dequantisation;
//   * warps 2-5 then read the accumulator (tcgen05.ld; warp w reads TMEM
//     lanes 32 (w % 4) ..) and apply bias / residual.
// Two tile shapes share the pipeline:
//   * tokens >= 128 (prefill; also 33-127 tokens of a very wide output, the
//     LM head of a decode batch): A = X (M = 128 tokens), B = W (N = 128 rows);
//   * fewer tokens (decode batches): A = W (M = 128 rows), B = X (N = the
//     token count rounded up to 16), so no tensor-core row is padding and W
//     is read once.  K is then split across the CTAs of a thread-block
//     cluster to fill the GPU; the fp32 partial tiles are summed through
//     distributed shared memory, each CTA finishing a slice of the rows.
// Every mbarrier wait is bounded (error flag, no hang).
#include "common.cuh"
#include "q4_tile.cuh"
#include "tcgen05.cuh"

namespace lmps {
namespace w4 {

using namespace tc;
using q4t::dequant8;

constexpr int kBK = 64;        // K per stage
constexpr int kRows = 128;     // weight rows per tile
constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 dequantise + epilogue
constexpr int kMaxStages = 8;
constexpr int kMaxSplits = 8;  // K splits of a tile = CTAs of one (portable) cluster
constexpr int kScaleAhead = 6; // K steps a dequantising thread's scale loads run ahead
constexpr int kStepBytes = kRows * kBK / 2;   // packed W bytes of one K step (4 KB)
constexpr int kWTileBytes = kRows * kBK * 2;  // 16 KB fp16

// EPI_SWIGLU: W holds gate and up rows interleaved (row 2t = gate row t, row
// 2t + 1 = up row t) and Y[m][t] = fp16(silu(fp16(gate)) * fp16(up)), the
// math of swiglu.metal:13-23 on the two fp16 projection outputs.
enum Epilogue { EPI_NONE = 0, EPI_BIAS = 1, EPI_RESIDUAL = 2, EPI_SWIGLU = 3 };

struct __align__(64) Params {
  CUtensorMap tx;  // X [m, k] fp16, box {64, xrows}, 128-byte swizzle
  CUtensorMap tw;  // packed W [n, k/2] u8, box {128, 128}, 128-byte swizzle
  const __half* s;
  const __half* bias;
  const __half* res;
  int ldr;
  __half* y;
  int ldy;
  int m, n, k, epi;
  int swap;    // 1: A = W (M = 128 rows), B = X (N = xrows tokens)
  int xrows;   // tokens per tile: 128, or (swap) 16..256 in steps of 16
  int xstages;  // X tiles in flight
  int dstages;  // dequantised W tiles
  int wslots;   // packed-W blocks in flight
  int wspb;     // K steps per packed-W block: 4 (128-byte rows, 128-byte swizzle) or 1 (32-byte rows)
  int* error;
  int ksteps_per_split;  // split K (gridDim.z > 1, swap tiles): K steps per cluster CTA
};

// Position in a ring of n stages: the slot of the current use and the
// parity of its fill (the fill count of the slot, mod 2).  Stepped once per
// use, so the loops carry no division by the run-time stage counts.
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

// 4-byte asynchronous global -> shared copy (completion by commit groups).
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Y[row][col] from an fp32 accumulator value and the epilogue operands.
__device__ __forceinline__ __half epi_value(const Params& P, float v, int row, int col) {
  if (P.epi == EPI_BIAS) return __float2half_rn(v + __half2float(P.bias[col]));
  if (P.epi == EPI_RESIDUAL) return __hadd(P.res[static_cast<size_t>(row) * P.ldr + col], __float2half_rn(v));
  return __float2half_rn(v);
}
__device__ __forceinline__ __half swiglu_value(float gate, float up) {
  return __float2half_rn(silu_mul(__half2float(__float2half_rn(gate)), __half2float(__float2half_rn(up))));
}

__global__ void __launch_bounds__(kThreads) w4a16_gemm_kernel(const __grid_constant__ Params P) {
  extern __shared__ unsigned char smem_raw[];
  const int SX = P.xstages, SD = P.dstages, R = P.wslots, SPB = P.wspb;
  const int wblk = kStepBytes * SPB;
  const int xbytes = P.xrows * 128;
  // 1024-byte aligned rings: [R] packed W blocks (128 rows x 128 bytes = 4 K
  // steps, 128-byte swizzle), [SX] X tiles, [SD] dequantised W tiles
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* wr = base;
  unsigned char* xs = wr + static_cast<size_t>(R) * wblk;
  unsigned char* wd = xs + static_cast<size_t>(SX) * xbytes;
  uint64_t* fullw = reinterpret_cast<uint64_t*>(wd + static_cast<size_t>(SD) * kWTileBytes);
  uint64_t* emptyw = fullw + kMaxStages;
  uint64_t* fullx = emptyw + kMaxStages;
  uint64_t* emptyx = fullx + kMaxStages;
  uint64_t* deq = emptyx + kMaxStages;
  uint64_t* emptyd = deq + kMaxStages;
  uint64_t* done = emptyd + kMaxStages;
  uint32_t* scale_ring = reinterpret_cast<uint32_t*>(done + 1);  // [kScaleAhead][128]
  uint32_t* tmem_slot = scale_ring + kScaleAhead * 128;
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_v = abort_flag;

  lmps_pdl_trigger();  // the next kernel may start its own prologue
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kRows, m0 = blockIdx.y * P.xrows;
  const int kbeg = blockIdx.z * P.ksteps_per_split;
  const int ksteps = max(0, min(P.ksteps_per_split, P.k / kBK - kbeg));
  const int nwb = (ksteps + SPB - 1) / SPB;  // packed W blocks of this CTA
  const uint32_t tcols = P.swap ? (P.xrows <= 32 ? 32u : P.xrows <= 64 ? 64u : P.xrows <= 128 ? 128u : 256u) : 128u;
  // split K (swap tiles only): CTA c of the cluster receives, from every
  // split, the partial rows [c * 128 / splits, ..) of the tile, fp32, in the
  // pipeline buffers (idle by then): [splits][128 / splits][xrows + 4]
  const bool split = gridDim.z > 1;
  float* red = reinterpret_cast<float*>(base);
  const int rs = P.xrows + 4;

  if (tid == 0) {
    for (int i = 0; i < R; ++i) {
      mbar_init(&fullw[i], 1);
      mbar_init(&emptyw[i], 128);
    }
    for (int i = 0; i < SX; ++i) {
      mbar_init(&fullx[i], 1);
      mbar_init(&emptyx[i], 1);
    }
    for (int i = 0; i < SD; ++i) {
      mbar_init(&deq[i], 128);
      mbar_init(&emptyd[i], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (tid == 64) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&P.tx)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&P.tw)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tcols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // ---- TMA producer (thread 0).  Packed W blocks run up to R blocks (4R K
  // steps) ahead, X tiles SX steps; the loads that need no free slot go out
  // before the block-wide sync.
  int wk = 0, xk = 0;
  RingPos wp, xp;  // ring positions of the next W block / X tile to load
  auto issue_w = [&]() {
    mbar_expect_tx(&fullw[wp.slot], static_cast<uint32_t>(wblk));
    tma_load_2d(wr + static_cast<size_t>(wp.slot) * wblk, &P.tw, (kbeg + wk * SPB) * (kBK / 2), n0,
                &fullw[wp.slot]);
    ++wk;
    wp.next(R);
  };
  auto issue_x = [&]() {
    mbar_expect_tx(&fullx[xp.slot], static_cast<uint32_t>(xbytes));
    tma_load_2d(xs + static_cast<size_t>(xp.slot) * xbytes, &P.tx, (kbeg + xk) * kBK, m0, &fullx[xp.slot]);
    ++xk;
    xp.next(SX);
  };
  if (tid == 0) {  // weights and scales are constant: they load before the previous kernel is done
    while (wk < nwb && wk < R) issue_w();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (tid == 0) {
    lmps_pdl_wait();  // X is the previous kernel's output
    while (xk < ksteps && xk < SX) issue_x();
    uint64_t t0 = globaltimer();
    while (wk < nwb || xk < ksteps) {
      bool progress = false;
      // a slot's previous use was fill phase ^ 1: wait for its release
      if (wk < nwb && mbar_try(&emptyw[wp.slot], wp.phase ^ 1u)) {
        issue_w();
        progress = true;
      }
      if (xk < ksteps && mbar_try(&emptyx[xp.slot], xp.phase ^ 1u)) {
        issue_x();
        progress = true;
      }
      if (progress) {
        t0 = globaltimer();
      } else if (*abort_v || globaltimer() - t0 > kTimeoutNs) {
        if (!*abort_v) {
          atomicExch(P.error, 1);
          *abort_flag = 1;
        }
        break;
      }
    }
    // every issued copy lands before the CTA may exit
    for (int b = max(0, wk - R); b < wk; ++b) {
      const uint64_t t1 = globaltimer();
      while (!mbar_try(&fullw[b % R], (b / R) & 1))
        if (globaltimer() - t1 > kTimeoutNs) break;
    }
    for (int kt = max(0, xk - SX); kt < xk; ++kt) {
      const uint64_t t1 = globaltimer();
      while (!mbar_try(&fullx[kt % SX], (kt / SX) & 1))
        if (globaltimer() - t1 > kTimeoutNs) break;
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = P.swap ? idesc_f16(128, P.xrows) : idesc_f16(128, 128);
      RingPos px, pd;
      for (int kt = 0; kt < ksteps; ++kt, px.next(SX), pd.next(SD)) {
        const int sx = px.slot, sd = pd.slot;
        if (!mbar_wait(&fullx[sx], px.phase, P.error, abort_v)) break;
        if (!mbar_wait(&deq[sd], pd.phase, P.error, abort_v)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t xd = sw128_desc(smem_u32(xs + static_cast<size_t>(sx) * xbytes));
        const uint64_t wdd = sw128_desc(smem_u32(wd + static_cast<size_t>(sd) * kWTileBytes));
        const uint64_t ad = P.swap ? wdd : xd, bd = P.swap ? xd : wdd;
#pragma unroll
        for (int j = 0; j < kBK / 16; ++j)  // K = 16 per MMA: 32 bytes further into the swizzle atom
          mma_f16(tmem, ad + 2 * j, bd + 2 * j, idesc, (kt > 0 || j > 0) ? 1u : 0u);
        mma_commit(&emptyx[sx]);
        mma_commit(&emptyd[sd]);
      }
      mma_commit(done);  // tracks every MMA issued above
    }
  } else if (warp >= 2) {
    // ---- dequantisation (thread t = weight row n0 + t)
    const int t = tid - 64;
    const uint32_t* srow = reinterpret_cast<const uint32_t*>(P.s + static_cast<size_t>(n0 + t) * (P.k / 32) + 2 * kbeg);
    // The two group scales of a step arrive kScaleAhead steps early through
    // cp.async into this thread's slots of a shared-memory ring (one commit
    // group per step, empty groups included, so wait_group counts steps).
    uint32_t* sring = scale_ring + t;
#pragma unroll
    for (int i = 0; i < kScaleAhead; ++i) {
      if (i < ksteps) cp_async4(sring + i * 128, srow + i);
      cp_async_commit();
    }
    const int sw = t & 7;
    RingPos pd, pw;  // dequantised stage, packed-W block
    int sub = 0, slot = 0;  // K step within the block, scale-ring slot
    for (int kt = 0; kt < ksteps; ++kt) {
      const int s = pd.slot, wsl = pw.slot;
      cp_async_wait<kScaleAhead - 1>();
      const uint32_t sc = sring[slot * 128];
      if (kt + kScaleAhead < ksteps) cp_async4(sring + slot * 128, srow + kt + kScaleAhead);
      cp_async_commit();
      slot = slot + 1 == kScaleAhead ? 0 : slot + 1;
      if (sub == 0 && !mbar_wait(&fullw[wsl], pw.phase, P.error, abort_v)) break;
      if (kt >= SD && !mbar_wait(&emptyd[s], pd.phase ^ 1u, P.error, abort_v)) break;  // MMA done with wd[s]
      // packed row t, bytes 32 sub .. 32 sub + 31: 16-byte chunks 2 sub and
      // 2 sub + 1 of a 32 SPB-byte row (128-byte rows are swizzled)
      const unsigned char* rrow = wr + static_cast<size_t>(wsl) * wblk + t * (32 * SPB);
      const int rsw = SPB == 4 ? sw : 0;
      const uint4 g0 = *reinterpret_cast<const uint4*>(rrow + (((2 * sub) ^ rsw) << 4));
      const uint4 g1 = *reinterpret_cast<const uint4*>(rrow + (((2 * sub + 1) ^ rsw) << 4));
      if (sub == SPB - 1 || kt == ksteps - 1) mbar_arrive(&emptyw[wsl]);  // packed block consumed
      const __half2 sc2 = *reinterpret_cast<const __half2*>(&sc);
      const __half2 s0 = __low2half2(sc2), s1 = __high2half2(sc2);
      unsigned char* row = wd + static_cast<size_t>(s) * kWTileBytes + t * 128;
      *reinterpret_cast<uint4*>(row + ((0 ^ sw) << 4)) = dequant8(g0.x, s0);
      *reinterpret_cast<uint4*>(row + ((1 ^ sw) << 4)) = dequant8(g0.y, s0);
      *reinterpret_cast<uint4*>(row + ((2 ^ sw) << 4)) = dequant8(g0.z, s0);
      *reinterpret_cast<uint4*>(row + ((3 ^ sw) << 4)) = dequant8(g0.w, s0);
      *reinterpret_cast<uint4*>(row + ((4 ^ sw) << 4)) = dequant8(g1.x, s1);
      *reinterpret_cast<uint4*>(row + ((5 ^ sw) << 4)) = dequant8(g1.y, s1);
      *reinterpret_cast<uint4*>(row + ((6 ^ sw) << 4)) = dequant8(g1.z, s1);
      *reinterpret_cast<uint4*>(row + ((7 ^ sw) << 4)) = dequant8(g1.w, s1);
      // generic-proxy shared-memory writes -> visible to the tensor core
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&deq[s]);
      pd.next(SD);
      if (++sub == SPB) {
        sub = 0;
        pw.next(R);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // no copy in flight past the loop (abort path)
  }
  // ---- epilogue (warps 2-5: warp w reads TMEM lanes 32 (w % 4) ..)
  __syncwarp();
  lmps_pdl_wait();  // before any read of the residual or write of Y
  const bool epi_warp = warp >= 2;
  bool ok = false;
  if (epi_warp) {
    ok = ksteps > 0 && mbar_wait(done, 0, P.error, abort_v);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  }
  const int q = warp & 3;  // TMEM lanes 32q .. 32q+31
  const uint32_t tl = tmem + (static_cast<uint32_t>(32 * q) << 16);
  if (split) {
    // Reduce-scatter over the cluster.  Barrier 1: every CTA is past its
    // main loop, so its pipeline buffers may receive partial rows.
    asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
    uint32_t rank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    const int nsplit = gridDim.z, rows_per = kRows / nsplit;
    if (epi_warp) {
      const int row = 32 * q + lane;  // weight row within the tile
      const uint32_t dst = static_cast<uint32_t>(row / rows_per);
      const uint32_t laddr =
          smem_u32(red) + static_cast<uint32_t>(((static_cast<int>(rank) * rows_per + row % rows_per) * rs) * 4);
      uint32_t raddr;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(raddr) : "r"(laddr), "r"(dst));
      for (int c0 = 0; c0 < P.xrows; c0 += 32) {
        uint32_t r[32];
        if (ok) {
          tmem_ld32(tl + c0, r);
        } else {  // no K steps (or aborted): this split adds zeros
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0u;
        }
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          if (c0 + j < P.xrows)
            asm volatile("st.shared::cluster.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(raddr + (c0 + j) * 4),
                         "f"(__uint_as_float(r[j])), "f"(__uint_as_float(r[j + 1])), "f"(__uint_as_float(r[j + 2])),
                         "f"(__uint_as_float(r[j + 3]))
                         : "memory");
      }
    }
    // Barrier 2: every partial row has arrived; each CTA sums and writes its rows.
    asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
    const int tok = min(P.xrows, P.m - m0), tok4 = (tok + 3) / 4;
    if (P.epi == EPI_SWIGLU) {  // a thread per (gate, up) row pair and 4 tokens
      const int pairs = rows_per / 2;
      for (int i = tid; i < pairs * tok4; i += kThreads) {
        const int lp = i % pairs, j = 4 * (i / pairs);
        float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
        for (int c = 0; c < nsplit; ++c) {
          const float4 vg = *reinterpret_cast<const float4*>(red + (c * rows_per + 2 * lp) * rs + j);
          const float4 vu = *reinterpret_cast<const float4*>(red + (c * rows_per + 2 * lp + 1) * rs + j);
          g.x += vg.x; g.y += vg.y; g.z += vg.z; g.w += vg.w;
          u.x += vu.x; u.y += vu.y; u.z += vu.z; u.w += vu.w;
        }
        const float ga[4] = {g.x, g.y, g.z, g.w}, ua[4] = {u.x, u.y, u.z, u.w};
        const int col = (n0 + static_cast<int>(rank) * rows_per) / 2 + lp;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (j + e < tok) P.y[static_cast<size_t>(m0 + j + e) * P.ldy + col] = swiglu_value(ga[e], ua[e]);
      }
    }
    for (int i = tid; P.epi != EPI_SWIGLU && i < rows_per * tok4; i += kThreads) {
      const int lr = i % rows_per, j = 4 * (i / rows_per);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c = 0; c < nsplit; ++c) {
        const float4 v = *reinterpret_cast<const float4*>(red + (c * rows_per + lr) * rs + j);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const float a[4] = {acc.x, acc.y, acc.z, acc.w};
      const int col = n0 + static_cast<int>(rank) * rows_per + lr;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rw = m0 + j + e;
        if (j + e < tok) P.y[static_cast<size_t>(rw) * P.ldy + col] = epi_value(P, a[e], rw, col);
      }
    }
  } else if (ok && P.swap) {
    // lane = weight row n0 + 32q + lane, columns = tokens m0 ..
    const int col = n0 + 32 * q + lane;
    for (int c0 = 0; c0 < P.xrows; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tl + c0, r);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int rw = m0 + c0 + j;
        if (P.epi == EPI_SWIGLU) {  // gate row in the even lane, its up row in the next
          const float up = __shfl_down_sync(0xffffffffu, __uint_as_float(r[j]), 1);
          if ((lane & 1) == 0 && rw < P.m)
            P.y[static_cast<size_t>(rw) * P.ldy + col / 2] = swiglu_value(__uint_as_float(r[j]), up);
        } else if (rw < P.m) {
          P.y[static_cast<size_t>(rw) * P.ldy + col] = epi_value(P, __uint_as_float(r[j]), rw, col);
        }
      }
    }
  } else if (ok) {
    // lane = token m0 + 32q + lane, columns = weight rows n0 ..
    const int rw = m0 + 32 * q + lane;
#pragma unroll 1
    for (int c0 = 0; c0 < kRows; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tl + c0, r);
      if (rw < P.m && P.epi == EPI_SWIGLU) {  // 16 (gate, up) pairs -> 16 outputs
        __half* yrow = P.y + static_cast<size_t>(rw) * P.ldy + (n0 + c0) / 2;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = 16 * g + 4 * e;  // pairs (i, i + 1), (i + 2, i + 3)
            const __half2 hh = __halves2half2(swiglu_value(__uint_as_float(r[i]), __uint_as_float(r[i + 1])),
                                              swiglu_value(__uint_as_float(r[i + 2]), __uint_as_float(r[i + 3])));
            o[e] = *reinterpret_cast<const uint32_t*>(&hh);
          }
          *reinterpret_cast<uint4*>(yrow + 8 * g) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      } else if (rw < P.m) {
        __half* yrow = P.y + static_cast<size_t>(rw) * P.ldy + n0 + c0;
#pragma unroll
        for (int g = 0; g < 4; ++g) {  // 8 columns per 16-byte store
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int cc = n0 + c0 + 8 * g + 2 * e;
            const __half2 hh = __halves2half2(epi_value(P, __uint_as_float(r[8 * g + 2 * e]), rw, cc),
                                              epi_value(P, __uint_as_float(r[8 * g + 2 * e + 1]), rw, cc + 1));
            o[e] = *reinterpret_cast<const uint32_t*>(&hh);
          }
          *reinterpret_cast<uint4*>(yrow + 8 * g) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
}

// Epilogue of 32 accumulator columns of a prefill tile: lane = token row rw,
// r[j] = column n0 + c0 + j (a weight row; gate/up pairs for SwiGLU).
__device__ __forceinline__ void tiles_epilogue_chunk(const Params& P, const uint32_t (&r)[32], int rw, int n0,
                                                     int c0) {
  if (rw < P.m && P.epi == EPI_SWIGLU) {  // 16 (gate, up) pairs -> 16 outputs
    __half* yrow = P.y + static_cast<size_t>(rw) * P.ldy + (n0 + c0) / 2;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 16 * g + 4 * e;  // pairs (i, i + 1), (i + 2, i + 3)
        const __half2 hh = __halves2half2(swiglu_value(__uint_as_float(r[i]), __uint_as_float(r[i + 1])),
                                          swiglu_value(__uint_as_float(r[i + 2]), __uint_as_float(r[i + 3])));
        o[e] = *reinterpret_cast<const uint32_t*>(&hh);
      }
      *reinterpret_cast<uint4*>(yrow + 8 * g) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else if (rw < P.m && P.epi == EPI_RESIDUAL) {  // residual rows read 16 bytes at a time
    __half* yrow = P.y + static_cast<size_t>(rw) * P.ldy + n0 + c0;
    const __half* rrow = P.res + static_cast<size_t>(rw) * P.ldr + n0 + c0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint4 rv = *reinterpret_cast<const uint4*>(rrow + 8 * g);
      const __half2* r2 = reinterpret_cast<const __half2*>(&rv);
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __half2 hh = __hadd2(r2[e], __floats2half2_rn(__uint_as_float(r[8 * g + 2 * e]),
                                                            __uint_as_float(r[8 * g + 2 * e + 1])));
        o[e] = *reinterpret_cast<const uint32_t*>(&hh);
      }
      *reinterpret_cast<uint4*>(yrow + 8 * g) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else if (rw < P.m) {
    __half* yrow = P.y + static_cast<size_t>(rw) * P.ldy + n0 + c0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {  // 8 columns per 16-byte store
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int cc = n0 + c0 + 8 * g + 2 * e;
        const __half2 hh = __halves2half2(epi_value(P, __uint_as_float(r[8 * g + 2 * e]), rw, cc),
                                          epi_value(P, __uint_as_float(r[8 * g + 2 * e + 1]), rw, cc + 1));
        o[e] = *reinterpret_cast<const uint32_t*>(&hh);
      }
      *reinterpret_cast<uint4*>(yrow + 8 * g) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Prefill tiles (MT x 128 tokens x 128 weight rows): one ring of S stages,
// each holding the MT X tiles, the step's packed W (128 rows x 32 bytes, one
// TMA box) and the dequantised W tile, which serves the MT token halves (one
// M = 128 MMA each, accumulators side by side in TMEM).  Warp 0 lane 0
// loads, warps 2-5 dequantise and then run the epilogue, warp 1 lane 0
// issues the MMAs.
template <int MT>
__global__ void __launch_bounds__(kThreads) w4a16_gemm_tiles_kernel(const __grid_constant__ Params P) {
  extern __shared__ unsigned char smem_raw[];
  const int S = P.xstages;
  constexpr int kX = MT * 128 * 128;  // X tile bytes of a stage (MT halves of 128 tokens)
  constexpr uint32_t kCols = 128 * MT;  // TMEM columns
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* xs = base;
  unsigned char* wd = xs + static_cast<size_t>(S) * kX;
  unsigned char* wr = wd + static_cast<size_t>(S) * kWTileBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(wr + static_cast<size_t>(S) * kStepBytes);
  uint64_t* deq = full + kMaxStages;
  uint64_t* empty = deq + kMaxStages;
  uint64_t* done = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_v = abort_flag;

  lmps_pdl_trigger();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kRows, m0 = blockIdx.y * 128 * MT;
  const int ksteps = P.k / kBK;
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&deq[i], 128);
      mbar_init(&empty[i], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      lmps_pdl_wait();  // X is the previous kernel's output
      int issued = 0;
      RingPos ps;
      for (int kt = 0; kt < ksteps; ++kt, ps.next(S)) {
        const int s = ps.slot;
        if (kt >= S && !mbar_wait(&empty[s], ps.phase ^ 1u, P.error, abort_v)) break;
        mbar_expect_tx(&full[s], static_cast<uint32_t>(kX + kStepBytes));
#pragma unroll
        for (int mh = 0; mh < MT; ++mh)
          tma_load_2d(xs + static_cast<size_t>(s) * kX + mh * 128 * 128, &P.tx, kt * kBK, m0 + 128 * mh, &full[s]);
        tma_load_2d(wr + static_cast<size_t>(s) * kStepBytes, &P.tw, kt * (kBK / 2), n0, &full[s]);
        issued = kt + 1;
      }
      for (int kt = max(0, issued - S); kt < issued; ++kt) {  // every issued copy lands before exit
        const uint64_t t0 = globaltimer();
        while (!mbar_try(&full[kt % S], (kt / S) & 1))
          if (globaltimer() - t0 > kTimeoutNs) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      const uint32_t idesc = idesc_f16(128, 128);
      RingPos ps;
      for (int kt = 0; kt < ksteps; ++kt, ps.next(S)) {
        const int s = ps.slot;
        if (!mbar_wait(&deq[s], ps.phase, P.error, abort_v)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t bd = sw128_desc(smem_u32(wd + static_cast<size_t>(s) * kWTileBytes));
#pragma unroll
        for (int mh = 0; mh < MT; ++mh) {
          const uint64_t ad = sw128_desc(smem_u32(xs + static_cast<size_t>(s) * kX + mh * 128 * 128));
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j)
            mma_f16(tmem + 128 * mh, ad + 2 * j, bd + 2 * j, idesc, (kt > 0 || j > 0) ? 1u : 0u);
        }
        mma_commit(&empty[s]);
      }
      mma_commit(done);
    }
  } else {
    // ---- dequantisation (thread t = weight row n0 + t); the full barrier of
    // a stage completes only after the MMAs that last read it (the producer
    // waited for them before refilling), so wd[s] is free once it is full
    const int t = tid - 64, sw = t & 7, hs = q4t::half_swap(t);
    const uint32_t* srow = reinterpret_cast<const uint32_t*>(P.s + static_cast<size_t>(n0 + t) * (P.k / 32));
    uint32_t sc_next = ksteps > 0 ? __ldg(srow) : 0u;
    RingPos ps;
    for (int kt = 0; kt < ksteps; ++kt, ps.next(S)) {
      const int s = ps.slot;
      const uint32_t sc = sc_next;
      if (kt + 1 < ksteps) sc_next = __ldg(srow + kt + 1);
      if (!mbar_wait(&full[s], ps.phase, P.error, abort_v)) break;
      // row t's two 16-byte halves, swapped by the 32-byte TMA swizzle when (t >> 2) & 1
      const uint4* raw = reinterpret_cast<const uint4*>(wr + static_cast<size_t>(s) * kStepBytes + t * 32);
      const uint4 g0 = raw[hs], g1 = raw[hs ^ 1];
      const __half2 sc2 = *reinterpret_cast<const __half2*>(&sc);
      const __half2 s0 = __low2half2(sc2), s1 = __high2half2(sc2);
      unsigned char* row = wd + static_cast<size_t>(s) * kWTileBytes + t * 128;
      *reinterpret_cast<uint4*>(row + ((0 ^ sw) << 4)) = dequant8(g0.x, s0);
      *reinterpret_cast<uint4*>(row + ((1 ^ sw) << 4)) = dequant8(g0.y, s0);
      *reinterpret_cast<uint4*>(row + ((2 ^ sw) << 4)) = dequant8(g0.z, s0);
      *reinterpret_cast<uint4*>(row + ((3 ^ sw) << 4)) = dequant8(g0.w, s0);
      *reinterpret_cast<uint4*>(row + ((4 ^ sw) << 4)) = dequant8(g1.x, s1);
      *reinterpret_cast<uint4*>(row + ((5 ^ sw) << 4)) = dequant8(g1.y, s1);
      *reinterpret_cast<uint4*>(row + ((6 ^ sw) << 4)) = dequant8(g1.z, s1);
      *reinterpret_cast<uint4*>(row + ((7 ^ sw) << 4)) = dequant8(g1.w, s1);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&deq[s]);
    }
    // ---- epilogue: lane = token m0 + 32q + lane, columns = weight rows n0 ..
    lmps_pdl_wait();  // before any read of the residual or write of Y
    const bool ok = ksteps > 0 && mbar_wait(done, 0, P.error, abort_v);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int q = warp & 3;
#pragma unroll 1
    for (int mh = 0; ok && mh < MT; ++mh) {
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * q) << 16) + 128 * mh;
    const int rw = m0 + 128 * mh + 32 * q + lane;
    {
#pragma unroll 1
      for (int c0 = 0; c0 < kRows; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tl + c0, r);
        tiles_epilogue_chunk(P, r, rw, n0, c0);
      }
    }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

// Persistent prefill GEMM (256 tokens x 128 weight rows per tile): one CTA
// per SM walks the tiles blockIdx.x, + gridDim.x, .. (weight-row tiles
// fastest, so the CTAs at work share the same X rows in L2).  The load ring
// and the dequantisation run on across tile boundaries; the accumulators
// alternate between two 256-column halves of TMEM, so the epilogue of a tile
// (warps 6-9) overlaps the main loop of the next; no per-tile prologue.
//   warp 0 lane 0: TMA loads (two X boxes + the packed W of a K step per stage)
//   warp 1 lane 0: tcgen05.mma (two M = 128 halves per K step), commits
//   warps 2-5:     dequantisation (thread t = weight row t of the tile)
//   warps 6-9:     epilogue (warp w reads TMEM lanes 32 (w % 4) ..)
constexpr int kPThreads = 320;
constexpr int kPMT = 2;
__global__ void __launch_bounds__(kPThreads, 1) w4a16_gemm_persist_kernel(const __grid_constant__ Params P) {
  extern __shared__ unsigned char smem_raw[];
  const int S = P.xstages;
  constexpr int kX = kPMT * 128 * 128;
  constexpr uint32_t kAcc = 128 * kPMT;  // TMEM columns of one accumulator set
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* xs = base;
  unsigned char* wd = xs + static_cast<size_t>(S) * kX;
  unsigned char* wr = wd + static_cast<size_t>(S) * kWTileBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(wr + static_cast<size_t>(S) * kStepBytes);
  uint64_t* deq = full + kMaxStages;
  uint64_t* empty = deq + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;  // [2] accumulator set complete
  uint64_t* tempty = tfull + 2;          // [2] accumulator set drained by the epilogue
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_v = abort_flag;

  lmps_pdl_trigger();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ksteps = P.k / kBK;
  const int n_tiles = P.n / kRows, m_tiles = (P.m + 128 * kPMT - 1) / (128 * kPMT);
  const int tiles = n_tiles * m_tiles;
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&deq[i], 128);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * kAcc)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      lmps_pdl_wait();  // X is the previous kernel's output
      RingPos ps;
      int issued = 0;  // K steps issued over all tiles
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        const int n0 = (tile % n_tiles) * kRows, m0 = (tile / n_tiles) * 128 * kPMT;
        for (int kt = 0; kt < ksteps; ++kt, ps.next(S)) {
          const int s = ps.slot;
          if (issued >= S && !mbar_wait(&empty[s], ps.phase ^ 1u, P.error, abort_v)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], static_cast<uint32_t>(kX + kStepBytes));
#pragma unroll
          for (int mh = 0; mh < kPMT; ++mh)
            tma_load_2d(xs + static_cast<size_t>(s) * kX + mh * 128 * 128, &P.tx, kt * kBK, m0 + 128 * mh, &full[s]);
          tma_load_2d(wr + static_cast<size_t>(s) * kStepBytes, &P.tw, kt * (kBK / 2), n0, &full[s]);
          ++issued;
        }
      }
      for (int g = max(0, issued - S); g < issued; ++g) {  // every issued copy lands before exit
        const uint64_t t0 = globaltimer();
        while (!mbar_try(&full[g % S], (g / S) & 1))
          if (globaltimer() - t0 > kTimeoutNs) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      const uint32_t idesc = idesc_f16(128, 128);
      RingPos ps;
      uint32_t uses[2] = {0u, 0u};
      int buf = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, buf ^= 1) {
        // the epilogue has drained this accumulator set's previous tile
        if (!mbar_wait(&tempty[buf], (uses[buf] & 1u) ^ 1u, P.error, abort_v)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + static_cast<uint32_t>(buf) * kAcc;
        for (int kt = 0; kt < ksteps; ++kt, ps.next(S)) {
          const int s = ps.slot;
          if (!mbar_wait(&deq[s], ps.phase, P.error, abort_v)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t bd = sw128_desc(smem_u32(wd + static_cast<size_t>(s) * kWTileBytes));
#pragma unroll
          for (int mh = 0; mh < kPMT; ++mh) {
            const uint64_t ad = sw128_desc(smem_u32(xs + static_cast<size_t>(s) * kX + mh * 128 * 128));
#pragma unroll
            for (int j = 0; j < kBK / 16; ++j)
              mma_f16(acc + 128 * mh, ad + 2 * j, bd + 2 * j, idesc, (kt > 0 || j > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&tfull[buf]);
        ++uses[buf];
      }
      // every MMA issued above finishes before the tensor memory is freed
      mma_commit(done);
      const uint64_t t0 = globaltimer();
      while (!mbar_try(done, 0u))
        if (globaltimer() - t0 > kTimeoutNs) break;
    }
  } else if (warp < 6) {
    // ---- dequantisation (thread t = weight row n0 + t of the current tile);
    // a stage's full barrier completes only after the MMAs that last read it
    // (the producer waited for them before refilling), so wd[s] is free then
    const int t = tid - 64, sw = t & 7, hs = q4t::half_swap(t);
    RingPos ps;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int n0 = (tile % n_tiles) * kRows;
      const uint32_t* srow = reinterpret_cast<const uint32_t*>(P.s + static_cast<size_t>(n0 + t) * (P.k / 32));
      uint32_t sc_next = ksteps > 0 ? __ldg(srow) : 0u;
      bool ok = true;
      for (int kt = 0; kt < ksteps; ++kt, ps.next(S)) {
        const int s = ps.slot;
        const uint32_t sc = sc_next;
        if (kt + 1 < ksteps) sc_next = __ldg(srow + kt + 1);
        if (!mbar_wait(&full[s], ps.phase, P.error, abort_v)) {
          ok = false;
          break;
        }
        // row t's two 16-byte halves, swapped by the 32-byte TMA swizzle when (t >> 2) & 1
        const uint4* raw = reinterpret_cast<const uint4*>(wr + static_cast<size_t>(s) * kStepBytes + t * 32);
        const uint4 g0 = raw[hs], g1 = raw[hs ^ 1];
        const __half2 sc2 = *reinterpret_cast<const __half2*>(&sc);
        const __half2 s0 = __low2half2(sc2), s1 = __high2half2(sc2);
        unsigned char* row = wd + static_cast<size_t>(s) * kWTileBytes + t * 128;
        *reinterpret_cast<uint4*>(row + ((0 ^ sw) << 4)) = dequant8(g0.x, s0);
        *reinterpret_cast<uint4*>(row + ((1 ^ sw) << 4)) = dequant8(g0.y, s0);
        *reinterpret_cast<uint4*>(row + ((2 ^ sw) << 4)) = dequant8(g0.z, s0);
        *reinterpret_cast<uint4*>(row + ((3 ^ sw) << 4)) = dequant8(g0.w, s0);
        *reinterpret_cast<uint4*>(row + ((4 ^ sw) << 4)) = dequant8(g1.x, s1);
        *reinterpret_cast<uint4*>(row + ((5 ^ sw) << 4)) = dequant8(g1.y, s1);
        *reinterpret_cast<uint4*>(row + ((6 ^ sw) << 4)) = dequant8(g1.z, s1);
        *reinterpret_cast<uint4*>(row + ((7 ^ sw) << 4)) = dequant8(g1.w, s1);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&deq[s]);
      }
      if (!ok) break;
    }
  } else {
    // ---- epilogue (warps 6-9): lane = token m0 + 128 mh + 32 q + lane
    lmps_pdl_wait();  // before any read of the residual or write of Y
    const int q = warp & 3;
    uint32_t uses[2] = {0u, 0u};
    int buf = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, buf ^= 1) {
      const int n0 = (tile % n_tiles) * kRows, m0 = (tile / n_tiles) * 128 * kPMT;
      if (!mbar_wait(&tfull[buf], uses[buf] & 1u, P.error, abort_v)) break;
      ++uses[buf];
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll 1
      for (int mh = 0; mh < kPMT; ++mh) {
        const uint32_t tl = tmem + static_cast<uint32_t>(buf) * kAcc + (static_cast<uint32_t>(32 * q) << 16) + 128 * mh;
        const int rw = m0 + 128 * mh + 32 * q + lane;
#pragma unroll 1
        for (int c0 = 0; c0 < kRows; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tl + c0, r);
          tiles_epilogue_chunk(P, r, rw, n0, c0);
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&tempty[buf]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kAcc) : "memory");
}

static size_t tiles_smem_bytes(int stages, int mt) {
  return static_cast<size_t>(stages) * (mt * 128 * 128 + kWTileBytes + kStepBytes) + 1024 +
         (3 * kMaxStages + 1) * sizeof(uint64_t) + 16;
}

static size_t ring_bytes(int xrows, int xstages, int dstages, int wslots, int spb) {
  return static_cast<size_t>(wslots) * kStepBytes * spb + static_cast<size_t>(xstages) * xrows * 128 +
         static_cast<size_t>(dstages) * kWTileBytes;
}
static size_t smem_bytes(int xrows, int xstages, int dstages, int wslots, int spb) {
  return ring_bytes(xrows, xstages, dstages, wslots, spb) + 1024 + (6 * kMaxStages + 1) * sizeof(uint64_t) +
         kScaleAhead * 128 * sizeof(uint32_t) + 16;
}

}  // namespace w4
}  // namespace lmps

using namespace lmps;
using tc::encode_2d;

// Token-tile geometry: fewer than 128 tokens run one token tile with the
// weight rows as the MMA's M (rounded up to 16 tokens); otherwise 128-token
// tiles.
// The swapped decode tile (weights as M, tokens as N, split K) below 128
// tokens -- except for very wide outputs (the LM head) from 33 tokens on,
// where the 128-token prefill tile (rows past m read as zero) is faster:
// 64 x 151936 x 1536 116 -> 89 us, 100 tokens 142 -> 92 us (16 tokens
// 95 -> 151 us, so not there).
static bool w4_swap(int m, int n) { return m < 128 && (m <= 32 || n < 65536); }
static int w4_xrows(int m, int n) { return w4_swap(m, n) ? ((m + 15) / 16) * 16 : 128; }

extern "C" size_t lmps_w4a16_gemm_workspace_size(int m, int n) {
  (void)m;
  (void)n;
  return 0;  // split K reduces inside a thread-block cluster
}

// K splits of the swap tiles: about two CTAs per SM, a power of two up to the
// portable cluster size, at least two 64-wide K steps per split.
static int choose_splits(int tiles, int ksteps, int sms) {
  const int want = (2 * sms) / (tiles > 0 ? tiles : 1);
  int s = 1;
  while (2 * s <= want && 2 * s <= w4::kMaxSplits && 2 * (2 * s) <= ksteps) s *= 2;
  return s;
}

extern "C" int lmps_w4a16_gemm(const uint16_t* x, int ldx, const uint8_t* packed, const uint16_t* scales,
                               const uint16_t* bias, const uint16_t* residual, int ldr, uint16_t* y, int ldy,
                               int m, int n, int k, int epilogue, int32_t* error, void* workspace,
                               size_t workspace_bytes, void* stream) {
  LMPS_CHECK_ARG(x && packed && scales && y && error);
  LMPS_CHECK_ARG(m >= 1 && n >= 1 && k >= 1);
  if (n % w4::kRows != 0 || k % w4::kBK != 0) return LMPS_ERR_UNSUPPORTED;
  LMPS_CHECK_ARG(epilogue >= w4::EPI_NONE && epilogue <= w4::EPI_SWIGLU);
  LMPS_CHECK_ARG(epilogue != w4::EPI_BIAS || bias);
  LMPS_CHECK_ARG(epilogue != w4::EPI_RESIDUAL || (residual && ldr >= n && ldr % 8 == 0 && lmps_aligned(residual, 16)));
  const int ncols = epilogue == w4::EPI_SWIGLU ? n / 2 : n;  // Y columns
  LMPS_CHECK_ARG(ldx >= k && ldx % 8 == 0 && ldy >= ncols && ldy % 8 == 0);
  LMPS_CHECK_ARG(lmps_aligned(x, 16) && lmps_aligned(y, 16) && lmps_aligned(packed, 16) && lmps_aligned(scales, 4));
  w4::Params P{};
  const int xr = w4_xrows(m, n);
  P.swap = w4_swap(m, n) ? 1 : 0;
  P.xrows = xr;
  // decode tiles stream packed W in 128-byte row pieces (4 K steps per load);
  // prefill tiles in 32-byte pieces, one per K step
  P.wspb = P.swap ? 4 : 1;
  if (!encode_2d(&P.tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, static_cast<uint64_t>(k), static_cast<uint64_t>(m),
                 static_cast<uint64_t>(ldx) * 2, w4::kBK, static_cast<uint32_t>(xr), CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&P.tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, packed, static_cast<uint64_t>(k / 2), static_cast<uint64_t>(n),
                 static_cast<uint64_t>(k / 2), static_cast<uint32_t>(w4::kBK / 2 * P.wspb), w4::kRows,
                 P.wspb == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B))
    return LMPS_ERR_INVALID_ARGUMENT;
  P.s = reinterpret_cast<const __half*>(scales);
  P.bias = reinterpret_cast<const __half*>(bias);
  P.res = reinterpret_cast<const __half*>(residual);
  P.ldr = ldr;
  P.y = reinterpret_cast<__half*>(y);
  P.ldy = ldy;
  P.m = m;
  P.n = n;
  P.k = k;
  P.epi = epilogue;
  P.error = error;
  const int ksteps = k / w4::kBK, mt = (m + xr - 1) / xr, nt = n / w4::kRows;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  (void)workspace;
  (void)workspace_bytes;
  if (!P.swap) {  // prefill tiles: the single-ring kernel
    if (m >= 256) {  // persistent: 256 tokens x 128 rows per tile, four stages, one CTA per SM
      P.xstages = 4;
      const size_t smem = w4::tiles_smem_bytes(P.xstages, 2) + 64;  // + the accumulator-set barriers
      const int st_attr = lmps_max_dyn_smem<w4::w4a16_gemm_persist_kernel>(static_cast<int>(smem));
      if (st_attr != LMPS_OK) return st_attr;
      const int tiles = nt * ((m + 255) / 256);
      return lmps_launch_pdl(w4::w4a16_gemm_persist_kernel, dim3(tiles < sms ? tiles : sms), dim3(w4::kPThreads),
                             smem, lmps_stream(stream), P);
    }
    P.xstages = 3;  // three stages, two CTAs per SM
    const size_t smem = w4::tiles_smem_bytes(P.xstages, 1);
    const int st_attr = lmps_max_dyn_smem<w4::w4a16_gemm_tiles_kernel<1>>(static_cast<int>(smem));
    if (st_attr != LMPS_OK) return st_attr;
    return lmps_launch_pdl(w4::w4a16_gemm_tiles_kernel<1>, dim3(nt, mt), dim3(w4::kThreads), smem,
                           lmps_stream(stream), P);
  }
  const int splits = choose_splits(nt, ksteps, sms);
  P.ksteps_per_split = (ksteps + splits - 1) / splits;  // trailing splits may get none: they add zeros
  // Two CTAs per SM: 2 packed-W blocks (8 K steps), 3 dequantised-W stages,
  // then as many X tiles as fit (up to 8).
  int max_smem = 0;
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t budget = static_cast<size_t>(max_smem) / 2 - 1024;
  const int spb = P.wspb;
  int xst = 2, dst = 3, wsl = 2;
  if (w4::smem_bytes(xr, xst, dst, wsl, spb) > budget) dst = 2;
  if (w4::smem_bytes(xr, xst, dst, wsl, spb) > budget) xst = 2;
  if (w4::smem_bytes(xr, xst, dst, wsl, spb) > budget) return LMPS_ERR_UNSUPPORTED;
  while (xst < w4::kMaxStages && w4::smem_bytes(xr, xst + 1, dst, wsl, spb) <= budget) ++xst;
  P.xstages = xst;
  P.dstages = dst;
  P.wslots = wsl;
  const size_t smem = w4::smem_bytes(xr, xst, dst, wsl, spb);
  // the split partial rows reuse the pipeline buffers
  if (splits > 1 &&
      static_cast<size_t>(w4::kRows) * (xr + 4) * sizeof(float) > w4::ring_bytes(xr, xst, dst, wsl, spb))
    return LMPS_ERR_UNSUPPORTED;
  cudaError_t e = cudaFuncSetAttribute(w4::w4a16_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return static_cast<int>(e);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(nt, mt, splits);
  cfg.blockDim = dim3(w4::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = lmps_stream(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = static_cast<unsigned>(splits);
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, w4::w4a16_gemm_kernel, P);
  if (e != cudaSuccess) return static_cast<int>(e);
  return lmps_launch_status();
}
