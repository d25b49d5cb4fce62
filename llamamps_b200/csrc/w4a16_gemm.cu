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
// One CTA computes a 128 x 128 tile of Y over K in steps of 64:
//   * all four warps stage the step's X tile (128 tokens x 64) and dequantise
//     the W tile (128 rows x 64, fp16 (nibble - 8) * scale) into shared
//     memory, in the 128-byte-swizzled K-major layout the tensor core reads
//     (16-byte chunk c of row r at chunk c ^ (r % 8));
//   * one thread issues four tcgen05.mma.kind::f16 (K = 16 each; M = 128
//     tokens, N = 128 rows) into the TMEM accumulator and commits them to the
//     stage's mbarrier, so the next step's staging overlaps the MMAs (two
//     stages);
//   * the epilogue reads the accumulator with tcgen05.ld (warp w owns TMEM
//     lanes 32w..32w+31 = tokens), applies bias / residual and writes fp16.
// Every mbarrier wait is bounded (error flag, no hang).
#include "common.cuh"

namespace lmps {
namespace w4 {

constexpr int kBM = 128;  // tokens per tile (TMEM lanes)
constexpr int kBN = 128;  // weight rows per tile (TMEM columns)
constexpr int kBK = 64;   // K per stage: one 128-byte swizzle atom of fp16
constexpr int kStages = 2;
constexpr int kThreads = 128;
constexpr uint32_t kTmemCols = 128;
constexpr int kTileBytes = kBM * kBK * 2;
constexpr unsigned long long kTimeoutNs = 2000000000ull;

enum Epilogue { EPI_NONE = 0, EPI_BIAS = 1, EPI_RESIDUAL = 2 };

struct Params {
  const __half* x;
  int ldx;
  const uint8_t* w;
  const __half* s;
  const __half* bias;
  const __half* res;
  int ldr;
  __half* y;
  int ldy;
  int m, n, k, epi;
  int* error;
  // split-K (gridDim.z > 1): fp32 partial tiles meet in acc32 [m_tiles*128, n]
  // (zero between calls); the last CTA of a tile finishes it and re-zeroes it
  float* acc32;
  uint32_t* tile_cnt;  // [m_tiles * n_tiles], zero between calls
  int ksteps_per_split;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled tile whose
// rows are 128 bytes and whose 8-row groups are 1024 bytes apart (the tile
// base is 1024-byte aligned): start address >> 4, leading byte offset 1
// (unused by swizzled K-major layouts), stride byte offset 1024 >> 4,
// descriptor version 1, layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor of kind::f16: fp16 A and B, fp32 D, both K-major,
// N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdesc = (1u << 4) | (static_cast<uint32_t>(kBN >> 3) << 17) |
                            (static_cast<uint32_t>(kBM >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait of the whole CTA for a phase of `bar`; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try(bar, parity)) {
    if (globaltimer() - t0 > kTimeoutNs) {
      atomicExch(err, 1);
      return false;
    }
  }
  return true;
}

// fp16 (nibble - 8) * scale of 8 consecutive elements (4 packed bytes).
__device__ __forceinline__ uint4 dequant8(uint32_t packed, __half scale) {
  const __half2 s2 = __halves2half2(scale, scale);
  uint32_t out[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t byte = (packed >> (8 * e)) & 0xFFu;
    const __half lo = __int2half_rn(static_cast<int>(byte & 0xFu) - 8);
    const __half hi = __int2half_rn(static_cast<int>(byte >> 4) - 8);
    const __half2 v = __hmul2(__halves2half2(lo, hi), s2);
    out[e] = *reinterpret_cast<const uint32_t*>(&v);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

__global__ void __launch_bounds__(kThreads, 1) w4a16_gemm_kernel(const __grid_constant__ Params P) {
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte aligned operand tiles
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* a_tiles = base;                                   // [kStages][16 KB]
  unsigned char* b_tiles = base + kStages * kTileBytes;            // [kStages][16 KB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + 2 * kStages * kTileBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kStages);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
  const int K = P.k;
  const int kbeg = blockIdx.z * P.ksteps_per_split;
  const int ksteps = min(P.ksteps_per_split, K / kBK - kbeg);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[i])) : "memory");
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  // Global loads run one K step ahead of the shared-memory stores: step
  // kt+1's X rows and packed weights are in flight while step kt is staged
  // and its MMAs are issued.
  constexpr int kPer = (kBM * kBK / 8) / kThreads;  // 16-byte chunks per thread and operand
  uint4 xr[kPer];
  uint32_t wr[kPer];
  __half sr[kPer];
  auto load_step = [&](int kt) {
    const int k0 = (kbeg + kt) * kBK;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int idx = tid + i * kThreads, r = idx >> 3, c = idx & 7;
      xr[i] = (m0 + r < P.m) ? __ldg(reinterpret_cast<const uint4*>(P.x + static_cast<size_t>(m0 + r) * P.ldx + k0 + 8 * c))
                             : make_uint4(0u, 0u, 0u, 0u);
      const size_t row = static_cast<size_t>(n0 + r);
      wr[i] = __ldg(reinterpret_cast<const uint32_t*>(P.w + row * (K / 2) + (k0 + 8 * c) / 2));
      sr[i] = P.s[row * (K / 32) + (k0 + 8 * c) / 32];
    }
  };
  if (ksteps > 0) load_step(0);
  for (int kt = 0; kt < ksteps; ++kt) {
    const int st = kt % kStages;
    if (kt >= kStages) {  // the MMAs that read this stage two steps ago are done
      if (tid == 0 && !mbar_wait(&bars[st], (kt / kStages - 1) & 1, P.error)) *abort_flag = 1;
      __syncthreads();
      if (*abort_flag) break;
    }
    unsigned char* at = a_tiles + st * kTileBytes;
    unsigned char* bt = b_tiles + st * kTileBytes;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int idx = tid + i * kThreads, r = idx >> 3, c = idx & 7;
      *reinterpret_cast<uint4*>(at + r * 128 + ((c ^ (r & 7)) << 4)) = xr[i];
      *reinterpret_cast<uint4*>(bt + r * 128 + ((c ^ (r & 7)) << 4)) = dequant8(wr[i], sr[i]);
    }
    if (kt + 1 < ksteps) load_step(kt + 1);
    // generic-proxy shared-memory writes -> visible to the tensor core
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint64_t ad = sw128_desc(smem_u32(at)), bd = sw128_desc(smem_u32(bt));
#pragma unroll
      for (int j = 0; j < kBK / 16; ++j)  // K = 16 per MMA: 32 bytes further into the swizzle atom
        mma_f16(tmem, ad + 2 * j, bd + 2 * j, (kt > 0 || j > 0) ? 1u : 0u);
      mma_commit(&bars[st]);
    }
  }
  // all MMAs done (the last commit covers every earlier one)
  if (!*abort_flag && ksteps > 0) {
    const int last = ksteps - 1;
    if (tid == 0 && !mbar_wait(&bars[last % kStages], (last / kStages) & 1, P.error)) *abort_flag = 1;
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const bool split = gridDim.z > 1;
  if (!*abort_flag && split) {
    // fp32 partial tile -> acc32 (red.add); the last split of the tile finishes it
    const int trow = m0 + warp * 32 + lane;
#pragma unroll 1
    for (int cc = 0; cc < kBN / 32; ++cc) {
      uint32_t r[32];
      const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16) + cc * 32;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
          "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
            "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
            "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
            "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
          : "r"(taddr)
          : "memory");
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (trow < P.m) {
        float* dst = P.acc32 + static_cast<size_t>(trow) * P.n + n0 + cc * 32;
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(dst + j), "f"(__uint_as_float(r[j])),
                       "f"(__uint_as_float(r[j + 1])), "f"(__uint_as_float(r[j + 2])), "f"(__uint_as_float(r[j + 3]))
                       : "memory");
      }
    }
    __threadfence();
    __syncthreads();
    uint32_t* cnt = P.tile_cnt + blockIdx.y * gridDim.x + blockIdx.x;
    if (tid == 0) *abort_flag = (atomicAdd(cnt, 1u) == gridDim.z - 1) ? 2 : 0;
    __syncthreads();
    if (*abort_flag == 2) {  // last split of this tile: epilogue from acc32, then clear it
      __threadfence();
      for (int i = tid; i < kBM * (kBN / 8); i += kThreads) {
        const int rr = i / (kBN / 8), c8 = i - rr * (kBN / 8);
        const int row = m0 + rr;
        if (row >= P.m) continue;
        float* src = P.acc32 + static_cast<size_t>(row) * P.n + n0 + 8 * c8;
        const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
        const float4 b = __ldcg(reinterpret_cast<const float4*>(src + 4));
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        *reinterpret_cast<float4*>(src) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(src + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
        const int col = n0 + 8 * c8;
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __half h0, h1;
          if (P.epi == EPI_BIAS) {
            h0 = __float2half_rn(v[2 * e] + __half2float(P.bias[col + 2 * e]));
            h1 = __float2half_rn(v[2 * e + 1] + __half2float(P.bias[col + 2 * e + 1]));
          } else if (P.epi == EPI_RESIDUAL) {
            const __half* rr2 = P.res + static_cast<size_t>(row) * P.ldr + col + 2 * e;
            h0 = __hadd(rr2[0], __float2half_rn(v[2 * e]));
            h1 = __hadd(rr2[1], __float2half_rn(v[2 * e + 1]));
          } else {
            h0 = __float2half_rn(v[2 * e]);
            h1 = __float2half_rn(v[2 * e + 1]);
          }
          const __half2 hh = __halves2half2(h0, h1);
          o[e] = *reinterpret_cast<const uint32_t*>(&hh);
        }
        *reinterpret_cast<uint4*>(P.y + static_cast<size_t>(row) * P.ldy + col) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      if (tid == 0) *cnt = 0u;
    }
  }
  if (!*abort_flag && !split) {
    const int row = m0 + warp * 32 + lane;  // token of this thread's TMEM lane
#pragma unroll 1
    for (int cc = 0; cc < kBN / 32; ++cc) {
      uint32_t r[32];
      const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16) + cc * 32;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
          "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
            "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
            "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
            "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
          : "r"(taddr)
          : "memory");
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (row < P.m) {
        const int c0 = n0 + cc * 32;
        __half* yrow = P.y + static_cast<size_t>(row) * P.ldy + c0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // 8 columns per 16-byte store
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float v0 = __uint_as_float(r[8 * q + 2 * e]), v1 = __uint_as_float(r[8 * q + 2 * e + 1]);
            __half h0, h1;
            if (P.epi == EPI_BIAS) {
              h0 = __float2half_rn(v0 + __half2float(P.bias[c0 + 8 * q + 2 * e]));
              h1 = __float2half_rn(v1 + __half2float(P.bias[c0 + 8 * q + 2 * e + 1]));
            } else if (P.epi == EPI_RESIDUAL) {
              const __half* rr = P.res + static_cast<size_t>(row) * P.ldr + c0 + 8 * q + 2 * e;
              h0 = __hadd(rr[0], __float2half_rn(v0));
              h1 = __hadd(rr[1], __float2half_rn(v1));
            } else {
              h0 = __float2half_rn(v0);
              h1 = __float2half_rn(v1);
            }
            const __half2 hh = __halves2half2(h0, h1);
            o[e] = *reinterpret_cast<const uint32_t*>(&hh);
          }
          *reinterpret_cast<uint4*>(yrow + 8 * q) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

constexpr size_t kSmemBytes = 2 * kStages * kTileBytes + 1024 /* alignment */ + 64;

}  // namespace w4
}  // namespace lmps

using namespace lmps;

extern "C" size_t lmps_w4a16_gemm_workspace_size(int m, int n) {
  if (m <= 0 || n <= 0) return 0;
  const size_t mt = (m + w4::kBM - 1) / w4::kBM, nt = (n + w4::kBN - 1) / w4::kBN;
  return mt * w4::kBM * n * sizeof(float) + ((mt * nt * sizeof(uint32_t) + 255) & ~static_cast<size_t>(255));
}

// Splits of K for a grid of `tiles` output tiles: about two CTAs per SM, at
// least two 64-wide K steps per split.
static int choose_splits(int tiles, int ksteps, int sms) {
  int s = (2 * sms) / (tiles > 0 ? tiles : 1);
  if (s > ksteps / 2) s = ksteps / 2;
  return s < 1 ? 1 : s;
}

extern "C" int lmps_w4a16_gemm(const uint16_t* x, int ldx, const uint8_t* packed, const uint16_t* scales,
                               const uint16_t* bias, const uint16_t* residual, int ldr, uint16_t* y, int ldy,
                               int m, int n, int k, int epilogue, int32_t* error, void* workspace,
                               size_t workspace_bytes, void* stream) {
  LMPS_CHECK_ARG(x && packed && scales && y && error);
  LMPS_CHECK_ARG(m >= 1 && n >= 1 && k >= 1);
  if (n % w4::kBN != 0 || k % w4::kBK != 0) return LMPS_ERR_UNSUPPORTED;
  LMPS_CHECK_ARG(epilogue >= w4::EPI_NONE && epilogue <= w4::EPI_RESIDUAL);
  LMPS_CHECK_ARG(epilogue != w4::EPI_BIAS || bias);
  LMPS_CHECK_ARG(epilogue != w4::EPI_RESIDUAL || (residual && ldr >= n));
  LMPS_CHECK_ARG(ldx >= k && ldx % 8 == 0 && ldy >= n && ldy % 8 == 0);
  LMPS_CHECK_ARG(lmps_aligned(x, 16) && lmps_aligned(y, 16) && lmps_aligned(packed, 4) && lmps_aligned(scales, 2));
  w4::Params P{};
  P.x = reinterpret_cast<const __half*>(x);
  P.ldx = ldx;
  P.w = packed;
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
  const int ksteps = k / w4::kBK, mt = (m + w4::kBM - 1) / w4::kBM, nt = n / w4::kBN;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int splits = 1;
  if (workspace && workspace_bytes >= lmps_w4a16_gemm_workspace_size(m, n)) {
    LMPS_CHECK_ARG(lmps_aligned(workspace, 256));
    splits = choose_splits(mt * nt, ksteps, sms);
  }
  P.ksteps_per_split = (ksteps + splits - 1) / splits;
  splits = (ksteps + P.ksteps_per_split - 1) / P.ksteps_per_split;
  if (splits > 1) {
    P.acc32 = reinterpret_cast<float*>(workspace);
    P.tile_cnt = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(workspace) +
                                             static_cast<size_t>(mt) * w4::kBM * n * sizeof(float));
  }
  cudaError_t e = cudaFuncSetAttribute(w4::w4a16_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(w4::kSmemBytes));
  if (e != cudaSuccess) return static_cast<int>(e);
  dim3 grid(nt, mt, splits);
  w4::w4a16_gemm_kernel<<<grid, w4::kThreads, w4::kSmemBytes, lmps_stream(stream)>>>(P);
  return lmps_launch_status();
}
