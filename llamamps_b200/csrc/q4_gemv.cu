// Q4 GEMV family for sm_100a.
//
// Restates kernels/quant_matmul.metal:15-69 (`gemv_q4_0`) for B200:
//  * the matrix is streamed once from HBM with 128-bit non-allocating loads;
//    one 16-byte load is exactly one Q4 group (32 nibbles, one fp16 scale);
//  * LPR lanes cooperate on a row (LPR = the largest power of two <= 32 that
//    divides the row's group count, so no lane idles on 1536- or 8960-wide
//    rows), each walking groups sub, sub+LPR, ... so a warp's loads cover
//    contiguous 16*LPR-byte runs of 32/LPR rows;
//  * nibbles become exact fp16 codes (n - 8) with the 0x6400 magic-exponent
//    trick, are multiplied with the fp16 activations by the sm_100
//    mixed-precision FMA (fp16 x fp16 -> fp32 accumulate, exact products), and
//    each group's partial sum is scaled by the group scale held in a register;
//  * the LPR-lane partial sums are combined with a warp-shuffle reduction;
//  * activations (<= 8 rows of <= 8960) are staged once per CTA in shared
//    memory with an XOR swizzle on 16-byte chunks so the strided group reads
//    are bank-conflict free.
// Epilogues fuse what follows the GEMV in runners/engine.py: q/k/v bias,
// residual add (residual.metal), SwiGLU over a gate/up pair (swiglu.metal),
// the LM-head argmax (engine.py:180-181), and -- for two-way tensor
// parallelism -- the all-reduce of the partial o/down products with the
// residual add, over NVLink peer memory in the same kernel (EPI_TP2).
#include "common.cuh"

namespace lmps {

enum GemvEpi { EPI_PLAIN = 0, EPI_BIAS = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_ARGMAX = 4, EPI_TP2 = 5 };

struct GemvParams {
  const uint8_t* w;
  const __half* s;
  const uint8_t* w2;  // EPI_SWIGLU: up matrix
  const __half* s2;
  const __half* x;
  int ldx;
  __half* y;
  int ldy;
  const __half* bias;           // EPI_BIAS
  const __half* res;            // EPI_RESID
  unsigned long long* keys;     // EPI_ARGMAX
  int rows, k, batch;
  // EPI_TP2: y = this rank's partial [batch, ldy]; x_io the residual (same
  // layout), updated to x + (partial + the peer's partial)
  __half* x_io;
  __half* tp_peer_recv;         // the peer's two receive slots of the site
  const __half* tp_recv;        // this rank's
  uint32_t* tp_peer_flags;
  const uint32_t* tp_flags;
  uint32_t* tp_seen;            // this rank's call counts of the site, per CTA
  int32_t* tp_error;
  int tp_slot;                  // elements per receive slot
  unsigned long long tp_wait_ns;  // limit of the peer wait
};

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / kWarp;

// fp32 d = a * b + c with fp16 a, b (exact product), sm_100 mixed precision.
__device__ __forceinline__ float fma_h_h_f(uint16_t a, uint16_t b, float c) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}

__device__ __forceinline__ uint16_t lo16(uint32_t v) { return static_cast<uint16_t>(v & 0xFFFFu); }
__device__ __forceinline__ uint16_t hi16(uint32_t v) { return static_cast<uint16_t>(v >> 16); }

// Codes of the 8 nibbles of w as fp16 pairs: c0 = (e0, e4), c1 = (e1, e5),
// c2 = (e2, e6), c3 = (e3, e7), each value exactly n - 8.
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t& c0, uint32_t& c1, uint32_t& c2,
                                        uint32_t& c3) {
  const uint32_t kMask = 0x000F000Fu, kMagic = 0x64006400u;  // fp16 1024.0 in both halves
  const __half2 kBias = __halves2half2(__ushort_as_half(0xE408u), __ushort_as_half(0xE408u));
  uint32_t t0 = (w & kMask) | kMagic;
  uint32_t t1 = ((w >> 4) & kMask) | kMagic;
  uint32_t t2 = ((w >> 8) & kMask) | kMagic;
  uint32_t t3 = ((w >> 12) & kMask) | kMagic;
  __half2 h0 = __hadd2(*reinterpret_cast<__half2*>(&t0), kBias);  // (1024 + n) - 1032
  __half2 h1 = __hadd2(*reinterpret_cast<__half2*>(&t1), kBias);
  __half2 h2 = __hadd2(*reinterpret_cast<__half2*>(&t2), kBias);
  __half2 h3 = __hadd2(*reinterpret_cast<__half2*>(&t3), kBias);
  c0 = *reinterpret_cast<uint32_t*>(&h0);
  c1 = *reinterpret_cast<uint32_t*>(&h1);
  c2 = *reinterpret_cast<uint32_t*>(&h2);
  c3 = *reinterpret_cast<uint32_t*>(&h3);
}

// acc += sum_{e<8} code(w, e) * x_e, x = 8 fp16 values (uint4 = 4 half2).
__device__ __forceinline__ float dot8(uint32_t w, const uint4& xv, float acc) {
  uint32_t c0, c1, c2, c3;
  unpack8(w, c0, c1, c2, c3);
  acc = fma_h_h_f(lo16(c0), lo16(xv.x), acc);  // e0 * x0
  acc = fma_h_h_f(lo16(c1), hi16(xv.x), acc);  // e1 * x1
  acc = fma_h_h_f(lo16(c2), lo16(xv.y), acc);  // e2 * x2
  acc = fma_h_h_f(lo16(c3), hi16(xv.y), acc);  // e3 * x3
  acc = fma_h_h_f(hi16(c0), lo16(xv.z), acc);  // e4 * x4
  acc = fma_h_h_f(hi16(c1), hi16(xv.z), acc);  // e5 * x5
  acc = fma_h_h_f(hi16(c2), lo16(xv.w), acc);  // e6 * x6
  acc = fma_h_h_f(hi16(c3), hi16(xv.w), acc);  // e7 * x7
  return acc;
}

// Swizzled position of 16-byte chunk `vi` of a staged activation row: chunks
// are permuted inside each 128-byte line by XOR with the line index.
__device__ __forceinline__ int xswz(int vi) { return (vi & ~7) | ((vi & 7) ^ ((vi >> 3) & 7)); }

// Dot product of one Q4 group (16 bytes) with the matching 32 activations.
__device__ __forceinline__ float group_dot(const uint4& wv, const uint4* xrow, int c) {
  const int v0 = c * 4;
  uint4 x0 = xrow[xswz(v0 + 0)];
  uint4 x1 = xrow[xswz(v0 + 1)];
  uint4 x2 = xrow[xswz(v0 + 2)];
  uint4 x3 = xrow[xswz(v0 + 3)];
  float a0 = dot8(wv.x, x0, 0.0f);
  float a1 = dot8(wv.y, x1, 0.0f);
  a0 = dot8(wv.z, x2, a0);
  a1 = dot8(wv.w, x3, a1);
  return a0 + a1;
}

template <int LPR, int NB, int EPI>
__global__ void __launch_bounds__(kGemvThreads) q4_gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint4* xs = reinterpret_cast<uint4*>(smem_raw);  // [NB][k/8] swizzled 16-byte chunks
  const int k = p.k;
  // EPI_TP2: thread 0's decisions reach the CTA through __syncthreads_or
  // (no static shared memory: the dynamic limit is set to the maximum)
  bool tp_go = false;
  uint32_t tp_want = 0;
  size_t tp_sl = 0;
  if constexpr (EPI == EPI_TP2) {
    // one reading of the error word per CTA (an earlier exchange failed: leave)
    if (threadIdx.x == 0) tp_go = *reinterpret_cast<volatile int32_t*>(p.tp_error) == 0;
    tp_want = p.tp_seen[blockIdx.x] + 1u;
    tp_sl = static_cast<size_t>(tp_want & 1u) * p.tp_slot;
  }
  const int G = k / kQ4Group;
  const int vpr_real = k / 8;
  const int vpr = (vpr_real + 7) & ~7;  // row stride in chunks: whole 128-byte lines

  for (int i = threadIdx.x; i < NB * vpr; i += kGemvThreads) {
    const int b = i / vpr, c = i - b * vpr;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (b < p.batch && c < vpr_real)
      v = *reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(b) * p.ldx + c * 8);
    xs[b * vpr + xswz(c)] = v;
  }
  if constexpr (EPI == EPI_TP2) {
    if (!__syncthreads_or(tp_go)) return;
  } else {
    __syncthreads();
  }

  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  constexpr int RPW = kWarp / LPR;
  const int sub = lane % LPR;
  const int rsub = lane / LPR;
  const size_t row_bytes = static_cast<size_t>(k) / 2;

  unsigned long long best[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) best[b] = 0ull;

  for (int r0 = (blockIdx.x * kGemvWarps + warp) * RPW; r0 < p.rows;
       r0 += gridDim.x * kGemvWarps * RPW) {
    const int row = r0 + rsub;
    const bool valid = row < p.rows;
    float acc[NB], acc2[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) { acc[b] = 0.0f; acc2[b] = 0.0f; }
    if (valid) {
      const uint8_t* wrow = p.w + static_cast<size_t>(row) * row_bytes;
      const __half* srow = p.s + static_cast<size_t>(row) * G;
      const uint8_t* wrow2 = nullptr;
      const __half* srow2 = nullptr;
      if constexpr (EPI == EPI_SWIGLU) {
        wrow2 = p.w2 + static_cast<size_t>(row) * row_bytes;
        srow2 = p.s2 + static_cast<size_t>(row) * G;
      }
#pragma unroll 4
      for (int c = sub; c < G; c += LPR) {
        const uint4 wv = ld_stream_v4(wrow + static_cast<size_t>(c) * kQ4GroupBytes);
        const float sc = __half2float(srow[c]);
        uint4 wv2;
        float sc2 = 0.0f;
        if constexpr (EPI == EPI_SWIGLU) {
          wv2 = ld_stream_v4(wrow2 + static_cast<size_t>(c) * kQ4GroupBytes);
          sc2 = __half2float(srow2[c]);
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const uint4* xrow = xs + b * vpr;
          acc[b] = fmaf(sc, group_dot(wv, xrow, c), acc[b]);
          if constexpr (EPI == EPI_SWIGLU) acc2[b] = fmaf(sc2, group_dot(wv2, xrow, c), acc2[b]);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      acc[b] = segment_sum<LPR>(acc[b]);
      if constexpr (EPI == EPI_SWIGLU) acc2[b] = segment_sum<LPR>(acc2[b]);
    }
    if (valid && sub == 0) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b >= p.batch) break;
        __half* yp = p.y ? p.y + static_cast<size_t>(b) * p.ldy + row : nullptr;
        if constexpr (EPI == EPI_PLAIN) {
          *yp = __float2half_rn(acc[b]);
        } else if constexpr (EPI == EPI_BIAS) {
          *yp = __float2half_rn(acc[b] + __half2float(p.bias[row]));
        } else if constexpr (EPI == EPI_RESID) {
          // residual.metal:19 adds the fp16 GEMV output to the fp16 residual.
          const __half o = __float2half_rn(acc[b]);
          *yp = __hadd(p.res[static_cast<size_t>(b) * p.ldy + row], o);
        } else if constexpr (EPI == EPI_TP2) {
          // this rank's fp16 partial: kept, and stored into the peer's slot
          const __half o = __float2half_rn(acc[b]);
          *yp = o;
          p.tp_peer_recv[tp_sl + static_cast<size_t>(b) * p.ldy + row] = o;
        } else if constexpr (EPI == EPI_SWIGLU) {
          const float g = __half2float(__float2half_rn(acc[b]));
          const float u = __half2float(__float2half_rn(acc2[b]));
          *yp = __float2half_rn(silu_mul(g, u));
        } else {  // EPI_ARGMAX
          const __half v = __float2half_rn(acc[b]);
          if (yp) *yp = v;
          best[b] = u64_max(best[b], argmax_key(__half2float(v), static_cast<uint32_t>(row)));
        }
      }
    }
  }
  if constexpr (EPI == EPI_ARGMAX) {
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const unsigned long long m = warp_max_u64(best[b]);
      if (lane == 0 && b < p.batch && m != 0ull) atomicMax(p.keys + b, m);
    }
  }
  if constexpr (EPI == EPI_TP2) {
    // hand-off with the same CTA of the peer (same rows), then the rows of
    // this CTA: x + (own partial + the peer's), fp16, the peer computing the
    // same sums in the other order (commutative: bit-identical).  Only the
    // lanes that stored to the peer fence at system scope.
    if (sub == 0) __threadfence_system();
    __syncthreads();
    bool good = false;
    if (threadIdx.x == 0) {
      good = lmps_tp2_handshake(p.tp_peer_flags, p.tp_flags, blockIdx.x, tp_want, p.tp_error, p.tp_wait_ns);
      if (good) p.tp_seen[blockIdx.x] = tp_want;
    }
    if (!__syncthreads_or(good)) return;
    if (sub == 0) __threadfence_system();
    for (int r0 = (blockIdx.x * kGemvWarps + warp) * RPW; r0 < p.rows; r0 += gridDim.x * kGemvWarps * RPW) {
      const int row = r0 + rsub;
      if (row < p.rows && sub == 0) {
        for (int b = 0; b < p.batch; ++b) {
          const size_t i = static_cast<size_t>(b) * p.ldy + row;
          const __half s = __hadd(p.y[i], __ldcg(p.tp_recv + tp_sl + i));  // own write, same thread
          p.x_io[i] = __hadd(p.x_io[i], s);
        }
      }
    }
  }
}

__global__ void argmax_finalize_kernel(unsigned long long* keys, int32_t* ids, int batch) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) {
    const unsigned long long key = keys[b];
    ids[b] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
    keys[b] = 0ull;
  }
}

static int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

template <int LPR, int NB, int EPI>
static int launch_lpr_nb(const GemvParams& p, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(NB) * ((p.k / 8 + 7) & ~7) * 16;
  auto kern = q4_gemv_kernel<LPR, NB, EPI>;
  if (smem > 48 * 1024) {
    const int st_attr = lmps_max_dyn_smem<q4_gemv_kernel<LPR, NB, EPI>>(227 * 1024);
    if (st_attr != LMPS_OK) return st_attr;
  }
  constexpr int rows_per_cta = kGemvWarps * (kWarp / LPR);
  long long blocks = (p.rows + rows_per_cta - 1) / rows_per_cta;
  const long long cap = static_cast<long long>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  kern<<<static_cast<unsigned>(blocks), kGemvThreads, smem, st>>>(p);
  return lmps_launch_status();
}

template <int NB, int EPI>
static int launch_nb(const GemvParams& p, cudaStream_t st) {
  const int G = p.k / kQ4Group;
  if (G % 32 == 0) return launch_lpr_nb<32, NB, EPI>(p, st);
  if (G % 16 == 0) return launch_lpr_nb<16, NB, EPI>(p, st);
  if (G % 8 == 0) return launch_lpr_nb<8, NB, EPI>(p, st);
  return launch_lpr_nb<4, NB, EPI>(p, st);
}

template <int EPI>
static int launch_gemv(const GemvParams& p, cudaStream_t st) {
  if (p.batch <= 1) return launch_nb<1, EPI>(p, st);
  if (p.batch <= 2) return launch_nb<2, EPI>(p, st);
  if (p.batch <= 4) return launch_nb<4, EPI>(p, st);
  return launch_nb<8, EPI>(p, st);
}

static int check_common(const uint8_t* packed, const uint16_t* scales, const uint16_t* x, int ldx,
                        int rows, int k, int batch) {
  LMPS_CHECK_ARG(packed && scales && x);
  LMPS_CHECK_ARG(rows > 0 && k > 0 && k % kQ4Group == 0);
  LMPS_CHECK_ARG(batch >= 1 && batch <= 8);
  LMPS_CHECK_ARG(ldx >= k && ldx % 8 == 0);
  LMPS_CHECK_ARG(lmps_aligned(packed, 16) && lmps_aligned(x, 16) && lmps_aligned(scales, 2));
  return LMPS_OK;
}

static GemvParams make_params(const uint8_t* packed, const uint16_t* scales, const uint16_t* x,
                              int ldx, uint16_t* y, int ldy, int rows, int k, int batch) {
  GemvParams p{};
  p.w = packed;
  p.s = reinterpret_cast<const __half*>(scales);
  p.x = reinterpret_cast<const __half*>(x);
  p.ldx = ldx;
  p.y = reinterpret_cast<__half*>(y);
  p.ldy = ldy;
  p.rows = rows;
  p.k = k;
  p.batch = batch;
  return p;
}

}  // namespace lmps

using namespace lmps;

extern "C" int lmps_gemv_q4_0(const uint8_t* packed, const uint16_t* scales, const uint16_t* x,
                              int ldx, uint16_t* y, int ldy, int rows, int k, int batch,
                              void* stream) {
  int st = check_common(packed, scales, x, ldx, rows, k, batch);
  if (st) return st;
  LMPS_CHECK_ARG(y && ldy >= rows);
  return launch_gemv<EPI_PLAIN>(make_params(packed, scales, x, ldx, y, ldy, rows, k, batch),
                                lmps_stream(stream));
}

extern "C" int lmps_gemv_q4_bias(const uint8_t* packed, const uint16_t* scales,
                                 const uint16_t* bias, const uint16_t* x, int ldx, uint16_t* y,
                                 int ldy, int rows, int k, int batch, void* stream) {
  int st = check_common(packed, scales, x, ldx, rows, k, batch);
  if (st) return st;
  LMPS_CHECK_ARG(y && bias && ldy >= rows);
  GemvParams p = make_params(packed, scales, x, ldx, y, ldy, rows, k, batch);
  p.bias = reinterpret_cast<const __half*>(bias);
  return launch_gemv<EPI_BIAS>(p, lmps_stream(stream));
}

extern "C" int lmps_gemv_q4_residual(const uint8_t* packed, const uint16_t* scales,
                                     const uint16_t* x, int ldx, const uint16_t* residual,
                                     uint16_t* y, int ldy, int rows, int k, int batch,
                                     void* stream) {
  int st = check_common(packed, scales, x, ldx, rows, k, batch);
  if (st) return st;
  LMPS_CHECK_ARG(y && residual && ldy >= rows);
  GemvParams p = make_params(packed, scales, x, ldx, y, ldy, rows, k, batch);
  p.res = reinterpret_cast<const __half*>(residual);
  return launch_gemv<EPI_RESID>(p, lmps_stream(stream));
}

extern "C" int lmps_gemv_q4_tp2_residual(const uint8_t* packed, const uint16_t* scales, const uint16_t* a,
                                         int lda, uint16_t* x, uint16_t* part, int rows, int k, int batch,
                                         void* comm, void* peer_comm, uint32_t* seen, int site, int n_sites,
                                         int max_n, int32_t* error, unsigned long long wait_ns, void* stream) {
  int st = check_common(packed, scales, a, lda, rows, k, batch);
  if (st) return st;
  LMPS_CHECK_ARG(x && part && comm && peer_comm && seen && error);
  LMPS_CHECK_ARG(n_sites >= 1 && site >= 0 && site < n_sites && max_n >= 8 && max_n % 8 == 0);
  LMPS_CHECK_ARG(static_cast<long long>(batch) * rows <= max_n);
  LMPS_CHECK_ARG(lmps_aligned(comm, 16) && lmps_aligned(peer_comm, 16) && lmps_aligned(seen, 4));
  // every CTA must have a flag word and be resident at once (its counterpart
  // on the peer waits for it): at most kTp2MaxCtas CTAs, none grid-strided
  const int G = k / kQ4Group;
  const int lpr = G % 32 == 0 ? 32 : G % 16 == 0 ? 16 : G % 8 == 0 ? 8 : 4;
  const int rows_per_cta = kGemvWarps * (kWarp / lpr);
  if ((rows + rows_per_cta - 1) / rows_per_cta > kTp2MaxCtas) return LMPS_ERR_UNSUPPORTED;
  GemvParams p = make_params(packed, scales, a, lda, part, rows, rows, k, batch);
  const Tp2Site t = lmps_tp2_site(comm, peer_comm, site, n_sites, max_n);
  p.x_io = reinterpret_cast<__half*>(x);
  p.tp_peer_recv = reinterpret_cast<__half*>(t.peer_recv);
  p.tp_recv = reinterpret_cast<const __half*>(t.recv);
  p.tp_peer_flags = t.peer_flags;
  p.tp_flags = t.flags;
  p.tp_seen = seen + site * kTp2MaxCtas;
  p.tp_error = error;
  p.tp_slot = max_n;
  p.tp_wait_ns = wait_ns ? wait_ns : kTp2DefaultWaitNs;
  return launch_gemv<EPI_TP2>(p, lmps_stream(stream));
}

extern "C" int lmps_gemv_q4_swiglu(const uint8_t* gate_packed, const uint16_t* gate_scales,
                                   const uint8_t* up_packed, const uint16_t* up_scales,
                                   const uint16_t* x, int ldx, uint16_t* y, int ldy, int rows,
                                   int k, int batch, void* stream) {
  int st = check_common(gate_packed, gate_scales, x, ldx, rows, k, batch);
  if (st) return st;
  LMPS_CHECK_ARG(up_packed && up_scales && y && ldy >= rows && lmps_aligned(up_packed, 16));
  GemvParams p = make_params(gate_packed, gate_scales, x, ldx, y, ldy, rows, k, batch);
  p.w2 = up_packed;
  p.s2 = reinterpret_cast<const __half*>(up_scales);
  return launch_gemv<EPI_SWIGLU>(p, lmps_stream(stream));
}

extern "C" int lmps_lm_head_argmax(const uint8_t* packed, const uint16_t* scales,
                                   const uint16_t* x, int ldx, uint16_t* logits,
                                   unsigned long long* keys, int32_t* token_ids, int rows, int k,
                                   int batch, void* stream) {
  int st = check_common(packed, scales, x, ldx, rows, k, batch);
  if (st) return st;
  LMPS_CHECK_ARG(keys && token_ids && lmps_aligned(keys, 8));
  GemvParams p = make_params(packed, scales, x, ldx, logits, rows, rows, k, batch);
  p.keys = keys;
  st = launch_gemv<EPI_ARGMAX>(p, lmps_stream(stream));
  if (st) return st;
  argmax_finalize_kernel<<<1, 32, 0, lmps_stream(stream)>>>(keys, token_ids, batch);
  return lmps_launch_status();
}
