// Causal prefill attention over the paged KV cache (flash attention with
// mma.sync tiles): the attention.metal / softmax.metal / attn_sum.metal stages
// of runners/engine.py:202-212 for every prompt position of every sequence at
// once -- query p of a sequence attends to positions 0..p.
//
// One CTA per (sequence, KV head, 32 query positions), 2 x G warps: warp
// (j, h) takes query head kvh*G + h for the 16 positions q0 + 16 j .. + 15,
// so every staged key/value block serves all G query heads of the KV head
// (GQA, attention.metal:23) and both 16-row halves.  Key/value blocks of 64
// positions stream through two shared-memory stages with cp.async: block
// kb + 1 is in flight while block kb is computed.  Per block a warp computes
// S = Q K^T (8 n-tiles x 8 k-steps of m16n8k16, fp16 in / fp32 accumulate),
// the causal mask, its rows' online softmax in fp32, and O += P V (16
// n-tiles x 4 k-steps; P taken straight from the score fragments).  Scores
// use the reference's scale literal 0.088388.  The longest query tiles are
// scheduled first (blockIdx.x counts down from the last tile).
#include <cmath>

#include "common.cuh"

namespace lmps {
namespace pf {

constexpr int kHD = 128;
constexpr int kQT = 32;          // query positions per CTA (two 16-row halves)
constexpr int kKB = 64;          // key positions per block
constexpr int kMaxG = 6;           // 2 x 6 warps at up to 168 registers each
constexpr int kStride = kHD + 8; // padded shared row (halves): conflict-free ldmatrix rows
constexpr int kStageHalves = 2 * kKB * kStride;               // K and V of one block
constexpr int kSmemBytes = 2 * kStageHalves * 2;              // two stages

struct Params {
  const __half* q;  // [batch * seq_len, n_q_heads * 128], rotated
  int ldq;
  const __half* kp;
  const __half* vp;
  const int32_t* bt;  // [batch, max_pages]
  int max_pages, page_size;
  __half* out;      // [batch * seq_len, n_q_heads * 128]
  int ldo;
  int seq_len, n_q, n_kv;
};

__device__ __forceinline__ void ldsm_x2(const void* p, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_trans(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2_trans(const void* p, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 16 bytes global -> shared through cp.async; src_bytes 0 zero-fills the
// destination without reading (src must still be a valid address).
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

// Stage K and V rows of positions k0 .. k0+63 (zero rows past `last`).
__device__ __forceinline__ void stage_block(const Params& P, const int32_t* bt, int kvh, int k0, int last,
                                            __half* st) {
  for (int i = threadIdx.x; i < 2 * kKB * (kHD / 8); i += blockDim.x) {
    const int kv = i / (kKB * (kHD / 8));
    const int r = (i / (kHD / 8)) % kKB, c = i % (kHD / 8);
    const int p = k0 + r;
    const __half* pool = kv ? P.vp : P.kp;
    const __half* src = pool;
    uint32_t bytes = 0u;
    if (p <= last) {
      src = pool + ((static_cast<size_t>(bt[p / P.page_size]) * P.n_kv + kvh) * P.page_size + p % P.page_size) *
                       kHD + 8 * c;
      bytes = 16u;
    }
    cp_async16(st + (kv * kKB + r) * kStride + 8 * c, src, bytes);
  }
}

__global__ void __launch_bounds__(2 * kMaxG * 32, 1) prefill_attn_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(16) __half smem[];
  const int qt = gridDim.x - 1 - blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = P.n_q / P.n_kv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g8 = lane >> 2, t4 = lane & 3, mi = lane >> 3, r8 = lane & 7;
  const int half = warp / G, hw = warp - half * G;
  const int q0 = qt * kQT + 16 * half;  // this warp's first query position
  const int head = kvh * G + hw;
  const size_t row0 = static_cast<size_t>(b) * P.seq_len;
  const int32_t* bt = P.bt + static_cast<size_t>(b) * P.max_pages;
  const int last = min(qt * kQT + kQT, P.seq_len) - 1;  // last query (and key) position of the CTA
  const int nblk = last / kKB + 1;
  // the first block's copies go out before anything else
  stage_block(P, bt, kvh, 0, last, smem);
  asm volatile("cp.async.commit_group;" ::: "memory");

  // Q fragments (A operand, rows = query positions q0..q0+15, 8 k-steps over the dims)
  uint32_t qa[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    qa[ks][0] = qa[ks][1] = qa[ks][2] = qa[ks][3] = 0u;
    const int r0 = q0 + g8, r1 = q0 + g8 + 8;
    const int c = head * kHD + 16 * ks + 2 * t4;
    if (r0 < P.seq_len) {
      const __half* qr = P.q + (row0 + r0) * P.ldq + c;
      qa[ks][0] = *reinterpret_cast<const uint32_t*>(qr);
      qa[ks][2] = *reinterpret_cast<const uint32_t*>(qr + 8);
    }
    if (r1 < P.seq_len) {
      const __half* qr = P.q + (row0 + r1) * P.ldq + c;
      qa[ks][1] = *reinterpret_cast<const uint32_t*>(qr);
      qa[ks][3] = *reinterpret_cast<const uint32_t*>(qr + 8);
    }
  }
  float o[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // rows g8, g8+8 (m in the log2 domain)
  const int qp0 = q0 + g8, qp1 = q0 + g8 + 8;
  for (int kb = 0; kb < nblk; ++kb) {
    const int k0 = kb * kKB;
    if (kb + 1 < nblk) stage_block(P, bt, kvh, k0 + kKB, last, smem + ((kb + 1) & 1) * kStageHalves);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // block kb landed (this thread's copies)
    __syncthreads();                                        // ... and every thread's
    const __half* ks_ = smem + (kb & 1) * kStageHalves;
    const __half* vs_ = ks_ + kKB * kStride;
    if (k0 <= q0 + 15) {  // (warp-uniform) some key of the block is visible to this warp's rows
      // S = Q K^T: 8 n-tiles of 8 key positions; one ldmatrix.x4 brings the
      // B fragments of two k-steps (dims 16 ks2 .. 16 ks2 + 31)
      float s[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
        for (int ks2 = 0; ks2 < 8; ks2 += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(ks_ + (8 * j + r8) * kStride + 16 * ks2 + 8 * mi, b0, b1, b2, b3);
          mma_16816(s[j], qa[ks2][0], qa[ks2][1], qa[ks2][2], qa[ks2][3], b0, b1);
          mma_16816(s[j], qa[ks2 + 1][0], qa[ks2 + 1][1], qa[ks2 + 1][2], qa[ks2 + 1][3], b2, b3);
        }
      }
      // causal mask (key position <= query position) and the scores in the
      // log2 domain, scale * log2(e) folded in: exp(scale s - scale m) is
      // exp2(s' - m') with s' = s * scale * log2(e)
      constexpr float kScaleLog2 = kAttnScale * 1.4426950408889634f;
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kp = k0 + 8 * j + 2 * t4 + e;
          s[j][e] = (kp <= qp0) ? s[j][e] * kScaleLog2 : -INFINITY;
          s[j][2 + e] = (kp <= qp1) ? s[j][2 + e] * kScaleLog2 : -INFINITY;
          mx0 = fmaxf(mx0, s[j][e]);
          mx1 = fmaxf(mx1, s[j][2 + e]);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      // rows past the sequence or with no visible key yet keep -inf: guard the exponentials
      const float al0 = (mn0 == -INFINITY) ? 1.0f : exp2f(m0 - mn0);
      const float al1 = (mn1 == -INFINITY) ? 1.0f : exp2f(m1 - mn1);
      float su0 = 0.0f, su1 = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s[j][0] = (mn0 == -INFINITY) ? 0.0f : exp2f(s[j][0] - mn0);
        s[j][1] = (mn0 == -INFINITY) ? 0.0f : exp2f(s[j][1] - mn0);
        s[j][2] = (mn1 == -INFINITY) ? 0.0f : exp2f(s[j][2] - mn1);
        s[j][3] = (mn1 == -INFINITY) ? 0.0f : exp2f(s[j][3] - mn1);
        su0 += s[j][0] + s[j][1];
        su1 += s[j][2] + s[j][3];
      }
      su0 += __shfl_xor_sync(0xffffffffu, su0, 1);
      su0 += __shfl_xor_sync(0xffffffffu, su0, 2);
      su1 += __shfl_xor_sync(0xffffffffu, su1, 1);
      su1 += __shfl_xor_sync(0xffffffffu, su1, 2);
      l0 = l0 * al0 + su0;
      l1 = l1 * al1 + su1;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        o[nt][0] *= al0;
        o[nt][1] *= al0;
        o[nt][2] *= al1;
        o[nt][3] *= al1;
      }
      // O += P V over the block's 4 k-steps of 16 keys; P straight from the score fragments
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t pa0 = pack2(s[2 * kk][0], s[2 * kk][1]), pa1 = pack2(s[2 * kk][2], s[2 * kk][3]);
        const uint32_t pa2 = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        const uint32_t pa3 = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int nt = 0; nt < 16; nt += 2) {  // one ldmatrix.x4.trans: dims 8 nt .. 8 nt + 15
          uint32_t b0, b1, b2, b3;
          ldsm_x4_trans(vs_ + (16 * kk + (mi & 1) * 8 + r8) * kStride + 8 * nt + 8 * (mi >> 1), b0, b1, b2, b3);
          mma_16816(o[nt], pa0, pa1, pa2, pa3, b0, b1);
          mma_16816(o[nt + 1], pa0, pa1, pa2, pa3, b2, b3);
        }
      }
    }
    __syncthreads();  // every warp is done with this stage before it is refilled
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int c = head * kHD + 8 * nt + 2 * t4;
    if (qp0 < P.seq_len)
      *reinterpret_cast<uint32_t*>(P.out + (row0 + qp0) * P.ldo + c) = pack2(o[nt][0] * inv0, o[nt][1] * inv0);
    if (qp1 < P.seq_len)
      *reinterpret_cast<uint32_t*>(P.out + (row0 + qp1) * P.ldo + c) = pack2(o[nt][2] * inv1, o[nt][3] * inv1);
  }
}

}  // namespace pf
}  // namespace lmps

using namespace lmps;

extern "C" int lmps_prefill_attention(const uint16_t* q, int ldq, const uint16_t* k_pool, const uint16_t* v_pool,
                                      const int32_t* block_table, int max_pages, int page_size, uint16_t* out,
                                      int ldo, int batch, int seq_len, int n_q_heads, int n_kv_heads, int head_dim,
                                      void* stream) {
  LMPS_CHECK_ARG(q && k_pool && v_pool && block_table && out);
  LMPS_CHECK_ARG(batch >= 1 && seq_len >= 1 && max_pages >= 1 && page_size >= 1 && n_kv_heads >= 1);
  LMPS_CHECK_ARG(n_q_heads % n_kv_heads == 0 && seq_len <= max_pages * page_size);
  if (head_dim != pf::kHD || n_q_heads / n_kv_heads > pf::kMaxG) return LMPS_ERR_UNSUPPORTED;
  LMPS_CHECK_ARG(ldq >= n_q_heads * head_dim && ldo >= n_q_heads * head_dim && ldq % 2 == 0 && ldo % 2 == 0);
  LMPS_CHECK_ARG(lmps_aligned(q, 4) && lmps_aligned(out, 4) && lmps_aligned(k_pool, 16) && lmps_aligned(v_pool, 16));
  pf::Params P{};
  P.q = reinterpret_cast<const __half*>(q);
  P.ldq = ldq;
  P.kp = reinterpret_cast<const __half*>(k_pool);
  P.vp = reinterpret_cast<const __half*>(v_pool);
  P.bt = block_table;
  P.max_pages = max_pages;
  P.page_size = page_size;
  P.out = reinterpret_cast<__half*>(out);
  P.ldo = ldo;
  P.seq_len = seq_len;
  P.n_q = n_q_heads;
  P.n_kv = n_kv_heads;
  const int st_attr = lmps_max_dyn_smem<pf::prefill_attn_kernel>(pf::kSmemBytes);
  if (st_attr != LMPS_OK) return st_attr;
  dim3 grid((seq_len + pf::kQT - 1) / pf::kQT, n_kv_heads, batch);
  const int threads = 2 * 32 * (n_q_heads / n_kv_heads);
  pf::prefill_attn_kernel<<<grid, threads, pf::kSmemBytes, lmps_stream(stream)>>>(P);
  return lmps_launch_status();
}
