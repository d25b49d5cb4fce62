// Causal prefill attention over the paged KV cache (flash attention with
// mma.sync tiles): the attention.metal / softmax.metal / attn_sum.metal stages
// of runners/engine.py:202-212 for every prompt position of every sequence at
// once -- query p of a sequence attends to positions 0..p.
//
// One CTA per (sequence, KV head, 16 query positions); warp h takes query
// head kvh*G + h, i.e. 16 query rows.  The CTA walks the key/value blocks of
// 16 positions up to its diagonal: all warps stage the block (K and V rows of
// the KV head) in shared memory, then each warp computes S = Q K^T (2 n-tiles
// x 8 k-steps of m16n8k16, fp16 in / fp32 accumulate), the causal mask, its
// rows' online softmax in fp32, and O += P V (16 n-tiles; P reused from the
// score fragments).  Scores use the reference's scale literal 0.088388.
#include <cmath>

#include "common.cuh"

namespace lmps {
namespace pf {

constexpr int kHD = 128;
constexpr int kQT = 16;          // query positions per CTA
constexpr int kKB = 16;          // key positions per block
constexpr int kMaxG = 8;
constexpr int kStride = kHD + 8; // padded shared row (halves): conflict-free 16-byte row reads

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

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x2(const void* p, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
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

__global__ void __launch_bounds__(kMaxG * 32) prefill_attn_kernel(const __grid_constant__ Params P) {
  __shared__ __align__(16) __half ks[kKB][kStride];
  __shared__ __align__(16) __half vs[kKB][kStride];
  const int qt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = P.n_q / P.n_kv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g8 = lane >> 2, t4 = lane & 3, mi = lane >> 3, r8 = lane & 7;
  const int q0 = qt * kQT;
  const int head = kvh * G + warp;
  const bool active = warp < G;
  const size_t row0 = static_cast<size_t>(b) * P.seq_len;
  const int32_t* bt = P.bt + static_cast<size_t>(b) * P.max_pages;

  // Q fragments (A operand, rows = query positions q0..q0+15, 8 k-steps over the dims)
  uint32_t qa[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    qa[ks][0] = qa[ks][1] = qa[ks][2] = qa[ks][3] = 0u;
    if (active) {
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
  }
  float o[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // rows g8, g8+8
  const int qlast = min(q0 + kQT, P.seq_len) - 1;
  const int nblk = qlast / kKB + 1;
  for (int kb = 0; kb < nblk; ++kb) {
    const int k0 = kb * kKB;
    __syncthreads();  // the previous block's readers are done
    for (int i = threadIdx.x; i < kKB * (kHD / 8); i += blockDim.x) {
      const int r = i / (kHD / 8), c = i - r * (kHD / 8);
      const int p = k0 + r;
      uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
      if (p <= qlast) {
        const size_t off = ((static_cast<size_t>(bt[p / P.page_size]) * P.n_kv + kvh) * P.page_size + p % P.page_size) * kHD + 8 * c;
        kv = __ldcg(reinterpret_cast<const uint4*>(P.kp + off));
        vv = __ldcg(reinterpret_cast<const uint4*>(P.vp + off));
      }
      *reinterpret_cast<uint4*>(&ks[r][8 * c]) = kv;
      *reinterpret_cast<uint4*>(&vs[r][8 * c]) = vv;
    }
    __syncthreads();
    if (!active) continue;
    // S = Q K^T: two n-tiles of 8 key positions
    float s[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
      for (int ks2 = 0; ks2 < 8; ++ks2) {
        uint32_t b0, b1;
        ldsm_x2(&ks[8 * j + r8][16 * ks2 + (mi & 1) * 8], b0, b1);
        mma_16816(s[j], qa[ks2][0], qa[ks2][1], qa[ks2][2], qa[ks2][3], b0, b1);
      }
    }
    // scale, causal mask (key position <= query position), online softmax per row
    const int qp0 = q0 + g8, qp1 = q0 + g8 + 8;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kp = k0 + 8 * j + 2 * t4 + e;
        s[j][e] = (kp <= qp0) ? s[j][e] * kAttnScale : -INFINITY;
        s[j][2 + e] = (kp <= qp1) ? s[j][2 + e] * kAttnScale : -INFINITY;
      }
    }
    float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    // rows past the sequence or fully masked keep -inf: guard the exponentials
    const float al0 = (mn0 == -INFINITY) ? 1.0f : expf(m0 - mn0);
    const float al1 = (mn1 == -INFINITY) ? 1.0f : expf(m1 - mn1);
    float p[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      p[j][0] = (mn0 == -INFINITY) ? 0.0f : expf(s[j][0] - mn0);
      p[j][1] = (mn0 == -INFINITY) ? 0.0f : expf(s[j][1] - mn0);
      p[j][2] = (mn1 == -INFINITY) ? 0.0f : expf(s[j][2] - mn1);
      p[j][3] = (mn1 == -INFINITY) ? 0.0f : expf(s[j][3] - mn1);
    }
    float su0 = p[0][0] + p[0][1] + p[1][0] + p[1][1], su1 = p[0][2] + p[0][3] + p[1][2] + p[1][3];
    su0 += __shfl_xor_sync(0xffffffffu, su0, 1);
    su0 += __shfl_xor_sync(0xffffffffu, su0, 2);
    su1 += __shfl_xor_sync(0xffffffffu, su1, 1);
    su1 += __shfl_xor_sync(0xffffffffu, su1, 2);
    l0 = l0 * al0 + su0;
    l1 = l1 * al1 + su1;
    m0 = mn0;
    m1 = mn1;
    // O = O * alpha + P V; P as the A operand straight from the score fragments
    const uint32_t pa0 = pack2(p[0][0], p[0][1]), pa1 = pack2(p[0][2], p[0][3]);
    const uint32_t pa2 = pack2(p[1][0], p[1][1]), pa3 = pack2(p[1][2], p[1][3]);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      o[nt][0] *= al0;
      o[nt][1] *= al0;
      o[nt][2] *= al1;
      o[nt][3] *= al1;
      uint32_t b0, b1;
      ldsm_x2_trans(&vs[(mi & 1) * 8 + r8][8 * nt], b0, b1);
      mma_16816(o[nt], pa0, pa1, pa2, pa3, b0, b1);
    }
  }
  if (!active) return;
  const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
  const int r0 = q0 + g8, r1 = q0 + g8 + 8;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int c = head * kHD + 8 * nt + 2 * t4;
    if (r0 < P.seq_len)
      *reinterpret_cast<uint32_t*>(P.out + (row0 + r0) * P.ldo + c) = pack2(o[nt][0] * inv0, o[nt][1] * inv0);
    if (r1 < P.seq_len)
      *reinterpret_cast<uint32_t*>(P.out + (row0 + r1) * P.ldo + c) = pack2(o[nt][2] * inv1, o[nt][3] * inv1);
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
  dim3 grid((seq_len + pf::kQT - 1) / pf::kQT, n_kv_heads, batch);
  const int threads = 32 * (n_q_heads / n_kv_heads);
  pf::prefill_attn_kernel<<<grid, threads, 0, lmps_stream(stream)>>>(P);
  return lmps_launch_status();
}
