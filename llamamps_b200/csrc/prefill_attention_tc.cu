// Causal prefill attention on the 5th-generation tensor cores (tcgen05.mma,
// accumulators in tensor memory): the attention.metal / softmax.metal /
// attn_sum.metal stages of runners/engine.py:202-212 for every prompt
// position at once -- query p of a sequence attends to positions 0..p.
//
// One CTA per (128-query tile, pair of query heads of one KV head, KV head,
// sequence); the longest query tiles are scheduled first.  Per 64-key tile
// of the paged cache:
//   * warp 0 (one lane) loads the tile's K and V rows with plain (non-
//     multicast) TMA from this GPU's own pool into a three-stage ring (128-byte
//     swizzle; the queries of both heads once at the start);
//   * warp 1 (one lane) issues S_h = Q_h K^T (M = 128 queries, N = 64 keys,
//     K = 128 dims) into TMEM, then, once the softmax has written P_h,
//     O_h += P_h V (M = 128, N = 128 dims, K = 64 keys; V read MN-major
//     straight from the cache rows); S and P have two buffers per head, so
//     S of tile i + 1 is ready while the softmax works on tile i and the
//     softmax never waits for the O MMA of the tile before;
//   * warps 2-5 for head 0 and 6-9 for head 1 (thread = query row, its TMEM
//     lane) read a row of S_h in one TMEM load, apply the scale
//     0.088388 and the causal mask (diagonal tiles only), keep the running
//     max and sum in fp32 (exp2), write P_h as fp16 into a 128-byte-swizzled
//     K-major tile, and rescale O_h in TMEM only when the row max grows by
//     more than 2^8 (between rescales P stays below 2^8, so fp16 P and fp32
//     O are exact enough); at the end they read O_h, divide by the sum and
//     store fp16.
// The two heads' softmax warpgroups run side by side while the tensor core
// works on the other head.  Every mbarrier wait is bounded (error flag, no
// hang).
#include <cmath>

#include "common.cuh"
#include "tcgen05.cuh"

namespace lmps {
namespace fa {

using namespace tc;

constexpr int kD = 128;        // head dim
constexpr int kQ = 128;        // queries per tile (TMEM lanes)
constexpr int kKV = 64;        // keys per tile
constexpr int kH = 2;          // query heads per CTA
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-5 / 6-9 softmax + epilogue of head 0 / 1
constexpr int kStages = 3;     // K/V tiles in shared memory: loads run two tiles ahead
constexpr int kQSub = kQ * 128;    // 64 dims of a Q tile: 128 rows x 128 bytes
constexpr int kKVSub = kKV * 128;  // 64 dims of a K or V tile: 64 rows x 128 bytes
constexpr int kPTile = kQ * 128;   // P tile: 128 rows x 64 keys fp16
constexpr int kOffK = kH * 2 * kQSub;          // 64 KB of Q
constexpr int kOffV = kOffK + kStages * 2 * kKVSub;  // the stages of K
constexpr int kOffP = kOffV + kStages * 2 * kKVSub;  // the stages of V
constexpr int kOffBar = kOffP + kH * 2 * kPTile;  // two P buffers per head
constexpr int kSmemBytes = kOffBar + 24 * 8 + 1024;  // (kOffBar + 192 + 1024 <= 227 KB)  // barriers, TMEM slot, abort flag; 1024-byte alignment slack
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;    // S of head h, buffer u at columns 64 (2 h + u)
constexpr uint32_t kColO = 256;  // O_h at columns 256 + 128 h
constexpr float kScaleLog2 = 0.088388f * 1.4426950408889634f;  // attention.metal:40 scale, base 2
constexpr float kRescaleLog2 = 8.0f;

// 2^x with the hardware approximation (ex2.approx.ftz: relative error ~2^-22,
// far below the fp16 rounding P gets next).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct Params {
  CUtensorMap tq;  // q [batch * seq_len, ldq] fp16, box {64, 128}
  CUtensorMap tk;  // K pool [n_pages * n_kv * page_size, 128] fp16, box {64, 64}
  CUtensorMap tv;
  const int32_t* bt;  // [batch, max_pages]
  __half* out;        // [batch * seq_len, ldo]
  int ldo, seq_len, n_q, n_kv, max_pages, page_size, n_qtiles, head_pairs;
  int* error;
};

__global__ void __launch_bounds__(kThreads, 1) prefill_attn_tc_kernel(const __grid_constant__ Params P) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* sq = base;
  unsigned char* sk = base + kOffK;
  unsigned char* sv = base + kOffV;
  unsigned char* sp = base + kOffP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kOffBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;              // [kStages]
  uint64_t* kv_empty = kv_full + kStages;    // [kStages]
  // per head and buffer u (tile i uses buffer i & 1): S_h ready, P_h written
  // (and S_h read), O_h += P_h V of the tile done
  uint64_t* s_full = kv_empty + kStages;     // [kH][2]
  uint64_t* p_full = s_full + 2 * kH;        // [kH][2]
  uint64_t* o_done = p_full + 2 * kH;        // [kH][2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2 * kH);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_v = abort_flag;

  lmps_pdl_trigger();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // work item: the query tile varies slowest, longest first
  const int per_tile = static_cast<int>(gridDim.x) / P.n_qtiles;  // items per query tile
  const int qt = P.n_qtiles - 1 - static_cast<int>(blockIdx.x) / per_tile;
  int rest = static_cast<int>(blockIdx.x) % per_tile;
  const int hp = rest % P.head_pairs;
  rest /= P.head_pairs;
  const int kvh = rest % P.n_kv, b = rest / P.n_kv;
  const int G = P.n_q / P.n_kv;
  const int h0 = kvh * G + 2 * hp;  // first query head of the pair
  const int q0 = qt * kQ;
  const int qend = min(P.seq_len, q0 + kQ);
  const int nt = (qend + kKV - 1) / kKV;  // key tiles 0 .. nt-1 reach the tile's last query

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int u = 0; u < 2 * kH; ++u) {
      mbar_init(&s_full[u], 1);
      mbar_init(&p_full[u], kQ);
      mbar_init(&o_done[u], 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (tid == 32) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&P.tq)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&P.tk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&P.tv)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  lmps_pdl_wait();  // the queries and the cache rows come from the previous kernels

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      mbar_expect_tx(q_full, kH * 2 * kQSub);
      for (int h = 0; h < kH; ++h)
        for (int dh = 0; dh < 2; ++dh)
          tma_load_2d(sq + (2 * h + dh) * kQSub, &P.tq, (h0 + h) * kD + 64 * dh, b * P.seq_len + q0, q_full);
      const int32_t* bt = P.bt + static_cast<size_t>(b) * P.max_pages;
      int issued = 0;
      for (int i = 0; i < nt; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait(&kv_empty[s], (i / kStages - 1) & 1, P.error, abort_v)) break;
        const int k0 = i * kKV;
        const int row = (__ldg(bt + k0 / P.page_size) * P.n_kv + kvh) * P.page_size + k0 % P.page_size;
        mbar_expect_tx(&kv_full[s], 4 * kKVSub);
        for (int dh = 0; dh < 2; ++dh) {
          tma_load_2d(sk + (2 * s + dh) * kKVSub, &P.tk, 64 * dh, row, &kv_full[s]);
          tma_load_2d(sv + (2 * s + dh) * kKVSub, &P.tv, 64 * dh, row, &kv_full[s]);
        }
        issued = i + 1;
      }
      // every issued copy lands before the CTA may exit
      {
        const uint64_t t0 = globaltimer();
        while (!mbar_try(q_full, 0))
          if (globaltimer() - t0 > kTimeoutNs) break;
      }
      for (int i = max(0, issued - kStages); i < issued; ++i) {
        const uint64_t t0 = globaltimer();
        while (!mbar_try(&kv_full[i % kStages], (i / kStages) & 1))
          if (globaltimer() - t0 > kTimeoutNs) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      const uint32_t id_s = idesc_f16(kQ, kKV), id_o = idesc_f16(kQ, kD) | kBMajorMN;
      auto issue_s = [&](int h, int s, int u) {  // S_h (buffer u) = Q_h K^T over 8 k-steps of 16 dims
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint64_t a = sw128_desc(smem_u32(sq + (2 * h + (j >> 2)) * kQSub)) + 2 * (j & 3);
          const uint64_t bk = sw128_desc(smem_u32(sk + (2 * s + (j >> 2)) * kKVSub)) + 2 * (j & 3);
          mma_f16(tmem + kColS + kKV * (2 * h + u), a, bk, id_s, j > 0 ? 1u : 0u);
        }
      };
      auto issue_o = [&](int h, int s, int u, bool acc) {  // O_h += P_h (buffer u) V over 4 k-steps of 16 keys
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t a = sw128_desc(smem_u32(sp + (2 * h + u) * kPTile)) + 2 * j;
          const uint64_t bv = sw128_mn_desc(smem_u32(sv + (2 * s) * kKVSub + 2048 * j), kKVSub);
          mma_f16(tmem + kColO + kD * h, a, bv, id_o, (acc || j > 0) ? 1u : 0u);
        }
      };
      // S of tiles 0 and 1 up front (both S buffers are free), then per tile
      // and head: O += P V once the softmax wrote P, and S of the tile two
      // ahead into the buffer the softmax just finished reading.
      bool ok = mbar_wait(q_full, 0, P.error, abort_v);
      for (int i = 0; ok && i < 2 && i < nt; ++i) {
        ok = mbar_wait(&kv_full[i], 0, P.error, abort_v);
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (int h = 0; h < kH; ++h) {
          issue_s(h, i, i);
          mma_commit(&s_full[2 * h + i]);
        }
      }
      for (int i = 0; ok && i < nt; ++i) {
        const int s = i % kStages, u = i & 1, s2 = (i + 2) % kStages;
        for (int h = 0; h < kH; ++h) {
          if (!mbar_wait(&p_full[2 * h + u], (i >> 1) & 1, P.error, abort_v)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          issue_o(h, s, u, i > 0);
          mma_commit(&o_done[2 * h + u]);
          if (i + 2 < nt) {
            if (h == 0 && !mbar_wait(&kv_full[s2], ((i + 2) / kStages) & 1, P.error, abort_v)) {
              ok = false;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            issue_s(h, s2, u);
            mma_commit(&s_full[2 * h + u]);
          }
        }
        if (ok) mma_commit(&kv_empty[s]);  // this tile's K and V are free once the MMAs above are done
      }
    }
  } else {
    // ---- softmax of head h = (warp - 2) / 4 (thread = query row r, TMEM lane r)
    const int h = (warp - 2) >> 2, quad = warp & 3, r = 32 * quad + lane, qi = q0 + r;
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * quad) << 16);
    const uint32_t to = tl + kColO + kD * h;
    float m_used = -INFINITY, l = 0.0f;  // running max (scaled, base 2) and sum
    bool ok = true;
    for (int i = 0; ok && i < nt; ++i) {
      const int k0 = i * kKV;
      const bool diag = k0 + kKV - 1 > q0;  // (warp-uniform) the tile reaches past some query of the tile
      const int u = i & 1;                  // S / P buffer of this tile
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[2 * h + u], (i >> 1) & 1, P.error, abort_v));
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // the row's 64 raw scores in one TMEM load; their max (the scale is positive)
      uint32_t sc[64];
      tmem_ld64(tl + kColS + kKV * (2 * h + u), sc);
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four chains
      if (diag) {
#pragma unroll
        for (int c = 0; c < kKV; ++c)
          if (k0 + c <= qi) mx[c & 3] = fmaxf(mx[c & 3], __uint_as_float(sc[c]));
      } else {
#pragma unroll
        for (int c = 0; c < kKV; ++c) mx[c & 3] = fmaxf(mx[c & 3], __uint_as_float(sc[c]));
      }
      float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      mt *= kScaleLog2;
      if (i >= 2) {  // O_h of tile i - 2 is done: its P buffer may be rewritten
        ok = __all_sync(0xffffffffu, mbar_wait(&o_done[2 * h + u], ((i - 2) >> 1) & 1, P.error, abort_v));
        if (!ok) break;
      }
      const float mnew = fmaxf(m_used, mt);
      const bool grow = mnew > m_used + kRescaleLog2;  // (always on the first tile)
      const float alpha = grow ? exp2f(m_used - mnew) : 1.0f;
      if (i > 0 && __any_sync(0xffffffffu, grow)) {  // warp-wide read-modify-write of O_h
        // once O_h += P V of the previous tile (and so every earlier one) is done
        ok = __all_sync(0xffffffffu, mbar_wait(&o_done[2 * h + (u ^ 1)], ((i - 1) >> 1) & 1, P.error, abort_v));
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll 1
        for (int cc = 0; cc < kD; cc += 32) {
          uint32_t o[32];
          tmem_ld32(to + cc, o);
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_st32(to + cc, o);
        }
      }
      if (grow) {
        l *= alpha;
        m_used = mnew;
      }
      // P = 2^(s * scale - m) as fp16 into row r of the swizzled K-major P tile
      const float nm = -m_used;
      float sm[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // four chains
      unsigned char* prow = sp + (2 * h + u) * kPTile + r * 128;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {  // 16-byte chunk ch: keys 8 ch .. 8 ch + 7
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = 8 * ch + 2 * e;
          float a0 = fast_exp2(fmaf(__uint_as_float(sc[c]), kScaleLog2, nm));
          float a1 = fast_exp2(fmaf(__uint_as_float(sc[c + 1]), kScaleLog2, nm));
          if (diag) {
            a0 = k0 + c <= qi ? a0 : 0.0f;
            a1 = k0 + c + 1 <= qi ? a1 : 0.0f;
          }
          sm[e] += a0 + a1;
          const __half2 hh = __floats2half2_rn(a0, a1);
          pk[e] = *reinterpret_cast<const uint32_t*>(&hh);
        }
        *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l += (sm[0] + sm[1]) + (sm[2] + sm[3]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> the tensor core
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&p_full[2 * h + u]);
    }
    // ---- epilogue: O_h / l, fp16, this row of the output
    if (ok)  // the last O_h += P V (and so every earlier one) done
      ok = __all_sync(0xffffffffu, mbar_wait(&o_done[2 * h + ((nt - 1) & 1)], ((nt - 1) >> 1) & 1, P.error, abort_v));
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      __half* orow = P.out + static_cast<size_t>(b * P.seq_len + qi) * P.ldo + (h0 + h) * kD;
#pragma unroll 1
      for (int cc = 0; cc < kD; cc += 32) {
        uint32_t o[32];
        tmem_ld32(to + cc, o);
        if (qi < qend) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __half2 hh = __floats2half2_rn(__uint_as_float(o[8 * g + 2 * e]) * inv,
                                                   __uint_as_float(o[8 * g + 2 * e + 1]) * inv);
              w[e] = *reinterpret_cast<const uint32_t*>(&hh);
            }
            *reinterpret_cast<uint4*>(orow + cc + 8 * g) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

}  // namespace fa
}  // namespace lmps

using namespace lmps;

extern "C" int lmps_prefill_attention_tcgen05(const uint16_t* q, int ldq, const uint16_t* k_pool,
                                              const uint16_t* v_pool, int n_pages, const int32_t* block_table,
                                              int max_pages, int page_size, uint16_t* out, int ldo, int batch,
                                              int seq_len, int n_q_heads, int n_kv_heads, int head_dim,
                                              int32_t* error, void* stream) {
  LMPS_CHECK_ARG(q && k_pool && v_pool && block_table && out && error);
  LMPS_CHECK_ARG(batch >= 1 && seq_len >= 1 && n_pages >= 1 && max_pages >= 1 && page_size >= 1);
  LMPS_CHECK_ARG(n_kv_heads >= 1 && n_q_heads % n_kv_heads == 0);
  LMPS_CHECK_ARG(static_cast<long long>(seq_len) <= static_cast<long long>(max_pages) * page_size);
  const int G = n_q_heads / n_kv_heads;
  // 64-key tiles inside one page, head pairs, 128-dim heads
  if (head_dim != fa::kD || page_size % fa::kKV != 0 || G % fa::kH != 0) return LMPS_ERR_UNSUPPORTED;
  LMPS_CHECK_ARG(ldq >= n_q_heads * head_dim && ldq % 8 == 0 && ldo >= n_q_heads * head_dim && ldo % 8 == 0);
  LMPS_CHECK_ARG(lmps_aligned(q, 16) && lmps_aligned(k_pool, 16) && lmps_aligned(v_pool, 16) &&
                 lmps_aligned(out, 16));
  fa::Params P{};
  const uint64_t pool_rows = static_cast<uint64_t>(n_pages) * n_kv_heads * page_size;
  if (!tc::encode_2d(&P.tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, q, static_cast<uint64_t>(n_q_heads) * head_dim,
                     static_cast<uint64_t>(batch) * seq_len, static_cast<uint64_t>(ldq) * 2, 64, fa::kQ,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      !tc::encode_2d(&P.tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, k_pool, head_dim, pool_rows, head_dim * 2, 64,
                     fa::kKV, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !tc::encode_2d(&P.tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, v_pool, head_dim, pool_rows, head_dim * 2, 64,
                     fa::kKV, CU_TENSOR_MAP_SWIZZLE_128B))
    return LMPS_ERR_INVALID_ARGUMENT;
  P.bt = block_table;
  P.out = reinterpret_cast<__half*>(out);
  P.ldo = ldo;
  P.seq_len = seq_len;
  P.n_q = n_q_heads;
  P.n_kv = n_kv_heads;
  P.max_pages = max_pages;
  P.page_size = page_size;
  P.n_qtiles = (seq_len + fa::kQ - 1) / fa::kQ;
  P.head_pairs = G / fa::kH;
  P.error = error;
  const int st_attr = lmps_max_dyn_smem<fa::prefill_attn_tc_kernel>(fa::kSmemBytes);
  if (st_attr != LMPS_OK) return st_attr;
  const long long ctas = static_cast<long long>(P.n_qtiles) * P.head_pairs * n_kv_heads * batch;
  if (ctas > 0x7FFFFFFFLL) return LMPS_ERR_UNSUPPORTED;
  return lmps_launch_pdl(fa::prefill_attn_tc_kernel, dim3(static_cast<unsigned>(ctas)), dim3(fa::kThreads),
                         static_cast<size_t>(fa::kSmemBytes), lmps_stream(stream), P);
}
