// Fused GQA decode attention over the paged fp16 KV cache (sm_100a).
//
// One kernel does what kernels/attention.metal (scores), softmax.metal and
// attn_sum.metal do in three dispatches (runners/engine.py:202-212), for a
// real cache of seq_lens[b] positions:
//   s[h, i] = (q_h . K[i, h/G]) * 0.088388,  p = softmax_i(s),  o_h = sum_i p V[i, h/G].
// Grid = (splits, kv heads, sequences).  A CTA owns one KV head of one
// sequence and a contiguous range of positions; the G query heads that share
// the KV head (GQA, attention.metal:23) are processed together so each K/V
// tile is read from HBM once.  Tiles of 64 positions are staged in shared
// memory; the softmax is computed online (running max / sum per head) and
// each split writes an unnormalised partial (acc, max, sum) that a combine
// kernel merges with a log-sum-exp rescale.  With one split the CTA writes
// the normalised output directly.
// The _rope entry point also does rope_kv_append's work (kernels/rope.metal
// on q and k, then the cache append): each CTA rotates the query heads of its
// KV head from the q|k|v row, and the split that attends the new position
// rotates and writes that K row (and the V row) into the paged cache before
// it stages its tiles.
#include <cmath>

#include "common.cuh"

namespace lmps {

constexpr int kAttnThreads = 128;
constexpr int kAttnTile = 64;
constexpr int kHeadDim = 128;
constexpr int kMaxGroup = 8;
constexpr int kKStride = kHeadDim + 8;  // padded K row (halves): conflict-free 16-byte row reads

struct AttnParams {
  const __half* q;        // [B, Hq*128] (rotated)
  const __half* k_pool;   // [pages, Hkv, page_size, 128]
  const __half* v_pool;
  const int32_t* block_table;  // [B, max_pages]
  const int32_t* seq_lens;     // [B]
  __half* out;                 // [B, Hq*128]
  float* part_o;               // [B, Hq, splits, 128]
  float2* part_ml;             // [B, Hq, splits]
  int max_pages, page_size, n_q_heads, n_kv_heads, n_splits, chunk;
  // fused RoPE + append (qkv != nullptr): q|k|v rows [B, (Hq + 2 Hkv) * 128]
  // (bias applied), position of the new token per sequence (seq_lens = pos + 1)
  const __half* qkv;
  const int32_t* pos;
  const float* inv_freq;
  int rope_style;
  __half* k_new;  // the pools, writable
  __half* v_new;
};

struct __align__(16) AttnSmem {
  float q[kMaxGroup][kHeadDim];
  __half k[kAttnTile][kKStride];
  __half v[kAttnTile][kHeadDim];
  float p[kMaxGroup][kAttnTile];
  float m[kMaxGroup];
  float l[kMaxGroup];
  float alpha[kMaxGroup];
};

__global__ void __launch_bounds__(kAttnThreads) gqa_decode_attn_kernel(const AttnParams P) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>(smem_raw);
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = P.n_q_heads / P.n_kv_heads;
  const int tid = threadIdx.x;
  const int T = P.seq_lens[b];
  const int start = split * P.chunk;
  const int end = min(T, start + P.chunk);
  const int q_dim = P.n_q_heads * kHeadDim;

  if (P.qkv != nullptr) {
    // RoPE of the G query heads (rounded to fp16 as rope_kv_append's output)
    const int kv_dim = P.n_kv_heads * kHeadDim;
    const __half* row = P.qkv + static_cast<size_t>(b) * (q_dim + 2 * kv_dim);
    const int p = P.pos[b];
    const float m = static_cast<float>(p);
    for (int t = tid; t < G * (kHeadDim / 2); t += kAttnThreads) {
      const int hl = t / (kHeadDim / 2);
      int i1, i2, fi;
      rope_pair_index(t - hl * (kHeadDim / 2), kHeadDim, P.rope_style, i1, i2, fi);
      const __half* src = row + (kvh * G + hl) * kHeadDim;
      __half a = src[i1], c = src[i2];
      rope_rotate(a, c, m * P.inv_freq[fi]);
      S.q[hl][i1] = __half2float(a);
      S.q[hl][i2] = __half2float(c);
    }
    if (p >= start && p < end) {  // this split attends the new position: append its K/V rows first
      const int page = P.block_table[static_cast<size_t>(b) * P.max_pages + p / P.page_size];
      const size_t dst = ((static_cast<size_t>(page) * P.n_kv_heads + kvh) * P.page_size + p % P.page_size) * kHeadDim;
      const __half* ksrc = row + q_dim + kvh * kHeadDim;
      for (int t = tid; t < kHeadDim / 2; t += kAttnThreads) {
        int i1, i2, fi;
        rope_pair_index(t, kHeadDim, P.rope_style, i1, i2, fi);
        __half a = ksrc[i1], c = ksrc[i2];
        rope_rotate(a, c, m * P.inv_freq[fi]);
        P.k_new[dst + i1] = a;
        P.k_new[dst + i2] = c;
      }
      for (int t = tid; t < kHeadDim; t += kAttnThreads) P.v_new[dst + t] = row[q_dim + kv_dim + kvh * kHeadDim + t];
      __threadfence();  // the rows are read back below through L2 by the tile staging
    }
  } else {
    for (int i = tid; i < G * kHeadDim; i += kAttnThreads) {
      const int h = i / kHeadDim, d = i - h * kHeadDim;
      S.q[h][d] = __half2float(P.q[static_cast<size_t>(b) * q_dim + (kvh * G + h) * kHeadDim + d]);
    }
  }
  if (tid < kMaxGroup) {
    S.m[tid] = -INFINITY;
    S.l[tid] = 0.0f;
  }
  float acc[kMaxGroup];
#pragma unroll
  for (int h = 0; h < kMaxGroup; ++h) acc[h] = 0.0f;
  __syncthreads();

  const int32_t* bt = P.block_table + static_cast<size_t>(b) * P.max_pages;
  for (int t0 = start; t0 < end; t0 += kAttnTile) {
    const int n = min(kAttnTile, end - t0);
    // Stage K and V rows of this tile: 16 threads per 256-byte row.  All of a
    // thread's loads are issued before any of its shared-memory stores, so
    // the tile costs one memory round trip, not one per row it stages.
    constexpr int kPer = kAttnTile * (kHeadDim / 8) / kAttnThreads;
    uint4 kv[kPer], vv[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = tid + j * kAttnThreads, r = i / (kHeadDim / 8), c = i - r * (kHeadDim / 8);
      kv[j] = make_uint4(0u, 0u, 0u, 0u);
      vv[j] = kv[j];
      if (r < n) {
        const int pos = t0 + r;
        const int page = __ldg(bt + pos / P.page_size);
        const size_t off = ((static_cast<size_t>(page) * P.n_kv_heads + kvh) * P.page_size +
                             pos % P.page_size) * kHeadDim + c * 8;
        kv[j] = __ldcg(reinterpret_cast<const uint4*>(P.k_pool + off));
        vv[j] = __ldcg(reinterpret_cast<const uint4*>(P.v_pool + off));
      }
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = tid + j * kAttnThreads, r = i / (kHeadDim / 8), c = i - r * (kHeadDim / 8);
      *reinterpret_cast<uint4*>(&S.k[r][c * 8]) = kv[j];
      *reinterpret_cast<uint4*>(&S.v[r][c * 8]) = vv[j];
    }
    __syncthreads();
    // Scores: thread -> (position r, head parity hs); heads hs, hs+2, ...
    {
      const int r = tid % kAttnTile, hs = tid / kAttnTile;
      float dots[kMaxGroup / 2];
#pragma unroll
      for (int j = 0; j < kMaxGroup / 2; ++j) dots[j] = 0.0f;
#pragma unroll 4
      for (int c = 0; c < kHeadDim / 8; ++c) {
        const uint4 kk = *reinterpret_cast<const uint4*>(&S.k[r][c * 8]);
        const __half2* k2 = reinterpret_cast<const __half2*>(&kk);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(k2[e]);
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int j = 0; j < kMaxGroup / 2; ++j) {
          const int h = hs + 2 * j;
          if (h < G) {
#pragma unroll
            for (int e = 0; e < 8; ++e) dots[j] = fmaf(S.q[h][c * 8 + e], kf[e], dots[j]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kMaxGroup / 2; ++j) {
        const int h = hs + 2 * j;
        if (h < G) S.p[h][r] = (r < n) ? dots[j] * kAttnScale : -INFINITY;
      }
    }
    __syncthreads();
    // Online softmax update, one warp per head.
    {
      const int warp = tid / kWarp, lane = tid % kWarp;
      for (int h = warp; h < G; h += kAttnThreads / kWarp) {
        const float s0 = S.p[h][lane], s1 = S.p[h][lane + 32];
        const float tmax = warp_max(fmaxf(s0, s1));
        const float m_old = S.m[h];
        const float m_new = fmaxf(m_old, tmax);
        float e0 = 0.0f, e1 = 0.0f, alpha = 1.0f;
        if (m_new != -INFINITY) {
          e0 = expf(s0 - m_new);
          e1 = expf(s1 - m_new);
          alpha = expf(m_old - m_new);
        }
        const float sum = warp_sum(e0 + e1);
        S.p[h][lane] = e0;
        S.p[h][lane + 32] = e1;
        __syncwarp();
        if (lane == 0) {
          S.alpha[h] = alpha;
          S.m[h] = m_new;
          S.l[h] = S.l[h] * alpha + sum;
        }
      }
    }
    __syncthreads();
    // P.V: thread -> output dimension d.
    {
      const int d = tid;
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h)
        if (h < G) acc[h] *= S.alpha[h];
      for (int r = 0; r < n; ++r) {
        const float v = __half2float(S.v[r][d]);
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h)
          if (h < G) acc[h] = fmaf(S.p[h][r], v, acc[h]);
      }
    }
    __syncthreads();
  }

  const int d = tid;
  if (P.n_splits == 1) {
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
      if (h < G) {
        const float l = S.l[h];
        P.out[static_cast<size_t>(b) * q_dim + (kvh * G + h) * kHeadDim + d] =
            __float2half_rn(l > 0.0f ? acc[h] / l : 0.0f);
      }
    }
  } else {
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
      if (h < G) {
        const size_t row = (static_cast<size_t>(b) * P.n_q_heads + kvh * G + h) * P.n_splits + split;
        P.part_o[row * kHeadDim + d] = acc[h];
        if (d == 0) P.part_ml[row] = make_float2(S.m[h], S.l[h]);
      }
    }
  }
}

// Merge the per-split partials of one (sequence, query head): log-sum-exp.
__global__ void __launch_bounds__(kHeadDim) gqa_combine_kernel(const AttnParams P) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const size_t row0 = (static_cast<size_t>(b) * P.n_q_heads + h) * P.n_splits;
  float M = -INFINITY;
  for (int s = 0; s < P.n_splits; ++s) M = fmaxf(M, P.part_ml[row0 + s].x);
  float num = 0.0f, den = 0.0f;
  if (M != -INFINITY) {
    for (int s = 0; s < P.n_splits; ++s) {
      const float2 ml = P.part_ml[row0 + s];
      if (ml.y > 0.0f) {
        const float w = expf(ml.x - M);
        num = fmaf(w, P.part_o[(row0 + s) * kHeadDim + d], num);
        den = fmaf(w, ml.y, den);
      }
    }
  }
  P.out[static_cast<size_t>(b) * P.n_q_heads * kHeadDim + h * kHeadDim + d] =
      __float2half_rn(den > 0.0f ? num / den : 0.0f);
}

static int attn_chunk(int max_seq_len, int n_splits) {
  int chunk = (max_seq_len + n_splits - 1) / n_splits;
  return (chunk + kAttnTile - 1) / kAttnTile * kAttnTile;
}

}  // namespace lmps

using namespace lmps;

extern "C" int lmps_gqa_attention_splits(int batch, int n_kv_heads, int max_seq_len, int page_size) {
  (void)page_size;
  if (batch <= 0 || n_kv_heads <= 0 || max_seq_len <= 0) return 1;
  // The time of a call follows its longest split: take the fewest 64-position
  // tiles per split that a grid of at most ~4 CTAs per SM (148 SMs) allows,
  // then the fewest splits that reach it (a batch-64 sweep: 416-position
  // cache 33.3 -> 27.7 us, 1024-position 60.8 -> 48.9 us; batch 16, 1024
  // positions 27.8 -> 18.4 us against the earlier two-CTAs-per-SM rule).
  const int tiles = (max_seq_len + kAttnTile - 1) / kAttnTile;
  const int ctas = batch * n_kv_heads;
  int cap = (4 * 148) / ctas;
  if (cap < 1) cap = 1;
  if (cap > tiles) cap = tiles;
  if (cap > 256) cap = 256;
  const int per = (tiles + cap - 1) / cap;
  const int splits = (tiles + per - 1) / per;
  return splits < 1 ? 1 : splits;
}

extern "C" size_t lmps_gqa_attention_workspace_size(int batch, int n_q_heads, int head_dim,
                                                    int n_splits) {
  if (n_splits <= 1 || batch <= 0 || n_q_heads <= 0 || head_dim <= 0) return 0;
  const size_t rows = static_cast<size_t>(batch) * n_q_heads * n_splits;
  return rows * head_dim * sizeof(float) + rows * sizeof(float2);
}

static int attention_launch(AttnParams P, const uint16_t* k_pool, const uint16_t* v_pool,
                            const int32_t* block_table, const int32_t* seq_lens, uint16_t* out, void* workspace,
                            size_t workspace_bytes, int max_pages, int page_size, int n_q_heads, int n_kv_heads,
                            int head_dim, int batch, int max_seq_len, int n_splits, void* stream);

extern "C" int lmps_gqa_decode_attention(const uint16_t* q, const uint16_t* k_pool,
                                         const uint16_t* v_pool, const int32_t* block_table,
                                         const int32_t* seq_lens, uint16_t* out, void* workspace,
                                         size_t workspace_bytes, int max_pages, int page_size,
                                         int n_q_heads, int n_kv_heads, int head_dim, int batch,
                                         int max_seq_len, int n_splits, void* stream) {
  LMPS_CHECK_ARG(q);
  AttnParams P{};
  P.q = reinterpret_cast<const __half*>(q);
  return attention_launch(P, k_pool, v_pool, block_table, seq_lens, out, workspace, workspace_bytes, max_pages,
                          page_size, n_q_heads, n_kv_heads, head_dim, batch, max_seq_len, n_splits, stream);
}

extern "C" int lmps_gqa_decode_attention_rope(const uint16_t* qkv, const int32_t* pos, const float* inv_freq,
                                              int rope_style, uint16_t* k_pool, uint16_t* v_pool,
                                              const int32_t* block_table, const int32_t* seq_lens, uint16_t* out,
                                              void* workspace, size_t workspace_bytes, int max_pages,
                                              int page_size, int n_q_heads, int n_kv_heads, int head_dim,
                                              int batch, int max_seq_len, int n_splits, void* stream) {
  LMPS_CHECK_ARG(qkv && pos && inv_freq);
  LMPS_CHECK_ARG(rope_style == LMPS_ROPE_INTERLEAVED || rope_style == LMPS_ROPE_NEOX);
  AttnParams P{};
  P.qkv = reinterpret_cast<const __half*>(qkv);
  P.pos = pos;
  P.inv_freq = inv_freq;
  P.rope_style = rope_style;
  P.k_new = reinterpret_cast<__half*>(k_pool);
  P.v_new = reinterpret_cast<__half*>(v_pool);
  return attention_launch(P, k_pool, v_pool, block_table, seq_lens, out, workspace, workspace_bytes, max_pages,
                          page_size, n_q_heads, n_kv_heads, head_dim, batch, max_seq_len, n_splits, stream);
}

static int attention_launch(AttnParams P, const uint16_t* k_pool, const uint16_t* v_pool,
                            const int32_t* block_table, const int32_t* seq_lens, uint16_t* out, void* workspace,
                            size_t workspace_bytes, int max_pages, int page_size, int n_q_heads, int n_kv_heads,
                            int head_dim, int batch, int max_seq_len, int n_splits, void* stream) {
  LMPS_CHECK_ARG(k_pool && v_pool && block_table && seq_lens && out);
  LMPS_CHECK_ARG(batch > 0 && max_pages > 0 && page_size > 0 && max_seq_len > 0);
  LMPS_CHECK_ARG(max_seq_len <= max_pages * page_size);
  LMPS_CHECK_ARG(n_kv_heads > 0 && n_q_heads % n_kv_heads == 0);
  if (head_dim != kHeadDim || n_q_heads / n_kv_heads > kMaxGroup) return LMPS_ERR_UNSUPPORTED;
  LMPS_CHECK_ARG(n_splits >= 1 && n_splits <= 1024);
  LMPS_CHECK_ARG(lmps_aligned(k_pool, 16) && lmps_aligned(v_pool, 16));
  const size_t need = lmps_gqa_attention_workspace_size(batch, n_q_heads, head_dim, n_splits);
  if (need > 0 && (!workspace || workspace_bytes < need)) return LMPS_ERR_WORKSPACE;
  P.k_pool = reinterpret_cast<const __half*>(k_pool);
  P.v_pool = reinterpret_cast<const __half*>(v_pool);
  P.block_table = block_table;
  P.seq_lens = seq_lens;
  P.out = reinterpret_cast<__half*>(out);
  P.max_pages = max_pages;
  P.page_size = page_size;
  P.n_q_heads = n_q_heads;
  P.n_kv_heads = n_kv_heads;
  P.n_splits = n_splits;
  P.chunk = attn_chunk(max_seq_len, n_splits);
  if (n_splits > 1) {
    const size_t rows = static_cast<size_t>(batch) * n_q_heads * n_splits;
    P.part_o = reinterpret_cast<float*>(workspace);
    P.part_ml = reinterpret_cast<float2*>(reinterpret_cast<char*>(workspace) + rows * head_dim * sizeof(float));
  }
  const size_t smem = sizeof(AttnSmem);
  const int st_attr = lmps_max_dyn_smem<gqa_decode_attn_kernel>(static_cast<int>(smem));
  if (st_attr != LMPS_OK) return st_attr;
  cudaStream_t st = lmps_stream(stream);
  dim3 grid(n_splits, n_kv_heads, batch);
  int status = lmps_launch_pdl(gqa_decode_attn_kernel, grid, dim3(kAttnThreads), smem, st, P);
  if (status || n_splits == 1) return status;
  return lmps_launch_pdl(gqa_combine_kernel, dim3(n_q_heads, batch), dim3(kHeadDim), 0, st, P);
}

// ---------------------------------------------------------------------------
// lmps_gqa_decode_attention_noalloc: the same attention with its split
// partials kept in a fixed, library-owned device array instead of a
// caller-provided workspace.
//
// Who needs it: callers that cannot allocate device memory where they call
// the attention -- a foreign-language binding that only receives device
// pointers from another runtime and has no allocator behind this C interface,
// code running under a global-mode stream capture (where cudaMalloc is not
// permitted), or a serving loop that forbids allocation after warm-up because
// cudaMalloc/cudaFree can synchronise the device.
//
// The array below is LMPS_GQA_ATTENTION_NOALLOC_SCRATCH_BYTES (4 MiB) and is
// resident on every GPU that loads this library until the process exits.  In
// host code its name is only a host-side stand-in, not a device address, so
// the host looks the device address up with cudaGetSymbolAddress, once per
// device (with that device current) on the first call made on that device,
// and hands that address to the kernels as their workspace.  That first call
// should therefore come before any stream capture.  Every call shares the one
// array and it keeps whatever the previous call left there; nothing in it has
// to start at zero, because the combine kernel only reads partial slots that
// the partial kernel of the same call has written.  Calls whose work overlaps
// on the GPU (different streams, or different host threads without ordering)
// race on the array.
// ---------------------------------------------------------------------------
#include <mutex>

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[LMPS_GQA_ATTENTION_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_scratch_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once).
int noalloc_scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kNoAllocMaxDevices) return LMPS_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return e != cudaSuccess ? static_cast<int>(e) : LMPS_ERR_UNSUPPORTED;
    g_noalloc_scratch_ptr[dev] = p;
  }
  *out = g_noalloc_scratch_ptr[dev];
  return LMPS_OK;
}
}  // namespace

extern "C" int lmps_gqa_decode_attention_noalloc(const uint16_t* q, const uint16_t* k_pool,
                                                 const uint16_t* v_pool,
                                                 const int32_t* block_table,
                                                 const int32_t* seq_lens, uint16_t* out,
                                                 int max_pages, int page_size, int n_q_heads,
                                                 int n_kv_heads, int head_dim, int batch,
                                                 int max_seq_len, int n_splits, void* stream) {
  if (batch <= 0 || n_q_heads <= 0 || head_dim <= 0 || n_splits < 1) return LMPS_ERR_INVALID_ARGUMENT;
  const size_t need = lmps_gqa_attention_workspace_size(batch, n_q_heads, head_dim, n_splits);
  if (need > LMPS_GQA_ATTENTION_NOALLOC_SCRATCH_BYTES) return LMPS_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int st = noalloc_scratch_address(&scratch);
  if (st != LMPS_OK) return st;
  return lmps_gqa_decode_attention(q, k_pool, v_pool, block_table, seq_lens, out, scratch,
                                   LMPS_GQA_ATTENTION_NOALLOC_SCRATCH_BYTES, max_pages, page_size,
                                   n_q_heads, n_kv_heads, head_dim, batch, max_seq_len, n_splits,
                                   stream);
}
