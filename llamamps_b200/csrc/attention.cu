// Fused GQA decode attention over the paged fp16 KV cache (sm_100a).
//
// One kernel does what kernels/attention.metal (scores), softmax.metal and
// attn_sum.metal do in three dispatches (runners/engine.py:202-212), for a
// real cache of seq_lens[b] positions:
//   s[h, i] = (q_h . K[i, h/G]) * 0.088388,  p = softmax_i(s),  o_h = sum_i p V[i, h/G].
// Grid = (splits, kv heads, sequences).  A CTA owns one KV head of one
// sequence and a contiguous range of positions; the G query heads that share
// the KV head (GQA, attention.metal:23) are processed together so each K/V
// row is read from HBM once.  Tiles of 64 positions (K and V rows in the
// cache's layout, 32 KB) are staged in shared memory with cp.async, double
// buffered; each of the 4 warps folds one 16-position block of a tile into
// its own online softmax on the tensor cores (flash_decode.cuh), and the
// warps' states meet in shared memory at the end.  Each split writes an
// unnormalised partial (acc, max, sum) that a combine kernel merges with a
// log-sum-exp rescale; with one split the CTA writes the normalised output.
// The _rope entry point also does rope_kv_append's work (kernels/rope.metal
// on q and k, then the cache append): each CTA rotates the query heads of its
// KV head from the q|k|v row, and the split that attends the new position
// rotates and writes that K row (and the V row) into the paged cache and
// into its staged tile.
#include <cmath>

#include "common.cuh"
#include "flash_decode.cuh"

namespace lmps {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * kWarp;
constexpr int kAttnTile = kAttnWarps * fd::kBlk;  // positions per staged tile
constexpr int kAttnStages = 2;                     // tiles in shared memory: one in flight while one computes
constexpr int kHeadDim = 128;
constexpr int kMaxGroup = 8;

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
  int page_shift;  // log2(page_size) when it is a power of two, else -1
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
  union {
    uint4 kv[kAttnStages][2][kAttnTile][fd::kRowUnits];  // [stage][K, V][row][16-byte unit], the cache's layout
    float wo[kAttnWarps][32][32];                         // after the tiles: per-warp O^T fragments
  };
  __half q[kMaxGroup][kHeadDim];             // rotated q, natural dim order
  __half knew[kHeadDim], vnew[kHeadDim];     // the appended row (rope entry point)
  float wm[kAttnWarps][kMaxGroup];           // per-warp running max and sum
  float wl[kAttnWarps][kMaxGroup];
};

__global__ void __launch_bounds__(kAttnThreads) gqa_decode_attn_kernel(const AttnParams P) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>(smem_raw);
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = P.n_q_heads / P.n_kv_heads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, t4 = lane & 3;
  const int T = P.seq_lens[b];
  const int start = split * P.chunk;
  const int end = min(T, start + P.chunk);
  const int q_dim = P.n_q_heads * kHeadDim;
  int pnew = -1;  // position whose row comes from S.knew / S.vnew instead of the cache

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
      S.q[hl][i1] = a;
      S.q[hl][i2] = c;
    }
    if (p >= start && p < end) {  // this split attends the new position: append its K/V rows
      pnew = p;
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
        S.knew[i1] = a;
        S.knew[i2] = c;
      }
      for (int t = tid; t < kHeadDim; t += kAttnThreads) {
        const __half v = row[q_dim + kv_dim + kvh * kHeadDim + t];
        P.v_new[dst + t] = v;
        S.vnew[t] = v;
      }
    }
  } else {
    for (int i = tid; i < G * kHeadDim; i += kAttnThreads) {
      const int h = i / kHeadDim, d = i - h * kHeadDim;
      S.q[h][d] = P.q[static_cast<size_t>(b) * q_dim + (kvh * G + h) * kHeadDim + d];
    }
  }
  __syncthreads();  // S.q, S.knew / S.vnew

  // Stage tile ti (positions start + 64 ti ..) into buffer ti % stages: thread tid
  // copies 16-byte unit (tid & 15) of rows (tid >> 4) + 8 j of K and of V,
  // so a warp instruction reads two whole 256-byte rows.
  const int32_t* bt = P.block_table + static_cast<size_t>(b) * P.max_pages;
  auto stage = [&](int ti) {
    const int t0 = start + ti * kAttnTile, u = tid & (fd::kRowUnits - 1);
#pragma unroll 4
    for (int j = 0; j < kAttnTile * fd::kRowUnits / kAttnThreads; ++j) {
      const int r = (tid >> 4) + j * (kAttnThreads / fd::kRowUnits), p = t0 + r;
      uint4* dk = &S.kv[ti % kAttnStages][0][r][u];
      uint4* dv = &S.kv[ti % kAttnStages][1][r][u];
      if (p == pnew) {
        *dk = reinterpret_cast<const uint4*>(S.knew)[u];
        *dv = reinterpret_cast<const uint4*>(S.vnew)[u];
      } else if (p < end) {
        const int pi = P.page_shift >= 0 ? p >> P.page_shift : p / P.page_size;
        const int in_page = P.page_shift >= 0 ? p & (P.page_size - 1) : p - pi * P.page_size;
        const size_t off =
            ((static_cast<size_t>(__ldg(bt + pi)) * P.n_kv_heads + kvh) * P.page_size + in_page) * kHeadDim + 8 * u;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dk)), "l"(P.k_pool + off)
                     : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dv)), "l"(P.v_pool + off)
                     : "memory");
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const int n_tiles = end > start ? (end - start + kAttnTile - 1) / kAttnTile : 0;
  for (int ti = 0; ti < n_tiles && ti < kAttnStages - 1; ++ti) stage(ti);

  uint32_t qf[16];
  fd::load_qf(&S.q[0][0], G, qf);
  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
  float mrun0 = -INFINITY, mrun1 = -INFINITY, lrun0 = 0.0f, lrun1 = 0.0f;  // heads 2*t4, 2*t4+1
  for (int ti = 0; ti < n_tiles; ++ti) {
    if (ti + kAttnStages - 1 < n_tiles) stage(ti + kAttnStages - 1);  // into the buffer tile ti - 1 used
    // tile ti's group complete: the groups of later tiles may stay in flight
    const int later = min(n_tiles - 1, ti + kAttnStages - 1) - ti;
    if (later >= 2)
      asm volatile("cp.async.wait_group 2;" ::: "memory");
    else if (later == 1)
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    else
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // tile ti landed for every thread's copies
    const int p0 = start + ti * kAttnTile + warp * fd::kBlk;
    const int sb = ti % kAttnStages;
    if (p0 < end) {
      uint4 kr[2][4], vr[2][4];
      fd::load_rows(&S.kv[sb][0][warp * fd::kBlk][0], &S.kv[sb][1][warp * fd::kBlk][0], p0, end, kr, vr);
      fd::block_update(kr, vr, p0, end, qf, o, mrun0, mrun1, lrun0, lrun1);
    }
    __syncthreads();  // buffer sb is free for tile ti + stages
  }

  // -- the warps meet in shared memory; the reducing thread rescales each
  // warp's state to the merged max
  const int nw = min(kAttnWarps, (max(end - start, 0) + fd::kBlk - 1) / fd::kBlk);  // warps that saw positions
  if (warp < nw) {
    if ((lane >> 2) == 0) {
      S.wm[warp][2 * t4] = mrun0;
      S.wm[warp][2 * t4 + 1] = mrun1;
      S.wl[warp][2 * t4] = lrun0;
      S.wl[warp][2 * t4 + 1] = lrun1;
    }
    fd::store_frags(S.wo[warp], o);
  }
  __syncthreads();
  for (int w = tid; w < G * (kHeadDim / 2); w += kAttnThreads) {
    const int h = w / (kHeadDim / 2), d = 2 * (w - h * (kHeadDim / 2));
    int la, k;
    fd::frag_slot(h, d, la, k);
    float M = -INFINITY;
    for (int ww = 0; ww < nw; ++ww) M = fmaxf(M, S.wm[ww][h]);
    float n0 = 0.0f, n1 = 0.0f, den = 0.0f;
    for (int ww = 0; ww < nw; ++ww) {
      const float f = expf(S.wm[ww][h] - M);
      const float2 v = fd::load_frag_pair(S.wo[ww], la, k);
      n0 = fmaf(v.x, f, n0);
      n1 = fmaf(v.y, f, n1);
      den = fmaf(S.wl[ww][h], f, den);
    }
    if (P.n_splits == 1) {
      const float inv = den > 0.0f ? 1.0f / den : 0.0f;
      *reinterpret_cast<__half2*>(&P.out[static_cast<size_t>(b) * q_dim + (kvh * G + h) * kHeadDim + d]) =
          __floats2half2_rn(n0 * inv, n1 * inv);
    } else {
      const size_t prow = (static_cast<size_t>(b) * P.n_q_heads + kvh * G + h) * P.n_splits + split;
      *reinterpret_cast<float2*>(&P.part_o[prow * kHeadDim + d]) = make_float2(n0, n1);
      if (d == 0) P.part_ml[prow] = make_float2(M, den);
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
  // tiles per split that a grid of at most ~3 CTAs per SM (148 SMs; the
  // kernel's 67 KB of shared memory allow three) permits, then the fewest
  // splits that reach it.  Sweep, us per call with combine: batch 64,
  // 155-position cache 1 split 9.1 / 2 10.5 / 3 8.8; 416: 17.3 / 14.8 /
  // 3 13.4 / 4 14.5; 1024: 36.4 / 23.9 / 3 19.8 / 4 24.7 / 6 22.9; batch 16,
  // 1024: 4 12.0 / 8 10.8 / 16 13.6; batch 8, 2144: 12 13.2 / 17 12.4 / 24 12.9.
  const int tiles = (max_seq_len + kAttnTile - 1) / kAttnTile;
  const int ctas = batch * n_kv_heads;
  int cap = (3 * 148) / ctas;
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
  P.page_shift = (page_size & (page_size - 1)) == 0 ? __builtin_ctz(static_cast<unsigned>(page_size)) : -1;
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
