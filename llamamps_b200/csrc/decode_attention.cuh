// Split-KV GQA decode attention over the paged fp16 KV cache: the work of
// one (split, KV head, sequence) item and the log-sum-exp merge of the
// splits, as device functions shared by the standalone kernels
// (attention.cu) and the batched decode kernel's attention phase
// (decode_batched.cu).
//
// What one item computes -- kernels/attention.metal (scores), softmax.metal
// and attn_sum.metal over a real cache of seq_lens[b] positions:
//   s[h, i] = (q_h . K[i, h/G]) * 0.088388,  p = softmax_i(s),  o_h = sum_i p V[i, h/G]
// for the G query heads sharing the KV head (GQA, attention.metal:23), so
// each K/V row is read from HBM once.  Tiles of 64 positions (K and V rows in
// the cache's layout, 32 KB) are staged in shared memory with cp.async,
// double buffered; each of the 4 warps folds one 16-position block of a tile
// into its own online softmax on the tensor cores (flash_decode.cuh), and the
// warps' states meet in shared memory at the end.  Each split writes an
// unnormalised partial (acc, max, sum) that the merge combines with a
// log-sum-exp rescale; with one split the item writes the normalised output.
// With the fused RoPE + append (`fused`), q, k and v come from the
// sequence's q|k|v row (bias applied) through a loader: the item rotates its
// query heads (kernels/rope.metal), and the split that attends the new
// position rotates that K row and writes it and the V row into the paged
// cache and into its staged tile.
#pragma once

#include <cmath>

#include "common.cuh"
#include "flash_decode.cuh"

namespace lmps {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * kWarp;
constexpr int kAttnTile = kAttnWarps * fd::kBlk;  // positions per staged tile
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

// Shared memory of an item with `Stages` K/V tiles in flight (Stages - 1
// loading while one is folded).
template <int Stages>
struct __align__(16) AttnSmemT {
  union {
    uint4 kv[Stages][2][kAttnTile][fd::kRowUnits];  // [stage][K, V][row][16-byte unit], the cache's layout
    float wo[kAttnWarps][32][32];                         // after the tiles: per-warp O^T fragments
  };
  __half q[kMaxGroup][kHeadDim];             // rotated q, natural dim order
  __half knew[kHeadDim], vnew[kHeadDim];     // the appended row (fused entry)
  float wm[kAttnWarps][kMaxGroup];           // per-warp running max and sum
  float wl[kAttnWarps][kMaxGroup];
};

// Loader of the fused q|k|v values: element i of sequence b's row.
struct QkvRowLoader {
  const __half* qkv;
  int row_len;
  __device__ __forceinline__ __half operator()(int b, int i) const {
    return qkv[static_cast<size_t>(b) * row_len + i];
  }
};

// Barrier over the whole CTA (the standalone kernel's 128 threads).
struct CtaSync {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

// One item on kAttnThreads threads (tid = 0 .. 127 among them; `sync` is a
// barrier over exactly those threads).
template <int kAttnStages, class Loader, class Sync>
__device__ __forceinline__ void attn_item(const AttnParams& P, AttnSmemT<kAttnStages>& S, int split, int kvh, int b,
                                          int tid, bool fused, const Loader& qkv, Sync sync) {
  static_assert(kAttnStages >= 2 && kAttnStages <= 4, "K/V tile stages");
  const int G = P.n_q_heads / P.n_kv_heads;
  const int warp = tid >> 5, lane = tid & 31, t4 = lane & 3;
  const int T = P.seq_lens[b];
  const int start = split * P.chunk;
  const int end = min(T, start + P.chunk);
  const int q_dim = P.n_q_heads * kHeadDim;
  int pnew = -1;  // position whose row comes from S.knew / S.vnew instead of the cache

  if (fused) {
    // RoPE of the G query heads (rounded to fp16 as rope_kv_append's output)
    const int kv_dim = P.n_kv_heads * kHeadDim;
    const int p = P.pos[b];
    const float m = static_cast<float>(p);
    for (int t = tid; t < G * (kHeadDim / 2); t += kAttnThreads) {
      const int hl = t / (kHeadDim / 2);
      int i1, i2, fi;
      rope_pair_index(t - hl * (kHeadDim / 2), kHeadDim, P.rope_style, i1, i2, fi);
      const int src = (kvh * G + hl) * kHeadDim;
      __half a = qkv(b, src + i1), c = qkv(b, src + i2);
      rope_rotate(a, c, m * P.inv_freq[fi]);
      S.q[hl][i1] = a;
      S.q[hl][i2] = c;
    }
    if (p >= start && p < end) {  // this split attends the new position: append its K/V rows
      pnew = p;
      const int page = P.block_table[static_cast<size_t>(b) * P.max_pages + p / P.page_size];
      const size_t dst = ((static_cast<size_t>(page) * P.n_kv_heads + kvh) * P.page_size + p % P.page_size) * kHeadDim;
      const int ksrc = q_dim + kvh * kHeadDim;
      for (int t = tid; t < kHeadDim / 2; t += kAttnThreads) {
        int i1, i2, fi;
        rope_pair_index(t, kHeadDim, P.rope_style, i1, i2, fi);
        __half a = qkv(b, ksrc + i1), c = qkv(b, ksrc + i2);
        rope_rotate(a, c, m * P.inv_freq[fi]);
        P.k_new[dst + i1] = a;
        P.k_new[dst + i2] = c;
        S.knew[i1] = a;
        S.knew[i2] = c;
      }
      for (int t = tid; t < kHeadDim; t += kAttnThreads) {
        const __half v = qkv(b, q_dim + kv_dim + kvh * kHeadDim + t);
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
  sync();  // S.q, S.knew / S.vnew

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
    if (later >= 3)
      asm volatile("cp.async.wait_group 3;" ::: "memory");
    else if (later == 2)
      asm volatile("cp.async.wait_group 2;" ::: "memory");
    else if (later == 1)
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    else
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    sync();  // tile ti landed for every thread's copies
    const int p0 = start + ti * kAttnTile + warp * fd::kBlk;
    const int sb = ti % kAttnStages;
    if (p0 < end) {
      uint4 kr[2][4], vr[2][4];
      fd::load_rows(&S.kv[sb][0][warp * fd::kBlk][0], &S.kv[sb][1][warp * fd::kBlk][0], p0, end, kr, vr);
      fd::block_update(kr, vr, p0, end, qf, o, mrun0, mrun1, lrun0, lrun1);
    }
    sync();  // buffer sb is free for tile ti + stages
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
  sync();
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

// Merge of the per-split partials of one (sequence, query head), dim d:
// log-sum-exp.  The partials are read from L2 (they come from other CTAs of
// the same grid in the batched decode kernel).
__device__ __forceinline__ void attn_combine(const AttnParams& P, int h, int b, int d) {
  const size_t row0 = (static_cast<size_t>(b) * P.n_q_heads + h) * P.n_splits;
  float M = -INFINITY;
  for (int s = 0; s < P.n_splits; ++s) M = fmaxf(M, __ldcg(&P.part_ml[row0 + s]).x);
  float num = 0.0f, den = 0.0f;
  if (M != -INFINITY) {
    for (int s = 0; s < P.n_splits; ++s) {
      const float2 ml = __ldcg(&P.part_ml[row0 + s]);
      if (ml.y > 0.0f) {
        const float w = expf(ml.x - M);
        num = fmaf(w, __ldcg(&P.part_o[(row0 + s) * kHeadDim + d]), num);
        den = fmaf(w, ml.y, den);
      }
    }
  }
  P.out[static_cast<size_t>(b) * P.n_q_heads * kHeadDim + h * kHeadDim + d] =
      __float2half_rn(den > 0.0f ? num / den : 0.0f);
}

// Positions per split: the splits cover max_seq_len in whole 64-position tiles.
static inline int attn_chunk(int max_seq_len, int n_splits) {
  int chunk = (max_seq_len + n_splits - 1) / n_splits;
  return (chunk + kAttnTile - 1) / kAttnTile * kAttnTile;
}

}  // namespace lmps
