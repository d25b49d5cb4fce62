// Normalisation, RoPE + KV append, elementwise kernels, the reference's
// three-stage attention drop-ins, the device Q4 packer and decode bookkeeping.
#include <cmath>

#include "common.cuh"

namespace lmps {

// ---------------------------------------------------------------------------
// RMSNorm -- kernels/rms_norm.metal:20-39, reduced over the full vector (the
// Metal launch at runners/engine.py:190 splits it over two threadgroups and
// reads past its 32-entry partial-sum array; the intended math is used).
// One CTA per row; scale = 1 / sqrt(sum(x^2)/dim + eps) with IEEE sqrt and
// division; out = fp16(fp16(x*scale) * gamma).
// ---------------------------------------------------------------------------
constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum_256(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (lane < kNormThreads / kWarp) ? red[lane] : 0.0f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(kNormThreads)
rms_norm_kernel(const __half* __restrict__ x, const __half* __restrict__ gamma,
                __half* __restrict__ out, int dim, float eps) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  __shared__ float red[kNormThreads / kWarp];
  const __half* xr = x + static_cast<size_t>(blockIdx.x) * dim;
  __half* orow = out + static_cast<size_t>(blockIdx.x) * dim;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < dim; i += kNormThreads) {
    const float v = __half2float(xr[i]);
    ss = fmaf(v, v, ss);
  }
  ss = block_sum_256(ss, red);
  const float scale = 1.0f / sqrtf(ss / static_cast<float>(dim) + eps);
  for (int i = threadIdx.x; i < dim; i += kNormThreads) {
    const __half nrm = __float2half_rn(__half2float(xr[i]) * scale);
    orow[i] = __float2half_rn(__half2float(nrm) * __half2float(gamma[i]));
  }
}

// The same RMSNorm with one warp per row (8 rows per CTA) and 16-byte loads
// and stores: no block barrier, every load of a row in flight at once.  For
// at least 256 rows (the prefill's 16384 rows: 48 us per call with a CTA per
// row), dim % 8 == 0, dim <= 2048, 16-byte aligned rows.
constexpr int kNormRowsPerCta = 8;
constexpr int kNormMaxVec = 8;  // 16-byte groups per lane: dim <= 8 * 8 * 32
constexpr int kNormWarpMinRows = 256;
__global__ void __launch_bounds__(kNormRowsPerCta * kWarp)
rms_norm_warp_kernel(const __half* __restrict__ x, const __half* __restrict__ gamma, __half* __restrict__ out,
                     int dim, float eps, int rows) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  const int row = blockIdx.x * kNormRowsPerCta + static_cast<int>(threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nv = dim / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * dim);
  uint4 v[kNormMaxVec];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int j = lane + kWarp * i;
    if (j < nv) {
      v[i] = xr[j];
      const __half* h = reinterpret_cast<const __half*>(&v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = __half2float(h[e]);
        ss = fmaf(f, f, ss);
      }
    }
  }
  ss = warp_sum(ss);
  const float scale = 1.0f / sqrtf(ss / static_cast<float>(dim) + eps);
  const uint4* gr = reinterpret_cast<const uint4*>(gamma);
  uint4* orow = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * dim);
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int j = lane + kWarp * i;
    if (j < nv) {
      const uint4 gv = __ldg(gr + j);
      const __half* h = reinterpret_cast<const __half*>(&v[i]);
      const __half* g = reinterpret_cast<const __half*>(&gv);
      uint4 o;
      __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const __half nrm = __float2half_rn(__half2float(h[e]) * scale);
        oh[e] = __float2half_rn(__half2float(nrm) * __half2float(g[e]));
      }
      orow[j] = o;
    }
  }
}

// RoPE -- kernels/rope.metal:19-40 (rope_pair_index / rope_rotate in common.cuh).
__global__ void rope_kernel(__half* vec, const int32_t* pos, const float* inv_freq, int n_heads,
                            int head_dim, int style) {
  const int b = blockIdx.y;
  const int npairs = n_heads * head_dim / 2;
  const float m = static_cast<float>(pos[b]);
  __half* v = vec + static_cast<size_t>(b) * n_heads * head_dim;
  for (int pr = blockIdx.x * blockDim.x + threadIdx.x; pr < npairs; pr += gridDim.x * blockDim.x) {
    int i1, i2, fi;
    rope_pair_index(pr, head_dim, style, i1, i2, fi);
    __half a = v[i1], c = v[i2];
    rope_rotate(a, c, m * inv_freq[fi]);
    v[i1] = a;
    v[i2] = c;
  }
}

// RoPE on q and k of the fused q|k|v row, then the paged KV-cache append.
__global__ void rope_kv_append_scalar_kernel(const __half* __restrict__ qkv, const int32_t* __restrict__ pos,
                                      const float* __restrict__ inv_freq, __half* __restrict__ q_out,
                                      __half* __restrict__ k_pool, __half* __restrict__ v_pool,
                                      const int32_t* __restrict__ block_table, int max_pages,
                                      int page_size, int n_q_heads, int n_kv_heads, int head_dim,
                                      int style) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  const int b = blockIdx.x;
  const int q_dim = n_q_heads * head_dim, kv_dim = n_kv_heads * head_dim;
  const __half* row = qkv + static_cast<size_t>(b) * (q_dim + 2 * kv_dim);
  const int p = pos[b];
  const float m = static_cast<float>(p);
  const int page = block_table[static_cast<size_t>(b) * max_pages + p / page_size];
  const int off = p % page_size;
  const int q_pairs = q_dim / 2, k_pairs = kv_dim / 2;
  for (int t = threadIdx.x; t < q_pairs + k_pairs; t += blockDim.x) {
    const bool is_q = t < q_pairs;
    const int pr = is_q ? t : t - q_pairs;
    int i1, i2, fi;
    rope_pair_index(pr, head_dim, style, i1, i2, fi);
    const __half* src = is_q ? row : row + q_dim;
    __half a = src[i1], c = src[i2];
    rope_rotate(a, c, m * inv_freq[fi]);
    if (is_q) {
      q_out[static_cast<size_t>(b) * q_dim + i1] = a;
      q_out[static_cast<size_t>(b) * q_dim + i2] = c;
    } else {
      const int h1 = i1 / head_dim, h2 = i2 / head_dim;
      k_pool[((static_cast<size_t>(page) * n_kv_heads + h1) * page_size + off) * head_dim + (i1 - h1 * head_dim)] = a;
      k_pool[((static_cast<size_t>(page) * n_kv_heads + h2) * page_size + off) * head_dim + (i2 - h2 * head_dim)] = c;
    }
  }
  const __half* vsrc = row + q_dim + kv_dim;
  for (int i = threadIdx.x; i < kv_dim; i += blockDim.x) {
    const int h = i / head_dim;
    v_pool[((static_cast<size_t>(page) * n_kv_heads + h) * page_size + off) * head_dim + (i - h * head_dim)] = vsrc[i];
  }
}

// The same with each row's head_dim / 2 (cos, sin) pairs computed once (not
// once per head) and 16 bytes moved per thread: 4 adjacent pairs
// (interleaved) or 8 pairs of a head's two halves (NeoX) per step.  For
// head_dim % 16 == 0, head_dim <= 512, 16-byte aligned buffers.
constexpr int kRopeMaxHalf = 256;
__global__ void __launch_bounds__(256)
rope_kv_append_kernel(const __half* __restrict__ qkv, const int32_t* __restrict__ pos,
                      const float* __restrict__ inv_freq, __half* __restrict__ q_out, __half* __restrict__ k_pool,
                      __half* __restrict__ v_pool, const int32_t* __restrict__ block_table, int max_pages,
                      int page_size, int n_q_heads, int n_kv_heads, int head_dim, int style) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  __shared__ float2 cs[kRopeMaxHalf];
  const int b = blockIdx.x, tid = threadIdx.x, half_d = head_dim / 2;
  const int q_dim = n_q_heads * head_dim, kv_dim = n_kv_heads * head_dim;
  const __half* row = qkv + static_cast<size_t>(b) * (q_dim + 2 * kv_dim);
  const int p = pos[b];
  const float m = static_cast<float>(p);
  const int page = block_table[static_cast<size_t>(b) * max_pages + p / page_size];
  const int off = p % page_size;
  auto kv_row = [&](__half* pool, int h) {
    return pool + ((static_cast<size_t>(page) * n_kv_heads + h) * page_size + off) * head_dim;
  };
  // the V rows and this thread's first q|k unit are read before the table is
  // built (nothing of theirs depends on it)
  const __half* vsrc = row + q_dim + kv_dim;
  for (int u = tid; u < kv_dim / 8; u += blockDim.x) {
    const int e = 8 * u, h = e / head_dim;
    *reinterpret_cast<uint4*>(kv_row(v_pool, h) + (e - h * head_dim)) = *reinterpret_cast<const uint4*>(vsrc + e);
  }
  const bool il = style == LMPS_ROPE_INTERLEAVED;
  uint4 first = make_uint4(0u, 0u, 0u, 0u);
  if (il && tid < (q_dim + kv_dim) / 8) first = *reinterpret_cast<const uint4*>(row + 8 * tid);
  for (int j = tid; j < half_d; j += blockDim.x) {
    float sn, c;
    sincosf(m * inv_freq[j], &sn, &c);
    cs[j] = make_float2(c, sn);
  }
  __syncthreads();
  if (il) {  // element 2j pairs with 2j + 1, frequency j
    for (int u = tid; u < (q_dim + kv_dim) / 8; u += blockDim.x) {
      const int e0 = 8 * u;
      const bool is_q = e0 < q_dim;
      const int e = is_q ? e0 : e0 - q_dim, h = e / head_dim, d0 = e - h * head_dim;
      uint4 v = u == tid ? first : *reinterpret_cast<const uint4*>(row + e0);
      __half* hv = reinterpret_cast<__half*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 t = cs[d0 / 2 + i];
        rope_rotate_cs(hv[2 * i], hv[2 * i + 1], t.x, t.y);
      }
      __half* dst = is_q ? q_out + static_cast<size_t>(b) * q_dim + e : kv_row(k_pool, h) + d0;
      *reinterpret_cast<uint4*>(dst) = v;
    }
  } else {  // NeoX: element j pairs with j + head_dim / 2, frequency j
    const int upd = half_d / 8;  // 8-pair units per head
    for (int u = tid; u < (n_q_heads + n_kv_heads) * upd; u += blockDim.x) {
      const int hh = u / upd, j0 = 8 * (u - hh * upd);
      const bool is_q = hh < n_q_heads;
      const int h = is_q ? hh : hh - n_q_heads;
      const __half* src = row + (is_q ? 0 : q_dim) + h * head_dim;
      uint4 v1 = *reinterpret_cast<const uint4*>(src + j0), v2 = *reinterpret_cast<const uint4*>(src + j0 + half_d);
      __half* h1 = reinterpret_cast<__half*>(&v1);
      __half* h2 = reinterpret_cast<__half*>(&v2);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 t = cs[j0 + i];
        rope_rotate_cs(h1[i], h2[i], t.x, t.y);
      }
      __half* dst = is_q ? q_out + static_cast<size_t>(b) * q_dim + h * head_dim : kv_row(k_pool, h);
      *reinterpret_cast<uint4*>(dst + j0) = v1;
      *reinterpret_cast<uint4*>(dst + j0 + half_d) = v2;
    }
  }
}

// residual.metal:19 and swiglu.metal:19-22.
__global__ void residual_add_kernel(const __half* x, const __half* y, __half* out, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = __hadd(x[i], y[i]);
}

__global__ void swiglu_kernel(const __half* g, const __half* u, __half* out, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = __float2half_rn(silu_mul(__half2float(g[i]), __half2float(u[i])));
}

// utils/tokenizer.py:22-26 -- one fp16 row per sequence.
__global__ void embed_gather_kernel(const __half* table, const int32_t* ids, __half* out, int dim,
                                    int vocab, int32_t* bad) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  const int b = blockIdx.x;
  const int id = ids[b];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0 && bad) *bad = 1;
  const __half* src = table + static_cast<size_t>(ok ? id : 0) * dim;
  __half* dst = out + static_cast<size_t>(b) * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) dst[i] = ok ? src[i] : __float2half_rn(0.0f);
}

// ---------------------------------------------------------------------------
// The reference's three attention stages over a contiguous [seq, kv_dim]
// cache, one thread per (head, position) / head / output element as in
// attention.metal:22-40, softmax.metal:19-36, attn_sum.metal:21-33.
// ---------------------------------------------------------------------------
__global__ void attention_scores_kernel(const __half* q, const __half* k_cache, float* scores,
                                        int seq_len, int n_q_heads, int n_kv_heads, int head_dim) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_q_heads * seq_len) return;
  const int h = idx / seq_len, i = idx - h * seq_len;
  const int kvh = h / (n_q_heads / n_kv_heads);
  const __half* qp = q + static_cast<size_t>(h) * head_dim;
  const __half* kp = k_cache + static_cast<size_t>(i) * n_kv_heads * head_dim + kvh * head_dim;
  float dot = 0.0f;
  for (int d = 0; d < head_dim; ++d) dot = fmaf(__half2float(qp[d]), __half2float(kp[d]), dot);
  scores[static_cast<size_t>(h) * seq_len + i] = dot * kAttnScale;
}

__global__ void softmax_kernel(float* scores, int seq_len) {
  __shared__ float red[kNormThreads / kWarp];
  float* s = scores + static_cast<size_t>(blockIdx.x) * seq_len;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < seq_len; i += blockDim.x) m = fmaxf(m, s[i]);
  m = warp_max(m);
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = (lane < kNormThreads / kWarp) ? red[lane] : -INFINITY;
  m = warp_max(m);
  __syncthreads();
  float sum = 0.0f;
  for (int i = threadIdx.x; i < seq_len; i += blockDim.x) {
    const float e = expf(s[i] - m);
    s[i] = e;
    sum += e;
  }
  sum = block_sum_256(sum, red);
  for (int i = threadIdx.x; i < seq_len; i += blockDim.x) s[i] = s[i] / sum;
}

__global__ void attn_weighted_sum_kernel(const float* scores, const __half* v_cache, __half* out,
                                         int seq_len, int n_q_heads, int n_kv_heads, int head_dim) {
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  if (tid >= n_q_heads * head_dim) return;
  const int h = tid / head_dim, d = tid - h * head_dim;
  const int kvh = h / (n_q_heads / n_kv_heads);
  float acc = 0.0f;
  for (int i = 0; i < seq_len; ++i)
    acc = fmaf(scores[static_cast<size_t>(h) * seq_len + i],
               __half2float(v_cache[static_cast<size_t>(i) * n_kv_heads * head_dim + kvh * head_dim + d]), acc);
  out[tid] = __float2half_rn(acc);
}

// ---------------------------------------------------------------------------
// Device Q4 packer -- utils/pack_weights.py:18-46: one thread per group of 32.
// scale = max|w| / 7 (IEEE division), 0 -> 1; code = rint(w / scale) (ties to
// even, like torch.round) clamped to [-8, 7]; nibble = code + 8; byte b =
// nib[2b] | nib[2b+1] << 4; scale stored fp16 (round to nearest even).
// ---------------------------------------------------------------------------
__global__ void q4_pack_kernel(const float* __restrict__ w, long long n, uint8_t* __restrict__ packed,
                               __half* __restrict__ scales, long long n_groups) {
  for (long long g = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; g < n_groups;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    float v[32];
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const long long i = g * 32 + j;
      v[j] = i < n ? w[i] : 0.0f;
      amax = fmaxf(amax, fabsf(v[j]));
    }
    float scale = __fdiv_rn(amax, 7.0f);
    if (scale == 0.0f) scale = 1.0f;
    uint32_t words[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float q = rintf(__fdiv_rn(v[j], scale));
      q = fminf(fmaxf(q, -8.0f), 7.0f);
      const uint32_t nib = static_cast<uint32_t>(static_cast<int>(q) + 8) & 0xFu;
      words[j / 8] |= nib << (4 * (j % 8));
    }
    reinterpret_cast<uint4*>(packed)[g] = make_uint4(words[0], words[1], words[2], words[3]);
    scales[g] = __float2half_rn(scale);
  }
}

__global__ void decode_advance_kernel(const int32_t* next, int32_t* tokens, int32_t* pos,
                                      int32_t* seq_lens, int32_t* history, int32_t* step,
                                      int max_steps, int batch) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  const int s = (history && step) ? step[0] : 0;
  for (int b = threadIdx.x; b < batch; b += blockDim.x) {
    const int32_t t = next[b];
    tokens[b] = t;
    if (pos) pos[b] += 1;
    if (seq_lens) seq_lens[b] += 1;
    if (history && step && s < max_steps) history[static_cast<size_t>(s) * batch + b] = t;
  }
  __syncthreads();
  if (threadIdx.x == 0 && history && step) step[0] = s + 1;
}

// Row-wise first-index argmax of fp16 logits (runners/engine.py:180-181:
// numpy.argmax over fp32(logits)); one block per row.
__global__ void argmax_rows_kernel(const __half* logits, int ld, int n, int32_t* ids) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  const __half* row = logits + static_cast<size_t>(blockIdx.x) * ld;
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    best = u64_max(best, argmax_key(__half2float(row[i]), static_cast<uint32_t>(i)));
  best = warp_max_u64(best);
  __shared__ unsigned long long red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) best = u64_max(best, red[w]);
    best = u64_max(best, red[0]);
    ids[blockIdx.x] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
  }
}

// out[r][i] = silu(gu[r][i]) * gu[r][n + i]: SwiGLU of a fused gate|up
// projection row (swiglu.metal over the two halves of one GEMM output).
__global__ void swiglu_rows_kernel(const __half* gu, int ld, int n, __half* out, int ldo, int rows) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  const int total = rows * n;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int r = i / n, c = i - r * n;
    const __half* row = gu + static_cast<size_t>(r) * ld;
    out[static_cast<size_t>(r) * ldo + c] = __float2half_rn(silu_mul(__half2float(row[c]), __half2float(row[n + c])));
  }
}

// First-index argmax of each row, one thread-block cluster of kArgSplit
// CTAs per row: every CTA scans a contiguous slice with 16-byte loads, the
// cluster's rank 0 combines the CTAs' keys through distributed shared memory.
constexpr int kArgSplit = 8;
__global__ void argmax_rows_cluster_kernel(const __half* logits, int ld, int n, int32_t* ids) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  __shared__ unsigned long long red[32];
  __shared__ unsigned long long cta_best;
  const int row = blockIdx.y;
  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int chunk = ((n + kArgSplit - 1) / kArgSplit + 7) & ~7;
  const int lo = static_cast<int>(rank) * chunk, hi = min(n, lo + chunk);
  const __half* r = logits + static_cast<size_t>(row) * ld;
  unsigned long long best = 0ull;
  const int hi8 = lo + ((max(hi - lo, 0)) & ~7);
  for (int i = lo + 8 * static_cast<int>(threadIdx.x); i < hi8; i += 8 * blockDim.x) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(r + i));
    const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
    for (int e = 0; e < 8; ++e) best = u64_max(best, argmax_key(__half2float(h[e]), static_cast<uint32_t>(i + e)));
  }
  for (int i = hi8 + threadIdx.x; i < hi; i += blockDim.x)
    best = u64_max(best, argmax_key(__half2float(r[i]), static_cast<uint32_t>(i)));
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) best = u64_max(best, red[w]);
    cta_best = u64_max(best, red[0]);
  }
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (rank == 0 && threadIdx.x == 0) {
    unsigned long long b = 0ull;
    const uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(&cta_best));
    for (uint32_t c = 0; c < kArgSplit; ++c) {
      uint32_t ra;
      unsigned long long v;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(local), "r"(c));
      asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(ra) : "memory");
      b = u64_max(b, v);
    }
    ids[row] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(b & 0xFFFFFFFFull));
  }
  // no CTA leaves while rank 0 may still read its key
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

}  // namespace lmps

using namespace lmps;

#define H(p) reinterpret_cast<__half*>(p)
#define CH(p) reinterpret_cast<const __half*>(p)

extern "C" int lmps_version(void) { return 100; }

extern "C" const char* lmps_status_string(int status) {
  switch (status) {
    case LMPS_OK: return "ok";
    case LMPS_ERR_INVALID_ARGUMENT: return "invalid argument";
    case LMPS_ERR_UNSUPPORTED: return "unsupported shape";
    case LMPS_ERR_WORKSPACE: return "workspace too small";
    case LMPS_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    default: break;
  }
  if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
  return "unknown status";
}

extern "C" int lmps_rms_norm(const uint16_t* x, const uint16_t* gamma, uint16_t* out, int dim,
                             int batch, float eps, void* stream) {
  LMPS_CHECK_ARG(x && gamma && out && dim > 0 && batch > 0 && eps >= 0.0f);
  // the warp-per-row kernel for the prefill's thousands of rows; decode
  // batches keep a CTA per row (measured faster at 64 rows: c2 2.10 vs 2.17 ms)
  if (batch >= kNormWarpMinRows && dim % 8 == 0 && dim <= kNormMaxVec * 8 * kWarp && lmps_aligned(x, 16) &&
      lmps_aligned(gamma, 16) && lmps_aligned(out, 16))
    return lmps_launch_pdl(rms_norm_warp_kernel, dim3((batch + kNormRowsPerCta - 1) / kNormRowsPerCta),
                           dim3(kNormRowsPerCta * kWarp), 0, lmps_stream(stream), CH(x), CH(gamma), H(out), dim, eps,
                           batch);
  return lmps_launch_pdl(rms_norm_kernel, dim3(batch), dim3(kNormThreads), 0, lmps_stream(stream), CH(x), CH(gamma),
                         H(out), dim, eps);
}

extern "C" int lmps_rope(uint16_t* vec, const int32_t* pos, const float* inv_freq, int n_heads,
                         int head_dim, int batch, int style, void* stream) {
  LMPS_CHECK_ARG(vec && pos && inv_freq && n_heads > 0 && batch > 0);
  LMPS_CHECK_ARG(head_dim > 0 && head_dim % 2 == 0);
  LMPS_CHECK_ARG(style == LMPS_ROPE_INTERLEAVED || style == LMPS_ROPE_NEOX);
  const int npairs = n_heads * head_dim / 2;
  dim3 grid((npairs + 255) / 256, batch);
  rope_kernel<<<grid, 256, 0, lmps_stream(stream)>>>(H(vec), pos, inv_freq, n_heads, head_dim, style);
  return lmps_launch_status();
}

extern "C" int lmps_rope_kv_append(const uint16_t* qkv, const int32_t* pos, const float* inv_freq,
                                   uint16_t* q_out, uint16_t* k_pool, uint16_t* v_pool,
                                   const int32_t* block_table, int max_pages, int page_size,
                                   int n_q_heads, int n_kv_heads, int head_dim, int batch,
                                   int style, void* stream) {
  LMPS_CHECK_ARG(qkv && pos && inv_freq && q_out && k_pool && v_pool && block_table);
  LMPS_CHECK_ARG(max_pages > 0 && page_size > 0 && batch > 0 && head_dim > 0 && head_dim % 2 == 0);
  LMPS_CHECK_ARG(n_kv_heads > 0 && n_q_heads > 0 && n_q_heads % n_kv_heads == 0);
  LMPS_CHECK_ARG(style == LMPS_ROPE_INTERLEAVED || style == LMPS_ROPE_NEOX);
  if (head_dim % 16 == 0 && head_dim / 2 <= kRopeMaxHalf && lmps_aligned(qkv, 16) && lmps_aligned(q_out, 16) &&
      lmps_aligned(k_pool, 16) && lmps_aligned(v_pool, 16))
    return lmps_launch_pdl(rope_kv_append_kernel, dim3(batch), dim3(256), 0, lmps_stream(stream), CH(qkv), pos,
                           inv_freq, H(q_out), H(k_pool), H(v_pool), block_table, max_pages, page_size, n_q_heads,
                           n_kv_heads, head_dim, style);
  return lmps_launch_pdl(rope_kv_append_scalar_kernel, dim3(batch), dim3(256), 0, lmps_stream(stream), CH(qkv), pos,
                         inv_freq, H(q_out), H(k_pool), H(v_pool), block_table, max_pages, page_size, n_q_heads,
                         n_kv_heads, head_dim, style);
}

extern "C" int lmps_residual_add(const uint16_t* x, const uint16_t* y, uint16_t* out, int n,
                                 void* stream) {
  LMPS_CHECK_ARG(x && y && out && n > 0);
  residual_add_kernel<<<(n + 255) / 256, 256, 0, lmps_stream(stream)>>>(CH(x), CH(y), H(out), n);
  return lmps_launch_status();
}

extern "C" int lmps_swiglu(const uint16_t* gate, const uint16_t* up, uint16_t* out, int n,
                           void* stream) {
  LMPS_CHECK_ARG(gate && up && out && n > 0);
  swiglu_kernel<<<(n + 255) / 256, 256, 0, lmps_stream(stream)>>>(CH(gate), CH(up), H(out), n);
  return lmps_launch_status();
}

extern "C" int lmps_embed_gather(const uint16_t* table, const int32_t* ids, uint16_t* out, int dim,
                                 int vocab, int batch, int32_t* bad_ids, void* stream) {
  LMPS_CHECK_ARG(table && ids && out && dim > 0 && vocab > 0 && batch > 0);
  return lmps_launch_pdl(embed_gather_kernel, dim3(batch), dim3(256), 0, lmps_stream(stream), CH(table), ids, H(out),
                         dim, vocab, bad_ids);
}

extern "C" int lmps_attention_scores(const uint16_t* q, const uint16_t* k_cache, float* scores,
                                     int seq_len, int n_q_heads, int n_kv_heads, int head_dim,
                                     void* stream) {
  LMPS_CHECK_ARG(q && k_cache && scores && seq_len > 0 && head_dim > 0);
  LMPS_CHECK_ARG(n_kv_heads > 0 && n_q_heads > 0 && n_q_heads % n_kv_heads == 0);
  const int n = n_q_heads * seq_len;
  attention_scores_kernel<<<(n + 127) / 128, 128, 0, lmps_stream(stream)>>>(
      CH(q), CH(k_cache), scores, seq_len, n_q_heads, n_kv_heads, head_dim);
  return lmps_launch_status();
}

extern "C" int lmps_softmax(float* scores, int seq_len, int n_heads, void* stream) {
  LMPS_CHECK_ARG(scores && seq_len > 0 && n_heads > 0);
  softmax_kernel<<<n_heads, kNormThreads, 0, lmps_stream(stream)>>>(scores, seq_len);
  return lmps_launch_status();
}

extern "C" int lmps_attn_weighted_sum(const float* scores, const uint16_t* v_cache, uint16_t* out,
                                      int seq_len, int n_q_heads, int n_kv_heads, int head_dim,
                                      void* stream) {
  LMPS_CHECK_ARG(scores && v_cache && out && seq_len > 0 && head_dim > 0);
  LMPS_CHECK_ARG(n_kv_heads > 0 && n_q_heads > 0 && n_q_heads % n_kv_heads == 0);
  const int n = n_q_heads * head_dim;
  attn_weighted_sum_kernel<<<(n + 127) / 128, 128, 0, lmps_stream(stream)>>>(
      scores, CH(v_cache), H(out), seq_len, n_q_heads, n_kv_heads, head_dim);
  return lmps_launch_status();
}

extern "C" int lmps_q4_pack(const float* w, long long n, uint8_t* packed, uint16_t* scales,
                            void* stream) {
  LMPS_CHECK_ARG(w && packed && scales && n > 0 && lmps_aligned(packed, 16));
  const long long groups = (n + 31) / 32;
  long long blocks = (groups + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  q4_pack_kernel<<<static_cast<unsigned>(blocks), 256, 0, lmps_stream(stream)>>>(w, n, packed, H(scales), groups);
  return lmps_launch_status();
}

extern "C" int lmps_decode_advance(const int32_t* next, int32_t* tokens, int32_t* pos,
                                   int32_t* seq_lens, int32_t* history, int32_t* step,
                                   int max_steps, int batch, void* stream) {
  LMPS_CHECK_ARG(next && tokens && batch > 0 && batch <= 4096);
  LMPS_CHECK_ARG(!history || (step && max_steps > 0));
  return lmps_launch_pdl(decode_advance_kernel, dim3(1), dim3(256), 0, lmps_stream(stream), next, tokens, pos,
                         seq_lens, history, step, max_steps, batch);
}

extern "C" int lmps_argmax_rows(const uint16_t* logits, int ld, int rows, int n, int32_t* ids, void* stream) {
  LMPS_CHECK_ARG(logits && ids && rows > 0 && n > 0 && ld >= n);
  if (ld % 8 == 0 && lmps_aligned(logits, 16) && rows <= 65535 && n >= 8 * kArgSplit) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(kArgSplit, rows);
    cfg.blockDim = dim3(512);
    cfg.stream = lmps_stream(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kArgSplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, argmax_rows_cluster_kernel, CH(logits), ld, n, ids);
    if (e != cudaSuccess) return static_cast<int>(e);
    return lmps_launch_status();
  }
  return lmps_launch_pdl(argmax_rows_kernel, dim3(rows), dim3(512), 0, lmps_stream(stream), CH(logits), ld, n, ids);
}

extern "C" int lmps_swiglu_rows(const uint16_t* gate_up, int ld, int rows, int n, uint16_t* out, int ldo,
                                void* stream) {
  LMPS_CHECK_ARG(gate_up && out && rows > 0 && n > 0 && ld >= 2 * n && ldo >= n);
  const long long total = static_cast<long long>(rows) * n;
  LMPS_CHECK_ARG(total < (1LL << 31));
  const int blocks = static_cast<int>(min((total + 255) / 256, 148LL * 16));
  return lmps_launch_pdl(swiglu_rows_kernel, dim3(blocks), dim3(256), 0, lmps_stream(stream), CH(gate_up), ld, n,
                         H(out), ldo, rows);
}
