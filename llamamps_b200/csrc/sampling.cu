// Top-k / temperature sampling of the next token on the device, beside the
// greedy argmax (runners/engine.py:180-181 `predict_next_token` is greedy
// only).  One CTA per row of fp16 logits:
//
//  1. top-k set: the logits' fp16 bit patterns become order-preserving 16-bit
//     keys (NaN lowest); a radix select over the high byte, then the low byte,
//     finds the key T of the k-th largest logit.  The candidates are every
//     index with key > T plus the lowest-index ones with key == T until there
//     are exactly k.  Each thread owns a contiguous index range and a block
//     prefix sum gives it its output slots, so the candidates come out in
//     ascending index order on every run (no atomics in the selection).
//  2. weights p_i = exp((v_i - v_max) * (1 / temperature)) in fp32 over the
//     candidates; warp 0 sums them in a fixed order (lane l the candidates
//     l*ceil(k/32) .. in order, then lane 0 the 32 lane sums in order).
//  3. u = 24 random bits of Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel
//     random numbers: as easy as 1, 2, 3", SC 2011) with key = seed and
//     counter = (row, offset low, offset high, 0), times 2^-24; the sampled
//     id is the first candidate whose running sum (same fixed order) exceeds
//     u * sum.
// temperature <= 0 or top_k == 1 gives the first-index argmax.
#include "common.cuh"

namespace lmps {
namespace smp {

constexpr int kThreads = 1024;
constexpr int kMaxK = 1024;

// Order-preserving 16-bit key of an fp16 bit pattern (larger float -> larger
// key); NaNs get key 0, below every number.
__device__ __forceinline__ uint32_t f16_key(uint16_t b) {
  if ((b & 0x7C00u) == 0x7C00u && (b & 0x03FFu)) return 0u;
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}

// Philox4x32-10 (the SC 2011 paper's constants), first output word.
__device__ __forceinline__ uint32_t philox_first(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                                 uint32_t k1) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c0), lo0 = M0 * c0;
    const uint32_t hi1 = __umulhi(M1, c2), lo1 = M1 * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += W0;
    k1 += W1;
  }
  return c0;
}

struct SampleSmem {
  uint32_t hist[256];
  uint32_t scan[kThreads / kWarp];
  int cand_idx[kMaxK];
  float cand_w[kMaxK];
  float lane_sum[kWarp];
  uint32_t sel_hi, above_hi, sel_key, above;
  int result;
};

// Block exclusive prefix sum of one count per thread; returns this thread's
// offset, *total the sum.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* scan, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scan[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t s = lane < kThreads / kWarp ? scan[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < kThreads / kWarp) scan[lane] = s;  // inclusive over warps
  }
  __syncthreads();
  const uint32_t before = (warp ? scan[warp - 1] : 0u) + x - v;
  *total = scan[kThreads / kWarp - 1];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(kThreads) sample_rows_kernel(const uint16_t* __restrict__ logits, int ld, int n,
                                                               int k, float inv_t, uint32_t seed_lo,
                                                               uint32_t seed_hi, uint32_t off_lo, uint32_t off_hi,
                                                               int32_t* __restrict__ ids,
                                                               int32_t* __restrict__ ids2) {
  __shared__ SampleSmem S;
  const int row = blockIdx.x, tid = threadIdx.x;
  const uint16_t* x = logits + static_cast<size_t>(row) * ld;
  const int per = (n + kThreads - 1) / kThreads;
  const int lo = min(n, tid * per), hi = min(n, lo + per);
  // -- 1a. high byte of the k-th largest key
  for (int i = tid; i < 256; i += kThreads) S.hist[i] = 0u;
  __syncthreads();
  for (int i = lo; i < hi; ++i) atomicAdd(&S.hist[f16_key(x[i]) >> 8], 1u);
  __syncthreads();
  if (tid == 0) {
    uint32_t acc = 0u;
    int b = 255;
    for (; b > 0; --b) {
      if (acc + S.hist[b] >= static_cast<uint32_t>(k)) break;
      acc += S.hist[b];
    }
    S.sel_hi = static_cast<uint32_t>(b);
    S.above_hi = acc;  // keys with a larger high byte
  }
  __syncthreads();
  const uint32_t sel_hi = S.sel_hi;
  // -- 1b. low byte within that high byte
  for (int i = tid; i < 256; i += kThreads) S.hist[i] = 0u;
  __syncthreads();
  for (int i = lo; i < hi; ++i) {
    const uint32_t key = f16_key(x[i]);
    if ((key >> 8) == sel_hi) atomicAdd(&S.hist[key & 0xFFu], 1u);
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t acc = S.above_hi;
    int b = 255;
    for (; b > 0; --b) {
      if (acc + S.hist[b] >= static_cast<uint32_t>(k)) break;
      acc += S.hist[b];
    }
    S.sel_key = (sel_hi << 8) | static_cast<uint32_t>(b);
    S.above = acc;  // keys > sel_key: fewer than k; with the ties at sel_key, at least k
  }
  __syncthreads();
  const uint32_t T = S.sel_key, n_above = S.above;
  // -- 1c. candidates in index order: all keys > T, then the lowest-index ties
  uint32_t c_above = 0u, c_eq = 0u;
  for (int i = lo; i < hi; ++i) {
    const uint32_t key = f16_key(x[i]);
    c_above += key > T;
    c_eq += key == T;
  }
  uint32_t tot;
  const uint32_t eq_before = block_exclusive_scan(c_eq, S.scan, &tot);
  const uint32_t ties_taken = static_cast<uint32_t>(k) - n_above;
  // a candidate's slot = the candidates of lower index: keys above T and
  // taken ties before it; both counted in index order through a second scan
  uint32_t mine = 0u;
  {
    uint32_t e = eq_before;
    for (int i = lo; i < hi; ++i) {
      const uint32_t key = f16_key(x[i]);
      if (key > T) ++mine;
      else if (key == T) {
        if (e < ties_taken) ++mine;
        ++e;
      }
    }
  }
  const uint32_t slot0 = block_exclusive_scan(mine, S.scan, &tot);
  {
    uint32_t e = eq_before, s = slot0;
    for (int i = lo; i < hi; ++i) {
      const uint32_t key = f16_key(x[i]);
      bool take = key > T;
      if (key == T) {
        take = e < ties_taken;
        ++e;
      }
      if (take) {
        S.cand_idx[s] = i;
        S.cand_w[s] = __half2float(__ushort_as_half(x[i]));
        ++s;
      }
    }
  }
  (void)c_above;
  __syncthreads();
  // -- 2./3. weights, fixed-order sums, inverse CDF (warp 0)
  if (tid < kWarp) {
    const int lane = tid;
    float vmax = -INFINITY;
    for (int i = lane; i < k; i += kWarp) vmax = fmaxf(vmax, S.cand_w[i]);
    vmax = warp_max(vmax);
    const int seg = (k + kWarp - 1) / kWarp;
    const int s0 = min(k, lane * seg), s1 = min(k, s0 + seg);
    float part = 0.0f;
    for (int i = s0; i < s1; ++i) {
      const float w = expf((S.cand_w[i] - vmax) * inv_t);
      S.cand_w[i] = w;
      part += w;
    }
    S.lane_sum[lane] = part;
    __syncwarp();
    if (lane == 0) {
      float z = 0.0f;
      for (int l = 0; l < kWarp; ++l) z += S.lane_sum[l];
      const uint32_t r = philox_first(static_cast<uint32_t>(row), off_lo, off_hi, 0u, seed_lo, seed_hi);
      const float target = static_cast<float>(r >> 8) * (1.0f / 16777216.0f) * z;
      // the lane segment holding the target, then the candidate inside it
      float run = 0.0f;
      int l = 0;
      for (; l < kWarp - 1; ++l) {
        if (run + S.lane_sum[l] > target) break;
        run += S.lane_sum[l];
      }
      int pick = -1;
      const int a = min(k, l * seg), b = min(k, a + seg);
      for (int i = a; i < b; ++i) {
        run += S.cand_w[i];
        if (run > target) {
          pick = i;
          break;
        }
      }
      if (pick < 0) {  // rounding left the target at the very end: the last candidate with weight
        pick = k - 1;
        while (pick > 0 && S.cand_w[pick] == 0.0f) --pick;
      }
      S.result = S.cand_idx[pick];
    }
  }
  __syncthreads();
  if (tid == 0) {
    ids[row] = S.result;
    if (ids2) ids2[row] = S.result;
  }
}

}  // namespace smp
}  // namespace lmps

using namespace lmps;

extern "C" int lmps_sample_rows(const uint16_t* logits, int ld, int rows, int n, int top_k, float temperature,
                                unsigned long long seed, unsigned long long offset, int32_t* ids, int32_t* ids2,
                                void* stream) {
  LMPS_CHECK_ARG(logits && ids && rows >= 1 && n >= 1 && ld >= n && top_k >= 1);
  LMPS_CHECK_ARG(top_k <= smp::kMaxK && top_k <= n);
  if (temperature <= 0.0f) top_k = 1;
  // top_k == 1: the largest logit, lowest index on ties -- the argmax
  const float inv_t = top_k == 1 ? 1.0f : 1.0f / temperature;
  smp::sample_rows_kernel<<<rows, smp::kThreads, 0, lmps_stream(stream)>>>(
      logits, ld, n, top_k, inv_t, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32),
      static_cast<uint32_t>(offset), static_cast<uint32_t>(offset >> 32), ids, ids2);
  return lmps_launch_status();
}
