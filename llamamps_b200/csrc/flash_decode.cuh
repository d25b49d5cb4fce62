// Flash-decoding block math of the decode attention kernels: one warp
// folds a 16-position block of one KV head's cache into
// its running softmax state for the G <= 8 query heads sharing that head
// (softmax.metal:23-36 online; attention.metal:32-40 scores, attn_sum.metal:26-32
// weighted sum), on the tensor cores (mma.sync m16n8k16, fp16 in, fp32
// accumulate):
//   S^T  = K Q^T   (M = 16 positions, N = 8 heads, K = 128 dims)
//   O^T += V^T P^T (M = 16 dims per m-tile, N = 8 heads, K = 16 positions)
// Both products sum over dims or positions, so the order of the dims inside
// them is free: fragment word w (k-step w >> 1) of lane t holds physical
// dims 8t + 32(w >> 2) + 2(w & 3) + {0, 1}, so a lane's K and V operands are
// four 16-byte runs of a cache row (runs t, t + 4, t + 8, t + 12), and
// output row r of m-tile mt is physical dim
// 8((r & 7) >> 1) + 32(mt >> 1) + 4(mt & 1) + 2(r >> 3) + (r & 1);
// movmatrix transposes V rows and probabilities in registers.
// The split-KV gqa_decode_attn kernel uses all of it; the persistent
// decoder's attention stage uses the helpers and the same dim mapping with
// its own inlined fold (one S accumulator chain: inside that kernel the two
// chains below cost registers it does not have -- bs1 decode 662 vs 625
// us/step).
#pragma once

#include "common.cuh"

namespace lmps {
namespace fd {

constexpr int kBlk = 16;   // positions per warp block
constexpr int kDim = 128;  // head dim
constexpr int kRowUnits = kDim / 8;  // 16-byte units per cache row

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t word_of(const uint4 (&v)[4], int w) {
  const uint4 q = v[w >> 2];
  return (w & 3) == 0 ? q.x : (w & 3) == 1 ? q.y : (w & 3) == 2 ? q.z : q.w;
}
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// B operand Q^T of this lane: head g8 (zero for g8 >= G), its four runs
// from q[h][dim] (fp16, natural dim order, 16-byte aligned rows).
__device__ __forceinline__ void load_qf(const __half* q, int G, uint32_t (&qf)[16]) {
  const int lane = threadIdx.x & 31, g8 = lane >> 2, t4 = lane & 3;
  const uint4* qs = reinterpret_cast<const uint4*>(q + (g8 < G ? g8 : 0) * kDim + 8 * t4);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 v = g8 < G ? qs[4 * c] : make_uint4(0u, 0u, 0u, 0u);
    qf[4 * c] = v.x;
    qf[4 * c + 1] = v.y;
    qf[4 * c + 2] = v.z;
    qf[4 * c + 3] = v.w;
  }
}

// K/V operands of a 16-position block from shared-memory rows in the
// cache's layout (krow / vrow: the block's first row, 16 units per row;
// rows p0 + i for i < 16).  Read without bank conflicts: at load c the
// lanes of even rows take their run c and those of odd rows run c ^ 1 --
// the other half of the banks -- and swap back in registers.  V rows of
// positions >= end read as zero.
__device__ __forceinline__ void load_rows(const uint4* krow, const uint4* vrow, int p0, int end,
                                          uint4 (&kr)[2][4], uint4 (&vr)[2][4]) {
  const int lane = threadIdx.x & 31, g8 = lane >> 2, t4 = lane & 3, odd = g8 & 1;
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    const bool ok = p0 + 8 * h2 + g8 < end;
    const uint4* kp = krow + (8 * h2 + g8) * kRowUnits;
    const uint4* vp = vrow + (8 * h2 + g8) * kRowUnits;
    uint4 tk[4], tv[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      tk[c] = kp[t4 + 4 * (c ^ odd)];
      tv[c] = ok ? vp[t4 + 4 * (c ^ odd)] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      kr[h2][c] = odd ? tk[c ^ 1] : tk[c];
      vr[h2][c] = odd ? tv[c ^ 1] : tv[c];
    }
  }
}

// Fold one block (first position p0; positions >= end masked) into the
// running state: the max and sum of heads 2*t4, 2*t4+1 and O^T fragments.
__device__ __forceinline__ void block_update(const uint4 (&kr)[2][4], const uint4 (&vr)[2][4], int p0, int end,
                                             const uint32_t (&qf)[16], float (&o)[8][4], float& mrun0,
                                             float& mrun1, float& lrun0, float& lrun1) {
  const int lane = threadIdx.x & 31, g8 = lane >> 2;
  // two accumulators (even / odd k-steps) halve the dependent mma chain
  float s[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int ks = 0; ks < kDim / 16; ks += 2) {
    mma_16816(s, word_of(kr[0], 2 * ks), word_of(kr[1], 2 * ks), word_of(kr[0], 2 * ks + 1),
              word_of(kr[1], 2 * ks + 1), qf[2 * ks], qf[2 * ks + 1]);
    mma_16816(s2, word_of(kr[0], 2 * ks + 2), word_of(kr[1], 2 * ks + 2), word_of(kr[0], 2 * ks + 3),
              word_of(kr[1], 2 * ks + 3), qf[2 * ks + 2], qf[2 * ks + 3]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) s[i] += s2[i];
  const bool v0 = p0 + g8 < end, v1 = p0 + 8 + g8 < end;
  s[0] = v0 ? s[0] * kAttnScale : -INFINITY;
  s[1] = v0 ? s[1] * kAttnScale : -INFINITY;
  s[2] = v1 ? s[2] * kAttnScale : -INFINITY;
  s[3] = v1 ? s[3] * kAttnScale : -INFINITY;
  // online softmax per head (columns 2*t4, 2*t4+1; positions over g8 and the two row halves)
  float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
  for (int ofs = 4; ofs < 32; ofs <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, ofs));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, ofs));
  }
  const float mn0 = fmaxf(mrun0, mx0), mn1 = fmaxf(mrun1, mx1);  // finite: position p0 is valid
  const float al0 = expf(mrun0 - mn0), al1 = expf(mrun1 - mn1);
  const float e0 = expf(s[0] - mn0), e1 = expf(s[1] - mn1), e2 = expf(s[2] - mn0), e3 = expf(s[3] - mn1);
  float su0 = e0 + e2, su1 = e1 + e3;
#pragma unroll
  for (int ofs = 4; ofs < 32; ofs <<= 1) {
    su0 += __shfl_xor_sync(0xffffffffu, su0, ofs);
    su1 += __shfl_xor_sync(0xffffffffu, su1, ofs);
  }
  lrun0 = lrun0 * al0 + su0;
  lrun1 = lrun1 * al1 + su1;
  mrun0 = mn0;
  mrun1 = mn1;
  // O^T = O^T * alpha + V^T P^T
  const uint32_t pb0 = movmatrix_t(pack_half2(e0, e1)), pb1 = movmatrix_t(pack_half2(e2, e3));
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    o[mt][0] *= al0;
    o[mt][2] *= al0;
    o[mt][1] *= al1;
    o[mt][3] *= al1;
    mma_16816(o[mt], movmatrix_t(word_of(vr[0], 2 * mt)), movmatrix_t(word_of(vr[0], 2 * mt + 1)),
              movmatrix_t(word_of(vr[1], 2 * mt)), movmatrix_t(word_of(vr[1], 2 * mt + 1)), pb0, pb1);
  }
}

// Where a warp's fragments hold head h, dims d and d + 1 (d even): value k
// (o[k >> 2][k & 3]) of lanes `lane` and lane + 4.
__device__ __forceinline__ void frag_slot(int h, int d, int& lane, int& k) {
  const int mt = 2 * (d >> 5) + ((d >> 2) & 1);
  k = 4 * mt + 2 * ((d >> 1) & 1) + (h & 1);
  lane = 8 * ((d >> 3) & 3) + (h >> 1);
}

// A warp's fragments into its [32][32] shared-memory block: value k of a
// lane at (k + 4 * lane) mod 32 (16-byte stores, conflict-free); read back
// with frag_slot.
__device__ __forceinline__ void store_frags(float (*wo)[32], const float (&o)[8][4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt)
    *reinterpret_cast<float4*>(&wo[lane][(4 * mt + 4 * lane) & 31]) = make_float4(o[mt][0], o[mt][1], o[mt][2], o[mt][3]);
}
__device__ __forceinline__ float2 load_frag_pair(const float (*wo)[32], int la, int k) {
  return make_float2(wo[la][(k + 4 * la) & 31], wo[la + 4][(k + 4 * (la + 4)) & 31]);
}

}  // namespace fd
}  // namespace lmps
