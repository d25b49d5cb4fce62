// Q4 weights (utils/pack_weights.py:11-47: packed u8 [N, K/2], element 2b in
// the low nibble of byte b; fp16 scales [N, K/32]; w = (nibble - 8) * scale,
// quant_matmul.metal:39-47) as fp16 on the tensor-core path, and the
// tile-major copy the batched decode kernel streams.
//
// Tile-major blocks: for weight-row tile i (rows 128 i .. 128 i + 127) and
// K step j (elements 64 j .. 64 j + 63), block i * (K / 64) + j is
//   bytes [0, 4096):    row r's 32 packed bytes at 32 r, its two 16-byte
//                       halves swapped when (r >> 2) & 1 (so eight threads
//                       reading the same half of eight rows hit distinct banks)
//   bytes [4096, 4608): row r's two group scales (groups 2 j, 2 j + 1) at 4 r
// so one bulk copy brings a whole K step of a tile, scales included.
#pragma once

#include "common.cuh"

namespace lmps {
namespace q4t {

constexpr int kTileRows = 128;
constexpr int kStepK = 64;
constexpr int kPackedBytes = kTileRows * kStepK / 2;           // 4096
constexpr int kBlockBytes = kPackedBytes + kTileRows * 4;      // 4608

__device__ __forceinline__ int half_swap(int r) { return (r >> 2) & 1; }

// fp16 (nibble - 8) * scale of the 8 elements of one packed word, in element
// order.  Halves of t_i hold the nibbles (i, i + 4) as 1024 + n: (n | 0x6400)
// is the fp16 1024 + n, minus 1032 gives n - 8 exactly, times the group scale
// rounds once.
__device__ __forceinline__ uint4 dequant8(uint32_t w, __half2 s2) {
  const __half2 k1032 = __halves2half2(__ushort_as_half(0x6408u), __ushort_as_half(0x6408u));
  uint32_t t[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t v = ((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u;
    const __half2 h = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&v), k1032), s2);
    t[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(__byte_perm(t[0], t[1], 0x5410), __byte_perm(t[2], t[3], 0x5410),
                    __byte_perm(t[0], t[1], 0x7632), __byte_perm(t[2], t[3], 0x7632));
}

}  // namespace q4t
}  // namespace lmps
