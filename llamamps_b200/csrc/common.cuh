// Shared helpers for the LlamaMPS B200 kernels (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/llamamps_b200.h"

#define LMPS_CHECK_ARG(cond)                      \
  do {                                            \
    if (!(cond)) return LMPS_ERR_INVALID_ARGUMENT; \
  } while (0)

// Status after a launch: 0, or the CUDA error code (always > 0).
static inline int lmps_launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LMPS_OK : static_cast<int>(e);
}

static inline cudaStream_t lmps_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Programmatic dependent launch: the kernel may begin while its predecessor
// in the stream is still running.  Such a kernel triggers its own dependents
// early (lmps_pdl_trigger) and calls lmps_pdl_wait() in every thread before
// it reads or writes anything an earlier kernel writes or reads (waiting
// means the predecessor -- and through it every earlier grid -- completed).
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void lmps_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void lmps_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
static inline int lmps_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                  Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  return e == cudaSuccess ? lmps_launch_status() : static_cast<int>(e);
}

static inline bool lmps_aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// Opt a kernel into `bytes` of dynamic shared memory on the current device.
// The attribute belongs to the kernel in one device's context, so it is set
// once per (kernel, device): a process that drives several GPUs sets it on
// each of them before that device's first launch above 48 KB.  `Kern` is the
// kernel itself (one flag table per kernel, not per signature).
template <auto Kern>
static inline int lmps_max_dyn_smem(int bytes) {
  constexpr int kMaxDevices = 64;
  static int done[kMaxDevices] = {};  // largest size set so far, per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev >= 0 && dev < kMaxDevices && __atomic_load_n(&done[dev], __ATOMIC_ACQUIRE) >= bytes) return LMPS_OK;
  e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev >= 0 && dev < kMaxDevices) {
    int cur = __atomic_load_n(&done[dev], __ATOMIC_ACQUIRE);
    while (cur < bytes && !__atomic_compare_exchange_n(&done[dev], &cur, bytes, false, __ATOMIC_ACQ_REL,
                                                        __ATOMIC_ACQUIRE)) {
    }
  }
  return LMPS_OK;
}

namespace lmps {

constexpr int kWarp = 32;
constexpr int kQ4Group = 32;        // elements per scale (utils/pack_weights.py:9)
constexpr int kQ4GroupBytes = 16;   // 32 nibbles
constexpr float kAttnScale = 0.088388f;  // kernels/attention.metal:40

// Shared-memory address of a generic pointer into this CTA's shared memory.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over aligned segments of SEG lanes (SEG a power of two <= 32).
template <int SEG>
__device__ __forceinline__ float segment_sum(float v) {
#pragma unroll
  for (int o = SEG / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 128-bit streaming load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Nibble k (k = 0..7) of a 32-bit word as the signed code (n - 8) in fp32.
// 0x4B000000 is 2^23 as a float: OR-ing a 4-bit value into its mantissa gives
// exactly 2^23 + n, and subtracting 2^23 + 8 leaves n - 8 with no rounding.
__device__ __forceinline__ float nib_code(uint32_t w, int k) {
  return __uint_as_float(0x4B000000u | ((w >> (4 * k)) & 0xFu)) - 8388616.0f;
}

// Order-preserving map of a float onto uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// 64-bit argmax key: value in the high word, (0xffffffff - index) in the low
// word, so that atomicMax keeps the largest value and, among equal values,
// the smallest index -- numpy.argmax's first-index rule (runners/engine.py:181).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  return (static_cast<unsigned long long>(float_order_key(v)) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - idx);
}

__device__ __forceinline__ unsigned long long u64_max(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = u64_max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  return (g / (1.0f + expf(-g))) * u;
}

// ---------------------------------------------------------------------------
// RoPE -- kernels/rope.metal:19-40 with the position and frequency table as
// inputs: angle = float(pos) * inv_freq[i]; (x1, x2) -> (x1 c - x2 s, x1 s + x2 c).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void rope_pair_index(int pair, int head_dim, int style, int& i1, int& i2,
                                                int& fi) {
  const int half_d = head_dim / 2;
  const int h = pair / half_d;
  const int j = pair - h * half_d;
  if (style == LMPS_ROPE_INTERLEAVED) {
    i1 = h * head_dim + 2 * j;
    i2 = i1 + 1;
  } else {
    i1 = h * head_dim + j;
    i2 = i1 + half_d;
  }
  fi = j;
}

// The rotation with cos / sin already computed (rope_rotate's arithmetic).
__device__ __forceinline__ void rope_rotate_cs(__half& a, __half& b, float c, float s) {
  const float x1 = __half2float(a), x2 = __half2float(b);
  a = __float2half_rn(x1 * c - x2 * s);
  b = __float2half_rn(x1 * s + x2 * c);
}
__device__ __forceinline__ void rope_rotate(__half& a, __half& b, float ang) {
  float s, c;
  sincosf(ang, &s, &c);
  rope_rotate_cs(a, b, c, s);
}

}  // namespace lmps

// Exchange-buffer layout of the two-way tensor-parallel kernels (tp_comm.cu,
// q4_gemv.cu): [n_sites][2][max_n] fp16 receive slots, then
// [n_sites][kTp2MaxCtas] uint32 flags, in this rank's buffer and the peer's.
constexpr int kTp2MaxCtas = 64;
struct Tp2Site {
  uint16_t* recv;       // this rank's two slots of the site
  uint16_t* peer_recv;  // the peer's two slots (mapped)
  uint32_t* flags;      // this rank's flag words of the site (written by the peer)
  uint32_t* peer_flags;
};
static inline Tp2Site lmps_tp2_site(void* comm, void* peer_comm, int site, int n_sites, int max_n) {
  const size_t slots = static_cast<size_t>(n_sites) * 2u * static_cast<size_t>(max_n);
  const size_t off = static_cast<size_t>(site) * 2u * static_cast<size_t>(max_n);
  Tp2Site t;
  t.recv = static_cast<uint16_t*>(comm) + off;
  t.peer_recv = static_cast<uint16_t*>(peer_comm) + off;
  t.flags = reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(comm) + slots) + site * kTp2MaxCtas;
  t.peer_flags = reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(peer_comm) + slots) + site * kTp2MaxCtas;
  return t;
}
__device__ __forceinline__ void lmps_st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t lmps_ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long lmps_globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Default limit of the peer wait (wait_ns = 0): the host-side skew between
// two ranks that make the same calls stays far below it.
constexpr unsigned long long kTp2DefaultWaitNs = 5000000000ull;
// Thread 0 of a CTA: publish `want` to the peer's flag `cta`, then wait
// (bounded by wait_ns of %globaltimer) until this rank's flag `cta` reaches
// it.  False after a timeout (error raised).
__device__ __forceinline__ bool lmps_tp2_handshake(uint32_t* peer_flags, const uint32_t* flags, int cta,
                                                   uint32_t want, int32_t* error, unsigned long long wait_ns) {
  lmps_st_release_sys(peer_flags + cta, want);
  const unsigned long long t0 = lmps_globaltimer();
  while (static_cast<int>(lmps_ld_acquire_sys(flags + cta) - want) < 0) {
    if (lmps_globaltimer() - t0 > wait_ns) {
      atomicExch(error, 1);
      return false;
    }
  }
  return true;
}

