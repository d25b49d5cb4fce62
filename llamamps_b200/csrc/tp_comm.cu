// Two-way tensor-parallel exchange over peer memory (NVLink P2P, one process
// per GPU): the all-reduce (sum) of the partial o_proj / down_proj products
// that follows each of them in a tensor-parallel decoder layer
// (runners/engine.py:215-221,237-243 with the projection split by K across
// two GPUs), fused with the residual add:
//
//   x <- x + (part_self + part_peer)        (fp16, two roundings)
//
// which is what an NCCL fp16 sum of the two partials followed by
// residual_add computes.  fp16 addition is commutative, so both ranks derive
// bit-identical x.
//
// Each rank owns one exchange buffer (cudaMalloc'd here so that a CUDA IPC
// handle covers it exactly) and maps the peer's through CUDA IPC.  Per call
// site ("site": one all-reduce position in the decode step) the buffer
// holds two receive slots of max_n halves and one flag word per CTA; the
// rank keeps a private count of completed calls per (site, CTA).
//
// Call protocol, per CTA c of the grid (both ranks launch the same grid):
//   1. store this rank's slice of `part` into the peer's receive slot
//      (call count + 1) & 1 -- plain stores over NVLink, no multicast;
//   2. fence (system scope), then release-store the new call count into the
//      peer's flag c;
//   3. wait (acquire, bounded) until this rank's flag c, written by the peer,
//      has reached the same count; a wait that runs out raises *error and
//      returns without touching x (and later calls return at once while
//      *error is set);
//   4. x <- x + (part + received) over the slice.
// A CTA only waits for its counterpart CTA on the other GPU, so there is no
// grid-wide barrier.  Two receive slots make back-to-back calls on one site
// safe: the peer cannot start call k + 2 (slot k & 1 again) before this rank
// has finished call k + 1, which is after it read call k.  The flags only
// grow, so a peer that has already moved one call ahead still satisfies the
// wait (>= in wrap-around arithmetic).
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace lmps {
namespace tp {

constexpr int kThreads = 256;
constexpr int kMaxCtas = kTp2MaxCtas;  // flag words per site

__device__ __forceinline__ uint32_t hadd2u(uint32_t a, uint32_t b) {
  const __half2 r = __hadd2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}

__global__ void __launch_bounds__(kThreads)
    allreduce_residual_kernel(const uint4* __restrict__ part, uint4* __restrict__ x, int n8, int slot8,
                              uint4* peer_recv, const uint4* recv, uint32_t* peer_flags, const uint32_t* flags,
                              uint32_t* seen, int32_t* error, unsigned long long wait_ns) {
  __shared__ int ok;
  // an earlier exchange failed (the pair is out of step): the whole CTA
  // leaves, on one reading of the flag
  if (threadIdx.x == 0) ok = *reinterpret_cast<volatile int32_t*>(error) == 0;
  __syncthreads();
  if (!ok) return;
  const int per = (n8 + gridDim.x - 1) / gridDim.x;
  const int lo = blockIdx.x * per, hi = min(n8, lo + per);
  const uint32_t want = seen[blockIdx.x] + 1u;
  const int sl = static_cast<int>(want & 1u) * slot8;
  for (int i = lo + threadIdx.x; i < hi; i += kThreads) peer_recv[sl + i] = part[i];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool good = lmps_tp2_handshake(peer_flags, flags, blockIdx.x, want, error, wait_ns);
    if (good) seen[blockIdx.x] = want;
    ok = good ? 1 : 0;
  }
  __syncthreads();
  if (!ok) return;
  __threadfence_system();
  for (int i = lo + threadIdx.x; i < hi; i += kThreads) {
    const uint4 a = part[i], b = __ldcg(recv + sl + i), r = x[i];
    x[i] = make_uint4(hadd2u(r.x, hadd2u(a.x, b.x)), hadd2u(r.y, hadd2u(a.y, b.y)), hadd2u(r.z, hadd2u(a.z, b.z)),
                      hadd2u(r.w, hadd2u(a.w, b.w)));
  }
}

// Vocabulary-split LM head, the cross-rank step (runners/engine.py:171-181
// with the head's rows divided between two GPUs): each rank found the
// first-index argmax of its own rows; one CTA turns it into a key (value
// key | 0xffffffff - global row, so the larger value and then the lower
// global row wins, numpy's first-index rule), stores it into the peer's
// receive slot, hands off with the peer's CTA and keeps the larger key.
// Both ranks derive the same id.  Same slots, flags and error behaviour as
// allreduce_residual_kernel (flag word 0 of the site).
__global__ void argmax_exchange_kernel(const __half* __restrict__ logits, int ld, const int32_t* __restrict__ local,
                                       int rows, uint32_t row_offset, int32_t* __restrict__ ids, int slot_u64,
                                       unsigned long long* peer_recv, const unsigned long long* recv,
                                       uint32_t* peer_flags, const uint32_t* flags, uint32_t* seen, int32_t* error,
                                       unsigned long long wait_ns) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = *reinterpret_cast<volatile int32_t*>(error) == 0;
  __syncthreads();
  if (!ok) return;
  const uint32_t want = seen[0] + 1u;
  const int sl = static_cast<int>(want & 1u) * slot_u64;
  const int b = threadIdx.x;
  unsigned long long key = 0ull;
  if (b < rows) {
    const int32_t i = local[b];
    const float v = __half2float(logits[static_cast<size_t>(b) * ld + i]);
    key = argmax_key(v, row_offset + static_cast<uint32_t>(i));
    peer_recv[sl + b] = key;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool good = lmps_tp2_handshake(peer_flags, flags, 0, want, error, wait_ns);
    if (good) seen[0] = want;
    ok = good ? 1 : 0;
  }
  __syncthreads();
  if (!ok) return;
  __threadfence_system();
  if (b < rows) {
    const unsigned long long best = u64_max(key, __ldcg(recv + sl + b));
    ids[b] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
  }
}

}  // namespace tp
}  // namespace lmps

using namespace lmps;

extern "C" int lmps_comm_alloc(size_t bytes, void** ptr) {
  LMPS_CHECK_ARG(ptr && bytes > 0);
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return static_cast<int>(e);
  }
  return LMPS_OK;
}

extern "C" int lmps_comm_free(void* ptr) {
  LMPS_CHECK_ARG(ptr);
  return static_cast<int>(cudaFree(ptr));
}

extern "C" int lmps_ipc_handle(const void* ptr, void* handle) {
  LMPS_CHECK_ARG(ptr && handle);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return static_cast<int>(e);
  memcpy(handle, &h, sizeof(h));
  return LMPS_OK;
}

extern "C" int lmps_ipc_open(const void* handle, void** ptr) {
  LMPS_CHECK_ARG(handle && ptr);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return static_cast<int>(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int lmps_ipc_close(void* ptr) {
  LMPS_CHECK_ARG(ptr);
  return static_cast<int>(cudaIpcCloseMemHandle(ptr));
}

extern "C" size_t lmps_tp2_comm_bytes(int n_sites, int max_n) {
  if (n_sites < 1 || max_n < 8 || max_n % 8) return 0;
  return static_cast<size_t>(n_sites) * (2u * static_cast<size_t>(max_n) * 2u + tp::kMaxCtas * 4u);
}

extern "C" int lmps_tp2_allreduce_residual(const uint16_t* part, uint16_t* x, int n, void* comm, void* peer_comm,
                                           uint32_t* seen, int site, int n_sites, int max_n, int32_t* error,
                                           unsigned long long wait_ns, void* stream) {
  LMPS_CHECK_ARG(part && x && comm && peer_comm && seen && error);
  LMPS_CHECK_ARG(n_sites >= 1 && site >= 0 && site < n_sites && max_n >= 8 && max_n % 8 == 0);
  LMPS_CHECK_ARG(n >= 8 && n % 8 == 0 && n <= max_n);
  LMPS_CHECK_ARG(lmps_aligned(part, 16) && lmps_aligned(x, 16) && lmps_aligned(comm, 16) &&
                 lmps_aligned(peer_comm, 16) && lmps_aligned(seen, 4));
  const Tp2Site t = lmps_tp2_site(comm, peer_comm, site, n_sites, max_n);
  const int n8 = n / 8;
  // One CTA per 2048 elements of the site's largest call, at most kMaxCtas:
  // every CTA of the grid is resident at once, so each one's counterpart on
  // the peer GPU runs too.  The grid depends on max_n only, never on n: every
  // CTA of a site takes part in every call of that site (a CTA whose slice is
  // empty still hands off), so the per-CTA call counts -- and with them the
  // receive slot each call uses -- stay equal across the CTAs of the site
  // whatever sizes successive calls have.
  const int grid = std::min(tp::kMaxCtas, (max_n / 8 + tp::kThreads - 1) / tp::kThreads);
  tp::allreduce_residual_kernel<<<grid, tp::kThreads, 0, lmps_stream(stream)>>>(
      reinterpret_cast<const uint4*>(part), reinterpret_cast<uint4*>(x), n8, max_n / 8,
      reinterpret_cast<uint4*>(t.peer_recv), reinterpret_cast<const uint4*>(t.recv), t.peer_flags, t.flags,
      seen + site * tp::kMaxCtas, error, wait_ns ? wait_ns : kTp2DefaultWaitNs);
  return lmps_launch_status();
}

extern "C" int lmps_tp2_argmax_exchange(const uint16_t* logits, int ld, const int32_t* local_ids, int rows,
                                        int row_offset, int32_t* ids, void* comm, void* peer_comm, uint32_t* seen,
                                        int site, int n_sites, int max_n, int32_t* error,
                                        unsigned long long wait_ns, void* stream) {
  LMPS_CHECK_ARG(logits && local_ids && ids && comm && peer_comm && seen && error);
  LMPS_CHECK_ARG(rows >= 1 && rows <= tp::kThreads && ld >= 1 && row_offset >= 0);
  LMPS_CHECK_ARG(n_sites >= 1 && site >= 0 && site < n_sites && max_n >= 8 && max_n % 8 == 0);
  LMPS_CHECK_ARG(4LL * rows <= max_n);  // rows 64-bit keys per receive slot of max_n halves
  LMPS_CHECK_ARG(lmps_aligned(comm, 16) && lmps_aligned(peer_comm, 16) && lmps_aligned(seen, 4));
  const Tp2Site t = lmps_tp2_site(comm, peer_comm, site, n_sites, max_n);
  tp::argmax_exchange_kernel<<<1, tp::kThreads, 0, lmps_stream(stream)>>>(
      reinterpret_cast<const __half*>(logits), ld, local_ids, rows, static_cast<uint32_t>(row_offset), ids,
      max_n / 4, reinterpret_cast<unsigned long long*>(t.peer_recv), reinterpret_cast<const unsigned long long*>(t.recv),
      t.peer_flags, t.flags, seen + site * tp::kMaxCtas, error, wait_ns ? wait_ns : kTp2DefaultWaitNs);
  return lmps_launch_status();
}
