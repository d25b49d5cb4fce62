// Fused GQA decode attention over the paged fp16 KV cache (sm_100a).
//
// One kernel does what kernels/attention.metal (scores), softmax.metal and
// attn_sum.metal do in three dispatches (runners/engine.py:202-212), for a
// real cache of seq_lens[b] positions.  Grid = (splits, kv heads,
// sequences): each CTA runs one split-KV item (decode_attention.cuh: the
// G query heads of a KV head over a contiguous range of positions, K/V
// tiles staged with cp.async, the folds on the tensor cores); with more than
// one split a combine kernel merges the partials.  The _rope entry point
// also does rope_kv_append's work (RoPE on q and k, the cache append).
#include "decode_attention.cuh"

namespace lmps {

using AttnSmem = AttnSmemT<2>;  // two K/V tiles: 67 KB, three CTAs per SM

__global__ void __launch_bounds__(kAttnThreads) gqa_decode_attn_kernel(const AttnParams P) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>(smem_raw);
  const QkvRowLoader qkv{P.qkv, (P.n_q_heads + 2 * P.n_kv_heads) * kHeadDim};
  attn_item(P, S, blockIdx.x, blockIdx.y, blockIdx.z, threadIdx.x, P.qkv != nullptr, qkv, CtaSync{});
}

// Merge the per-split partials of one (sequence, query head): log-sum-exp.
__global__ void __launch_bounds__(kHeadDim) gqa_combine_kernel(const AttnParams P) {
  lmps_pdl_trigger();
  lmps_pdl_wait();
  attn_combine(P, blockIdx.x, blockIdx.y, threadIdx.x);
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
