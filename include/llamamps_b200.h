/*
 * llamamps_b200.h -- C ABI of the B200 (sm_100a) LlamaMPS decode kernels.
 *
 * Conventions (mirroring the reference's Metal binding, runners/engine.py:49-58,
 * where every kernel takes positional device buffers and never allocates):
 *   - every pointer is a device pointer owned by the caller; fp16 tensors are
 *     passed as uint16_t* holding IEEE binary16 bits;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream);
 *   - a call enqueues work and returns LMPS_OK (0), a negative LMPS_ERR_* for
 *     rejected arguments (nothing is launched), or a positive cudaError_t from
 *     the launch; lmps_status_string() names any of them;
 *   - no entry point allocates device memory: scratch is passed in, with a
 *     *_workspace_size() query beside the call that needs it.
 *
 * Weight format (utils/pack_weights.py:18-46): a [rows, k] matrix is packed
 * row-major as uint8[rows*k/2] (element 2b in the low nibble of byte b, 2b+1
 * in the high nibble, code+8) plus fp16 scales[rows*k/32] (one per 32
 * consecutive elements, code = round(w / scale), scale = max|w| / 7).
 */
#ifndef LLAMAMPS_B200_H_
#define LLAMAMPS_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  LMPS_OK = 0,
  LMPS_ERR_INVALID_ARGUMENT = -1, /* shape/pointer/alignment rejected */
  LMPS_ERR_UNSUPPORTED = -2,      /* shape outside the compiled variants */
  LMPS_ERR_WORKSPACE = -3,        /* workspace too small */
  LMPS_ERR_DEVICE_TIMEOUT = -4    /* a bounded device-side wait gave up */
};

enum { LMPS_ROPE_INTERLEAVED = 0, LMPS_ROPE_NEOX = 1 };

/* Library version (major*10000 + minor*100 + patch). */
int lmps_version(void);
/* Human-readable name of a status code returned by any entry point. */
const char* lmps_status_string(int status);

/* ---- Q4 GEMV family ------------------------------------------------------
 * y[b, r] = sum_k W[r, k] * x[b, k] with W in the Q4 format above, fp32
 * accumulation, y rounded to fp16.  x is [batch, k] with row stride ldx
 * elements, y is [batch, rows] with row stride ldy.  k % 32 == 0,
 * 1 <= batch <= 8, packed 16-byte aligned.
 */

/* Replaces kernels/quant_matmul.metal:15-22 `gemv_q4_0` (dispatched at
 * runners/engine.py:192-195, :215-217, :228-231, :237-239, :171-175). */
int lmps_gemv_q4_0(const uint8_t* packed, const uint16_t* scales, const uint16_t* x, int ldx,
                   uint16_t* y, int ldy, int rows, int k, int batch, void* stream);

/* gemv_q4_0 + bias epilogue: y = fp16(acc + bias[r]).  Qwen2 q/k/v biases
 * (absent from the reference, runners/engine.py:124-141). */
int lmps_gemv_q4_bias(const uint8_t* packed, const uint16_t* scales, const uint16_t* bias,
                      const uint16_t* x, int ldx, uint16_t* y, int ldy, int rows, int k,
                      int batch, void* stream);

/* gemv_q4_0 + residual_add: y = residual + fp16(acc) in fp16.  Replaces the
 * o_proj/down_proj GEMV + kernels/residual.metal:13-20 pair
 * (runners/engine.py:215-221, :237-243).  y may alias residual. */
int lmps_gemv_q4_residual(const uint8_t* packed, const uint16_t* scales, const uint16_t* x,
                          int ldx, const uint16_t* residual, uint16_t* y, int ldy, int rows,
                          int k, int batch, void* stream);

/* gate/up GEMVs + kernels/swiglu.metal:13-23: y = fp16(silu(g) * u) with
 * g = fp16(acc_gate), u = fp16(acc_up) (runners/engine.py:228-235). */
int lmps_gemv_q4_swiglu(const uint8_t* gate_packed, const uint16_t* gate_scales,
                        const uint8_t* up_packed, const uint16_t* up_scales, const uint16_t* x,
                        int ldx, uint16_t* y, int ldy, int rows, int k, int batch, void* stream);

/* LM head GEMV + argmax.  Replaces runners/engine.py:171-181 (Q4 tied head
 * GEMV, logits read-back, host argmax over fp32(logits) with first-index
 * ties).  logits (may be NULL) receives fp16[batch, rows].  keys is a
 * caller-owned uint64[batch] workspace that must be zero on entry and is left
 * zero on return; token_ids receives int32[batch]. */
int lmps_lm_head_argmax(const uint8_t* packed, const uint16_t* scales, const uint16_t* x,
                        int ldx, uint16_t* logits, unsigned long long* keys,
                        int32_t* token_ids, int rows, int k, int batch, void* stream);

/* ---- normalisation / elementwise ---------------------------------------- */

/* Replaces kernels/rms_norm.metal:14-19 `rms_norm_q4` (runners/engine.py:188-190,
 * :224-226, :165-169): out = fp16(fp16(x * rsqrt(mean(x^2) + eps)) * gamma),
 * reduced over the full vector.  x/out are [batch, dim]. */
int lmps_rms_norm(const uint16_t* x, const uint16_t* gamma, uint16_t* out, int dim, int batch,
                  float eps, void* stream);

/* Replaces kernels/rope.metal:13-16 `apply_rope_q4` (runners/engine.py:198-200),
 * in place on vec [batch, n_heads*head_dim] at position pos[b].  inv_freq is
 * fp32[head_dim/2] (base^-(2i/head_dim)); style LMPS_ROPE_*. */
int lmps_rope(uint16_t* vec, const int32_t* pos, const float* inv_freq, int n_heads,
              int head_dim, int batch, int style, void* stream);

/* Replaces kernels/residual.metal:13-20 `residual_add`: out = x + y (fp16). */
int lmps_residual_add(const uint16_t* x, const uint16_t* y, uint16_t* out, int n, void* stream);

/* Replaces kernels/swiglu.metal:13-23 `swiglu`. */
int lmps_swiglu(const uint16_t* gate, const uint16_t* up, uint16_t* out, int n, void* stream);
/* SwiGLU of a fused gate|up projection: out[r][i] = silu(gu[r][i]) * gu[r][n + i]
 * for rows x n (swiglu.metal; the gate and up halves of one GEMM output row,
 * row stride ld >= 2n; out row stride ldo). */
int lmps_swiglu_rows(const uint16_t* gate_up, int ld, int rows, int n, uint16_t* out, int ldo, void* stream);

/* Replaces the embedding-row lookup of utils/tokenizer.py:22-26 on the device:
 * out[b, :] = table[ids[b], :] for an fp16 [vocab, dim] table.  Ids outside
 * [0, vocab) produce a zero row and set *bad_ids (may be NULL) to 1. */
int lmps_embed_gather(const uint16_t* table, const int32_t* ids, uint16_t* out, int dim,
                      int vocab, int batch, int32_t* bad_ids, void* stream);

/* ---- attention ------------------------------------------------------------
 * The reference's three-stage attention over a contiguous cache
 * k_cache/v_cache [seq_len, n_kv_heads*head_dim] (kernels/attention.metal:33,
 * kernels/attn_sum.metal:30), scores fp32 [n_q_heads, seq_len]. */

/* Replaces kernels/attention.metal:13-18 `attention_scores` (engine.py:202-204). */
int lmps_attention_scores(const uint16_t* q, const uint16_t* k_cache, float* scores,
                          int seq_len, int n_q_heads, int n_kv_heads, int head_dim,
                          void* stream);
/* Replaces kernels/softmax.metal:14-18 `softmax` (engine.py:206-208), in place. */
int lmps_softmax(float* scores, int seq_len, int n_heads, void* stream);
/* Replaces kernels/attn_sum.metal:14-19 `attn_weighted_sum` (engine.py:210-212). */
int lmps_attn_weighted_sum(const float* scores, const uint16_t* v_cache, uint16_t* out,
                           int seq_len, int n_q_heads, int n_kv_heads, int head_dim,
                           void* stream);

/* Paged KV cache: one layer's K (and V) pool is fp16
 * [n_pages, n_kv_heads, page_size, head_dim]; block_table is int32
 * [batch, max_pages] mapping page j of sequence b to a pool page. */

/* RoPE + KV append, the q/k half of runners/engine.py:198-200 plus the cache
 * write the reference lacks (engine.py:90-91 hold one token).  qkv is the
 * fused q|k|v GEMV output [batch, (n_q+2*n_kv)*head_dim]; q_out receives the
 * rotated q [batch, n_q*head_dim]; rotated k and raw v go to position pos[b]. */
int lmps_rope_kv_append(const uint16_t* qkv, const int32_t* pos, const float* inv_freq,
                        uint16_t* q_out, uint16_t* k_pool, uint16_t* v_pool,
                        const int32_t* block_table, int max_pages, int page_size,
                        int n_q_heads, int n_kv_heads, int head_dim, int batch, int style,
                        void* stream);

/* Fused GQA decode attention (scores + softmax + weighted sum of
 * kernels/attention.metal, softmax.metal, attn_sum.metal) over the paged
 * cache for seq_lens[b] positions, split over the sequence with a
 * log-sum-exp combine.  out is fp16 [batch, n_q_heads*head_dim].  workspace
 * must hold lmps_gqa_attention_workspace_size(...) bytes. */
int lmps_gqa_attention_splits(int batch, int n_kv_heads, int max_seq_len, int page_size);
size_t lmps_gqa_attention_workspace_size(int batch, int n_q_heads, int head_dim, int n_splits);
int lmps_gqa_decode_attention(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                              const int32_t* block_table, const int32_t* seq_lens, uint16_t* out,
                              void* workspace, size_t workspace_bytes, int max_pages,
                              int page_size, int n_q_heads, int n_kv_heads, int head_dim,
                              int batch, int max_seq_len, int n_splits, void* stream);

/* lmps_rope_kv_append followed by lmps_gqa_decode_attention in one launch
 * (kernels/rope.metal + the cache append, then attention.metal, softmax.metal,
 * attn_sum.metal): qkv is the biased q|k|v row of each sequence
 * [batch, (n_q_heads + 2 n_kv_heads) * head_dim]; pos[b] is the new token's
 * position and seq_lens[b] must be pos[b] + 1.  The rotated K row and the V
 * row of pos[b] are written into the pools (as lmps_rope_kv_append writes
 * them) and attended in the same call; out and the workspace as for
 * lmps_gqa_decode_attention.  Outputs are bit-identical to the two calls. */
int lmps_gqa_decode_attention_rope(const uint16_t* qkv, const int32_t* pos, const float* inv_freq,
                                   int rope_style, uint16_t* k_pool, uint16_t* v_pool,
                                   const int32_t* block_table, const int32_t* seq_lens, uint16_t* out,
                                   void* workspace, size_t workspace_bytes, int max_pages, int page_size,
                                   int n_q_heads, int n_kv_heads, int head_dim, int batch, int max_seq_len,
                                   int n_splits, void* stream);

/* Size of the fixed device scratch used by lmps_gqa_decode_attention_noalloc. */
#define LMPS_GQA_ATTENTION_NOALLOC_SCRATCH_BYTES (4u * 1024u * 1024u)

/* No counterpart in the reference.  lmps_gqa_decode_attention for callers
 * that cannot allocate device memory where they call it (a binding that only
 * receives device pointers from another runtime, code under a global-mode
 * stream capture, a serving loop that bans allocation after warm-up): the
 * split partials live in a 4 MiB array compiled into the library and resident
 * on every GPU that loads it until exit, so no workspace is passed and nothing
 * is allocated.  The first call on each device looks the array's device
 * address up (cudaGetSymbolAddress) and should come before any stream
 * capture.  Returns LMPS_ERR_WORKSPACE without launching when
 * lmps_gqa_attention_workspace_size(batch, n_q_heads, head_dim, n_splits)
 * exceeds LMPS_GQA_ATTENTION_NOALLOC_SCRATCH_BYTES.  All calls share the
 * array: calls that overlap on the GPU race. */
int lmps_gqa_decode_attention_noalloc(const uint16_t* q, const uint16_t* k_pool,
                                      const uint16_t* v_pool, const int32_t* block_table,
                                      const int32_t* seq_lens, uint16_t* out, int max_pages,
                                      int page_size, int n_q_heads, int n_kv_heads, int head_dim,
                                      int batch, int max_seq_len, int n_splits, void* stream);

/* ---- prefill / large-batch projections ------------------------------------ */

/* W4A16 GEMM on the tcgen05 tensor cores (TMEM accumulators), for prefill and
 * large-batch decode where the Q4 projections of quant_matmul.metal:15-69 are
 * dense contractions: y[m, :n] = x[m, :k] . W^T with W the Q4 [n, k] layout of
 * lmps_gemv_q4_0 (dequantised to fp16 tile by tile), fp32 accumulate, fp16 out.
 * epilogue: 0 none, 1 + bias[n], 2 residual[m, n] + fp16(acc) (residual may
 * alias y; 16-byte aligned, ldr a multiple of 8), 3 SwiGLU (swiglu.metal:13-23): W's rows interleave gate and up
 * (row 2t = gate row t, 2t + 1 = up row t) and y[m, t] =
 * fp16(silu(fp16(gate)) * fp16(up)) for t < n/2 (ldy >= n/2).
 * n must be a multiple of 128 and k of 64 (else UNSUPPORTED); any
 * m >= 1.  error[0] is set to 1 if a bounded wait for the tensor core gives up.
 * Calls with fewer than 128 tokens split K over the CTAs of a thread-block
 * cluster and sum the partial tiles in distributed shared memory, so the
 * workspace arguments are unused (lmps_w4a16_gemm_workspace_size returns 0;
 * pass NULL, 0).  packed must be 16-byte aligned (TMA).  Replaces the
 * per-token dispatch of runners/engine.py:188-243 at B > 1. */
#define LMPS_EPI_NONE 0
#define LMPS_EPI_BIAS 1
#define LMPS_EPI_RESIDUAL 2
#define LMPS_EPI_SWIGLU 3
size_t lmps_w4a16_gemm_workspace_size(int m, int n);
int lmps_w4a16_gemm(const uint16_t* x, int ldx, const uint8_t* packed, const uint16_t* scales,
                    const uint16_t* bias, const uint16_t* residual, int ldr, uint16_t* y, int ldy,
                    int m, int n, int k, int epilogue, int32_t* error, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Causal prefill attention (attention.metal + softmax.metal + attn_sum.metal,
 * runners/engine.py:202-212, for every prompt position at once): q holds the
 * rotated queries of seq_len positions of each of `batch` sequences, row
 * b*seq_len + p, [.., n_q_heads*head_dim] with leading dimension ldq; their
 * K/V rows are already in the paged cache (block_table [batch, max_pages]).
 * Query p attends to positions 0..p; out has q's row layout.  head_dim 128,
 * n_q_heads / n_kv_heads <= 6. */
int lmps_prefill_attention(const uint16_t* q, int ldq, const uint16_t* k_pool, const uint16_t* v_pool,
                           const int32_t* block_table, int max_pages, int page_size, uint16_t* out, int ldo,
                           int batch, int seq_len, int n_q_heads, int n_kv_heads, int head_dim, void* stream);

/* The same causal prefill attention on the tcgen05 tensor cores with S and O
 * accumulators in tensor memory and K/V tiles loaded by TMA from the pools
 * (n_pages pages of [n_kv_heads, page_size, head_dim] each).  Takes head_dim
 * 128, page_size a multiple of 64 and an even n_q_heads / n_kv_heads (else
 * UNSUPPORTED: use lmps_prefill_attention).  q, the pools and out 16-byte
 * aligned, ldq and ldo multiples of 8.  error[0] is set to 1 if a bounded
 * wait for the tensor core gives up. */
int lmps_prefill_attention_tcgen05(const uint16_t* q, int ldq, const uint16_t* k_pool, const uint16_t* v_pool,
                                   int n_pages, const int32_t* block_table, int max_pages, int page_size,
                                   uint16_t* out, int ldo, int batch, int seq_len, int n_q_heads,
                                   int n_kv_heads, int head_dim, int32_t* error, void* stream);

/* First-index argmax of each row of fp16 logits [rows, ld] over n columns
 * (runners/engine.py:180-181), the large-batch companion of the LM-head GEMM. */
int lmps_argmax_rows(const uint16_t* logits, int ld, int rows, int n, int32_t* ids, void* stream);

/* Top-k / temperature sampling of each row of fp16 logits [rows, ld] over n
 * columns, beside the greedy argmax of runners/engine.py:180-181 (the
 * reference has no sampling).  The k largest logits (ties at the k-th value:
 * lowest indices first) in ascending index order get weights
 * exp((v - max) / temperature) (fp32); u = the top 24 bits of the first
 * Philox4x32-10 word for key = seed and counter = (row, offset low 32 bits,
 * offset high 32 bits, 0), times 2^-24; ids[row] = the first candidate whose
 * running weight sum exceeds u times the total (sums in a fixed order: see
 * csrc/sampling.cu).  Same seed, offset and logits give the same ids.
 * temperature <= 0 or top_k == 1: the largest logit, lowest index on ties.
 * NaN logits are never chosen.  1 <= top_k <= min(1024, n).  ids2, when not
 * NULL, receives a copy (e.g. a history row). */
int lmps_sample_rows(const uint16_t* logits, int ld, int rows, int n, int top_k, float temperature,
                     unsigned long long seed, unsigned long long offset, int32_t* ids, int32_t* ids2,
                     void* stream);

/* ---- two-way tensor parallelism over peer memory ------------------------
 * The all-reduce (sum) of the two ranks' partial o_proj / down_proj products
 * that follows each split projection (runners/engine.py:215-221,237-243 with
 * K split across two GPUs), fused with the residual add, over NVLink P2P
 * stores into the peer's buffer (one process per GPU, CUDA IPC mapping).
 *
 * lmps_comm_alloc: a zero-filled device buffer of `bytes` (its own cudaMalloc,
 * so an IPC handle covers it exactly); lmps_comm_free releases it.
 * lmps_ipc_handle writes the 64-byte cudaIpcMemHandle_t of such a buffer;
 * lmps_ipc_open maps a peer's handle (peer access enabled lazily);
 * lmps_ipc_close unmaps it.
 * lmps_tp2_comm_bytes: the exchange buffer size for n_sites call sites of at
 * most max_n fp16 elements each (max_n a multiple of 8), 0 if invalid. */
int lmps_comm_alloc(size_t bytes, void** ptr);
int lmps_comm_free(void* ptr);
int lmps_ipc_handle(const void* ptr, void* handle);
int lmps_ipc_open(const void* handle, void** ptr);
int lmps_ipc_close(void* ptr);
size_t lmps_tp2_comm_bytes(int n_sites, int max_n);

/* x[i] <- x[i] + (part[i] + peer's part[i]) for i < n (fp16; both ranks get
 * bit-identical x).  comm = this rank's exchange buffer, peer_comm = the
 * peer's, mapped; seen = this rank's private uint32 [n_sites * 64] call
 * counters (zeroed with the buffers).  Both ranks must make the same calls
 * (site, n) in the same order; calls on one site may follow each other
 * directly, with any n <= max_n.  A wait for the peer that runs out
 * (wait_ns nanoseconds of the GPU's global timer; 0 = 5 s) sets *error and
 * leaves x unchanged, and later calls return at once while *error is set;
 * the buffers and counters of both ranks must then be zeroed again.  The
 * grid is ceil(max_n / 2048) CTAs, at most 64, all resident at once; it
 * depends on max_n only, so every CTA takes part in every call of a site. */
int lmps_tp2_allreduce_residual(const uint16_t* part, uint16_t* x, int n, void* comm, void* peer_comm,
                                uint32_t* seen, int site, int n_sites, int max_n, int32_t* error,
                                unsigned long long wait_ns, void* stream);

/* The split o_proj / down_proj GEMV and its all-reduce in ONE kernel
 * (kernels/quant_matmul.metal:15-69 on this rank's K slice, then
 * runners/engine.py:219-221 / 241-243 over both ranks): part[b, r] =
 * fp16(W_r . a[b]) for the `rows` rows, stored locally and into the peer's
 * receive slot; after a hand-off between the same CTA on both GPUs,
 * x[b, r] <- x[b, r] + (part[b, r] + peer's part[b, r]).  x and part are
 * [batch, rows] contiguous, batch * rows <= max_n; same exchange buffers,
 * counters, call rules, wait limit and error behaviour as
 * lmps_tp2_allreduce_residual (use other sites than it; the grid depends on
 * rows only).  LMPS_ERR_UNSUPPORTED when the GEMV grid would
 * exceed 64 CTAs. */
int lmps_gemv_q4_tp2_residual(const uint8_t* packed, const uint16_t* scales, const uint16_t* a, int lda,
                              uint16_t* x, uint16_t* part, int rows, int k, int batch, void* comm,
                              void* peer_comm, uint32_t* seen, int site, int n_sites, int max_n,
                              int32_t* error, unsigned long long wait_ns, void* stream);

/* Vocabulary-split LM head (runners/engine.py:171-181 with the head's rows
 * divided between the two ranks): rank r ran lmps_lm_head_argmax over its
 * own rows [row_offset, row_offset + its row count), writing its fp16
 * logits [rows, ld] and local first-index argmax local_ids; this call
 * exchanges (logit, global row) with the peer and writes the global
 * first-index argmax to ids on both ranks (the larger logit, then the lower
 * global row).  rows <= 256 sequences, 4 * rows <= max_n; same exchange
 * buffers, counters, call rules, wait limit and error behaviour as
 * lmps_tp2_allreduce_residual (a site of its own; one CTA). */
int lmps_tp2_argmax_exchange(const uint16_t* logits, int ld, const int32_t* local_ids, int rows, int row_offset,
                             int32_t* ids, void* comm, void* peer_comm, uint32_t* seen, int site, int n_sites,
                             int max_n, int32_t* error, unsigned long long wait_ns, void* stream);

/* ---- weight format ---------------------------------------------------- */

/* Device Q4 packer, bit-exact with utils/pack_weights.py:18-46
 * `pack_tensor_4bit`: w is fp32[n]; packed receives ceil(n/32)*16 bytes and
 * scales ceil(n/32) fp16 values (the tail group is zero-padded). */
int lmps_q4_pack(const float* w, long long n, uint8_t* packed, uint16_t* scales, void* stream);

/* ---- decode loop bookkeeping ------------------------------------------- */

/* After an argmax: tokens[b] = next[b]; pos[b] += 1; seq_lens[b] += 1 and,
 * when history != NULL, history[step[0]*batch + b] = next[b], step[0] += 1
 * (history has room for max_steps rows; later steps are dropped). */
int lmps_decode_advance(const int32_t* next, int32_t* tokens, int32_t* pos, int32_t* seq_lens,
                        int32_t* history, int32_t* step, int max_steps, int batch,
                        void* stream);

/* ---- persistent decode step -----------------------------------------------
 * The whole of runners/engine.py:157-181 (28 x _execute_block, final norm,
 * LM head, argmax) for `batch` sequences as ONE cooperative kernel launch of
 * one CTA per SM, repeated for n_steps tokens: weights stream from HBM into a
 * shared-memory ring through TMA bulk copies issued by a producer warp while
 * consumer warps compute, and stages hand activations to each other through
 * device-side counters instead of kernel boundaries. */

typedef struct lmps_layer_desc {
  const uint8_t* qkv_packed;    /* [n_q+2*n_kv)*head_dim, hidden] Q4 (q|k|v rows) */
  const uint16_t* qkv_scales;
  const uint16_t* qkv_bias;     /* fp16 [(n_q+2*n_kv)*head_dim] */
  const uint8_t* o_packed;      /* [hidden, n_q*head_dim] */
  const uint16_t* o_scales;
  const uint8_t* gate_packed;   /* [intermediate, hidden] */
  const uint16_t* gate_scales;
  const uint8_t* up_packed;     /* [intermediate, hidden] */
  const uint16_t* up_scales;
  const uint8_t* down_packed;   /* [hidden, intermediate] */
  const uint16_t* down_scales;
  const uint16_t* in_norm;      /* fp16 [hidden] */
  const uint16_t* post_norm;    /* fp16 [hidden] */
  uint16_t* k_pool;             /* fp16 [n_pages, n_kv, page_size, head_dim] */
  uint16_t* v_pool;
} lmps_layer_desc;

typedef struct lmps_model_desc {
  int n_layers, hidden, intermediate, vocab, n_q_heads, n_kv_heads, head_dim;
  float eps;
  int rope_style;                   /* LMPS_ROPE_* */
  const lmps_layer_desc* layers;    /* DEVICE array of n_layers descriptors */
  const uint16_t* final_norm;       /* fp16 [hidden] */
  const uint8_t* lm_packed;         /* [vocab, hidden] Q4 tied head */
  const uint16_t* lm_scales;
  const uint16_t* embed;            /* fp16 [vocab, hidden] */
  const float* inv_freq;            /* fp32 [head_dim/2] */
} lmps_model_desc;

typedef struct lmps_decode_state {
  int batch, page_size, max_pages, max_seq_len;   /* page_size: a power of two */
  const int32_t* block_table;   /* [batch, max_pages] */
  const float* rope_table;      /* fp32 [max_seq_len, head_dim/2, 2]: cos and sin of the
                                   fp32 angle p * inv_freq[j] (rope.metal:28-33) */
  int32_t* tokens;              /* [batch] token fed at the next step; updated */
  int32_t* pos;                 /* [batch] position of that token; updated */
  const int32_t* forced;        /* [batch, forced_stride] tokens fed after steps 0..n_forced-1 (or NULL) */
  int forced_stride, n_forced;
  const uint16_t* x_in;         /* fp16 [batch, hidden] replaces the step-0 embedding (or NULL) */
  uint16_t* logits;             /* fp16 [batch, vocab] of the last step (or NULL) */
  int32_t* history;             /* [history_rows, batch] argmax of every step (or NULL) */
  int32_t* step_counter;        /* [1] history row of the first step (rows outside
                                   [0, history_rows) are skipped); advanced by n_steps */
  int history_rows;
  void* workspace;              /* lmps_decode_persistent_workspace_size() bytes, zeroed once */
  size_t workspace_bytes;
  int32_t* error;               /* [1] set to 1 when a bounded device wait gives up */
  unsigned long long* trace;    /* optional stage timeline (or NULL): [3 * grid, trace_events]
                                   %globaltimer stamps; rows 0..grid-1 compute warps (stage
                                   start, input staged, compute done, stage end; four
                                   per stage), rows grid.. the producer
                                   (first and last chunk issue of each stage), rows 2*grid..
                                   the compute warps' cumulative ns spent waiting for weights */
  int trace_events;
  int trace_rows;               /* rows allocated in trace (>= 3 * grid) */
} lmps_decode_state;

/* Bytes of workspace the persistent step needs (tagged activations, split
 * partials, counters, the launch sequence number the activation tags are
 * derived from).  The workspace must be zero-filled before the first call;
 * each call leaves it ready for the next one. */
size_t lmps_decode_persistent_workspace_size(const lmps_model_desc* model, int batch,
                                             int max_seq_len);

/* Run n_steps decode steps (1 <= batch <= 4, head_dim 128, hidden a multiple
 * of 512 and <= 1536, intermediate a multiple of 32 and <= 11264, vocab <=
 * 262144).  model/state are HOST
 * structs (copied into the launch).  Failures found on the device are reported
 * through state->error, which the caller reads after synchronising: 1 = a
 * bounded wait timed out, 2 = a position past max_seq_len or a token id
 * outside the vocabulary (nothing ran), 3 = no finite logit.  After a non-zero
 * error the workspace must be zeroed again. */
int lmps_decode_persistent(const lmps_model_desc* model, const lmps_decode_state* state,
                           int n_steps, void* stream);

/* ---- Batched decode: all layers of a decode step for 1..64 sequences in one
 * cooperative launch, the Q4 projections on the tcgen05 tensor cores
 * (replaces the per-layer loop of runners/engine.py:183-245 run once per
 * sequence; the LM head and argmax of :163-181 stay separate calls).
 * Weights are read from tile-major copies of the Q4 matrices: */

/* Bytes of the tile-major copy of an [n, k] Q4 matrix (n % 128 == 0,
 * k % 64 == 0; 0 otherwise). */
size_t lmps_q4_tile_blocks_size(int n, int k);
/* Write the tile-major copy: for every 128 rows and 64-wide K step one
 * 4608-byte block, the rows' 32 packed bytes (two 16-byte halves, swapped
 * when (row >> 2) & 1) followed by their two group scales (fp16 pairs).
 * packed/out 16-byte aligned. */
int lmps_q4_tile_blocks(const uint8_t* packed, const uint16_t* scales, int n, int k, void* out,
                        void* stream);

typedef struct lmps_batched_layer {
  const void* qkv_blocks;       /* tile-major W_q|k|v [(n_q+2*n_kv)*head_dim, hidden] */
  const void* o_blocks;         /* tile-major W_o [hidden, n_q*head_dim] */
  const void* gu_blocks;        /* tile-major W_gate|up, rows interleaved (2t gate t, 2t+1 up t)
                                   [2*intermediate, hidden] */
  const void* down_blocks;      /* tile-major W_down [hidden, intermediate] */
  const uint16_t* qkv_bias;     /* fp16 [(n_q+2*n_kv)*head_dim] */
  const uint16_t* in_norm;      /* fp16 [hidden] */
  const uint16_t* post_norm;    /* fp16 [hidden] */
  uint16_t* k_pool;             /* fp16 [n_pages, n_kv, page_size, head_dim] */
  uint16_t* v_pool;
} lmps_batched_layer;

typedef struct lmps_batched_desc {
  const lmps_batched_layer* layers;  /* DEVICE array of n_layers descriptors */
  int n_layers, hidden, intermediate, n_q_heads, n_kv_heads, head_dim;
  float eps;
  int rope_style;                    /* LMPS_ROPE_* */
  const float* inv_freq;             /* fp32 [head_dim/2] */
} lmps_batched_desc;

/* Workspace bytes for `batch` sequences (0 if the model is unsupported:
 * head_dim 128, hidden a multiple of 512 and <= 2048, every projection's rows
 * a multiple of 128 and at most one 128-row tile per SM, K a multiple of 64). */
size_t lmps_decode_batched_workspace_size(const lmps_batched_desc* model, int batch, int max_seq_len);

/* Grid barriers of one launch (rows of its trace per CTA; 0 if unsupported). */
int lmps_decode_batched_barriers(const lmps_batched_desc* model, int batch, int max_seq_len);

/* One decode step of every layer: x (fp16 [batch, hidden], the embedded
 * tokens) becomes the residual after the last layer (the final norm is the
 * caller's); the K/V rows of position pos[b] are appended to each layer's
 * pools and attention covers seq_lens[b] = pos[b] + 1 positions.  workspace:
 * 256-byte aligned, zeroed once (it carries a grid-barrier counter from
 * launch to launch) and again after a reported error.  error: 1 = a bounded
 * device wait gave up, 2 = a position outside the cache (nothing ran).
 * trace (or NULL): %globaltimer stamps [grid][barriers][4] -- when each CTA's
 * workers arrived at each grid barrier, when they saw it complete (0 where
 * they did not wait), and for a barrier that ends a projection stage, when
 * the CTA's weight tiles were all dequantised and when its accumulator was
 * ready; barriers: lmps_decode_batched_barriers(). */
int lmps_decode_batched(const lmps_batched_desc* model, uint16_t* x, const int32_t* pos,
                        const int32_t* seq_lens, const int32_t* block_table, int max_pages,
                        int page_size, int batch, int max_seq_len, void* workspace,
                        size_t workspace_bytes, int32_t* error, unsigned long long* trace,
                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LLAMAMPS_B200_H_ */
