// Persistent decode kernel: one cooperative launch runs n decode steps of the
// whole model (runners/engine.py:157-181 repeated), one CTA per SM.
//
// Why: a bs1 decode step reads 868.6 MB of Q4 weights in ~230 dependent
// pieces (28 x 5 stages + head); as separate kernels each piece pays launch
// latency and a cold start of its memory stream (the fused gate/up GEMV alone
// reaches ~23% of HBM bandwidth).  Here the weight stream never stops:
//
//  * the last warp of every CTA (the producer) walks the same static schedule as the
//    compute warps and issues TMA bulk copies (cp.async.bulk, L2 evict-first)
//    of the CTA's row slice of every matrix, layer after layer, into a ring of
//    shared-memory slots guarded by full/empty mbarriers.  Weights do not
//    depend on activations, so the producer runs up to a ring (~160 KB, about
//    one layer per SM) ahead of the compute;
//  * the other warps (the consumers) wait for a stage's input activation, stage it
//    in shared memory (RMSNorm'd where the reference normalises) as exact
//    integer activation planes, consume their slots (dp4a group dots of the
//    weight nibbles against the planes, scaled per group into fp32, warp-
//    shuffle reduction) and publish the stage output with the fused epilogue;
//  * stages hand data across CTAs through global memory as tagged words: a
//    64-bit word holds two fp16 outputs and the 32-bit tag of the stage (and
//    step and launch) that wrote them, stored with st.relaxed.gpu.  A reader
//    polls the words it needs until every tag matches -- the data is its own
//    flag, so there is no grid-wide barrier in a step and a stage starts as
//    soon as its inputs exist.  The LM head publishes one tagged argmax slot
//    per CTA.  Every wait is bounded (2 s of %globaltimer): on expiry the CTA
//    raises state.error, stops the producer, drains its in-flight copies and
//    returns.
//
// Stages per layer (rows split evenly over the CTAs):
//   QKV  rmsnorm(x, in_norm) -> q|k|v = Wqkv x + b              (engine.py:188-195)
//   ATT  per (seq, kv head, position split): RoPE q/k, KV append at pos, GQA
//        scores/softmax/weighted sum over the paged cache; the last split to
//        finish merges the partials (log-sum-exp)                (engine.py:198-212)
//   O    x1 = x + fp16(Wo attn)                                  (engine.py:215-221)
//   GU   a = swiglu(Wg n, Wu n), n = rmsnorm(x1, post_norm)      (engine.py:224-235)
//   DN   x = x1 + fp16(Wd a)                                     (engine.py:237-243)
// then HEAD: logits = Wlm rmsnorm(x, final_norm) with the first-index argmax
// (engine.py:163-181), and every CTA derives the next token from the argmax.
#include <cmath>

#include <mutex>

#include "common.cuh"
#include "flash_decode.cuh"

namespace lmps {
namespace pk {

constexpr int kConsumerWarps = 11;   // + 1 producer warp = 12 warps (registers are allocated per 4 warps)
constexpr int kConsumers = kConsumerWarps * kWarp;        // 352
constexpr int kThreads = kConsumers + kWarp;              // + producer warp
constexpr int kSlotBytes = 20160;
constexpr int kRows1536 = 2 * kConsumerWarps;  // rows per ring chunk when k = hidden
constexpr int kPairsGU = kConsumerWarps;    // gate/up row pairs per chunk
constexpr int kRowsDown = 4;      // rows per chunk when k = intermediate
// Batches of 2-4 (the tensor-core GEMV, see gemv_rows_mma): ring chunks of
// 16 weight rows (one m16n8k32 tile; gate/up: 8 gate + 8 up rows); the down
// projection's 16-row tile comes in k-parts of a few groups each.
constexpr int kTileRows = 16;
constexpr int kHD = 128;
constexpr int kMaxG = 8;
constexpr unsigned long long kTimeoutNs = 2000000000ull;
constexpr int kMaxB = 4;
constexpr int kOwnMax = 32;  // hidden / qkv rows one CTA owns
constexpr int kOutMax = 128; // gate/up output rows one CTA computes
constexpr int kMaxGrid = 256;
constexpr int kMaxLayers = 64;

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Non-blocking probe of a phase (try_wait may suspend the thread for a while).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Potentially blocking probe: the thread is suspended (it issues nothing)
// until the phase completes or about kSuspendNs pass.
constexpr uint32_t kSuspendNs = 20000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// Plain (non-multicast) TMA bulk copy global -> this CTA's shared memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }

struct Params {
  lmps_model_desc m;
  lmps_decode_state s;
  int n_steps;
  int slots;       // ring slots
  int act_bytes;   // activation / attention staging bytes
  // workspace carve-up.  Stage outputs are tagged words: two fp16 values (low
  // 32 bits, element 2i in the low half) and the 32-bit tag of the stage that
  // wrote them (high 32 bits); readers poll the words themselves.
  unsigned long long* xt;     // [B, hidden/2] residual after a layer (down stage)
  unsigned long long* x1t;    // [B, hidden/2] residual after attention (o stage)
  unsigned long long* qkvt;   // [B, qkv_rows/2]
  unsigned long long* attnt;  // [B, q_dim/2]
  unsigned long long* at;     // [B, intermediate/2] SwiGLU output
  unsigned long long* kslot;  // [grid, kMaxB] per-CTA argmax of the LM head rows, tagged
  float* part_o;    // [B, Hq, max_splits, 128]
  float2* part_ml;  // [B, Hq, max_splits]
  uint32_t* att_cnt;  // [kMaxB, Hkv] split arrivals (reset by the last split)
  uint32_t* epoch;    // [1] tag base of the next launch
  int max_splits;
};

enum StageKind { ST_QKV = 0, ST_O = 1, ST_GU = 2, ST_DN = 3, ST_HEAD = 4 };

// Shared-memory copy of the per-layer pointers on the consumers' critical
// path (the descriptor array itself is in global memory).
struct LayerPtrs {
  const __half* in_norm;
  const __half* post_norm;
  __half* k_pool;
  __half* v_pool;
};

struct Smem {
  unsigned char* ring;
  unsigned char* act;
  uint64_t* full;
  uint64_t* empty;
  float* red8;       // [warps * kMaxB] block-reduction scratch
  unsigned long long* best;  // [warps][kMaxB]
  int* misc;         // [0] abort
  struct LayerPtrs* lp;  // [n_layers] the layer pointers the consumers read, staged once per launch
  __half* xown;     // [kMaxB][kOwnMax] residual x of the hidden rows this CTA owns
  __half* x1own;     // [kMaxB][kOwnMax] residual after attention, same rows
  __half* bias_own;  // [n_layers][kOwnMax] q|k|v bias of the qkv rows this CTA owns
  int gemv_grid;     // CTAs [0, gemv_grid) run the projections; the others attention only
  int n_att;         // CTAs dedicated to attention (0: attention spread over every CTA)
};

// Rows [r0, r1) of a stage this CTA computes: row pairs split evenly over the
// CTAs (stage outputs are published as pairs).  rows * ctas < 2^32.
__device__ __forceinline__ void row_range(int rows, int cta, int ctas, int& r0, int& r1) {
  const uint32_t pairs = static_cast<uint32_t>(rows) / 2;
  r0 = 2 * static_cast<int>(pairs * cta / static_cast<uint32_t>(ctas));
  r1 = 2 * static_cast<int>(pairs * (cta + 1) / static_cast<uint32_t>(ctas));
}

// Weight chunk geometry of a stage for this CTA.
struct Chunking {
  const uint8_t* w;
  const __half* s;
  const uint8_t* w2;
  const __half* s2;
  int k, r0, r1, rows_per_chunk;
  int kparts;  // tensor-core down projection: k-parts per 16-row tile (1 otherwise)
};

// k-parts of the down projection's 16-row tiles on the tensor-core path: the
// fewest that keep a part's scales a multiple of 16 bytes and the part
// (padded rows and scales) in a ring slot.
__host__ __device__ __forceinline__ int down_kparts(int groups) {
  for (int kp = 1; kp <= groups; ++kp)
    if (groups % kp == 0 && (groups / kp) % 8 == 0 && kTileRows * ((groups / kp) * 18 + 16) <= kSlotBytes) return kp;
  return 0;
}

// kMma (batches 2-4, decided per kernel instantiation): the tensor-core
// chunking of gemv_rows_mma / gemv_down_mma.
template <bool kMma>
__device__ __forceinline__ Chunking stage_chunks(const Params& P, int kind, int layer, int ctas) {
  Chunking c{};
  const lmps_model_desc& m = P.m;
  int rows = 0;
  if (kind == ST_HEAD) {
    c.w = m.lm_packed; c.s = reinterpret_cast<const __half*>(m.lm_scales);
    c.k = m.hidden; rows = m.vocab; c.rows_per_chunk = kMma ? kTileRows : kRows1536;
  } else {
    const lmps_layer_desc& L = m.layers[layer];
    if (kind == ST_QKV) {
      c.w = L.qkv_packed; c.s = reinterpret_cast<const __half*>(L.qkv_scales);
      c.k = m.hidden; rows = (m.n_q_heads + 2 * m.n_kv_heads) * m.head_dim;
      c.rows_per_chunk = kMma ? kTileRows : kRows1536;
    } else if (kind == ST_O) {
      c.w = L.o_packed; c.s = reinterpret_cast<const __half*>(L.o_scales);
      c.k = m.n_q_heads * m.head_dim; rows = m.hidden; c.rows_per_chunk = kMma ? kTileRows : kRows1536;
    } else if (kind == ST_GU) {
      c.w = L.gate_packed; c.s = reinterpret_cast<const __half*>(L.gate_scales);
      c.w2 = L.up_packed; c.s2 = reinterpret_cast<const __half*>(L.up_scales);
      c.k = m.hidden; rows = m.intermediate; c.rows_per_chunk = kMma ? kTileRows / 2 : kPairsGU;
    } else {
      c.w = L.down_packed; c.s = reinterpret_cast<const __half*>(L.down_scales);
      c.k = m.intermediate; rows = m.hidden; c.rows_per_chunk = kMma ? kTileRows : kRowsDown;
      if (kMma) c.kparts = down_kparts(m.intermediate / kQ4Group);
    }
  }
  row_range(rows, blockIdx.x, ctas, c.r0, c.r1);
  if (c.kparts == 0) c.kparts = 1;
  return c;
}

// Optional timeline: one %globaltimer stamp per event and row (see the header).
__device__ __forceinline__ void trace_event(const Params& P, int row, int& ev,
                                            unsigned long long wait_ns = ~0ull) {
  if (P.s.trace) {
    if (ev < P.s.trace_events) {
      P.s.trace[static_cast<size_t>(row) * P.s.trace_events + ev] = globaltimer();
      if (wait_ns != ~0ull)   // consumer rows: cumulative ring wait in rows [2*grid, 3*grid)
        P.s.trace[(static_cast<size_t>(row) + 2 * gridDim.x) * P.s.trace_events + ev] = wait_ns;
    }
    ++ev;
  }
}

// ---------------------------------------------------------------------------
// Producer: one lane streams every chunk of every stage into the ring (TMA
// bulk copies): the weight rows of the projections and, with attention
// spread over the CTAs, the cached K/V rows of the attention stages.
// ---------------------------------------------------------------------------
__device__ bool produce_kv(const Params& P, Smem& S, int layer, int step, uint32_t& chunk, int& pslot,
                           uint32_t& pphase);

// Wait until the consumers released ring slot `slot` from its previous fill
// (chunk - slots).
__device__ __forceinline__ bool acquire_slot(const Params& P, Smem& S, uint32_t chunk, int slot, uint32_t phase) {
  if (chunk < static_cast<uint32_t>(P.slots)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(&S.empty[slot], phase ^ 1u))
    if (*reinterpret_cast<volatile int*>(&S.misc[0]) || globaltimer() - t0 > kTimeoutNs) return false;
  return true;
}

template <bool kMma>
__device__ void producer(const Params& P, Smem& S) {
  const uint64_t policy = evict_first_policy();
  uint32_t chunk = 0, pphase = 0;
  int pslot = 0;
  bool ok = true;
  int pev = 0;
  const int n_stages = P.m.n_layers * 4 + 1;  // q|k|v, o, gate/up, down per layer, then the LM head
  for (int step = 0; step < P.n_steps && ok; ++step) {
    for (int st = 0; st < n_stages && ok; ++st) {
      const int kind = (st == n_stages - 1) ? ST_HEAD : (st & 3);
      // spread attention sits between a layer's q|k|v and o chunks
      if (kind == ST_O && S.n_att == 0 && !produce_kv(P, S, st >> 2, step, chunk, pslot, pphase)) {
        ok = false;
        break;
      }
      const Chunking c = stage_chunks<kMma>(P, kind, st >> 2, S.gemv_grid);
      const uint32_t row_bytes = c.k / 2, row_sbytes = c.k / 16;
      const uint32_t ncopy = (kind == ST_GU) ? 2u : 1u;
      trace_event(P, gridDim.x + blockIdx.x, pev);
      const int kparts = (kind == ST_DN) ? c.kparts : 1;
      for (int ci = 0; ok && c.r0 + (ci / kparts) * c.rows_per_chunk < c.r1; ++ci, ++chunk) {
        const int r = c.r0 + (ci / kparts) * c.rows_per_chunk, part = ci % kparts;
        const uint32_t n = min(c.rows_per_chunk, c.r1 - r);
        const int slot = pslot;
        const uint32_t phase = pphase;
        if (++pslot == P.slots) {
          pslot = 0;
          pphase ^= 1u;
        }
        if (!acquire_slot(P, S, chunk, slot, phase)) {
          ok = false;
          break;
        }
        // slot layout: packed rows [, second matrix's packed rows], scales [, second matrix's scales]
        unsigned char* dst = S.ring + static_cast<size_t>(slot) * kSlotBytes;
        if (kMma && kind == ST_DN) {
          // Down projection (batches 2-4): one k-part of 16 tile rows at a
          // padded stride (part bytes + 16: the 8 rows one fragment load
          // touches fall in different banks), then the rows' part scales.
          const uint32_t pbr = row_bytes / kparts, sbr = row_sbytes / kparts, pbs = pbr + 16;
          mbar_expect_tx(&S.full[slot], n * (pbr + sbr));
          const unsigned char* sc = reinterpret_cast<const unsigned char*>(c.s);
          for (uint32_t i = 0; i < n; ++i) {
            bulk_g2s(dst + i * pbs, c.w + static_cast<size_t>(r + i) * row_bytes + part * pbr, pbr, &S.full[slot],
                     policy);
            bulk_g2s(dst + kTileRows * pbs + i * sbr, sc + static_cast<size_t>(r + i) * row_sbytes + part * sbr, sbr,
                     &S.full[slot], policy);
          }
          continue;
        }
        if (kMma) {
          // Row tiles (batches 2-4): pairs of adjacent weight rows, one bulk
          // copy each, at a padded pair stride (2 rows + 16 bytes): pair j
          // holds tile rows j and j + 8, so the 8 rows one fragment load
          // touches fall in different banks; then the rows' scales in weight
          // row order.  Gate/up: gate pairs in pairs 0-3, up pairs in 4-7.
          const uint32_t pps = 2 * row_bytes + 16;
          mbar_expect_tx(&S.full[slot], ncopy * n * (row_bytes + row_sbytes));
          for (uint32_t m2 = 0; m2 < ncopy; ++m2) {
            const uint8_t* w = m2 ? c.w2 : c.w;
            const unsigned char* sc = reinterpret_cast<const unsigned char*>(m2 ? c.s2 : c.s);
            for (uint32_t i = 0; 2 * i < n; ++i)
              bulk_g2s(dst + (m2 * (kTileRows / 4) + i) * pps, w + static_cast<size_t>(r + 2 * i) * row_bytes,
                       min(2u, n - 2 * i) * row_bytes, &S.full[slot], policy);
            bulk_g2s(dst + (kTileRows / 2) * pps + m2 * (kTileRows / 2) * row_sbytes,
                     sc + static_cast<size_t>(r) * row_sbytes, n * row_sbytes, &S.full[slot], policy);
          }
          continue;
        }
        const uint32_t pb = n * row_bytes, sb = n * row_sbytes;
        mbar_expect_tx(&S.full[slot], ncopy * (pb + sb));
        for (uint32_t i = 0; i < ncopy; ++i) {
          const uint8_t* w = i ? c.w2 : c.w;
          const unsigned char* s = reinterpret_cast<const unsigned char*>(i ? c.s2 : c.s);
          bulk_g2s(dst + i * pb, w + static_cast<size_t>(r) * row_bytes, pb, &S.full[slot], policy);
          bulk_g2s(dst + ncopy * pb + i * sb, s + static_cast<size_t>(r) * row_sbytes, sb, &S.full[slot], policy);
        }
      }
      trace_event(P, gridDim.x + blockIdx.x, pev);
    }
  }
  // Drain: every issued copy must land before this CTA may exit.
  const uint32_t issued = chunk;
  const uint32_t first = issued > static_cast<uint32_t>(P.slots) ? issued - P.slots : 0u;
  for (uint32_t c = first; c < issued; ++c) {
    const int slot = c % P.slots;
    const uint32_t phase = (c / P.slots) & 1u;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(&S.full[slot], phase)) {
      if (globaltimer() - t0 > kTimeoutNs) break;
    }
  }
}

// ---------------------------------------------------------------------------
// Consumer helpers
// ---------------------------------------------------------------------------
struct CState {
  int slot;           // ring slot of the next chunk (same sequence as the producer)
  uint32_t phase;     // its full-barrier phase parity
  unsigned long long wait_ns;  // time thread 0 spent waiting for ring chunks (timeline only)
  int ev;             // next timeline event of this CTA (thread 0, timeline only)
};

// Timeline stamp of thread 0 between the stages' own stamps: where a
// stage's compute ends and its epilogue (reduction, publish) begins.
__device__ __forceinline__ void trace_mid(const Params& P, CState& cs) {
  if (threadIdx.x == 0) trace_event(P, blockIdx.x, cs.ev, cs.wait_ns);
}

__device__ __forceinline__ bool aborting(Smem& S) { return *reinterpret_cast<volatile int*>(&S.misc[0]) != 0; }
__device__ __forceinline__ void raise_abort(const Params& P, Smem& S, int code) {
  atomicExch(P.s.error, code);
  *reinterpret_cast<volatile int*>(&S.misc[0]) = 1;
}

__device__ __forceinline__ void ld_tagged2(const unsigned long long* p, unsigned long long& a,
                                           unsigned long long& b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0,%1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_tagged(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long tagged(uint32_t tag, uint32_t payload) {
  return (static_cast<unsigned long long>(tag) << 32) | payload;
}
__device__ __forceinline__ bool has_tag(unsigned long long w, uint32_t tag) {
  return static_cast<uint32_t>(w >> 32) == tag;
}

// Eight fp16 values from four tagged words at p (16-byte aligned) once all
// four carry `tag`: tagged4_issue loads them, tagged4_finish checks the tags
// and re-polls if needed (bounded: on timeout the CTA's abort flag is raised
// and zeros are returned).  Issuing several groups before finishing any keeps
// their loads in flight together.
// Pause between re-polls of words that are not ready yet: every CTA polls
// the same few KB of a stage output, so unthrottled polling crowds the L2
// slices holding them.
constexpr unsigned kPollBackoffNs = 0;
struct Tagged4 {
  unsigned long long w[4];
};
__device__ __forceinline__ void tagged4_issue(const unsigned long long* p, Tagged4& t) {
  ld_tagged2(p, t.w[0], t.w[1]);
  ld_tagged2(p + 2, t.w[2], t.w[3]);
}
__device__ __forceinline__ bool tagged4_ok(const Tagged4& t, uint32_t tag) {
  return has_tag(t.w[0], tag) && has_tag(t.w[1], tag) && has_tag(t.w[2], tag) && has_tag(t.w[3], tag);
}
__device__ __forceinline__ uint4 tagged4_payload(const Tagged4& t) {
  return make_uint4(static_cast<uint32_t>(t.w[0]), static_cast<uint32_t>(t.w[1]), static_cast<uint32_t>(t.w[2]),
                    static_cast<uint32_t>(t.w[3]));
}
__device__ __noinline__ uint4 tagged4_spin(int32_t* error, volatile int* abort_flag, const unsigned long long* p,
                                           uint32_t tag) {
  const uint64_t t0 = globaltimer();
  Tagged4 t;
  while (true) {
    if (kPollBackoffNs) __nanosleep(kPollBackoffNs);
    tagged4_issue(p, t);
    if (tagged4_ok(t, tag)) return tagged4_payload(t);
    if (*abort_flag || globaltimer() - t0 > kTimeoutNs) break;
  }
  if (!*abort_flag) {
    atomicExch(error, 1);
    *abort_flag = 1;
  }
  return make_uint4(0u, 0u, 0u, 0u);
}
__device__ __forceinline__ uint4 tagged4_finish(const Params& P, Smem& S, const unsigned long long* p,
                                                uint32_t tag, const Tagged4& t) {
  if (tagged4_ok(t, tag)) return tagged4_payload(t);
  return tagged4_spin(P.s.error, reinterpret_cast<volatile int*>(&S.misc[0]), p, tag);
}

// One tagged word (acquire: later loads of this thread see what the writer
// published before it).
__device__ __forceinline__ uint32_t poll1(const Params& P, Smem& S, const unsigned long long* p, uint32_t tag) {
  unsigned long long w = ld_tagged_acquire(p);
  if (!has_tag(w, tag)) {
    const uint64_t t0 = globaltimer();
    while (true) {
      w = ld_tagged_acquire(p);
      if (has_tag(w, tag)) break;
      if (aborting(S)) return 0u;
      if (globaltimer() - t0 > kTimeoutNs) {
        raise_abort(P, S, 1);
        return 0u;
      }
    }
  }
  return static_cast<uint32_t>(w);
}


// Wait for the next ring chunk.  Control flow stays uniform across the
// consumers: a thread that gives up (timeout, or the CTA already aborting)
// raises the abort flag and carries on with the slot's stale contents -- all
// reads stay inside shared memory and all writes inside the stage's outputs --
// and the CTA leaves together at its next abort check (after a block sync).
__device__ void slot_wait(Smem& S, const Params& P, CState& cs) {
  const int slot = cs.slot;
  const uint32_t phase = cs.phase;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(&S.misc[0]);
  if (mbar_test_wait(&S.full[slot], phase)) return;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(&S.full[slot], phase)) {
    if (*abort_flag) return;
    if (globaltimer() - t0 > kTimeoutNs) {
      raise_abort(P, S, 1);
      return;
    }
  }
  if (P.s.trace && threadIdx.x == 0) cs.wait_ns += globaltimer() - t0;
}

// Block (consumer) sums of NB floats per thread; every consumer gets the totals.
template <int NB>
__device__ __forceinline__ void consumer_sum_n(float (&v)[NB], float* red8) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const float w = warp_sum(v[b]);
    if (lane == 0) red8[warp * kMaxB + b] = w;
  }
  consumer_sync();
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) t += red8[w * kMaxB + b];
    v[b] = t;
  }
  // (no trailing sync: red8 is written again only after later block syncs)
}

// ---------------------------------------------------------------------------
// Activation planes.  A staged activation vector (RMSNorm'd x, attention
// output, SwiGLU output) is kept per 32-element group -- the Q4 group of the
// weights it meets -- as a 16-bit block fixed point X = rint(x * 2^(15-e)),
// with e the smallest exponent such that every |x| of the group is < 2^e,
// split into a signed high byte H and an unsigned low byte L (X = 256 H + L).
// With the weight nibbles n (0..15) as bytes, dp4a gives the group's dot
// product exactly in integers:
//     sum_k (n_k - 8) X_k = 256 * sum n H + sum n L - 8 * sum X,
// and the fp32 accumulation across groups applies scale * 2^(e-15) once per
// group.  The only rounding is x -> X (below 2^-15 of the group's largest
// |x|).  Word layout of one group: He[4] Ho[4] Le[4] Lo[4]; word c of He holds
// H of elements 8c, 8c+2, 8c+4, 8c+6 (the low nibbles of packed bytes
// 4c..4c+3), Ho the odd elements 8c+1, 8c+3, 8c+5, 8c+7.
// ---------------------------------------------------------------------------
struct Planes {
  uint32_t* w;  // [NB][G][16]; the tensor-core path: [G][He, Le, Ho, Lo][NB][4]
  float* scl;   // [NB][G]   2^(e-15) (tensor-core path: 2^(e-14))
  int* xs8;     // [NB][G]   8 * sum X
  int G;
  int nb;
};

__device__ __forceinline__ Planes planes_view(Smem& S, int G, int nb) {
  Planes pl;
  pl.w = reinterpret_cast<uint32_t*>(S.act);
  pl.scl = reinterpret_cast<float*>(pl.w + static_cast<size_t>(nb) * G * 16);
  pl.xs8 = reinterpret_cast<int*>(pl.scl + nb * G);
  pl.G = G;
  pl.nb = nb;
  return pl;
}

// Convert the 8 values v (elements 8c..8c+7 of group g, c = lane & 3; the 4
// lanes of a group are consecutive) into their plane words.  Every lane of the
// warp must call this (shuffles); `active` marks lanes holding real data.
// S8 (the tensor-core path of batches 2-4): X = rint(x * 2^(14-e)) and both
// planes signed bytes, L = ((X + 128) & 255) - 128, H = (X - L) / 256, so a
// signed 8-bit mma multiplies them (|X| <= 2^14, |H| <= 64); the scale word
// is then 2^(e-14).  Otherwise X = rint(x * 2^(15-e)) with an unsigned L.
template <bool S8 = false>
__device__ __forceinline__ void store_planes(const float (&v)[8], bool active, const Planes& pl,
                                             int b, int g) {
  float mx = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(v[e]));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  // frexp exponent: mx = f * 2^e, f in [0.5, 1); e = 0 for mx == 0
  const int ebits = (__float_as_int(mx) >> 23) & 0xFF;
  const int e = (mx > 0.0f) ? ebits - 126 : 0;
  constexpr int kFrac = S8 ? 14 : 15;
  const float q = __int_as_float((127 + kFrac - e) << 23);   // 2^(kFrac-e)
  int X[8], sx = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int xi = __float2int_rn(v[i] * q);
    xi = max(-32768, min(32767, xi));
    if constexpr (S8) {  // H * 256 + L with L in [-128, 127]: store L and H as bytes
      const int lo = ((xi + 128) & 255) - 128;
      sx += xi;
      xi = ((xi - lo) / 256) * 256 + (lo & 255);  // same byte layout as 256 H + L below
      X[i] = xi;
      continue;
    }
    X[i] = xi;
    sx += xi;
  }
  sx += __shfl_xor_sync(0xffffffffu, sx, 1);
  sx += __shfl_xor_sync(0xffffffffu, sx, 2);
  if (active) {
    // byte 0 (L) and byte 1 (H) of the even / odd elements, four per word
    const uint32_t pe0 = __byte_perm(X[0], X[2], 0x5140), pe1 = __byte_perm(X[4], X[6], 0x5140);
    const uint32_t po0 = __byte_perm(X[1], X[3], 0x5140), po1 = __byte_perm(X[5], X[7], 0x5140);
    const uint32_t le = __byte_perm(pe0, pe1, 0x5410), he = __byte_perm(pe0, pe1, 0x7632);
    const uint32_t lo = __byte_perm(po0, po1, 0x5410), ho = __byte_perm(po0, po1, 0x7632);
    const int c = threadIdx.x & 3;
    if constexpr (S8) {  // [g][He, Le, Ho, Lo][sequence][word]: one B fragment row per lane, no conflicts
      uint32_t* gw = pl.w + static_cast<size_t>(g) * 16 * pl.nb + 4 * b + c;
      gw[0] = he;
      gw[4 * pl.nb] = le;
      gw[8 * pl.nb] = ho;
      gw[12 * pl.nb] = lo;
    } else {
      const int sw = (g >> 1) & 3;  // quad swizzle, see load_xgroup
      uint32_t* gw = pl.w + (static_cast<size_t>(b) * pl.G + g) * 16;
      gw[4 * (0 ^ sw) + c] = he;
      gw[4 * (1 ^ sw) + c] = ho;
      gw[4 * (2 ^ sw) + c] = le;
      gw[4 * (3 ^ sw) + c] = lo;
    }
    if (c == 0) {
      pl.scl[b * pl.G + g] = __int_as_float((127 + e - kFrac) << 23);  // 2^(e-kFrac)
      pl.xs8[b * pl.G + g] = 8 * sx;
    }
  }
}

// Planes of fp16(fp16(x*scale) * gamma) -- rms_norm.metal:20-39 over the full
// vector (k <= 8 * consumer threads) -- for every sequence; the sums of squares
// share one block reduction.  x comes from the tagged rows tsrc[b * k/2 ..]
// written by the stage tagged `tag`, or (tsrc == nullptr) from the plain fp16
// rows[b] (embedding / caller input).
template <int NB>
__device__ void stage_norm(const Params& P, Smem& S, const __half* const (&rows)[NB],
                           const unsigned long long* tsrc, uint32_t tag, const __half* gamma, int k) {
  const int vpr = k / 8;
  const Planes pl = planes_view(S, k / 32, NB);
  const int c = threadIdx.x;
  const bool active = c < vpr;
  uint4 gv = make_uint4(0u, 0u, 0u, 0u);
  if (active) gv = __ldg(reinterpret_cast<const uint4*>(gamma) + c);
  uint4 v[NB];
  float ss[NB];
  if (tsrc) {
    Tagged4 t[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b)
      if (active && b < P.s.batch) tagged4_issue(tsrc + static_cast<size_t>(b) * (k / 2) + 4 * c, t[b]);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      v[b] = make_uint4(0u, 0u, 0u, 0u);
      if (active && b < P.s.batch) v[b] = tagged4_finish(P, S, tsrc + static_cast<size_t>(b) * (k / 2) + 4 * c, tag, t[b]);
    }
  } else {
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      v[b] = make_uint4(0u, 0u, 0u, 0u);
      if (active && b < P.s.batch) v[b] = __ldg(reinterpret_cast<const uint4*>(rows[b]) + c);
    }
  }
#pragma unroll
  for (int b = 0; b < NB; ++b) ss[b] = 0.0f;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const __half2* h = reinterpret_cast<const __half2*>(&v[b]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      ss[b] = fmaf(f.x, f.x, ss[b]);
      ss[b] = fmaf(f.y, f.y, ss[b]);
    }
  }
  consumer_sum_n<NB>(ss, S.red8);
  const __half* gh = reinterpret_cast<const __half*>(&gv);
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    if (b >= P.s.batch) break;
    const float scale = 1.0f / sqrtf(ss[b] / static_cast<float>(k) + P.m.eps);
    const __half* xh = reinterpret_cast<const __half*>(&v[b]);
    float nv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const __half nrm = __float2half_rn(__half2float(xh[e]) * scale);
      nv[e] = __half2float(__float2half_rn(__half2float(nrm) * __half2float(gh[e])));
    }
    store_planes<(NB > 1)>(nv, active, pl, b, c >> 2);
  }
  consumer_sync();
}

// Planes of the tagged rows src[b * k/2 ..] (k fp16 elements) of every sequence.
template <int NB>
__device__ void stage_copy(const Params& P, Smem& S, const unsigned long long* src, uint32_t tag, int k) {
  const int vpr = k / 8;
  const Planes pl = planes_view(S, k / 32, NB);
  const int total = NB * vpr;
  const int rounds = (total + kConsumers - 1) / kConsumers;
  constexpr int kBatch = 4;  // chunks in flight per thread
  for (int r0 = 0; r0 < rounds; r0 += kBatch) {
    Tagged4 t[kBatch];
#pragma unroll
    for (int q = 0; q < kBatch; ++q) {
      const int i = threadIdx.x + (r0 + q) * kConsumers;
      const int b = i / vpr, c = i - b * vpr;
      if (r0 + q < rounds && i < total && b < P.s.batch) tagged4_issue(src + static_cast<size_t>(b) * (k / 2) + 4 * c, t[q]);
    }
    // One loop body finishes and converts the chunks in turn (t[0] is the
    // current one; the array shifts down), keeping the code compact.
#pragma unroll 1
    for (int q = 0; q < kBatch && r0 + q < rounds; ++q) {  // uniform across the CTA
      const int i = threadIdx.x + (r0 + q) * kConsumers;
      const int b = i / vpr, c = i - b * vpr;
      const bool active = i < total && b < P.s.batch;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (active) v = tagged4_finish(P, S, src + static_cast<size_t>(b) * (k / 2) + 4 * c, tag, t[0]);
      const __half* h = reinterpret_cast<const __half*>(&v);
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = __half2float(h[e]);
      store_planes<(NB > 1)>(f, active, pl, active ? b : 0, c >> 2);
#pragma unroll
      for (int j = 0; j + 1 < kBatch; ++j) t[j] = t[j + 1];
    }
  }
  consumer_sync();
}

// Exact sum_k (n_k - 8) X_k of one group: wv = 16 packed bytes, x = plane
// words.  The nibble bytes (0..15) are non-negative, so the signed dp4a is
// exact for the signed H plane and the unsigned one for the L plane; four
// independent accumulators keep the dependent chains short.
__device__ __forceinline__ int group_idot(const uint4& wv, const uint32_t (&x)[16], int xs8) {
  const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
  int he = 0, ho = 0;
  unsigned le = 0u, lo = 0u;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t ne = ws[c] & 0x0F0F0F0Fu, no = (ws[c] >> 4) & 0x0F0F0F0Fu;
    he = __dp4a(static_cast<int>(ne), static_cast<int>(x[c]), he);
    ho = __dp4a(static_cast<int>(no), static_cast<int>(x[4 + c]), ho);
    le = __dp4a(ne, x[8 + c], le);
    lo = __dp4a(no, x[12 + c], lo);
  }
  return (he + ho) * 256 + static_cast<int>(le + lo) - xs8;
}

struct XGroup {
  uint32_t w[16];
  float scl;
  int xs8;
};

// A group's four 16-byte quads (He, Ho, Le, Lo) are stored in the order
// q ^ ((g >> 1) & 3): lanes reading the same quad of 8 consecutive groups then
// touch 8 different 16-byte bank groups (one wavefront) instead of two.
__device__ __forceinline__ void load_xgroup(const Planes& pl, int b, int g, XGroup& x) {
  const uint4* src = reinterpret_cast<const uint4*>(pl.w + (static_cast<size_t>(b) * pl.G + g) * 16);
  const int sw = (g >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 v = src[q ^ sw];
    x.w[4 * q] = v.x;
    x.w[4 * q + 1] = v.y;
    x.w[4 * q + 2] = v.z;
    x.w[4 * q + 3] = v.w;
  }
  x.scl = pl.scl[b * pl.G + g];
  x.xs8 = pl.xs8[b * pl.G + g];
}

constexpr int kJH = 3;    // groups per lane when k = hidden: G / 16 <= 3 (hidden <= 1536)
constexpr int kMaxJ = 4;  // groups per lane in the down projection: ceil(G / warps / 8) <= 4

__device__ __forceinline__ void slot_release(Smem& S, const Params& P, CState& cs) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&S.empty[cs.slot]);
  if (++cs.slot == P.slots) {
    cs.slot = 0;
    cs.phase ^= 1u;
  }
}

// acc[b] += scale * dot(weights of group gi, activation group gi of sequence b)
template <int NB>
__device__ __forceinline__ void group_fma(const Planes& pl, int gi, const uint4& wv, float sc, float (&acc)[NB]) {
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    XGroup xg;
    load_xgroup(pl, b, gi, xg);
    acc[b] = fmaf(sc * xg.scl, static_cast<float>(group_idot(wv, xg.w, xg.xs8)), acc[b]);
  }
}

// ---------------------------------------------------------------------------
// GEMV stages over ring chunks
// ---------------------------------------------------------------------------
// A chunk only computes: every lane stores its partial dot products in shared
// memory and the chunk's slot is released; the reductions and epilogues of
// all rows run once per stage, spread over the block, fused with publishing
// the tagged output.  (Per-chunk shuffle trees and single-lane epilogues were
// a serial tail after every chunk.)
constexpr int kPartRows = 2 * kOutMax;  // row entries of a stage (gate/up: a gate and an up entry per row)
constexpr int kRedStride = 16;          // down projection: per-row stride of the warp partials

// Partial-sum area after the activation planes of a k = hidden stage:
// [NB][kPartRows][16 lanes] floats.
__device__ __forceinline__ float* partials_view(const Planes& pl, int nb) {
  // 16-byte aligned: the epilogues read the partials as float4
  const uintptr_t p = reinterpret_cast<uintptr_t>(pl.xs8 + nb * pl.G);
  return reinterpret_cast<float*>((p + 15) & ~static_cast<uintptr_t>(15));
}

// Row GEMVs with k = hidden: q|k|v (+bias), o (+residual), gate/up (SwiGLU) and
// the LM head (argmax).  A chunk holds <= 2*warps rows (gate/up: <= warps row
// pairs); warp w takes rows 2w (lanes 0-15) and 2w+1 (lanes 16-31) -- for
// gate/up, gate row w and up row w -- and lane sub groups sub, sub+16, sub+32.
// One code path for every kind keeps the kernel's instruction footprint small.
template <int NB>
__device__ void gemv_rows(const Params& P, Smem& S, CState& cs, int kind, int layer, __half* logits, uint32_t tag,
                          const Chunking& c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = c.k / 32, JG = G / 16;
  const int half = lane >> 4, sub = lane & 15;
  const bool gu = kind == ST_GU, head = kind == ST_HEAD;
  const int lrow = gu ? warp : 2 * warp + half;  // row of the chunk this half-warp computes
  const int rpc = c.rows_per_chunk;
  const size_t rb = c.k / 2;
  const Planes pl = planes_view(S, G, NB);
  float* part = partials_view(pl, NB);
  unsigned long long best[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) best[b] = 0ull;
  // Two ring chunks per pass (when the stage has them): every activation
  // group is read from shared memory once for both chunks' rows.
  for (int r = c.r0; r < c.r1; r += 2 * rpc) {
    const int nc[2] = {min(rpc, c.r1 - r), min(rpc, max(0, c.r1 - r - rpc))};  // nc[1] == 0: one chunk
    const int slot0 = cs.slot;
    slot_wait(S, P, cs);
    int slot1 = slot0;
    if (nc[1] > 0) {
      CState nx = cs;
      if (++nx.slot == P.slots) {
        nx.slot = 0;
        nx.phase ^= 1u;
      }
      slot1 = nx.slot;
      slot_wait(S, P, nx);
      cs.wait_ns = nx.wait_ns;
    }
    float acc[2][NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[0][b] = acc[1][b] = 0.0f;
    const unsigned char* wrow[2];
    const __half* srow[2];
    bool ok[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int n = nc[q];
      ok[q] = lrow < n;
      const unsigned char* base = S.ring + static_cast<size_t>(q ? slot1 : slot0) * kSlotBytes;
      const size_t pbytes = n * rb * (gu ? 2 : 1);
      const int srow_i = gu ? half * n + warp : lrow;  // scale row within the slot's scale block
      wrow[q] = base + (gu ? half * n * rb : 0) + lrow * rb;
      srow[q] = reinterpret_cast<const __half*>(base + pbytes) + srow_i * G;
    }
#pragma unroll
    for (int j = 0; j < kJH; ++j) {
      if (j < JG) {
        const int g = sub + 16 * j;
        uint4 wv[2];
        float sc[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          wv[q] = ok[q] ? *reinterpret_cast<const uint4*>(wrow[q] + g * 16) : make_uint4(0u, 0u, 0u, 0u);
          sc[q] = ok[q] ? __half2float(srow[q][g]) : 0.0f;
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          XGroup xg;
          load_xgroup(pl, b, g, xg);
          acc[0][b] = fmaf(sc[0] * xg.scl, static_cast<float>(group_idot(wv[0], xg.w, xg.xs8)), acc[0][b]);
          if (nc[1] > 0)
            acc[1][b] = fmaf(sc[1] * xg.scl, static_cast<float>(group_idot(wv[1], xg.w, xg.xs8)), acc[1][b]);
        }
      }
    }
    if (!head) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        if (ok[q]) {
          const int r0 = r + q * rpc - c.r0;
          const int e = gu ? 2 * (r0 + warp) + half : r0 + lrow;
#pragma unroll
          for (int b = 0; b < NB; ++b) part[(b * kPartRows + e) * 16 + sub] = acc[q][b];
        }
      }
    }
    slot_release(S, P, cs);
    if (nc[1] > 0) slot_release(S, P, cs);
    if (head) {  // LM head: argmax keys only, kept per lane-0 of each row
#pragma unroll
      for (int q = 0; q < 2; ++q) {
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[q][b] = segment_sum<16>(acc[q][b]);
        if (sub == 0 && ok[q]) {
          const int row = r + q * rpc + lrow;
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            if (b >= P.s.batch) break;
            const __half v = __float2half_rn(acc[q][b]);
            if (logits) logits[static_cast<size_t>(b) * P.m.vocab + row] = v;
            best[b] = u64_max(best[b], argmax_key(__half2float(v), static_cast<uint32_t>(row)));
          }
        }
      }
    }
  }
  trace_mid(P, cs);
  if (head) {
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const unsigned long long w = warp_max_u64(best[b]);
      if (lane == 0) S.best[warp * kMaxB + b] = w;
    }
    return;
  }
  // -- epilogue of every row pair, published as tagged words.  Four lanes
  // per row: they reduce its 16 partials (gate/up: lanes 0-1 the gate
  // entry, 2-3 the up entry, eight partials each), and the two rows of a
  // pair are an aligned group of 8 lanes in one warp.
  consumer_sync();
  unsigned long long* dst = kind == ST_QKV ? P.qkvt : kind == ST_O ? P.x1t : P.at;
  const int dld = kind == ST_QKV ? (P.m.n_q_heads + 2 * P.m.n_kv_heads) * kHD / 2
                                 : (kind == ST_O ? P.m.hidden : P.m.intermediate) / 2;
  const int per_b = (c.r1 - c.r0) * 4;  // lanes per sequence
  for (int t0 = 0; t0 < NB * per_b; t0 += kConsumers) {
    const int t = t0 + threadIdx.x;
    const int b = t / per_b, rem = t - b * per_b;
    const int i = rem >> 2, q4 = rem & 3;  // i = row - c.r0
    const bool live = t < NB * per_b && b < P.s.batch;
    float v = 0.0f;
    if (live) {
      if (gu) {
        const float* pp = part + (b * kPartRows + 2 * i + (q4 >> 1)) * 16 + 8 * (q4 & 1);
        const float4 a0 = *reinterpret_cast<const float4*>(pp), a1 = *reinterpret_cast<const float4*>(pp + 4);
        v = ((a0.x + a0.y) + (a0.z + a0.w)) + ((a1.x + a1.y) + (a1.z + a1.w));
      } else {
        const float4 p4 = *reinterpret_cast<const float4*>(part + (b * kPartRows + i) * 16 + 4 * q4);
        v = (p4.x + p4.y) + (p4.z + p4.w);
      }
    }
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    if (!gu) v += __shfl_xor_sync(0xffffffffu, v, 2);
    const float u = __shfl_down_sync(0xffffffffu, v, 2);  // gate/up: the row's up entry
    const bool row_lane = live && q4 == 0;
    __half h;
    if (gu) {
      h = __float2half_rn(silu_mul(__half2float(__float2half_rn(v)), __half2float(__float2half_rn(u))));
    } else if (kind == ST_QKV) {
      h = __float2half_rn(v + __half2float(S.bias_own[layer * kOwnMax + i]));
    } else {  // ST_O
      h = __hadd(S.xown[(live ? b : 0) * kOwnMax + i], __float2half_rn(v));
      if (row_lane) S.x1own[b * kOwnMax + i] = h;
    }
    const uint32_t hb = __half_as_ushort(h);
    const uint32_t hp = __shfl_down_sync(0xffffffffu, hb, 4);  // the pair's second row
    if (row_lane && (i & 1) == 0)
      st_tagged(dst + static_cast<size_t>(b) * dld + (c.r0 + i) / 2, tagged(tag, hb | (hp << 16)));
  }
  consumer_sync();  // the partials' area is the next stage's staging area
}

// ---------------------------------------------------------------------------
// Tensor-core GEMV stages for batches 2-4: mma.sync m16n8k32, s8 x s8 -> s32.
// A = 16 weight rows x one 32-element group as bytes (the nibbles 0..15): a
// lane's 32-bit word t of a row's group holds 8 nibbles, the even ones are
// fragment k 4t..4t+3 and the odd ones k 16+4t..16+4t+3 -- the element order
// of the activation planes' He / Ho words, so both fragments come straight
// from shared memory.  B = the planes of the same group, column 2s = H and
// 2s+1 = L of sequence s.  Per group the int32 results give each sequence's
// exact dot 256 H + L - 8 sum X (4-bit codes times 15-bit fixed point),
// scaled into fp32 by the row's scale and the group's 2^(e-14).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// The ring state `n` chunks after `c`.
__device__ __forceinline__ CState cs_after(const Params& P, CState c, int n) {
  const int t = c.slot + n;
  if ((t / P.slots) & 1) c.phase ^= 1u;
  c.slot = t % P.slots;
  return c;
}

// acc0 / acc1 += the group dots of tile rows g / g + 8 with sequence t's
// activation group gx (plane group index) -- one mma and its per-group scaling.
template <int NB>
__device__ __forceinline__ void tile_group(const Planes& pl, const unsigned char* wa, const unsigned char* wb,
                                           float sa, float sb, int gx, float& acc0, float& acc1) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int seq = g >> 1, plane = g & 1;
  const uint32_t w0 = *reinterpret_cast<const uint32_t*>(wa + 4 * t);
  const uint32_t w1 = *reinterpret_cast<const uint32_t*>(wb + 4 * t);
  const uint32_t* pw = pl.w + static_cast<size_t>(gx) * 16 * NB + 4 * seq + t;
  uint32_t b0 = 0u, b1 = 0u;
  if (seq < NB) {
    b0 = pw[4 * NB * plane];          // He / Le
    b1 = pw[4 * NB * (2 + plane)];    // Ho / Lo
  }
  int d[4];
  mma_s8_16832(d, w0 & 0x0F0F0F0Fu, w1 & 0x0F0F0F0Fu, (w0 >> 4) & 0x0F0F0F0Fu, (w1 >> 4) & 0x0F0F0F0Fu, b0, b1);
  const int ts = t < NB ? t : 0;  // columns 2t, 2t+1: sequence t
  const float xsc = pl.scl[ts * pl.G + gx];
  const int xs = pl.xs8[ts * pl.G + gx];
  acc0 = fmaf(sa * xsc, static_cast<float>(256 * d[0] + d[1] - xs), acc0);
  acc1 = fmaf(sb * xsc, static_cast<float>(256 * d[2] + d[3] - xs), acc1);
}

// Row GEMVs with k = hidden (q|k|v, o, gate/up, LM head) for batches 2-4:
// each warp takes whole 16-row ring chunks (chunk i of the stage goes to
// warp i mod min(warps, slots), which releases its slot alone) and runs all groups of
// its tile, so a lane ends with the dots of tile rows g and g + 8 for
// sequence t and applies the stage's epilogue itself -- gate/up tiles hold
// 8 gate and the matching 8 up rows, so SwiGLU needs no exchange either.
template <int NB>
__device__ void gemv_rows_mma(const Params& P, Smem& S, CState& cs, int kind, int layer, __half* logits,
                              uint32_t tag, const Chunking& c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int G = c.k / 32;
  const bool gu = kind == ST_GU, head = kind == ST_HEAD;
  const int rpc = c.rows_per_chunk;
  const int nch = (c.r1 - c.r0 + rpc - 1) / rpc;
  const size_t rb = c.k / 2, pps = 2 * rb + 16;  // row bytes, pair stride
  const Planes pl = planes_view(S, G, NB);
  const int B = P.s.batch;
  unsigned long long best = 0ull;  // LM head: this lane's sequence t
  const CState base = cs;
  unsigned long long wns = cs.wait_ns;  // warp 0's ring waits (timeline only)
  unsigned long long* dst = kind == ST_QKV ? P.qkvt : kind == ST_O ? P.x1t : P.at;
  const int dld = kind == ST_QKV ? (P.m.n_q_heads + 2 * P.m.n_kv_heads) * kHD / 2
                                 : (kind == ST_O ? P.m.hidden : P.m.intermediate) / 2;
  // At most `slots` warps take chunks: a warp then only ever waits on a chunk
  // whose slot's previous contents (the chunk `slots` earlier) it has seen
  // land already (its own previous chunk is no older), so the full barrier's
  // parity cannot match a phase two fills old.
  const int nw = min(kConsumerWarps, P.slots);
  for (int ch = warp; warp < nw && ch < nch; ch += nw) {
    CState my = cs_after(P, base, ch);
    my.wait_ns = wns;
    slot_wait(S, P, my);
    wns = my.wait_ns;
    const int r = c.r0 + ch * rpc;
    const int n = min(rpc, c.r1 - r);
    const unsigned char* sl = S.ring + static_cast<size_t>(my.slot) * kSlotBytes;
    // tile rows g, g + 8 = weight rows 2j, 2j + 1 of pair j = g (gate/up:
    // gate pair g for g < 4, up pair g - 4 above)
    const __half* sc = reinterpret_cast<const __half*>(sl + (kTileRows / 2) * pps);
    const unsigned char* wa = sl + g * pps;
    const unsigned char* wb = wa + rb;
    const int srow = gu ? 8 * (g >> 2) + 2 * (g & 3) : 2 * g;  // scale row of tile row g
    const __half* sa = sc + srow * G;
    const __half* sb = sa + G;
    float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll 4
    for (int grp = 0; grp < G; ++grp)
      tile_group<NB>(pl, wa + grp * 16, wb + grp * 16, __half2float(sa[grp]), __half2float(sb[grp]), grp, acc0, acc1);
    __syncwarp();
    if (lane == 0)
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&S.empty[my.slot])),
                   "r"(kConsumerWarps)
                   : "memory");
    // -- epilogue: this lane holds stage rows i0, i0 + 1 (gate/up: the
    // gate rows, and lane + 16 the up rows) for sequence t
    const int pr = gu ? 2 * (g & 3) : 2 * g;  // first row of the lane's pair within the chunk
    const int i0 = r - c.r0 + pr;
    const bool v = pr < n;  // (rows come in pairs)
    const bool lt = t < B;
    if (head) {
      if (lt && v) {
        const __half h0 = __float2half_rn(acc0), h1 = __float2half_rn(acc1);
        if (logits) {
          logits[static_cast<size_t>(t) * P.m.vocab + r + pr] = h0;
          logits[static_cast<size_t>(t) * P.m.vocab + r + pr + 1] = h1;
        }
        best = u64_max(best, argmax_key(__half2float(h0), static_cast<uint32_t>(r + pr)));
        best = u64_max(best, argmax_key(__half2float(h1), static_cast<uint32_t>(r + pr + 1)));
      }
      continue;
    }
    __half h0, h1;
    if (gu) {
      const float u0 = __shfl_down_sync(0xffffffffu, acc0, 16), u1 = __shfl_down_sync(0xffffffffu, acc1, 16);
      h0 = __float2half_rn(silu_mul(__half2float(__float2half_rn(acc0)), __half2float(__float2half_rn(u0))));
      h1 = __float2half_rn(silu_mul(__half2float(__float2half_rn(acc1)), __half2float(__float2half_rn(u1))));
    } else if (kind == ST_QKV) {
      h0 = __float2half_rn(acc0 + __half2float(S.bias_own[layer * kOwnMax + min(i0, kOwnMax - 1)]));
      h1 = __float2half_rn(acc1 + __half2float(S.bias_own[layer * kOwnMax + min(i0 + 1, kOwnMax - 1)]));
    } else {  // ST_O
      const int tb = lt ? t : 0;
      h0 = __hadd(S.xown[tb * kOwnMax + min(i0, kOwnMax - 1)], __float2half_rn(acc0));
      h1 = __hadd(S.xown[tb * kOwnMax + min(i0 + 1, kOwnMax - 1)], __float2half_rn(acc1));
      if (lt && v) {
        S.x1own[t * kOwnMax + i0] = h0;
        S.x1own[t * kOwnMax + i0 + 1] = h1;
      }
    }
    if (lt && v && (!gu || g < 4))
      st_tagged(dst + static_cast<size_t>(t) * dld + (r + pr) / 2,
                tagged(tag, static_cast<uint32_t>(__half_as_ushort(h0)) |
                                (static_cast<uint32_t>(__half_as_ushort(h1)) << 16)));
  }
  cs = cs_after(P, base, nch);
  cs.wait_ns = wns;
  trace_mid(P, cs);
  if (head) {  // per sequence over the warp's lanes (same t), then one slot per warp
    best = u64_max(best, __shfl_xor_sync(0xffffffffu, best, 4));
    best = u64_max(best, __shfl_xor_sync(0xffffffffu, best, 8));
    best = u64_max(best, __shfl_xor_sync(0xffffffffu, best, 16));
    if (lane < kMaxB) S.best[warp * kMaxB + lane] = lane < NB ? best : 0ull;
    return;
  }
  consumer_sync();  // the planes' area is the next stage's staging area
}

// Down projection (k = intermediate) for batches 2-4: the CTA's hidden rows
// (<= 16) are one tile; its k-parts arrive as ring chunks every warp reads,
// warp w taking groups w, w + warps, .. of each part; the warps' fp32
// partials meet in shared memory: x = x1 + fp16(sum).
template <int NB>
__device__ void gemv_down_mma(const Params& P, Smem& S, CState& cs, uint32_t tag, const Chunking& c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int G = c.k / 32, Gp = G / c.kparts;
  const size_t pbs = static_cast<size_t>(Gp) * 16 + 16;
  const Planes pl = planes_view(S, G, NB);
  const int n = c.r1 - c.r0;  // <= kTileRows (host-checked)
  float acc0 = 0.0f, acc1 = 0.0f;
  for (int part = 0; part < c.kparts; ++part) {
    const int slot = cs.slot;
    slot_wait(S, P, cs);
    const unsigned char* sl = S.ring + static_cast<size_t>(slot) * kSlotBytes;
    const __half* sc = reinterpret_cast<const __half*>(sl + kTileRows * pbs);
    for (int j = warp; j < Gp; j += kConsumerWarps)
      tile_group<NB>(pl, sl + g * pbs + j * 16, sl + (g + 8) * pbs + j * 16, __half2float(sc[g * Gp + j]),
                     __half2float(sc[(g + 8) * Gp + j]), part * Gp + j, acc0, acc1);
    slot_release(S, P, cs);
  }
  // warp partials: red[warp][row][sequence] after the planes
  float* red = reinterpret_cast<float*>(pl.xs8 + NB * G);
  if (t < NB) {
    red[(warp * kTileRows + g) * kMaxB + t] = acc0;
    red[(warp * kTileRows + g + 8) * kMaxB + t] = acc1;
  }
  trace_mid(P, cs);
  consumer_sync();
  const int pairs = n / 2;
  for (int q = threadIdx.x; q < NB * pairs; q += kConsumers) {
    const int b = q / pairs, i = 2 * (q - b * pairs);
    if (b >= P.s.batch) break;
    float s0 = 0.0f, s1 = 0.0f;
    for (int w = 0; w < kConsumerWarps; ++w) {
      s0 += red[(w * kTileRows + i) * kMaxB + b];
      s1 += red[(w * kTileRows + i + 1) * kMaxB + b];
    }
    const __half h0 = __hadd(S.x1own[b * kOwnMax + i], __float2half_rn(s0));
    const __half h1 = __hadd(S.x1own[b * kOwnMax + i + 1], __float2half_rn(s1));
    S.xown[b * kOwnMax + i] = h0;
    S.xown[b * kOwnMax + i + 1] = h1;
    st_tagged(P.xt + static_cast<size_t>(b) * (P.m.hidden / 2) + (c.r0 + i) / 2,
              tagged(tag, static_cast<uint32_t>(__half_as_ushort(h0)) |
                              (static_cast<uint32_t>(__half_as_ushort(h1)) << 16)));
  }
  consumer_sync();  // the partials' area is the next stage's staging area
}

// Down projection (k = intermediate): chunks of <= 4 rows; warp w sums groups
// [G*w/warps, G*(w+1)/warps) of every row (lane = row*8 + sub, groups
// g0+sub+8j); each warp leaves one partial per (row, sequence) in shared
// memory and the block finishes all rows at the end: x = x1 + fp16(sum).
template <int NB>
__device__ void gemv_down(const Params& P, Smem& S, CState& cs, int layer, uint32_t tag, const Chunking& c) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = c.k / 32;
  const int g0 = G * warp / kConsumerWarps, g1 = G * (warp + 1) / kConsumerWarps;
  const int lrow = lane >> 3, sub = lane & 7;
  const int rpc = c.rows_per_chunk;
  const Planes pl = planes_view(S, G, NB);
  float* red = partials_view(pl, NB);  // [NB][kOwnMax rows][kRedStride >= warps]
  for (int r = c.r0; r < c.r1; r += rpc) {
    const int n = min(rpc, c.r1 - r);
    const int slot = cs.slot;
    slot_wait(S, P, cs);
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.0f;
    if (lrow < n) {
      const unsigned char* base = S.ring + static_cast<size_t>(slot) * kSlotBytes;
      const unsigned char* wrow = base + static_cast<size_t>(lrow) * (c.k / 2);
      const __half* srow = reinterpret_cast<const __half*>(base + static_cast<size_t>(n) * (c.k / 2)) + lrow * G;
#pragma unroll
      for (int j = 0; j < kMaxJ; ++j) {
        const int g = g0 + sub + 8 * j;
        if (g < g1) group_fma<NB>(pl, g, *reinterpret_cast<const uint4*>(wrow + g * 16), __half2float(srow[g]), acc);
      }
    }
    slot_release(S, P, cs);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const float v = segment_sum<8>(acc[b]);
      if (sub == 0 && lrow < n) red[(b * kOwnMax + r - c.r0 + lrow) * kRedStride + warp] = v;
    }
  }
  trace_mid(P, cs);
  // -- epilogue: four lanes per row (quarters of the 11 warp partials), the
  // two rows of a pair in an aligned group of 8 lanes
  consumer_sync();
  const int per_b = (c.r1 - c.r0) * 4;
  for (int t0 = 0; t0 < NB * per_b; t0 += kConsumers) {
    const int t = t0 + threadIdx.x;
    const int b = t / per_b, rem = t - b * per_b;
    const int i = rem >> 2, qq = rem & 3;
    const bool live = t < NB * per_b && b < P.s.batch;
    float v = 0.0f;
    if (live && 4 * qq < kConsumerWarps) {
      const float4 p4 = *reinterpret_cast<const float4*>(red + (b * kOwnMax + i) * kRedStride + 4 * qq);
      v = (p4.x + p4.y) + (p4.z + (4 * qq + 3 < kConsumerWarps ? p4.w : 0.0f));
    }
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    const __half h = __hadd(S.x1own[(live ? b : 0) * kOwnMax + i], __float2half_rn(v));
    const bool row_lane = live && qq == 0;
    if (row_lane) S.xown[b * kOwnMax + i] = h;
    const uint32_t hb = __half_as_ushort(h);
    const uint32_t hp = __shfl_down_sync(0xffffffffu, hb, 4);
    if (row_lane && (i & 1) == 0)
      st_tagged(P.xt + static_cast<size_t>(b) * (P.m.hidden / 2) + (c.r0 + i) / 2, tagged(tag, hb | (hp << 16)));
  }
  consumer_sync();  // the partials' area is the next stage's staging area
}

// ---------------------------------------------------------------------------
// Attention stage: one work item = (sequence b, kv head, split of positions)
// ---------------------------------------------------------------------------
// Flash-decoding inside the CTA: every warp takes 16-position blocks of the
// split and keeps its own online softmax (softmax.metal:23-36); the warps'
// (max, sum, output) meet in shared memory at the end.  Per block, on the
// tensor cores (mma.sync m16n8k16, fp16 in, fp32 accumulate):
//   S^T  = K Q^T   (M = 16 positions, N = 8 heads, K = 128 dims)   attention.metal:32-40
//   O^T += V^T P^T (M = 16 dims per m-tile, N = 8 heads, K = 16 positions)   attn_sum.metal:26-32
// Both products sum over dims or positions, so the order of the dims inside
// them is free: fragment word w (k-step w >> 1) of lane t holds physical
// dims 8t + 32(w >> 2) + 2(w & 3) + {0, 1}, so every lane's K and V operands
// are four 16-byte runs of a cache row (runs t, t + 4, t + 8, t + 12), and
// output row r of m-tile mt is physical dim
// 8((r & 7) >> 1) + 32(mt >> 1) + 4(mt & 1) + 2(r >> 3) + (r & 1);
// movmatrix transposes V rows and probabilities in registers.
using fd::kBlk;                 // positions per warp block
constexpr int kMinSplit = 512;  // positions per work item before the positions split across CTAs
constexpr int kKvSlotPos = 2 * kBlk;  // positions per ring slot (spread attention): K and V tiles, 16 KB

struct AttnSmem {
  __half raw[(kMaxG + 2) * kHD];          // polled q heads, k, v (before RoPE)
  float2 rot[kHD / 2];                    // (cos, sin) of pos * inv_freq[j]
  __half q[kMaxG][kHD];                   // rotated q, natural dim order
  float wm[kConsumerWarps][kMaxG];        // per-warp running max and sum (then merge weights)
  float wl[kConsumerWarps][kMaxG];
  float wo[kConsumerWarps][32][32];       // per-warp unnormalised O^T fragments, [lane][value, rotated by 4*lane]
  int is_last;
};

// KV cache rows are written (and prefetched) with an L2 evict_last policy so
// that they stay in L2 while the weight stream passes through evict_first.
__device__ __forceinline__ uint64_t evict_last_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void st_kv(__half* p, __half v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.b16 [%0], %1, %2;" ::"l"(p), "h"(__half_as_ushort(v)), "l"(pol) : "memory");
}
__device__ __forceinline__ void st_kv8(__half* p, const uint4& v, uint64_t pol) {  // 8 values, 16-byte aligned
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1,%2,%3,%4}, %5;" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w), "l"(pol)
               : "memory");
}

// mma / movmatrix helpers of flash_decode.cuh
using fd::mma_16816;
using fd::movmatrix_t;
using fd::pack_half2;
using fd::word_of;

__device__ __forceinline__ void rope_pair(int j, int style, int& i1, int& i2) {
  if (style == LMPS_ROPE_INTERLEAVED) {
    i1 = 2 * j;
    i2 = i1 + 1;
  } else {
    i1 = j;
    i2 = j + kHD / 2;
  }
}

// Shared-memory K/V tiles of the dedicated attention CTAs: per 16-position
// block, K then V, each [chunk 4*h2 + c][lane 4*g8 + t4] of 16 bytes = dims
// 8*t4 + 32*c .. +7 of row 8*h2 + g8 (the lanes' mma operand runs).
constexpr int kKvTileBytes = 2 * 8 * 32 * 16;  // K and V of one block: 8 KB
constexpr int kMaxAttCtas = 8;
__device__ __forceinline__ int kv_tile_idx(int blk, int kv, int h2, int c, int lane) {
  return ((blk * 2 + kv) * 8 + 4 * h2 + c) * 32 + lane;
}
__device__ __forceinline__ __half& tile_half(uint4* kvs, int rel, int kv, int d) {
  uint4& u = kvs[kv_tile_idx(rel >> 4, kv, (rel >> 3) & 1, d >> 5, 4 * (rel & 7) + ((d >> 3) & 3))];
  return reinterpret_cast<__half*>(&u)[d & 7];
}

// One 16-position block of a warp's flash loop from shared memory (block
// bi; first position p0; positions >= end are masked and their V rows read
// as zero): S^T = K Q^T, the online softmax of heads 2*t4, 2*t4+1,
// O^T = O^T * alpha + V^T P^T.  kRows: K rows [32][head_dim] then V rows
// (a ring slot, as in the cache), read conflict-free -- at load c the lanes
// of even rows take their run c and those of odd rows run c ^ 1, which fall
// in the other half of the banks, and swap back in registers; otherwise
// the lane tiles of kv_tile_idx.
template <bool kRows>
__device__ __forceinline__ void flash_block(const uint4* tiles, int bi, int p0, int end, const uint32_t (&qf)[16],
                                            float (&o)[8][4], float& mrun0, float& mrun1, float& lrun0,
                                            float& lrun1) {
  const int lane = threadIdx.x & 31, g8 = lane >> 2, t4 = lane & 3;
  uint4 kr[2][4], vr[2][4];
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    const bool ok = p0 + 8 * h2 + g8 < end;
    if constexpr (kRows) {
      const int odd = g8 & 1;
      const uint4* krow = tiles + (kBlk * bi + 8 * h2 + g8) * (kHD / 8);
      const uint4* vrow = krow + kKvSlotPos * (kHD / 8);
      uint4 tk[4], tv[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tk[c] = krow[t4 + 4 * (c ^ odd)];
        tv[c] = ok ? vrow[t4 + 4 * (c ^ odd)] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        kr[h2][c] = odd ? tk[c ^ 1] : tk[c];
        vr[h2][c] = odd ? tv[c ^ 1] : tv[c];
      }
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        kr[h2][c] = tiles[kv_tile_idx(bi, 0, h2, c, lane)];
        vr[h2][c] = ok ? tiles[kv_tile_idx(bi, 1, h2, c, lane)] : make_uint4(0u, 0u, 0u, 0u);
      }
    }
  }
  // S^T = K Q^T
  float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int ks = 0; ks < kHD / 16; ++ks)
    mma_16816(s, word_of(kr[0], 2 * ks), word_of(kr[1], 2 * ks), word_of(kr[0], 2 * ks + 1),
              word_of(kr[1], 2 * ks + 1), qf[2 * ks], qf[2 * ks + 1]);
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

__device__ void attn_item(const Params& P, Smem& S, const LayerPtrs& L, int b, int kvh,
                          int split, int n_splits, int chunk, int pos, uint32_t in_tag, uint32_t out_tag,
                          uint4* kvs, CState* ring) {
  AttnSmem& A = *reinterpret_cast<AttnSmem*>(S.act);
  const lmps_model_desc& m = P.m;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int Hq = m.n_q_heads, Hkv = m.n_kv_heads, G = Hq / Hkv;
  const int qkv_rows = (Hq + 2 * Hkv) * kHD;
  const int T = pos + 1;
  const int start = split * chunk, end = min(T, start + chunk);
  const unsigned long long* row = P.qkvt + static_cast<size_t>(b) * (qkv_rows / 2);
  unsigned long long* out = P.attnt + static_cast<size_t>(b) * (Hq * kHD / 2);
  const int ps = P.s.page_size, pshift = __ffs(ps) - 1;  // page_size is a power of two
  const int32_t* bt = P.s.block_table + static_cast<size_t>(b) * P.s.max_pages;
  __half* kpool = L.k_pool;
  __half* vpool = L.v_pool;
  const bool has_pos = pos >= start && pos < end;
  const uint64_t kvpol = evict_last_policy();

  // Where the cached K/V rows come from: the caller's shared-memory tiles
  // (dedicated attention CTAs, kvs), or ring slots of 32 positions that the
  // producer warp fills while the q|k|v stage runs (produce_kv); the row of
  // pos itself is appended below and patched into its tile after the sync.
  const int nblk = (end - start + kBlk - 1) / kBlk;
  // cache offset of position pos (the KV append of the split holding it)
  const size_t app =
      has_pos ? ((static_cast<size_t>(__ldg(bt + (pos >> pshift))) * Hkv + kvh) * ps + (pos & (ps - 1))) * kHD : 0;
  // q rows of this KV head's G query heads and (the split holding the new
  // position) its k and v rows, polled from the tagged q|k|v output as groups
  // of 8 dims.  With adjacent RoPE pairs (rope.metal:19-40) a group holds
  // whole pairs: the polling thread rotates it in registers, with the cos/sin
  // of its four pairs (a row of the position's RoPE table) loaded while it
  // waits.
  const bool adj = m.rope_style == LMPS_ROPE_INTERLEAVED;
  const float4* rope_row = reinterpret_cast<const float4*>(P.s.rope_table + static_cast<size_t>(pos) * kHD);
  {
    const int nq4 = G * (kHD / 8), n4 = nq4 + (has_pos ? 2 * (kHD / 8) : 0);
    if (tid < n4) {
      const int c8 = tid % (kHD / 8);  // dims 8*c8 .. 8*c8+7
      const int kind = tid < nq4 ? 0 : (tid - nq4 < kHD / 8 ? 1 : 2);  // q, k, v
      const int seg = kind == 0 ? kvh * G + tid / (kHD / 8) : kind == 1 ? Hq + kvh : Hq + Hkv + kvh;
      const unsigned long long* src = row + seg * (kHD / 2) + 4 * c8;
      Tagged4 t;
      tagged4_issue(src, t);
      float4 cs[2];  // (cos, sin) of pairs 4*c8 .. 4*c8+3 at this position
      if (adj && kind < 2) {
        cs[0] = __ldg(rope_row + 2 * c8);
        cs[1] = __ldg(rope_row + 2 * c8 + 1);
      }
      uint4 v = tagged4_finish(P, S, src, in_tag, t);
      if (adj && kind < 2) {
        uint32_t* w = reinterpret_cast<uint32_t*>(&v);
        const float* r = reinterpret_cast<const float*>(cs);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
          w[e] = pack_half2(f.x * r[2 * e] - f.y * r[2 * e + 1], f.x * r[2 * e + 1] + f.y * r[2 * e]);
        }
      }
      if (!adj) {
        *reinterpret_cast<uint4*>(&A.raw[8 * tid]) = v;
      } else if (kind == 0) {
        *reinterpret_cast<uint4*>(&A.q[tid / (kHD / 8)][8 * c8]) = v;
      } else {
        st_kv8((kind == 1 ? kpool : vpool) + app + 8 * c8, v, kvpol);
        if (kvs) {  // and into its tile: row pos, dims 8*c8 .. (lane (pos & 7, c8 / 4), chunk c8 % 4)
          const int rel = pos - start;
          kvs[kv_tile_idx(rel >> 4, kind - 1, (rel >> 3) & 1, c8 >> 2, 4 * (rel & 7) + (c8 & 3))] = v;
        }
      }
    }
  }
  if (!adj && tid < kHD / 2)  // RoPE (cos, sin) of this position, (j, j + head_dim/2) pairs
    A.rot[tid] = __ldg(reinterpret_cast<const float2*>(rope_row) + tid);
  consumer_sync();
  if (!adj) {
    for (int i = tid; i < G * (kHD / 2); i += kConsumers) {  // RoPE'd q, fp16-rounded
      const int h = i / (kHD / 2), j = i - h * (kHD / 2);
      int i1, i2;
      rope_pair(j, m.rope_style, i1, i2);
      const float2 r = A.rot[j];
      const float qa = __half2float(A.raw[h * kHD + i1]), qb = __half2float(A.raw[h * kHD + i2]);
      A.q[h][i1] = __float2half_rn(qa * r.x - qb * r.y);
      A.q[h][i2] = __float2half_rn(qa * r.y + qb * r.x);
    }
    if (has_pos) {  // KV append: rotated k and raw v at position pos
      const __half* kraw = A.raw + G * kHD;
      if (tid < kHD / 2) {
        int i1, i2;
        rope_pair(tid, m.rope_style, i1, i2);
        const float2 r = A.rot[tid];
        const float ka = __half2float(kraw[i1]), kb = __half2float(kraw[i2]);
        const __half k1 = __float2half_rn(ka * r.x - kb * r.y), k2 = __float2half_rn(ka * r.y + kb * r.x);
        st_kv(kpool + app + i1, k1, kvpol);
        st_kv(kpool + app + i2, k2, kvpol);
        if (kvs) {
          tile_half(kvs, pos - start, 0, i1) = k1;
          tile_half(kvs, pos - start, 0, i2) = k2;
        }
      } else if (tid < kHD / 2 + kHD) {
        st_kv(vpool + app + tid - kHD / 2, kraw[kHD + tid - kHD / 2], kvpol);
        if (kvs) tile_half(kvs, pos - start, 1, tid - kHD / 2) = kraw[kHD + tid - kHD / 2];
      }
    }
    consumer_sync();
  }
  // rotated q in shared memory, the new k/v row in the cache

  // -- per-warp flash loop over 16-position blocks
  uint32_t qf[16];  // B operand Q^T: head g8, physical dims 8*t4 + 32*c .. +7 (c = 0..3)
  {
    const uint4* qs = reinterpret_cast<const uint4*>(&A.q[g8 < G ? g8 : 0][8 * t4]);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 v = g8 < G ? qs[4 * c] : make_uint4(0u, 0u, 0u, 0u);
      qf[4 * c] = v.x;
      qf[4 * c + 1] = v.y;
      qf[4 * c + 2] = v.z;
      qf[4 * c + 3] = v.w;
    }
  }
  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
  float mrun0 = -INFINITY, mrun1 = -INFINITY, lrun0 = 0.0f, lrun1 = 0.0f;  // heads 2*t4, 2*t4+1
  // Work units: 16-position blocks of the caller's tiles (kvs: warp w takes
  // blocks w, w + warps, ..), or ring slots of 32 positions (slot i of the
  // item goes to warp i mod min(warps, slots) and is released by it alone;
  // the bound keeps every wait within one fill of its slot).
  if (kvs) asm volatile("cp.async.wait_all;" ::: "memory");  // this thread's staged tile rows
  const int n_units = kvs ? nblk : (end - start + kKvSlotPos - 1) / kKvSlotPos;
  const int nwu = kvs ? kConsumerWarps : min(kConsumerWarps, P.slots);
  const int upos = kvs ? kBlk : kKvSlotPos;
  const CState base = ring ? *ring : CState{};
  for (int i = warp; warp < nwu && i < n_units; i += nwu) {
    const int s0 = start + i * upos;
    const uint4* tiles = kvs;
    int bi = i;
    CState my{};
    if (!kvs) {
      my = cs_after(P, base, i);
      slot_wait(S, P, my);
      uint4* slot_tiles = reinterpret_cast<uint4*>(S.ring + static_cast<size_t>(my.slot) * kSlotBytes);
      if (has_pos && pos >= s0 && pos < s0 + kKvSlotPos) {  // the new row (lanes 0-15 K, 16-31 V)
        const int kv = lane >> 4, u = lane & 15;
        slot_tiles[(kv * kKvSlotPos + pos - s0) * (kHD / 8) + u] =
            __ldcg(reinterpret_cast<const uint4*>((kv ? vpool : kpool) + app) + u);
        __syncwarp();
      }
      tiles = slot_tiles;
      bi = 0;
    }
#pragma unroll 1
    for (int p0 = s0; p0 < min(end, s0 + upos); p0 += kBlk, ++bi) {
      if (kvs)
        flash_block<false>(tiles, bi, p0, end, qf, o, mrun0, mrun1, lrun0, lrun1);
      else
        flash_block<true>(tiles, bi, p0, end, qf, o, mrun0, mrun1, lrun0, lrun1);
    }
    if (!kvs) {
      // (the slot's next fill may be a TMA copy: order this warp's writes before it)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&S.empty[my.slot])),
                     "r"(kConsumerWarps)
                     : "memory");
    }
  }
  if (ring) *ring = cs_after(P, base, n_units);
  const int nw = min(nwu, n_units);  // warps that saw positions
  const size_t ms = P.max_splits;
  // -- warps meet in shared memory: each leaves its running max, sum and
  // output; the reducing thread rescales them to the merged max
  if (warp < nw) {
    if (g8 == 0) {
      A.wm[warp][2 * t4] = mrun0;
      A.wm[warp][2 * t4 + 1] = mrun1;
      A.wl[warp][2 * t4] = lrun0;
      A.wl[warp][2 * t4 + 1] = lrun1;
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)  // 16-byte stores, value k of this lane at (k + 4 lane) mod 32
      *reinterpret_cast<float4*>(&A.wo[warp][lane][(4 * mt + 4 * lane) & 31]) =
          make_float4(o[mt][0], o[mt][1], o[mt][2], o[mt][3]);
  }
  consumer_sync();
  for (int w = tid; w < G * (kHD / 2); w += kConsumers) {
    const int h = w / (kHD / 2), dp = w - h * (kHD / 2);
    // dims d = 2dp, d + 1 of head h: fragment value 4mt + 2e + (h & 1) of
    // lanes (g8, t4) = (2b + {0, 1}, h >> 1), d = 32(mt >> 1) + 8b + 4(mt & 1) + 2e
    const int d = 2 * dp, mt = 2 * (d >> 5) + ((d >> 2) & 1);
    const int k = 4 * mt + 2 * ((d >> 1) & 1) + (h & 1);
    const int la = 4 * (2 * ((d >> 3) & 3)) + (h >> 1);
    const int ka = (k + 4 * la) & 31, kb = (k + 4 * (la + 4)) & 31;
    float M = -INFINITY;
    for (int ww = 0; ww < nw; ++ww) M = fmaxf(M, A.wm[ww][h]);
    float n0 = 0.0f, n1 = 0.0f, den = 0.0f;
    for (int ww = 0; ww < nw; ++ww) {
      const float f = expf(A.wm[ww][h] - M);
      n0 += A.wo[ww][la][ka] * f;
      n1 += A.wo[ww][la + 4][kb] * f;
      den += A.wl[ww][h] * f;
    }
    if (n_splits == 1) {
      const float inv = den > 0.0f ? 1.0f / den : 0.0f;
      st_tagged(out + (kvh * G + h) * (kHD / 2) + dp, tagged(out_tag, pack_half2(n0 * inv, n1 * inv)));
    } else {
      const size_t prow = (static_cast<size_t>(b) * Hq + kvh * G + h) * ms + split;
      *reinterpret_cast<float2*>(&P.part_o[prow * kHD + 2 * dp]) = make_float2(n0, n1);
      if (dp == 0) P.part_ml[prow] = make_float2(M, den);
    }
  }
  if (n_splits == 1) {
    consumer_sync();  // the shared area is the next stage's staging area
    return;
  }
  __threadfence();
  consumer_sync();
  if (tid == 0) {
    const uint32_t old = atomicAdd(P.att_cnt + b * Hkv + kvh, 1u);
    A.is_last = (old == static_cast<uint32_t>(n_splits - 1)) ? 1 : 0;
  }
  consumer_sync();
  if (A.is_last) {  // the last split merges all partials of (b, kvh) by log-sum-exp
    if (tid == 0) {   // ready for the next layer before any output is published
      P.att_cnt[b * Hkv + kvh] = 0u;
      __threadfence();
    }
    consumer_sync();
    __threadfence();
    // split weights exp(m_sp - M) of every (head, split), one warp per head
    // with the splits across its lanes; then every (head, dim pair) adds the
    // weighted partial outputs (loads unrolled, several in flight)
    float* wsm = &A.wo[0][0][0];      // [G][n_splits] weights
    float* inv_den = wsm + G * n_splits;  // [G]
    if (warp < G) {
      // each lane loads its first kMergeLane splits' (max, sum) pairs once,
      // all in flight together, and keeps them in registers for both passes
      constexpr int kMergeLane = 4;
      const size_t prow0 = (static_cast<size_t>(b) * Hq + kvh * G + warp) * ms;
      float2 mls[kMergeLane];
#pragma unroll
      for (int i = 0; i < kMergeLane; ++i) {
        const int sp = lane + kWarp * i;
        mls[i] = sp < n_splits ? __ldcg(&P.part_ml[prow0 + sp]) : make_float2(-INFINITY, 0.0f);
      }
      float M = -INFINITY;
#pragma unroll
      for (int i = 0; i < kMergeLane; ++i)
        if (mls[i].y > 0.0f) M = fmaxf(M, mls[i].x);
      for (int sp = lane + kWarp * kMergeLane; sp < n_splits; sp += kWarp) {
        const float2 ml = __ldcg(&P.part_ml[prow0 + sp]);
        if (ml.y > 0.0f) M = fmaxf(M, ml.x);
      }
      M = warp_max(M);
      float den = 0.0f;
#pragma unroll
      for (int i = 0; i < kMergeLane; ++i) {
        const int sp = lane + kWarp * i;
        if (sp < n_splits) {
          const float wgt = mls[i].y > 0.0f ? expf(mls[i].x - M) : 0.0f;
          wsm[warp * n_splits + sp] = wgt;
          den = fmaf(wgt, mls[i].y, den);
        }
      }
      for (int sp = lane + kWarp * kMergeLane; sp < n_splits; sp += kWarp) {
        const float2 ml = __ldcg(&P.part_ml[prow0 + sp]);
        const float wgt = ml.y > 0.0f ? expf(ml.x - M) : 0.0f;
        wsm[warp * n_splits + sp] = wgt;
        den = fmaf(wgt, ml.y, den);
      }
      den = warp_sum(den);
      if (lane == 0) inv_den[warp] = den > 0.0f ? 1.0f / den : 0.0f;
    }
    consumer_sync();
    for (int w = tid; w < G * (kHD / 2); w += kConsumers) {
      const int h = w / (kHD / 2), dp = w - h * (kHD / 2);
      const size_t prow0 = (static_cast<size_t>(b) * Hq + kvh * G + h) * ms;
      const float* wh = wsm + h * n_splits;
      float n0 = 0.0f, n1 = 0.0f;
#pragma unroll 16  // the partial outputs' loads issue together
      for (int sp = 0; sp < n_splits; ++sp) {
        const float wgt = wh[sp];
        const float2 po = __ldcg(reinterpret_cast<const float2*>(&P.part_o[(prow0 + sp) * kHD + 2 * dp]));
        if (wgt != 0.0f) {
          n0 = fmaf(wgt, po.x, n0);
          n1 = fmaf(wgt, po.y, n1);
        }
      }
      const float inv = inv_den[h];
      st_tagged(out + (kvh * G + h) * (kHD / 2) + dp, tagged(out_tag, pack_half2(n0 * inv, n1 * inv)));
    }
  }
  consumer_sync();
}

// Positions per attention work item this step (all CTAs compute the same
// value): a whole sequence up to kMinSplit positions (one CTA, no cross-CTA
// merge), longer contexts split so that the items about fill the grid.
__device__ __forceinline__ int attn_chunk_len(const int* pos, int batch, int n_kv) {
  uint32_t total = 0;  // < 2^32: max_seq_len * batch * n_kv is bounded on the host
  for (int b = 0; b < batch; ++b) total += static_cast<uint32_t>(pos[b] + 1);
  if (total * static_cast<uint32_t>(n_kv) <= static_cast<uint32_t>(kMinSplit)) return kMinSplit;
  // ceil() of each (sequence, KV head) adds at most one item: keep the
  // item count within the grid so no CTA gets a second item
  const int slots_i = static_cast<int>(gridDim.x) - batch * n_kv;
  const uint32_t slots = slots_i > 0 ? static_cast<uint32_t>(slots_i) : 1u;
  uint32_t c = (total * static_cast<uint32_t>(n_kv) + slots - 1) / slots;
  c = (c + kKvSlotPos - 1) / kKvSlotPos * kKvSlotPos;  // ring slots never straddle two items
  return c < static_cast<uint32_t>(kMinSplit) ? kMinSplit : static_cast<int>(c);
}

// The cached K/V rows of this CTA's attention items of one layer (spread
// attention: the items, in the order, the consumers' attention stage runs),
// 32 positions per ring slot: K rows [32][head_dim] then V rows, as in the
// cache.  Items start at multiples of 32 positions, so a slot's rows span
// whole runs of cache pages: one TMA bulk copy per page run and matrix.
// The row of the new position (appended by the consumers during the
// stage; always the item's last row) is not copied.
__device__ bool produce_kv(const Params& P, Smem& S, int layer, int step, uint32_t& chunk, int& pslot,
                           uint32_t& pphase) {
  const int B = P.s.batch, Hkv = P.m.n_kv_heads;
  const int ps = P.s.page_size, pshift = __ffs(ps) - 1;  // a power of two
  const LayerPtrs& L = S.lp[layer];
  const uint64_t pol = evict_last_policy();
  int pos[kMaxB];
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) pos[b] = b < B ? P.s.pos[b] + step : 0;
  const int chunk_len = attn_chunk_len(pos, B, Hkv);
  int n_items = 0;
  for (int b = 0; b < B; ++b) n_items += Hkv * ((pos[b] + chunk_len) / chunk_len);
  for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
    // item -> (sequence, KV head, split) as the consumers number them
    int rem = it, b = 0, nsp = (pos[0] + chunk_len) / chunk_len;
    while (rem >= Hkv * nsp) {
      rem -= Hkv * nsp;
      ++b;
      nsp = (pos[b] + chunk_len) / chunk_len;
    }
    const int kvh = rem / nsp, sp = rem - kvh * nsp;
    const int start = sp * chunk_len, end = min(pos[b] + 1, start + chunk_len);
    const int32_t* bt = P.s.block_table + static_cast<size_t>(b) * P.s.max_pages;
    for (int s0 = start; s0 < end; s0 += kKvSlotPos) {
      const int slot = pslot;
      const uint32_t phase = pphase;
      if (++pslot == P.slots) {
        pslot = 0;
        pphase ^= 1u;
      }
      if (!acquire_slot(P, S, chunk, slot, phase)) return false;
      unsigned char* dst = S.ring + static_cast<size_t>(slot) * kSlotBytes;
      const int e = min(end, s0 + kKvSlotPos);
      const int e2 = (pos[b] >= s0 && pos[b] < e) ? pos[b] : e;  // rows [s0, e2) come from the cache
      constexpr uint32_t kRowBytes = kHD * sizeof(__half);
      mbar_expect_tx(&S.full[slot], 2u * static_cast<uint32_t>(e2 - s0) * kRowBytes);
      for (int p = s0; p < e2;) {
        const int in_page = p & (ps - 1), run = min(e2 - p, ps - in_page);
        const size_t off = ((static_cast<size_t>(__ldg(bt + (p >> pshift))) * Hkv + kvh) * ps + in_page) * kHD;
        unsigned char* d = dst + static_cast<size_t>(p - s0) * kRowBytes;
        bulk_g2s(d, L.k_pool + off, run * kRowBytes, &S.full[slot], pol);
        bulk_g2s(d + kKvSlotPos * kRowBytes, L.v_pool + off, run * kRowBytes, &S.full[slot], pol);
        p += run;
      }
      ++chunk;
    }
  }
  return true;
}

// The next token of every sequence from the tagged per-CTA argmax slots of a
// LM head stage (tag14 = low 14 bits of its tag): slot = value key (32) |
// (0x3FFFF - row) (18) | tag14 (14).  Every consumer thread gets the rows.
template <int NB>
__device__ void gather_argmax(const Params& P, Smem& S, uint32_t tag14, int (&row)[NB]) {
  const int B = P.s.batch;
  const int n = S.gemv_grid * kMaxB;
  unsigned long long best[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) best[b] = 0ull;
  unsigned long long w[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int i = threadIdx.x + q * kConsumers;
    w[q] = (i < n && (i % kMaxB) < B) ? ld_tagged_acquire(P.kslot + i) : 0ull;
  }
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int i = threadIdx.x + q * kConsumers;
    if (i < n && (i % kMaxB) < B) {
      if ((w[q] & 0x3FFFull) != tag14) {
        const uint64_t t0 = globaltimer();
        while (true) {
          w[q] = ld_tagged_acquire(P.kslot + i);
          if ((w[q] & 0x3FFFull) == tag14) break;
          if (aborting(S)) break;
          if (globaltimer() - t0 > kTimeoutNs) {
            raise_abort(P, S, 1);
            break;
          }
        }
      }
#pragma unroll
      for (int b = 0; b < NB; ++b)
        if (b == i % kMaxB) best[b] = u64_max(best[b], w[q]);
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const unsigned long long v = warp_max_u64(best[b]);
    if (lane == 0) S.best[warp * kMaxB + b] = v;
  }
  consumer_sync();
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    unsigned long long v = 0ull;
#pragma unroll
    for (int ww = 0; ww < kConsumerWarps; ++ww) v = u64_max(v, S.best[ww * kMaxB + b]);
    row[b] = 0x3FFFF - static_cast<int>((v >> 14) & 0x3FFFFull);
  }
  consumer_sync();
}

// Stages of a step (see consumer below).
enum StepStage { K_QKV = 0, K_ATT = 1, K_O = 2, K_GU = 3, K_DN = 4, K_HEAD = 5 };

// K/V rows [0, npos) of (sequence b, KV head kvh) of one layer into the
// shared-memory tiles: warp w stages blocks w, w + warps, .. (the blocks it
// reads in attn_item), each lane its own 16-byte runs (cp.async, waited for
// in attn_item before the flash loop).
__device__ void stage_kv_tiles(const Params& P, const LayerPtrs& L, int b, int kvh, int npos, uint4* kvs) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g8 = lane >> 2, t4 = lane & 3;
  const int ps = P.s.page_size, pshift = __ffs(ps) - 1, Hkv = P.m.n_kv_heads;
  const int32_t* bt = P.s.block_table + static_cast<size_t>(b) * P.s.max_pages;
  for (int bi = warp; bi * kBlk < npos; bi += kConsumerWarps) {
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int p = bi * kBlk + 8 * h2 + g8;
      if (p < npos) {
        const size_t off =
            ((static_cast<size_t>(__ldg(bt + (p >> pshift))) * Hkv + kvh) * ps + (p & (ps - 1))) * kHD + 8 * t4;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(&kvs[kv_tile_idx(bi, 0, h2, c, lane)])),
                       "l"(L.k_pool + off + 32 * c)
                       : "memory");
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(&kvs[kv_tile_idx(bi, 1, h2, c, lane)])),
                       "l"(L.v_pool + off + 32 * c)
                       : "memory");
        }
      }
    }
  }
}

// A dedicated attention CTA: item (sequence b, KV head kvh) of every layer
// and step.  While the projections of a layer run, it stages the next
// layer's cached K/V rows; then it waits for the layer's q|k|v like any
// attention item (attn_item, whole context, one split).
__device__ void att_consumer(const Params& P, Smem& S, uint32_t epoch) {
  const int a = static_cast<int>(blockIdx.x) - S.gemv_grid;
  const int Hkv = P.m.n_kv_heads, b = a / Hkv, kvh = a - b * Hkv;
  const int n_stage = P.m.n_layers * 5 + 1;
  const int pos0 = P.s.pos[b];
  uint4* kvs = reinterpret_cast<uint4*>(S.ring);
  for (int step = 0; step < P.n_steps; ++step) {
    const int pos = pos0 + step;
    const uint32_t tag0 = epoch + static_cast<uint32_t>(step * n_stage) + 1u;
    stage_kv_tiles(P, S.lp[0], b, kvh, pos, kvs);
    for (int l = 0; l < P.m.n_layers; ++l) {
      if (aborting(S)) return;
      const uint32_t tag = tag0 + static_cast<uint32_t>(5 * l + K_ATT);
      attn_item(P, S, S.lp[l], b, kvh, 0, 1, pos + 1, pos, tag - 1u, tag, kvs, nullptr);
      if (l + 1 < P.m.n_layers) stage_kv_tiles(P, S.lp[l + 1], b, kvh, pos, kvs);
    }
  }
}

// ---------------------------------------------------------------------------
// Consumers: the decode loop
// ---------------------------------------------------------------------------
// Stages of a step in order: per layer q|k|v, attention, o, gate/up, down;
// then the LM head.  Each stage function has exactly one call site below, so
// the kernel's code is one copy of every stage.  Stage si of step `step`
// publishes its output with tag epoch + step * n_stage + si + 1; the next
// stage polls for that tag, so no grid-wide barrier is needed.

template <int NB>
__device__ void consumer(const Params& P, Smem& S, uint32_t epoch) {
  CState cs{0, 0u, 0ull, 0};
  const lmps_model_desc& m = P.m;
  const int B = P.s.batch;
  const int hidden = m.hidden, Hkv = m.n_kv_heads;
  const int q_dim = m.n_q_heads * kHD;
  int tok[NB], pos[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    tok[b] = b < B ? P.s.tokens[b] : 0;
    pos[b] = b < B ? P.s.pos[b] : 0;
  }
  const int hist0 = (P.s.history && P.s.step_counter) ? P.s.step_counter[0] : 0;
  const bool tr = threadIdx.x == 0;
  const int n_stage = m.n_layers * 5 + 1;
  int o0, o1;
  row_range(hidden, blockIdx.x, S.gemv_grid, o0, o1);
  const __half* embed = reinterpret_cast<const __half*>(m.embed);
  const __half* x_in = reinterpret_cast<const __half*>(P.s.x_in);

  for (int step = 0; step < P.n_steps; ++step) {
    const uint32_t tag0 = epoch + static_cast<uint32_t>(step * n_stage) + 1u;  // tag of stage 0
    if (step > 0) {
      // next tokens from the previous step's LM head
      int nxt[NB];
      gather_argmax<NB>(P, S, (tag0 - 1u) & 0x3FFFu, nxt);
      if (aborting(S)) return;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b < B) {
          if (nxt[b] >= m.vocab) {  // no logit won (non-finite head output)
            if (threadIdx.x == 0) atomicExch(P.s.error, 3);
            nxt[b] = 0;
          }
          if (blockIdx.x == 0 && threadIdx.x == 0 && P.s.history && hist0 + step - 1 >= 0 &&
              hist0 + step - 1 < P.s.history_rows)
            P.s.history[static_cast<size_t>(hist0 + step - 1) * B + b] = nxt[b];
          tok[b] = (step - 1 < P.s.n_forced && P.s.forced) ? P.s.forced[static_cast<size_t>(b) * P.s.forced_stride + step - 1] : nxt[b];
          pos[b] += 1;
        }
      }
    }
    const bool from_x_in = step == 0 && x_in;
    {  // residual rows this CTA owns start as the step's input rows
      const int bb = threadIdx.x / kOwnMax, i = threadIdx.x - bb * kOwnMax;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b == bb && b < B && i < o1 - o0) {
          const __half* src = from_x_in ? x_in + static_cast<size_t>(b) * hidden : embed + static_cast<size_t>(tok[b]) * hidden;
          S.xown[b * kOwnMax + i] = src[o0 + i];
        }
      }
    }
    for (int si = 0; si < n_stage; ++si) {
      if (aborting(S)) return;  // uniform: every wait that raises it is followed by a block sync
      const int l = si / 5;
      const int kind = (l == m.n_layers) ? K_HEAD : si - 5 * l;
      const uint32_t tag = tag0 + static_cast<uint32_t>(si), in_tag = tag - 1u;
      if (tr) trace_event(P, blockIdx.x, cs.ev, cs.wait_ns);
      const LayerPtrs& L = S.lp[kind == K_HEAD ? 0 : l];
      // the stage's weight chunking does not depend on its input: set up
      // before the input is polled
      const int wk = kind == K_QKV ? ST_QKV : kind == K_O ? ST_O : kind == K_GU ? ST_GU : kind == K_DN ? ST_DN : ST_HEAD;
      Chunking ch{};
      if (kind != K_ATT) ch = stage_chunks<(NB > 1)>(P, wk, l, S.gemv_grid);
      // -- stage the input activation in shared memory
      if (kind == K_QKV || kind == K_GU || kind == K_HEAD) {
        const __half* rows[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const int bb = b < B ? b : 0;
          rows[b] = from_x_in ? x_in + static_cast<size_t>(bb) * hidden : embed + static_cast<size_t>(tok[bb]) * hidden;
        }
        const unsigned long long* tsrc = (kind == K_QKV && l == 0) ? nullptr : kind == K_GU ? P.x1t : P.xt;
        const __half* gamma = kind == K_QKV ? L.in_norm : kind == K_GU ? L.post_norm
                                                       : reinterpret_cast<const __half*>(m.final_norm);
        stage_norm<NB>(P, S, rows, tsrc, in_tag, gamma, hidden);
      } else if (kind == K_O || kind == K_DN) {
        stage_copy<NB>(P, S, kind == K_O ? P.attnt : P.at, in_tag, kind == K_O ? q_dim : m.intermediate);
      }
      if (tr) trace_event(P, blockIdx.x, cs.ev, cs.wait_ns);
      // -- compute and publish
      if (kind == K_ATT) {
        // (with dedicated attention CTAs they run this stage: no items here)
        const int chunk = attn_chunk_len(pos, B, Hkv);
        int n_items = 0;
#pragma unroll
        for (int b = 0; b < NB; ++b)
          if (b < B && S.n_att == 0) n_items += Hkv * ((pos[b] + chunk) / chunk);
        for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
          int rem = it, bsel = 0, nsp = 1;
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            if (b < B && bsel == b) {
              nsp = (pos[b] + chunk) / chunk;
              if (rem >= Hkv * nsp) {
                rem -= Hkv * nsp;
                ++bsel;
              }
            }
          }
          const int kvh = rem / nsp, sp = rem - kvh * nsp;
          int pb = pos[0];
#pragma unroll
          for (int b = 0; b < NB; ++b)
            if (b == bsel) pb = pos[b];
          attn_item(P, S, L, bsel, kvh, sp, nsp, chunk, pb, in_tag, tag, nullptr, &cs);
        }
        trace_mid(P, cs);
      } else if (kind == K_DN) {
        if constexpr (NB > 1)
          gemv_down_mma<NB>(P, S, cs, tag, ch);
        else
          gemv_down<NB>(P, S, cs, l, tag, ch);
      } else {
        __half* lg = (kind == K_HEAD && step == P.n_steps - 1) ? reinterpret_cast<__half*>(P.s.logits) : nullptr;
        if constexpr (NB > 1)
          gemv_rows_mma<NB>(P, S, cs, wk, l, lg, tag, ch);
        else
          gemv_rows<NB>(P, S, cs, wk, l, lg, tag, ch);
        if (kind == K_HEAD) {
          consumer_sync();
          if (threadIdx.x < B) {
            unsigned long long v = 0ull;
            for (int w = 0; w < kConsumerWarps; ++w) v = u64_max(v, S.best[w * kMaxB + threadIdx.x]);
            const uint32_t row = 0xFFFFFFFFu - static_cast<uint32_t>(v);
            const unsigned long long slot =
                v ? ((v >> 32) << 32) | (static_cast<unsigned long long>(0x3FFFFu - row) << 14) : 0ull;
            st_tagged(P.kslot + blockIdx.x * kMaxB + threadIdx.x, slot | (tag & 0x3FFFu));
          }
        }
      }
      if (tr) trace_event(P, blockIdx.x, cs.ev, cs.wait_ns);
    }
  }
  // ---- CTA 0: final tokens, state write-back, next launch's tag base
  if (blockIdx.x != 0) return;
  {
    const int last = P.n_steps - 1;
    int nxt[NB];
    gather_argmax<NB>(P, S, (epoch + static_cast<uint32_t>(P.n_steps * n_stage)) & 0x3FFFu, nxt);
    if (aborting(S)) return;
    if (threadIdx.x == 0) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b < B) {
          if (nxt[b] >= m.vocab) {
            atomicExch(P.s.error, 3);
            nxt[b] = 0;
          }
          if (P.s.history && hist0 + last >= 0 && hist0 + last < P.s.history_rows)
            P.s.history[static_cast<size_t>(hist0 + last) * B + b] = nxt[b];
          P.s.tokens[b] = (last < P.s.n_forced && P.s.forced) ? P.s.forced[static_cast<size_t>(b) * P.s.forced_stride + last] : nxt[b];
          P.s.pos[b] = pos[b] + 1;
        }
      }
      if (P.s.history && P.s.step_counter) P.s.step_counter[0] = hist0 + P.n_steps;
      *P.epoch = epoch + static_cast<uint32_t>(P.n_steps * n_stage) + 1u;
    }
  }
}

template <int NB>
__global__ void __launch_bounds__(kThreads, 1) decode_persistent_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(128) unsigned char smem[];
  Smem S;
  S.ring = smem;
  S.act = smem + static_cast<size_t>(P.slots) * kSlotBytes;
  unsigned char* tail = S.act + P.act_bytes;
  S.full = reinterpret_cast<uint64_t*>(tail);
  S.empty = S.full + 16;
  S.red8 = reinterpret_cast<float*>(S.empty + 16);
  S.best = reinterpret_cast<unsigned long long*>(S.red8 + kConsumerWarps * kMaxB);
  S.misc = reinterpret_cast<int*>(S.best + kConsumerWarps * kMaxB);
  S.lp = reinterpret_cast<LayerPtrs*>(S.misc + 16);
  S.xown = reinterpret_cast<__half*>(S.lp + P.m.n_layers);
  S.x1own = S.xown + kMaxB * kOwnMax;
  S.bias_own = S.x1own + kMaxB * kOwnMax;
  // tag base of this launch (CTA 0 advances it after every CTA has used it)
  const uint32_t epoch = __ldcg(P.epoch);
  {
    // Short contexts: the batch * n_kv attention items each get a CTA of
    // their own (the last CTAs of the grid), whose code stays resident in its
    // SM's instruction cache and which stages each layer's K/V rows in its
    // shared memory while the projections run; the other CTAs run the
    // projections.  Long contexts spread attention over every CTA.  Every CTA
    // derives the same choice from the launch's positions.
    int max_t = 0;
    for (int b = 0; b < P.s.batch; ++b) max_t = max(max_t, P.s.pos[b] + P.n_steps);
    const int items = P.s.batch * P.m.n_kv_heads;
    const int tile_blocks = static_cast<int>((static_cast<size_t>(P.slots) * kSlotBytes) / kKvTileBytes);
    S.n_att = (max_t <= tile_blocks * kBlk && items <= kMaxAttCtas) ? items : 0;
    S.gemv_grid = static_cast<int>(gridDim.x) - S.n_att;
  }
  for (int i = threadIdx.x; i < P.m.n_layers; i += blockDim.x) {
    const lmps_layer_desc& L = P.m.layers[i];
    S.lp[i] = LayerPtrs{reinterpret_cast<const __half*>(L.in_norm), reinterpret_cast<const __half*>(L.post_norm),
                        reinterpret_cast<__half*>(L.k_pool), reinterpret_cast<__half*>(L.v_pool)};
  }
  if (static_cast<int>(blockIdx.x) < S.gemv_grid) {  // q|k|v bias of this CTA's qkv rows, every layer
    const int qkv_rows = (P.m.n_q_heads + 2 * P.m.n_kv_heads) * kHD;
    int q0, q1;
    row_range(qkv_rows, blockIdx.x, S.gemv_grid, q0, q1);
    for (int i = threadIdx.x; i < P.m.n_layers * kOwnMax; i += blockDim.x) {
      const int l = i / kOwnMax, r = i - l * kOwnMax;
      if (r < q1 - q0) S.bias_own[i] = reinterpret_cast<const __half*>(P.m.layers[l].qkv_bias)[q0 + r];
    }
  }
  // Every position this launch touches must be inside the cache and every fed
  // token inside the vocabulary; all CTAs read the same values, so all leave
  // together (nothing has been issued yet).
  {
    bool bad = false;
    for (int b = 0; b < P.s.batch; ++b) {
      const int p0 = P.s.pos[b], t0 = P.s.tokens[b];
      if (p0 < 0 || p0 + P.n_steps > P.s.max_seq_len) bad = true;
      if (!P.s.x_in && (t0 < 0 || t0 >= P.m.vocab)) bad = true;
      for (int i = 0; P.s.forced && i < P.s.n_forced && i < P.n_steps; ++i) {
        const int f = P.s.forced[static_cast<size_t>(b) * P.s.forced_stride + i];
        if (f < 0 || f >= P.m.vocab) bad = true;
      }
    }
    if (bad) {
      if (threadIdx.x == 0) atomicExch(P.s.error, 2);
      return;
    }
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < P.slots; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.empty[i], kConsumerWarps);
    }
    S.misc[0] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const bool att_cta = static_cast<int>(blockIdx.x) >= S.gemv_grid;
  if (threadIdx.x >= kConsumers) {
    if (threadIdx.x == kConsumers && !att_cta) producer<(NB > 1)>(P, S);
    return;
  }
  if (att_cta)
    att_consumer(P, S, epoch);
  else
    consumer<NB>(P, S, epoch);
}

// Shared-memory tail after the ring and the activation area.
static int tail_bytes(int n_layers) {
  const size_t fixed = 32 * sizeof(uint64_t) +
                       kConsumerWarps * kMaxB * (sizeof(float) + sizeof(unsigned long long)) + 16 * sizeof(int) +
                       2 * kOwnMax * kMaxB * sizeof(__half);
  const size_t t = fixed + static_cast<size_t>(n_layers) * (kOwnMax * sizeof(__half) + sizeof(LayerPtrs));
  return static_cast<int>((t + 127) & ~static_cast<size_t>(127));
}

struct WsLayout {
  size_t xt, x1t, qkvt, attnt, at, kslot, part_o, part_ml, att_cnt, epoch, total;
  int max_splits;
};

static size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

static WsLayout ws_layout(const lmps_model_desc& m, int B, int max_seq_len) {
  WsLayout w{};
  const size_t qkv_rows = static_cast<size_t>(m.n_q_heads + 2 * m.n_kv_heads) * m.head_dim;
  const size_t q_dim = static_cast<size_t>(m.n_q_heads) * m.head_dim;
  const size_t tw = sizeof(unsigned long long) / 2;  // tagged bytes per element
  w.max_splits = (max_seq_len + kMinSplit - 1) / kMinSplit;
  size_t off = 0;
  // State that persists from one launch to the next comes first, at offsets
  // that do not depend on the batch size of the launch.
  w.epoch = off; off = align256(off + sizeof(uint32_t));
  w.att_cnt = off; off = align256(off + sizeof(uint32_t) * kMaxB * m.n_kv_heads);
  w.kslot = off; off = align256(off + sizeof(unsigned long long) * kMaxGrid * kMaxB);
  w.xt = off; off = align256(off + tw * B * m.hidden);
  w.x1t = off; off = align256(off + tw * B * m.hidden);
  w.qkvt = off; off = align256(off + tw * B * qkv_rows);
  w.attnt = off; off = align256(off + tw * B * q_dim);
  w.at = off; off = align256(off + tw * B * m.intermediate);
  w.part_o = off; off = align256(off + sizeof(float) * B * m.n_q_heads * w.max_splits * m.head_dim);
  w.part_ml = off; off = align256(off + sizeof(float2) * B * m.n_q_heads * w.max_splits);
  w.total = off;
  return w;
}

static int act_bytes_for(const lmps_model_desc& m, int nb) {
  size_t a = sizeof(AttnSmem);
  const size_t grp = 16 * 4 + 4 + 4;  // plane words + scl + xs8 per group
  // k = hidden stages: planes + per-lane partials of every row entry
  // (+16: the partials start 16-byte aligned)
  const size_t hid =
      static_cast<size_t>(nb) * (m.hidden / 32) * grp + static_cast<size_t>(nb) * kPartRows * 16 * 4 + 16;
  // down projection: planes + one partial per (row, warp)
  const size_t dn = static_cast<size_t>(nb) * (m.intermediate / 32) * grp +
                    static_cast<size_t>(nb) * kOwnMax * kRedStride * 4 + 16;
  a = a > hid ? a : hid;
  a = a > dn ? a : dn;
  return static_cast<int>((a + 127) & ~static_cast<size_t>(127));
}

// Launch configuration of one (device, batch instantiation, model shape):
// found once with the CUDA attribute and occupancy queries, then reused (the
// per-token path launches once per token, and those queries cost more host
// time than the launch).
struct LaunchCfg {
  int key_layers = -1, key_hidden = 0, key_inter = 0, key_qkv = 0, key_vocab = 0;
  int sms = 0, slots = 0;
  size_t smem = 0;
};
constexpr int kCfgDevices = 64;

template <int NB>
static int launch(const Params& P0, const lmps_model_desc& m, cudaStream_t st) {
  static LaunchCfg cache[kCfgDevices];
  static std::mutex cache_mutex;
  Params P = P0;
  int dev = 0;
  cudaError_t e0 = cudaGetDevice(&dev);
  if (e0 != cudaSuccess) return static_cast<int>(e0);
  P.act_bytes = act_bytes_for(m, NB);
  const int qkv_rows_k = (m.n_q_heads + 2 * m.n_kv_heads) * m.head_dim;
  if (dev >= 0 && dev < kCfgDevices) {
    std::lock_guard<std::mutex> lock(cache_mutex);
    const LaunchCfg& c = cache[dev];
    if (c.key_layers == m.n_layers && c.key_hidden == m.hidden && c.key_inter == m.intermediate &&
        c.key_qkv == qkv_rows_k && c.key_vocab == m.vocab) {
      P.slots = c.slots;
      void* args[] = {&P};
      const cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<void*>(decode_persistent_kernel<NB>),
                                                        dim3(c.sms), dim3(kThreads), args, c.smem, st);
      return e == cudaSuccess ? LMPS_OK : static_cast<int>(e);
    }
  }
  int sms = 0, max_smem = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  // rows of the hidden and q|k|v outputs one CTA owns (residual / bias kept in shared memory)
  const int qkv_rows = (m.n_q_heads + 2 * m.n_kv_heads) * m.head_dim;
  // (pair-aligned partitions: at most 2 * ceil(rows / 2 / ctas) rows per CTA,
  // with up to kMaxAttCtas CTAs set aside for attention)
  const int proj_ctas = sms - kMaxAttCtas;
  if (proj_ctas < 1) return LMPS_ERR_UNSUPPORTED;
  auto per_cta = [&](int rows) { return 2 * ((rows / 2 + proj_ctas - 1) / proj_ctas); };
  // tensor-core path: a CTA's hidden rows are one 16-row tile of the down projection
  if (NB > 1 && per_cta(m.hidden) > kTileRows) return LMPS_ERR_UNSUPPORTED;
  if (per_cta(m.hidden) > kOwnMax || per_cta(qkv_rows) > kOwnMax || per_cta(m.intermediate) > kOutMax ||
      m.n_layers > kMaxLayers || sms > kMaxGrid || m.vocab > 0x40000 || 2 * kConsumers < sms * kMaxB)
    return LMPS_ERR_UNSUPPORTED;
  auto kern = decode_persistent_kernel<NB>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return static_cast<int>(e);
  // As many ring slots as fit next to one resident CTA per SM.
  const int tail = tail_bytes(m.n_layers);
  int slots = (max_smem - P.act_bytes - tail) / kSlotBytes;
  // At most one slot per consumer warp: chunk i of a stage goes to warp
  // i mod min(warps, slots), so each slot's consecutive fills go to the same
  // warp and no parity wait can match a phase two fills old.  (227 KB of
  // shared memory holds at most 11 slots anyway.)
  if (slots > kConsumerWarps) slots = kConsumerWarps;
  size_t smem = 0;
  for (; slots >= 3; --slots) {
    smem = static_cast<size_t>(slots) * kSlotBytes + P.act_bytes + tail;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (per_sm >= 1) break;
  }
  if (slots < 3) return LMPS_ERR_UNSUPPORTED;
  P.slots = slots;
  if (dev >= 0 && dev < kCfgDevices) {
    std::lock_guard<std::mutex> lock(cache_mutex);
    LaunchCfg& c = cache[dev];
    c.key_layers = m.n_layers;
    c.key_hidden = m.hidden;
    c.key_inter = m.intermediate;
    c.key_qkv = qkv_rows_k;
    c.key_vocab = m.vocab;
    c.sms = sms;
    c.slots = slots;
    c.smem = smem;
  }
  void* args[] = {&P};
  e = cudaLaunchCooperativeKernel(reinterpret_cast<void*>(kern), dim3(sms), dim3(kThreads), args, smem, st);
  return e == cudaSuccess ? LMPS_OK : static_cast<int>(e);
}

}  // namespace pk
}  // namespace lmps

using namespace lmps;

extern "C" size_t lmps_decode_persistent_workspace_size(const lmps_model_desc* model, int batch,
                                                        int max_seq_len) {
  if (!model || batch <= 0 || max_seq_len <= 0) return 0;
  return pk::ws_layout(*model, batch, max_seq_len).total;
}

extern "C" int lmps_decode_persistent(const lmps_model_desc* model, const lmps_decode_state* state,
                                      int n_steps, void* stream) {
  LMPS_CHECK_ARG(model && state && n_steps >= 1);
  const lmps_model_desc& m = *model;
  const lmps_decode_state& s = *state;
  LMPS_CHECK_ARG(m.layers && m.final_norm && m.lm_packed && m.lm_scales && m.embed && m.inv_freq);
  LMPS_CHECK_ARG(m.n_layers >= 1 && m.n_kv_heads >= 1 && m.n_q_heads % m.n_kv_heads == 0);
  if (m.head_dim != pk::kHD || m.n_q_heads / m.n_kv_heads > pk::kMaxG) return LMPS_ERR_UNSUPPORTED;
  // lanes own hidden/512 groups of a row (<= 3) and G_down/16/8 groups of the
  // down projection (<= 3); see gemv_hidden / gemv_down
  if (m.hidden % 512 != 0 || m.hidden > 1536 || m.intermediate % 32 != 0 ||
      (m.intermediate / 32 + pk::kConsumerWarps - 1) / pk::kConsumerWarps > 8 * pk::kMaxJ ||
      m.n_q_heads * m.head_dim != m.hidden)
    return LMPS_ERR_UNSUPPORTED;
  // ring chunks must fit a slot
  if (static_cast<size_t>(pk::kRows1536) * (m.hidden / 2 + m.hidden / 16) > pk::kSlotBytes ||
      static_cast<size_t>(2 * pk::kPairsGU) * (m.hidden / 2 + m.hidden / 16) > pk::kSlotBytes ||
      static_cast<size_t>(pk::kRowsDown) * (m.intermediate / 2 + m.intermediate / 16) > pk::kSlotBytes)
    return LMPS_ERR_UNSUPPORTED;
  LMPS_CHECK_ARG(s.batch >= 1 && s.batch <= pk::kMaxB);
  LMPS_CHECK_ARG(s.block_table && s.rope_table && s.tokens && s.pos && s.workspace && s.error);
  LMPS_CHECK_ARG(s.page_size > 0 && (s.page_size & (s.page_size - 1)) == 0 && s.max_pages > 0 &&
                 s.max_seq_len > 0 && s.max_seq_len <= s.max_pages * s.page_size);
  // attention work-item arithmetic runs in 32 bits
  if (static_cast<long long>(s.max_seq_len) * pk::kMaxB * m.n_kv_heads >= (1LL << 31)) return LMPS_ERR_UNSUPPORTED;
  LMPS_CHECK_ARG(lmps_aligned(s.rope_table, 16));
  LMPS_CHECK_ARG(!s.forced || s.forced_stride >= s.n_forced);
  LMPS_CHECK_ARG(!s.history || (s.step_counter && s.history_rows > 0));
  const pk::WsLayout w = pk::ws_layout(m, s.batch, s.max_seq_len);
  if (s.workspace_bytes < w.total) return LMPS_ERR_WORKSPACE;
  LMPS_CHECK_ARG(lmps_aligned(s.workspace, 256) && lmps_aligned(m.lm_packed, 16));
  pk::Params P{};
  P.m = m;
  P.s = s;
  P.n_steps = n_steps;
  char* ws = reinterpret_cast<char*>(s.workspace);
  P.xt = reinterpret_cast<unsigned long long*>(ws + w.xt);
  P.x1t = reinterpret_cast<unsigned long long*>(ws + w.x1t);
  P.qkvt = reinterpret_cast<unsigned long long*>(ws + w.qkvt);
  P.attnt = reinterpret_cast<unsigned long long*>(ws + w.attnt);
  P.at = reinterpret_cast<unsigned long long*>(ws + w.at);
  P.kslot = reinterpret_cast<unsigned long long*>(ws + w.kslot);
  P.part_o = reinterpret_cast<float*>(ws + w.part_o);
  P.part_ml = reinterpret_cast<float2*>(ws + w.part_ml);
  P.att_cnt = reinterpret_cast<uint32_t*>(ws + w.att_cnt);
  P.epoch = reinterpret_cast<uint32_t*>(ws + w.epoch);
  P.max_splits = w.max_splits;
  // batches of 2-4: the GEMV stages on the tensor cores (16-row tiles)
  if (s.batch > 1 && pk::down_kparts(m.intermediate / 32) == 0) return LMPS_ERR_UNSUPPORTED;
  cudaStream_t st = lmps_stream(stream);
  switch (s.batch) {
    case 1: return pk::launch<1>(P, m, st);
    case 2: return pk::launch<2>(P, m, st);
    default: return pk::launch<4>(P, m, st);
  }
}
