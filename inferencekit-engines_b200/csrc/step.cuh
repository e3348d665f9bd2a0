// Persistent decode step: the whole batch-1 token (36 layers + lm_head + argmax + bookkeeping) in ONE launch.
//
// Why: at B200 bandwidth a layer's 193 MB of FP8 weights stream in ~30 us, while every kernel boundary costs
// several us (CTA turnover, the PDL wait, the activation prologue) during which DRAM idles. Here no boundary
// exists: every SM runs one CTA for the whole step and its weight stream never stops.
//
// Structure (grid = one CTA per SM, cooperative launch so all CTAs are resident):
//  * warp 8 (producer): lane 0 walks the CTA's static schedule of loads for the entire step and issues them
//    as bulk async copies into a 5 x 32 KiB shared-memory ring (full/empty mbarriers): for each layer its
//    slice range of W_qkv, the K and V chunks of its attention items (one stage per item), then its ranges of
//    W_o, W_gu, W_down; finally its range of the lm_head. Loads depend only on weights and on KV rows of earlier tokens, so the
//    producer runs ahead across phase boundaries and keeps DRAM busy while the consumers synchronise.
//  * warps 0-7 (consumers) execute the phases in order, separated by grid barriers (monotonic counter, bounded
//    spin): QKV, ATTN, MERGE, O, GU, DOWN per layer, then HEAD. A GEMV phase gives each CTA a contiguous range
//    of 2 KiB slices (16 rows x 128 k); each warp takes two slices per stage without waiting for the others and
//    stores their block dots in shared memory; once every warp has released a 16-row unit's last stage, one
//    warp folds the unit in K order (a unit split with the next CTA gets that CTA's dots through global
//    scratch; the CTA holding a unit's first K block always folds it). The attention
//    phase gives each CTA a range of (kv head, 64-key split) items and writes split partials; the merge phase
//    has 64 CTAs combine them (two per query head).
//  * The arithmetic is the per-op kernels' (csrc/gemv.cuh, csrc/attention.cuh), operation for operation, so
//    the step's outputs, logits and KV rows are bit-identical to the per-op path (and so to the reference).
// All data written by one CTA and read by another in a later phase is read with ld.global.cg (L2), never
// through L1, because L1 is not coherent across SMs.
#pragma once
#include <cuda.h>   // CUtensorMap
#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"

namespace qk {

constexpr int ST_WARPS = 8;                        // consumer warps (warpgroups 0 and 1)
constexpr int ST_THREADS = (ST_WARPS + 4) * 32;    // + a producer warpgroup: one warp loads, three fetch split units
// Register split (setmaxnreg): the CTA launches with 168 registers a thread (65,536 / 384, rounded down to 8),
// 384 x 168 = 64,512 in all. The producer warpgroup gives its share back down to ST_PRODUCER_REGS and the two
// consumer warpgroups grow to ST_CONSUMER_REGS: 128 x 56 + 256 x 216 = 62,464 <= 64,512, so the increase
// never waits on registers that no one returns.
constexpr int ST_PRODUCER_REGS = 56;
constexpr int ST_CONSUMER_REGS = 216;
static_assert(4 * 32 * ST_PRODUCER_REGS + ST_WARPS * 32 * ST_CONSUMER_REGS <= ST_THREADS * 168,
              "register split exceeds the launch's registers");
constexpr int ST_STAGE = 32768;
constexpr int ST_SLICE = 2048;                     // 16 rows x 128 k of fp8
constexpr int ST_SLICES = ST_STAGE / ST_SLICE;     // 16 slices per stage
constexpr int ST_SPW = ST_SLICES / ST_WARPS;       // 2 slices per consumer warp per stage (attention: stage share)
#ifndef ST_QUAD
#define ST_QUAD 4                                  // GEMV slices a consumer warp takes at a time
#endif
#ifndef ST_NSTAGE_N
#define ST_NSTAGE_N 5                              // ring stages (a tuning knob: the weight stream's depth per SM)
#endif
constexpr int ST_NSTAGE = ST_NSTAGE_N;
constexpr int ST_MAX_K = 12288;
constexpr int ST_CHUNK = 64;                       // attention keys per item
constexpr int ST_MAX_SPLITS = 1024;                // contexts up to 64k
// Block-dot slots: a slot holds one open unit's KB x 16*NG block dots (2-6 KiB); 24 KiB gives 12, 6 or 4 slots,
// enough for the units that can be open at once (see the bound in gemv_phase).
constexpr int ST_BD_FLOATS = 6144;
constexpr int ST_MERGE_ROUND = 128;                // splits staged per round of the attention merge
constexpr int ST_TAIL_FLOATS = 96 * 16;            // StepSmem::tail: the remote block dots of a split unit
constexpr int ST_FETCH_WARPS = 3;                  // warps 9-11 copy split units' remote block dots
constexpr int ST_ABATCH = ST_NSTAGE < 4 ? ST_NSTAGE : 4;   // attention items processed together (<= ST_NSTAGE)

struct StepLayer {
  const uint8_t *w_qkv, *w_o, *w_gu, *w_down;      // model.pack_fp8 layout
  const float *s_qkv, *s_o, *s_gu, *s_down;        // scales (layout per the kernel's SCALE)
  const bf16 *ln1, *ln2, *q_norm, *k_norm;
};

// K/V cache chunks reach shared memory through these TMA maps ({128 dims, max_seq, 8 kv heads, layers}, box
// {64, 64, 1, 1}, 128-byte swizzle): a 64-key chunk is two 8 KiB boxes (dims 0-63, 64-127) of 64 rows x 128 B,
// 16-byte chunk c of row r stored at chunk c ^ (r & 7), so eight keys read at the same dims hit eight
// different bank groups.
__device__ __forceinline__ uint32_t kv_swz(int r, int d) {   // byte offset of (row r, dim d) in a chunk
  return (uint32_t)((d >> 6) * 8192 + r * 128 + ((((d & 63) >> 3) ^ (r & 7)) << 4) + (d & 7) * 2);
}

// Tensor parallelism: each rank owns one TpArea in memory its peers map (CUDA IPC) and write over NVLink.
constexpr int ST_MAX_TP = 8;
// A partial row travels as one 64-bit word: the fp32 value in the low half and the exchange's tag (its
// sequence number since the areas were created, never 0) in the high half. An aligned 64-bit store is seen
// whole or not at all, so a reader that sees the expected tag has the value: no fence, no counter.
struct TpArea {
  unsigned long long recv[2][ST_MAX_TP][HIDDEN];   // exchange k: [k % 2][source rank][row]
  unsigned long long key_ctr;                      // argmax keys received (1 per rank per launch)
  unsigned long long keys[ST_MAX_TP];              // argmax key of each rank
  unsigned long long epoch;                        // launches completed by this rank (written by itself)
};

struct StepParams {
  CUtensorMap tm_k, tm_v;                          // see kv_swz
  bf16 *k_cache, *v_cache;                         // layer l: + l * kv_layer_elems, [8][max_seq][128]
  long long kv_layer_elems;
  const StepLayer* layers;                         // device array [n_layers]
  int n_layers;
  const bf16* embed;                               // [vocab][4096]
  const bf16* final_norm;                          // [4096]
  const uint8_t* w_head;                           // packed fp8 [vocab x 4096], or bf16 row-major [vocab][4096]
  const float* s_head;                             // [vocab] per-channel (fp8 head only)
  int vocab;
  const bf16 *cos_tab, *sin_tab;                   // [max_seq][128]
  int* token;                                      // [1]
  int* state;                                      // [pos, step]
  int* out_tokens;
  int out_len;
  unsigned long long* best;                        // [1], zero between launches
  bf16 *resid, *qkv, *attn, *h, *logits;           // activations [4096], [6144], [4096], [12288], [vocab]
  float* part;                                     // tagged block dots of split units: u64 [max N*K/128], zeroed once
  int* counters;                                   // [max N/16], zero between launches
  float *o_part, *ml_part;                         // attention partials [32][max_splits][128], [32][max_splits][2]
  int* attn_counters;                              // [8], zero between launches
  unsigned* sync;                                  // [4]: grid barrier counter, end counter (zero between
                                                   // launches), launches completed (never reset), unused
  int max_seq, max_splits;
  float eps, attn_scale;
  unsigned long long* tl;                          // optional timeline [CTA][phase][8], null when off
  // tensor parallelism (tp > 1; shapes per rank: see decode_step_kernel)
  int tp, tp_rank, vocab_offset;                   // this rank's lm_head rows start at global id vocab_offset
  bf16* resid_alt;                                 // second residual buffer: exchange k reads resid[k % 2]
  TpArea* const* areas;                            // device array [tp]: every rank's area ([tp_rank] = own)
};

// Phase p of a step: layer l's qkv, attn, o, gu, down are 5l + 0..4; the lm_head is 5 * n_layers.
// Timeline words per (CTA, phase): 0 consumers start (after the barrier), 1 prologue done, 2 work done
// (before the next barrier), 3 producer issues the phase's first load.
// Words 4-6 are cumulative clock64 cycles up to the end of the phase: 4 consumer warp 0 waiting for stages,
// 5 consumer warp 0 folding units, 6 producer waiting for free stages (cumulative at the phase's first load).
// Word 7: warp 0 leaves a GEMV phase's stage loop (before its last folds); the attention partials are done.
// Word 8: cumulative clock64 cycles consumer warp 0 spent waiting for the slowest warp to release a stage it
// must fold. Words 9-15: GEMV phases: consumer warps 1-7 leave the stage loop (%globaltimer). Words 16-18 (GEMV
// phases, consumer warp 0): cycles computing its slice pairs, cycles taking pairs and counting them, pairs taken.
// GEMV phases with a split unit: 19 the tail fetcher starts copying its remote block dots, 20 the copy is done,
// 21 the folding warp starts waiting for the copy, 22 it has it; 23 the prologue's input is in shared memory (and,
// for an RMSNorm, its scale known). Attention phase, thread 0, last batch of items: 9 its K/V stages have landed, 10 q/k/v setup done, 11 scores
// done, 12 softmax done; merge: 13 merge entered, 14 the KV head's counter complete, 15 split weights ready.
constexpr int ST_TL_WORDS = 32;
__device__ __forceinline__ void step_put(const StepParams& p, int phase, int i, unsigned long long v) {
  if (p.tl) p.tl[((size_t)blockIdx.x * (5 * p.n_layers + 1) + phase) * ST_TL_WORDS + i] = v;
}
__device__ __forceinline__ void step_stamp(const StepParams& p, int phase, int i) {
  if (p.tl) step_put(p, phase, i, globaltimer());
}
__device__ __forceinline__ unsigned long long* step_word(const StepParams& p, int phase, int i) {
  return p.tl ? p.tl + ((size_t)blockIdx.x * (5 * p.n_layers + 1) + phase) * ST_TL_WORDS + i : nullptr;
}

// A GEMV phase kind's per-CTA constants (slice range, stages, units, split unit), the same for every layer:
// computed once per launch (their integer divisions off the phases' critical path).
struct GemvPlan {
  int s0, s1;           // the CTA's slices
  int nst;              // ring stages of the phase
  int u_lo, u_hi;       // its first and last unit
  int nslots;           // block-dot slots of the shape
  int tu_u, tu_hi, tu_need, tu_any;   // the split last unit (TailUnit)
};
constexpr int ST_PLANS = 5;                        // qkv, o_proj, gate_up, down, lm_head

struct StepSmem {
  uint8_t ring[ST_NSTAGE][ST_STAGE];
  uint32_t xh[ST_MAX_K / 2];                       // x as f16 MMA fragments (see gemv_prologue)
  float xscale[ST_MAX_K / QB];
  union {
    float bd[ST_BD_FLOATS];                        // block dots of the 16-row units in flight (slots)
    bf16 xs[ST_MAX_K];                             // x during a prologue
    struct {
      float qs[ST_ABATCH][GQA][HEAD_DIM + 4];      // q per kv head of the batch; +4: 4 heads read conflict-free
      float sc[ST_ABATCH][GQA][ST_CHUNK];          // scores, then probabilities, per item and query head
      float m_s[ST_ABATCH][GQA], l_s[ST_ABATCH][GQA];
    } at;
    struct {
      float o[ST_MERGE_ROUND * 32];                // partial outputs of up to ST_MERGE_ROUND splits, 32 dims each
      float w[ST_MAX_SPLITS];                      // m_s, then exp(m_s - M), per split
      float l[ST_MAX_SPLITS];                      // l_s per split
      float cl;                                    // sum_s exp(m_s - M) * l_s
    } mg;
  } u;
  // Block dots of the last unit of a GEMV phase when it continues in the next CTA: the tail-fetcher warp copies
  // them (tagged words in `part`) into tail[n % 2] as soon as that CTA has published them (a unit has KB * NG
  // <= 96 slices of 16 dots; at most all but one come from the next CTA). tail_full[b]: the copy landed (the
  // fetcher's 32 lanes arrive); tail_empty[b]: the folding warp has used it.
  __align__(16) float tail[2][ST_TAIL_FLOATS];
  uint64_t tail_full[2], tail_empty[2];
  int grab;                                        // GEMV phase: slice pairs handed out so far
  int done[ST_BD_FLOATS / (4 * 16)];               // GEMV phase: finished slices per block-dot slot (K/128 >= 4)
  float red[8];
  unsigned long long bestbuf[ST_WARPS];
  uint64_t full[ST_NSTAGE], empty[ST_NSTAGE];
  int flag;
  GemvPlan plan[ST_PLANS];
};

static_assert(sizeof(StepSmem) <= 227 * 1024, "the fused step's shared memory exceeds a CTA's 227 KB");

// ---- small helpers -------------------------------------------------------------------------------------------
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(ST_WARPS * 32) : "memory"); }
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void red_add_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait until *p >= target (a counter other GPUs add to); sets DEVERR_GRID_TIMEOUT on timeout.
__device__ __forceinline__ void wait_sys_counter(const unsigned long long* p, unsigned long long target,
                                                 unsigned long long limit_ns = WAIT_LIMIT_NS) {
  const long long c0 = clock64();
  while (ld_acquire_sys_u64(p) < target && clock64() - c0 < 500000) {
  }
  if (ld_acquire_sys_u64(p) >= target) return;
  const unsigned long long t0 = globaltimer();
  while (ld_acquire_sys_u64(p) < target) {
    if (wait_failed()) return;
    if (globaltimer() - t0 > limit_ns) {
      atomicOr(&g_dev_error, DEVERR_GRID_TIMEOUT);
      return;
    }
  }
}
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Tag of the block dots a GEMV phase shares between CTAs: unique per (launch, phase) over 2^32 - 1 phases and
// never 0, so a zeroed `part` or an earlier phase's words never pass for this phase's.
__device__ __forceinline__ unsigned dots_tag(unsigned epoch, int n_layers, int phase) {
  const unsigned long long k = (unsigned long long)epoch * (unsigned)(5 * n_layers + 1) + (unsigned)phase;
  return 1u + (unsigned)(k % 0xFFFFFFFFull);
}
__device__ __forceinline__ void red_add_relaxed(int* p, int v) {
  asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bf16 ldcg_bf16(const bf16* p) {
  unsigned short v;
  asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return __ushort_as_bfloat16(v);
}
__device__ __forceinline__ uint2 ldcg_u2(const void* p) {
  uint2 r;
  asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
// 16-byte global -> shared copy through L2 only (data written by another SM), no registers involved
__device__ __forceinline__ void cp_async16_cg(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ uint4 ldcg_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// Consumer-side grid barrier number `idx` (0-based) of this launch. Bounded: on timeout it records the error and
// lets the CTA continue (wrong results, but no hang).
__device__ __forceinline__ void grid_barrier(unsigned* ctr, unsigned idx, unsigned long long* tl_word = nullptr) {
  consumer_sync();   // orders the CTA's writes before thread 0's release below
  if (threadIdx.x == 0) {
    if (tl_word) *tl_word = globaltimer();   // every consumer warp of the CTA has finished the phase
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
    const unsigned target = (idx + 1) * gridDim.x;
    const long long c0 = clock64();
    while (ld_acquire_u32(ctr) < target && clock64() - c0 < 500000) {
    }
    if (ld_acquire_u32(ctr) < target) {
      const unsigned long long t0 = globaltimer();
      while (ld_acquire_u32(ctr) < target) {
        if (wait_failed()) break;
        if (globaltimer() - t0 > WAIT_LIMIT_NS) {
          atomicOr(&g_dev_error, DEVERR_GRID_TIMEOUT);
          break;
        }
      }
    }
  }
  consumer_sync();   // the other threads read what the acquire made visible
}

// A GEMV phase's share for this CTA: a contiguous range of 2 KiB slices. Slice q of a matrix with NG
// sub-matrices is tile q/NG (unit (q/NG)/KB, block (q/NG)%KB) and sub-matrix q%NG (gate/up).
struct SliceRange {
  int s0, s1;
};
__device__ __forceinline__ SliceRange slice_range(int n_slices) {
  const long long G = gridDim.x, c = blockIdx.x;
  return SliceRange{(int)(c * n_slices / G), (int)((c + 1) * n_slices / G)};
}

struct AttnItems {
  int i0, i1, n_splits;
};
__device__ __forceinline__ AttnItems attn_items(int pos, int n_kv) {
  const int n_splits = (pos + 1 + ST_CHUNK - 1) / ST_CHUNK;
  const long long n = (long long)n_kv * n_splits, G = gridDim.x, c = blockIdx.x;
  return AttnItems{(int)(c * n / G), (int)((c + 1) * n / G), n_splits};
}

// ---- producer --------------------------------------------------------------------------------------------------
struct Producer {
  StepSmem* sm;
  int n;          // stages issued so far
  uint64_t pol;
  bool ok;
  long long wait_cycles;
  __device__ __forceinline__ void push(const void* src, uint32_t bytes) {
    if (!ok) return;
    const int s = n % ST_NSTAGE;
    const long long t0 = clock64();
    if (n >= ST_NSTAGE && !mbar_wait(&sm->empty[s], (uint32_t)(((n / ST_NSTAGE) - 1) & 1))) {
      ok = false;
      return;
    }
    wait_cycles += clock64() - t0;
    mbar_arrive_expect_tx(&sm->full[s], bytes);
    bulk_g2s(sm->ring[s], src, bytes, &sm->full[s], pol);
    ++n;
  }
  // K and V chunk (keys j0..j0+63 of kv head kvh, layer l) of one attention item into one stage: K in the first
  // half, V in the second, each as two swizzled 8 KiB boxes (rows past the cache end are zero-filled)
  __device__ __forceinline__ void push_kv(const StepParams& p, int l, int kvh, int j0) {
    if (!ok) return;
    const int s = n % ST_NSTAGE;
    const long long t0 = clock64();
    if (n >= ST_NSTAGE && !mbar_wait(&sm->empty[s], (uint32_t)(((n / ST_NSTAGE) - 1) & 1))) {
      ok = false;
      return;
    }
    wait_cycles += clock64() - t0;
    mbar_arrive_expect_tx(&sm->full[s], ST_STAGE);
    tma_load_4d(sm->ring[s], &p.tm_k, 0, j0, kvh, l, &sm->full[s]);
    tma_load_4d(sm->ring[s] + 8192, &p.tm_k, 64, j0, kvh, l, &sm->full[s]);
    tma_load_4d(sm->ring[s] + 16384, &p.tm_v, 0, j0, kvh, l, &sm->full[s]);
    tma_load_4d(sm->ring[s] + 24576, &p.tm_v, 64, j0, kvh, l, &sm->full[s]);
    ++n;
  }
  __device__ __forceinline__ void gemv(const uint8_t* w, int n_slices) {
    const SliceRange r = slice_range(n_slices);
    for (int q = r.s0; q < r.s1; q += ST_SLICES)
      push(w + (size_t)q * ST_SLICE, (uint32_t)(min(ST_SLICES, r.s1 - q) * ST_SLICE));
  }
};

// ---- consumer: GEMV phase ---------------------------------------------------------------------------------------
// ONE code path serves every GEMV phase of the step (qkv, o_proj, gate_up, down, lm_head): the matrix shape, the
// sub-matrix count, the scale layout and the epilogue are run-time fields of GemvPhase, and the step calls
// gemv_phase from a single site. A layer then executes one copy of the stage loop and of the fold instead of
// four specialised ones (~25-30 KB of code each), which keeps a layer's code inside the SM's instruction cache.
constexpr int EPI_TP_PARTIAL = 10;   // fp32 row partial into every rank's TpArea (row-parallel shard)

struct GemvPhase {
  const float* ws;    // weight scales: [N] per channel, or [N/128][KB] per 128x128 block
  int N, K;           // N = all rows (gate + up for NG = 2)
  int KB, NG;         // K / 128; sub-matrices per unit (1, or 2 = gate|up)
  int epi;            // EPI_STORE | EPI_RESIDUAL | EPI_SWIGLU | EPI_ARGMAX | EPI_TP_PARTIAL
  int scale_block;    // 1: block-128 scales, 0: per channel
  bf16* out;          // STORE: qkv; RESIDUAL: resid; SWIGLU: h; ARGMAX: logits
  float* part;
  int row_offset;     // ARGMAX: global id of row 0 (vocabulary shard)
  int xbuf;           // TP_PARTIAL: exchange buffer (k % 2)
  unsigned xtag;      // TP_PARTIAL: the exchange's tag
  unsigned dtag;      // tag of this phase's shared block dots (set by gemv_phase)
  int nslots;         // block-dot slots of this shape (set by gemv_phase)
};

// Block-dot slots: unit u uses slot u % nslots, next reused by unit u + nslots, whose first slice lies
// (nslots - 1) * spu slices past u's last. No warp works more than ST_NSTAGE stages past the oldest stage not yet
// released, and u's owner folds it at the latest after its next slice group once u is complete, so no writer of
// u + nslots can come first when this holds (checked for every shape the step runs, TP 1..8):
__host__ __device__ constexpr bool gemv_slots_ok(int KB, int NG) {
  return (ST_BD_FLOATS / (KB * 16 * NG) - 1) * KB * NG > (2 * ST_NSTAGE + 2) * ST_SLICES;
}
static_assert(gemv_slots_ok(32, 1) && gemv_slots_ok(32, 2) && gemv_slots_ok(96, 1) && gemv_slots_ok(16, 1) &&
                  gemv_slots_ok(48, 1) && gemv_slots_ok(8, 1) && gemv_slots_ok(24, 1) && gemv_slots_ok(4, 1) &&
                  gemv_slots_ok(12, 1),
              "too few block-dot slots");
static_assert(96 * 16 <= ST_TAIL_FLOATS, "a split unit's remote block dots must fit a tail buffer");
static_assert(ST_BD_FLOATS / (4 * 16) == sizeof(StepSmem::done) / sizeof(int), "a done counter per block-dot slot");

struct Consumer {
  StepSmem* sm;
  const StepParams* p;
  int n;              // stages consumed so far
  int lane, warp, g, t;
  float best_v;
  int best_i;
  long long wait_cycles, fold_cycles;
  int tl_phase = 0;   // timeline phase index of the phase being run
  long long relwait_cycles = 0;   // waiting for the slowest warp to release a stage this warp folds
  unsigned epoch = 0;             // launches completed before this one (the block-dot tags)
  unsigned long long tag_base = 0;   // tag_base(epoch, n_layers)
  int tail_n = 0;     // GEMV phases so far with a split unit folded here (the tail buffers' use count)

  __device__ __forceinline__ bool wait_stage(int s) { return wait_abs(n); }
  // wait for the load of the consumer's stage number `m` (counted over the whole launch)
  __device__ __forceinline__ bool wait_abs(int m) {
    const long long t0 = clock64();
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&sm->full[m % ST_NSTAGE], (uint32_t)((m / ST_NSTAGE) & 1)));
    wait_cycles += clock64() - t0;
    return ok;
  }
  __device__ __forceinline__ bool released_wait(int m) {
    const long long t0 = clock64();
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&sm->empty[m % ST_NSTAGE], (uint32_t)((m / ST_NSTAGE) & 1)));
    relwait_cycles += clock64() - t0;
    return ok;
  }
  __device__ __forceinline__ void release_stage(int s) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm->empty[s]);
  }
};

// Block-128 weight scale of `row` at K block `kb`.
__device__ __forceinline__ float block_row_scale(const float* ws, int row, int kb, int KB) {
  return __ldg(ws + (size_t)(row / QB) * KB + kb);
}

// Per-row inputs of a unit's epilogue that do not depend on this phase's block dots (the channel scale and,
// for a residual epilogue, the residual value). The owner loads them for its next unit long before the fold.
struct FoldPre {
  float sw, resid;
};
__device__ __forceinline__ FoldPre fold_prefetch(const Consumer& c, const GemvPhase& ph, int u, bool valid) {
  const int row = (ph.NG == 2 ? (c.lane >> 4) * (ph.N / 2) : 0) + u * 16 + (c.lane & 15);
  const bool active = valid && (ph.NG == 2 || c.lane < 16);
  FoldPre f;
  f.sw = (!ph.scale_block && active) ? __ldg(ph.ws + row) : 0.f;
  f.resid = (ph.epi == EPI_RESIDUAL && active) ? __bfloat162float(ldcg_bf16(ph.out + row)) : 0.f;
  return f;
}

// Copy n tagged block dots (u64 words: the fp32 value in the low half, the phase's tag in the high half) from
// `src` into `dst` (shared memory), each once it carries `tag`: a warp loads 128 words at a time and reloads only
// those not yet written. Bounded; returns false (error word set) on a timeout.
__device__ __forceinline__ bool copy_tagged_dots(const unsigned long long* src, float* dst, int n, unsigned tag, int lane,
                                                 int part = 0, int parts = 1) {
  const unsigned long long t0 = globaltimer();
  for (int b0 = 128 * part; b0 < n; b0 += 128 * parts) {   // this warp's passes of 128 words
    unsigned long long w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = b0 + 32 * k + lane;
      w[k] = i < n ? ld_relaxed_gpu_u64(src + i) : ((unsigned long long)tag << 32);
    }
    while (true) {
      bool all = true;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = b0 + 32 * k + lane;
        if ((unsigned)(w[k] >> 32) != tag) {
          all = false;
          w[k] = ld_relaxed_gpu_u64(src + i);
        }
      }
      if (__all_sync(0xffffffffu, all)) break;
      if (wait_failed()) return false;
      if (globaltimer() - t0 > WAIT_LIMIT_NS) {
        if (lane == 0) atomicOr(&g_dev_error, DEVERR_GRID_TIMEOUT);
        return false;
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = b0 + 32 * k + lane;
      if (i < n) dst[i] = __uint_as_float((unsigned)w[k]);
    }
  }
  return true;
}

// The split unit of a GEMV phase that this CTA folds: its last unit u when it ends past this CTA's range and
// starts inside it. `need` slices of it come from the following CTA(s), which publish them early in the phase.
struct TailUnit {
  int u, hi, need;
  bool any;
};
__device__ __forceinline__ TailUnit tail_unit(int N, int KB, int NG) {
  const int spu = KB * NG;
  const SliceRange r = slice_range(N / (16 * NG) * spu);
  const int u_lo = r.s0 / spu, u_hi = r.s1 > r.s0 ? (r.s1 - 1) / spu : u_lo - 1;
  TailUnit t{u_hi, r.s1, (u_hi + 1) * spu - r.s1, false};
  t.any = u_hi >= u_lo && t.need > 0 && u_hi * spu >= r.s0;
  return t;
}

__device__ __forceinline__ GemvPlan make_plan(int N, int KB, int NG) {
  const int spu = KB * NG;
  const SliceRange r = slice_range(N / (16 * NG) * spu);
  const TailUnit tu = tail_unit(N, KB, NG);
  GemvPlan g;
  g.s0 = r.s0;
  g.s1 = r.s1;
  g.nst = (r.s1 - r.s0 + ST_SLICES - 1) / ST_SLICES;
  g.u_lo = r.s0 / spu;
  g.u_hi = r.s1 > r.s0 ? (r.s1 - 1) / spu : g.u_lo - 1;
  g.nslots = ST_BD_FLOATS / (KB * 16 * NG);
  g.tu_u = tu.u;
  g.tu_hi = tu.hi;
  g.tu_need = tu.need;
  g.tu_any = tu.any;
  return g;
}
// Tag of launch `epoch`'s phase `phase` (dots_tag), from base = dots_tag's k for phase 0 modulo 2^32 - 1.
__device__ __forceinline__ unsigned phase_tag(unsigned long long base, int phase) {
  unsigned long long k = base + (unsigned)phase;
  if (k >= 0xFFFFFFFFull) k -= 0xFFFFFFFFull;
  return 1u + (unsigned)k;
}
__device__ __forceinline__ unsigned long long tag_base(unsigned epoch, int n_layers) {
  return ((unsigned long long)epoch * (unsigned)(5 * n_layers + 1)) % 0xFFFFFFFFull;
}

// Tail-fetcher warp, one GEMV phase (timeline phase index `phase`; n counts the phases with a split unit,
// identically on the consumer side): copy the following CTA's share of the split unit, tagged words published
// early in that CTA's phase, into tail[n % 2] and signal tail_full[n % 2] (one arrival per lane). It first
// waits until the folding warp has used the buffer two phases back. Every wait is bounded; on a timeout the
// error word is set and the fetch is skipped (the folding warp's own bounded wait then gives up).
__device__ __forceinline__ void tail_fetch(StepSmem& sm, const StepParams& p, const GemvPlan& pl, int KB, int NG,
                                           int phase, unsigned tag, int& n, int lane, int part) {
  const int spu = KB * NG, RPU = 16 * NG;
  const TailUnit tu{pl.tu_u, pl.tu_hi, pl.tu_need, pl.tu_any != 0};
  if (!tu.any) return;
  const int b = n & 1, use = n >> 1;
  ++n;
  if (use >= 1 && !__all_sync(0xffffffffu, mbar_wait(&sm.tail_empty[b], (uint32_t)((use - 1) & 1)))) return;
  const unsigned long long* src =
      reinterpret_cast<const unsigned long long*>(p.part) + (size_t)tu.u * KB * RPU + (tu.hi - tu.u * spu) * 16;
  if (lane == 0 && part == 0) step_stamp(p, phase, 19);
  const bool ok = copy_tagged_dots(src, sm.tail[b], tu.need * 16, tag, lane, part, ST_FETCH_WARPS);
  if (lane == 0 && part == 0) step_stamp(p, phase, 20);
  if (ok) mbar_arrive(&sm.tail_full[b]);
}

// In-order sum over a unit's K blocks, acc += d * s_x * s_w, reading FB block dots at a time (independent loads).
template <int FB>
__device__ __forceinline__ float fold_dots(const float* s, int RPU, int KB, const float* xscale, const float* ws,
                                           int scale_block, int row, float sw_ch) {
  float a = 0.f;
  for (int k0 = 0; k0 < KB; k0 += FB) {
    float d[FB], sw[FB];
#pragma unroll
    for (int j = 0; j < FB; ++j) {
      d[j] = s[(k0 + j) * RPU];
      sw[j] = scale_block ? block_row_scale(ws, row, k0 + j, KB) : sw_ch;
    }
#pragma unroll
    for (int j = 0; j < FB; ++j) a += d[j] * xscale[k0 + j] * sw[j];
  }
  return a;
}

// Fold of one 16-row unit (32 rows for gate|up) once this CTA's block dots of it are complete: the per-op
// kernel's in-order sum acc += d * sx * sw over K blocks, then the epilogue. Gate rows fold on lanes 0-15 and
// up rows on lanes 16-31. A unit shared with a neighbouring CTA is folded by the CTA holding its first K block,
// with the following CTA's block dots (tagged words in `part`, copied by the tail-fetcher warp).
__device__ __forceinline__ void fold_unit(Consumer& c, const GemvPhase& ph, const SliceRange& r, int u,
                                          const FoldPre& pre, int tail_use = -1) {
  StepSmem& sm = *c.sm;
  const int KB = ph.KB, NG = ph.NG, RPU = 16 * NG, spu = KB * NG, slot_floats = KB * RPU;
  const int hi = min((u + 1) * spu, r.s1);
  if (u * spu < r.s0) return;   // started in an earlier CTA, which folds it (this CTA's dots are in `part`, tagged)
  float* slot = &sm.u.bd[(u % ph.nslots) * slot_floats];
  if (hi < (u + 1) * spu) {
    // The unit continues in the following CTA(s), whose share the tail-fetcher warp has copied into tail[use % 2]:
    // a slice is 16 consecutive floats of the unit's [KB][NG][16] layout, so that share goes behind this CTA's.
    const int off = (hi - u * spu) * 16, nf = ((u + 1) * spu - hi) * 16;
    if (tail_use >= 0) {
      const int b = tail_use & 1;
      if (c.lane == 0) step_stamp(*c.p, c.tl_phase, 21);
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.tail_full[b], (uint32_t)((tail_use >> 1) & 1)));
      if (c.lane == 0) step_stamp(*c.p, c.tl_phase, 22);
      if (ok)
        for (int i4 = c.lane; i4 < nf / 4; i4 += 32)
          reinterpret_cast<uint4*>(slot + off)[i4] = reinterpret_cast<const uint4*>(sm.tail[b])[i4];
      __syncwarp();
      if (c.lane == 0) mbar_arrive(&sm.tail_empty[b]);
    } else {   // not expected (the fetcher covers every split unit): copy the tagged words here
      const unsigned long long* src = reinterpret_cast<const unsigned long long*>(ph.part) + (size_t)u * KB * RPU + off;
      copy_tagged_dots(src, slot + off, nf, ph.dtag, c.lane);
    }
    __syncwarp();
  }
  const int rr = c.lane & 15, gi = NG == 2 ? c.lane >> 4 : 0;
  const int row = gi * (ph.N / 2) + u * 16 + rr;            // gate (or only) row; up row on lanes 16-31
  const bool active = NG == 2 || c.lane < 16;
  float a = 0.f;
  if (active) {
    const float* s = slot + gi * 16 + rr;
    if (KB % 16 == 0) a = fold_dots<16>(s, RPU, KB, sm.xscale, ph.ws, ph.scale_block, row, pre.sw);
    else if (KB % 8 == 0) a = fold_dots<8>(s, RPU, KB, sm.xscale, ph.ws, ph.scale_block, row, pre.sw);
    else a = fold_dots<4>(s, RPU, KB, sm.xscale, ph.ws, ph.scale_block, row, pre.sw);
  }
  const float resid_in = pre.resid;
  if (ph.epi == EPI_SWIGLU) {
    const float a_up = __shfl_down_sync(0xffffffffu, a, 16);
    if (c.lane < 16) {
      const float gt = bf16r(a);
      const float up = bf16r(a_up);
      const float act = bf16r(gt / (1.0f + expf(-gt)));
      ph.out[row] = __float2bfloat16_rn(act * up);
    }
  } else if (c.lane < 16) {
    if (ph.epi == EPI_STORE) {
      ph.out[row] = __float2bfloat16_rn(a);
    } else if (ph.epi == EPI_RESIDUAL) {
      ph.out[row] = __float2bfloat16_rn(resid_in + bf16r(a));
    } else if (ph.epi == EPI_TP_PARTIAL) {   // this rank's fp32 partial of the row, to every rank (NVLink stores)
      const StepParams& p = *c.p;
      const unsigned long long w = ((unsigned long long)ph.xtag << 32) | __float_as_uint(a);
      for (int r2 = 0; r2 < p.tp; ++r2) st_relaxed_sys_u64(&p.areas[r2]->recv[ph.xbuf][p.tp_rank][row], w);
    } else {  // EPI_ARGMAX
      ph.out[row] = __float2bfloat16_rn(a);
      const float lv = bf16r(a);
      const int gid = row + ph.row_offset;
      if (lv > c.best_v || (lv == c.best_v && gid < c.best_i)) { c.best_v = lv; c.best_i = gid; }
    }
  }
}

__device__ void gemv_phase(Consumer& c, GemvPhase ph, const GemvPlan& pl) {
  StepSmem& sm = *c.sm;
  ph.dtag = phase_tag(c.tag_base, c.tl_phase);
  const int KB = ph.KB, NG = ph.NG, ngs = NG - 1;   // NG is 1 or 2: slice q is tile q >> ngs, sub-matrix q & ngs
  const int RPU = 16 * NG;                          // rows per unit
  const int spu = KB * NG;                          // slices per unit
  const int slot_floats = KB * RPU;
  const int nslots = pl.nslots;
  ph.nslots = nslots;
  constexpr int NQ = ST_SLICES / ST_QUAD;         // grabs per stage
  static_assert(ST_SLICES % ST_QUAD == 0 && ST_WARPS % NQ == 0, "a stage's grabs must add up to its ST_WARPS arrivals");
  static_assert(ST_QUAD <= 4, "a group of slices spans at most two units (4 <= every K / 128)");
  const SliceRange r{pl.s0, pl.s1};
  const int nst = pl.nst;   // stages of this phase (as the producer issues)
  const int n0 = c.n;
  const uint8_t* xh = reinterpret_cast<const uint8_t*>(sm.xh);
  // Work is handed out in groups of ST_QUAD consecutive slices: grab p is slices ST_QUAD * (p % NQ) .. +ST_QUAD-1
  // of stage p / NQ, taken by whichever warp asks next (sm.grab), so a warp that is delayed (a fold, a slow wait)
  // leaves its share to the others; each grab counts ST_WARPS / NQ arrivals on the stage's `empty` barrier. A
  // finished slice adds 1 to its unit's counter (sm.done, per slot); unit u is folded by warp
  // (u - u_lo) % ST_WARPS once all its slices in this CTA are done.
  const int u_lo = pl.u_lo, u_hi = pl.u_hi;
  int fu = u_lo + c.warp;                                       // next unit this warp folds
  // slices of unit u that this CTA computes and folds (none for a unit an earlier CTA started, which folds it)
  auto local_count = [&](int u) { return u * spu < r.s0 ? 0 : min((u + 1) * spu, r.s1) - u * spu; };
  FoldPre pre = fold_prefetch(c, ph, fu, fu <= u_hi);
  const int tail_use = pl.tu_any ? c.tail_n++ : -1;
  auto fold_ready = [&](int u) { return *reinterpret_cast<volatile int*>(&sm.done[u % nslots]) >= local_count(u); };
  auto fold_next = [&]() {   // fold unit fu, move on to this warp's next unit and prefetch its row inputs
    const long long t0 = clock64();
    __threadfence_block();   // the other warps' block dots, published before their counts
    fold_unit(c, ph, r, fu, pre, fu == u_hi ? tail_use : -1);
    __syncwarp();
    if (c.lane == 0) sm.done[fu % nslots] = 0;
    fu += ST_WARPS;
    pre = fold_prefetch(c, ph, fu, fu <= u_hi);
    c.fold_cycles += clock64() - t0;
  };
  long long cyc_compute = 0, cyc_sync = 0;
  int pairs = 0;
  while (true) {
    const long long tg0 = clock64();
    int pidx = 0;
    if (c.lane == 0) pidx = atomicAdd(&sm.grab, 1);
    pidx = __shfl_sync(0xffffffffu, pidx, 0);
    if (pidx >= NQ * nst) break;
    const int i = pidx / NQ, k0 = (pidx - i * NQ) * ST_QUAD;
    const long long tg1 = clock64();
    if (!c.wait_abs(n0 + i)) atomicOr(&g_dev_error, DEVERR_MBAR_TIMEOUT);
    const long long tc0 = clock64();
    // slice coordinates (also computed for slices past the range: kb stays in [0, KB), nothing is stored): one
    // division for the group, then steps (the group's tiles are consecutive and KB >= 4 > the step)
    const int qa = r.s0 + i * ST_SLICES + k0;
    const int tla = qa >> ngs;
    const int una = tla / KB, kba = tla - una * KB;
    const int sla = una % nslots, slb = sla + 1 == nslots ? 0 : sla + 1;   // slots of units una, una + 1
    int q[ST_QUAD], un[ST_QUAD], kb[ST_QUAD];
    const uint8_t* wp[ST_QUAD];
    const uint8_t* xp[ST_QUAD];
#pragma unroll
    for (int j = 0; j < ST_QUAD; ++j) {
      q[j] = qa + j;
      const int kk = kba + ((q[j] >> ngs) - tla);
      un[j] = kk >= KB ? una + 1 : una;
      kb[j] = kk >= KB ? kk - KB : kk;
      wp[j] = sm.ring[(n0 + i) % ST_NSTAGE] + (k0 + j) * ST_SLICE + c.lane * 16;
      xp[j] = xh + kb[j] * 256 + c.t * 16;
    }
    float d0[ST_QUAD], d1[ST_QUAD];
#pragma unroll
    for (int j = 0; j < ST_QUAD; ++j) d0[j] = d1[j] = 0.f;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {   // 32-k chunk ch of the group's slices (16-byte fragments per lane)
      uint4 W[ST_QUAD], X[ST_QUAD];
#pragma unroll
      for (int j = 0; j < ST_QUAD; ++j) {
        W[j] = *reinterpret_cast<const uint4*>(wp[j] + ch * 512);
        X[j] = *reinterpret_cast<const uint4*>(xp[j] + ch * 64);
      }
#pragma unroll
      for (int j = 0; j < ST_QUAD; ++j) {
        float e[4];
        fp8_chunk_dot(W[j], X[j], e);
        d0[j] += e[0];
        d1[j] += e[2];
      }
    }
#pragma unroll
    for (int j = 0; j < ST_QUAD; ++j) {
      if (q[j] < r.s1) {
        const int gi = q[j] & ngs;                              // sub-matrix of the slice (0 for NG == 1)
        const int u = un[j];
        const bool in = u * spu >= r.s0;                        // this CTA folds u: keep its dots here
        if (c.t == 0) {
          const int off = kb[j] * RPU + gi * 16 + c.g;
          if (in) {
            float* dst = &sm.u.bd[(u == una ? sla : slb) * slot_floats + off];
            dst[0] = d0[j];
            dst[8] = d1[j];
          } else {   // the earlier CTA folds u: publish the dots tagged (no fence or counter needed)
            unsigned long long* dst = reinterpret_cast<unsigned long long*>(ph.part) + (size_t)u * KB * RPU + off;
            const unsigned long long tg = (unsigned long long)ph.dtag << 32;
            st_relaxed_gpu_u64(dst, tg | __float_as_uint(d0[j]));
            st_relaxed_gpu_u64(dst + 8, tg | __float_as_uint(d1[j]));
          }
        }
      }
    }
    const long long tc1 = clock64();
    __syncwarp();
    if (c.lane == 0) {
      __threadfence_block();   // this group's block dots before its counts
      // the group's slices by unit (consecutive slices: at most two units), one count per unit
      int na = 0, nb = 0;
#pragma unroll
      for (int j = 0; j < ST_QUAD; ++j) {
        if (q[j] < r.s1 && un[j] * spu >= r.s0) {
          if (un[j] == una) ++na;
          else ++nb;
        }
      }
      if (na) atomicAdd(&sm.done[sla], na);
      if (nb) atomicAdd(&sm.done[slb], nb);
      mbar_arrive_n(&sm.empty[(n0 + i) % ST_NSTAGE], ST_WARPS / NQ);
    }
    __syncwarp();
    cyc_compute += tc1 - tc0;
    cyc_sync += (tg1 - tg0) + (clock64() - tc1);
    ++pairs;
    while (fu <= u_hi && fold_ready(fu)) fold_next();
  }
  if (c.lane == 0 && c.p->tl) step_stamp(*c.p, c.tl_phase, c.warp == 0 ? 7 : 8 + c.warp);
  // the rest of this warp's units: wait (bounded) until the other warps have finished their slices
  while (fu <= u_hi) {
    if (!fold_ready(fu)) {
      const long long t0 = clock64();
      const unsigned long long g0 = globaltimer();
      while (!fold_ready(fu)) {
        if (wait_failed()) break;
        if (globaltimer() - g0 > WAIT_LIMIT_NS) {
          if (c.lane == 0) atomicOr(&g_dev_error, DEVERR_MBAR_TIMEOUT);
          break;
        }
      }
      c.relwait_cycles += clock64() - t0;
    }
    fold_next();
  }
  c.n = n0 + nst;
  if (threadIdx.x == 0) {
    step_put(*c.p, c.tl_phase, 8, c.relwait_cycles);
    step_put(*c.p, c.tl_phase, 16, cyc_compute);
    step_put(*c.p, c.tl_phase, 17, cyc_sync);
    step_put(*c.p, c.tl_phase, 18, pairs);
  }
}

// ---- consumer: activation quantization of the staged x (sm.u.xs) -------------------------------------------
// B groups gq = warp + 8 i per batch, every chain independent: loads (+ the RMSNorm scale when `norm`: K == 4096,
// one batch, nraw[i] is group gq's weights), the group maxima reduced together by one butterfly, then the e4m3
// quantization into f16 MMA fragments (sm.xh) and the scales (sm.xscale). Groups past KB are zero and not stored.
template <int B>
__device__ __forceinline__ void prologue_quant(Consumer& c, int KB, bool norm, const uint2 (&nraw)[4], float rstd) {
  StepSmem& sm = *c.sm;
  const int lane = c.lane, warp = c.warp;
  const int ch = lane >> 3, hi = (lane >> 2) & 1, t = lane & 3;
  for (int g0 = warp; g0 < KB; g0 += B * ST_WARPS) {
    float v[B][4], amax[B];
#pragma unroll
    for (int i = 0; i < B; ++i) {
      const int gq = g0 + i * ST_WARPS;
      const uint2 raw = gq < KB ? *reinterpret_cast<const uint2*>(sm.u.xs + gq * QB + lane * 4) : make_uint2(0, 0);
      v[i][0] = bf16lo(raw.x);
      v[i][1] = bf16hi(raw.x);
      v[i][2] = bf16lo(raw.y);
      v[i][3] = bf16hi(raw.y);
      if (B == 4 && norm) {
        const float w[4] = {bf16lo(nraw[i & 3].x), bf16hi(nraw[i & 3].x), bf16lo(nraw[i & 3].y), bf16hi(nraw[i & 3].y)};
#pragma unroll
        for (int j = 0; j < 4; ++j) v[i][j] = bf16r(w[j] * bf16r(v[i][j] * rstd));
      }
      amax[i] = fmaxf(fmaxf(fabsf(v[i][0]), fabsf(v[i][1])), fmaxf(fabsf(v[i][2]), fabsf(v[i][3])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int i = 0; i < B; ++i) amax[i] = fmaxf(amax[i], __shfl_xor_sync(0xffffffffu, amax[i], o));
    }
#pragma unroll
    for (int i = 0; i < B; ++i) {
      const int gq = g0 + i * ST_WARPS;
      if (gq < KB) {
        const float sc = div_full(amax[i], 448.0f);
        const uint32_t qv = quant4(v[i][0], v[i][1], v[i][2], v[i][3], sc);
        uint32_t* dst = sm.xh + ((gq * 4 + ch) * 4 + t) * 4;
        dst[hi] = e4m3x2_to_f16x2(qv);
        dst[2 + hi] = e4m3x2_to_f16x2(qv >> 16);
        if (lane == 0) sm.xscale[gq] = sc;
      }
    }
  }
}

// ---- consumer: activation prologue ---------------------------------------------------------------------------
// x (global, K values) -> RMSNorm when norm_w is given (K == 4096; the reference's 128-thread reduction order) ->
// e4m3 per 128-group -> f16 fragments in sm.xh + scales in sm.xscale. x is read through L2 (other CTAs wrote it),
// every load in flight at once, and staged in shared memory: by the whole CTA for an RMSNorm (every thread needs
// the sum of squares), else by each warp for its own groups, so that only the warp waits. `resid_slice_dst`
// (layer 0): x is the token's embedding row and this CTA also writes its slice of it into the residual stream.
__device__ void step_prologue(Consumer& c, const bf16* x, const bf16* norm_w, int K, float eps, bf16* resid_slice_dst) {
  StepSmem& sm = *c.sm;
  const int tid = threadIdx.x, lane = c.lane, warp = c.warp;
  const int KB = K / QB;
  constexpr int NT = ST_WARPS * 32;
  if (tid == 0) sm.grab = 0;   // every warp left the previous GEMV phase (a grid barrier lies between)
  uint4* xs4 = reinterpret_cast<uint4*>(sm.u.xs);
  const uint4* x4 = reinterpret_cast<const uint4*>(x);
  float rstd = 0.f;
  uint2 nraw[4];   // RMSNorm: the norm weights of this lane's 4 values in each of the warp's 4 groups
  if (norm_w) {   // every thread loads two 8-value chunks (K == 4096), all loads in flight at once
    uint4 xv[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) xv[i] = ldcg_u4(x4 + tid + i * NT);
#pragma unroll
    for (int i = 0; i < 4; ++i) nraw[i] = __ldg(reinterpret_cast<const uint2*>(norm_w + (warp + i * ST_WARPS) * QB) + lane);
#pragma unroll
    for (int i = 0; i < 2; ++i) xs4[tid + i * NT] = xv[i];
    consumer_sync();
    if (resid_slice_dst) {
      const int per = (K / 8 + gridDim.x - 1) / gridDim.x;
      const int lo = blockIdx.x * per, hi = min(lo + per, K / 8);
      for (int i = lo + tid; i < hi; i += NT) reinterpret_cast<uint4*>(resid_slice_dst)[i] = xs4[i];
    }
    if (tid < 128) {
      float ss = 0.f;
      for (int i = tid; i < K / 8; i += 128) {
        const uint4 v = xs4[i];
        const bf16* e = reinterpret_cast<const bf16*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float f = __bfloat162float(e[j]);
          ss += f * f;
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) sm.red[warp] = ss;
    }
    consumer_sync();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) tot += sm.red[i];
    rstd = rsqrtf(tot / (float)K + eps);
  } else {   // each warp loads its own groups gq = warp + 8 i (up to 12), all at once, into its part of xs
    constexpr int MAXG = ST_MAX_K / QB / ST_WARPS;
    uint2 raw[MAXG];
#pragma unroll
    for (int i = 0; i < MAXG; ++i) {
      const int gq = warp + i * ST_WARPS;
      if (gq < KB) raw[i] = ldcg_u2(x + gq * QB + lane * 4);
    }
#pragma unroll
    for (int i = 0; i < MAXG; ++i) {
      const int gq = warp + i * ST_WARPS;
      if (gq < KB) *reinterpret_cast<uint2*>(sm.u.xs + gq * QB + lane * 4) = raw[i];
    }
    __syncwarp();
  }
  if (tid == 0 && c.p->tl) step_stamp(*c.p, c.tl_phase, 23);
  if (KB <= 4 * ST_WARPS) prologue_quant<4>(c, KB, norm_w != nullptr, nraw, rstd);
  else prologue_quant<ST_MAX_K / QB / ST_WARPS>(c, KB, false, nraw, rstd);
  consumer_sync();
}

// ---- consumer: attention phase ---------------------------------------------------------------------------------
// Attention items (kv head, 64-key split) of this CTA: partial (m, l, o) per query head into o_part/ml_part.
// The item owning position `pos` appends the new K/V row. Items go in batches of up to ST_ABATCH (one ring
// stage each) so that every thread carries independent dot chains of several items: scores with thread =
// (key, query head) over all items of the batch, softmax with one warp per (item, head) row, P @ V with two
// warps per item and thread = (2 dims, 4 heads). Every sum keeps the reference's order.
template <int NKV>   // KV heads of this rank (8 / TP); 4 query heads per KV head
__device__ void attention_phase(Consumer& c, const StepLayer& L, int l, int pos) {
  StepSmem& sm = *c.sm;
  const StepParams& p = *c.p;
  const int tid = threadIdx.x, lane = c.lane, warp = c.warp;
  constexpr int NQ = GQA * NKV;
  const AttnItems it = attn_items(pos, NKV);
  const int ctx = pos + 1;
  const int last_split = it.n_splits - 1;
  const bf16* cos_row = p.cos_tab + (size_t)pos * HEAD_DIM;
  const bf16* sin_row = p.sin_tab + (size_t)pos * HEAD_DIM;
  bf16* k_cache = p.k_cache + (size_t)l * p.kv_layer_elems;
  bf16* v_cache = p.v_cache + (size_t)l * p.kv_layer_elems;
  for (int b0 = it.i0; b0 < it.i1; b0 += ST_ABATCH) {
    const int nb = min(ST_ABATCH, it.i1 - b0);
    const int kv0 = b0 / it.n_splits, nkv = (b0 + nb - 1) / it.n_splits - kv0 + 1;   // kv heads in the batch
    bool ok = true;
    for (int k = 0; k < nb; ++k) ok = c.wait_abs(c.n + k) && ok;
    if (!ok) atomicOr(&g_dev_error, DEVERR_MBAR_TIMEOUT);
    const bool tl = p.tl != nullptr && tid == 0;
    if (tl) step_stamp(p, c.tl_phase, 9);
    auto stage = [&](int k) { return sm.ring[(c.n + k) % ST_NSTAGE]; };
    // setup tasks, one warp each: q of every query head of the batch's kv heads (RMSNorm + RoPE), and the new
    // K row (RMSNorm + RoPE) and V row of every kv head whose last split is in the batch
    const int n_tasks = 4 * nkv + 2 * nkv;
    for (int t = warp; t < n_tasks; t += ST_WARPS) {
      const bool is_q = t < 4 * nkv;
      const int kvh = kv0 + ((t - 4 * nkv) >> 1), is_v = is_q ? 0 : (t - 4 * nkv) & 1;
      const int k = kvh * it.n_splits + last_split - b0;     // K/V tasks: batch index of the item owning pos
      if (!is_q && (k < 0 || k >= nb)) continue;
      const int row = is_q ? (kv0 + (t >> 2)) * GQA + (t & 3) : (is_v ? NQ + NKV : NQ) + kvh;   // qkv head row
      const uint2 raw = ldcg_u2(p.qkv + row * HEAD_DIM + lane * 4);
      const int jn = pos - last_split * ST_CHUNK;
      uint8_t* st = is_q ? nullptr : stage(k) + (is_v ? ST_STAGE / 2 : 0);
      if (is_v) {
        *reinterpret_cast<uint2*>(v_cache + ((size_t)kvh * p.max_seq + pos) * HEAD_DIM + lane * 4) = raw;
        *reinterpret_cast<uint2*>(st + kv_swz(jn, lane * 4)) = raw;
        fence_proxy_async_smem();   // this stage is refilled by TMA (async proxy) after its release
        continue;
      }
      float v[4] = {bf16lo(raw.x), bf16hi(raw.x), bf16lo(raw.y), bf16hi(raw.y)};
      float o[4];
      head_norm_rope(v, is_q ? L.q_norm : L.k_norm, cos_row, sin_row, lane, p.eps, o);
      if (is_q) {
#pragma unroll
        for (int j = 0; j < 4; ++j) sm.u.at.qs[t >> 2][t & 3][lane * 4 + j] = bf16r(o[j]);
      } else {
        bf16* dst = k_cache + ((size_t)kvh * p.max_seq + pos) * HEAD_DIM + lane * 4;
        bf16* sdst = reinterpret_cast<bf16*>(st + kv_swz(jn, lane * 4));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          dst[j] = __float2bfloat16_rn(o[j]);
          sdst[j] = __float2bfloat16_rn(o[j]);
        }
        fence_proxy_async_smem();
      }
    }
    consumer_sync();
    if (tl) step_stamp(p, c.tl_phase, 10);
    // scores: thread (item k = tid / 64, key j = tid % 64), all 4 query heads: dims 0..63 and 64..127 each
    // summed in order, then added. Each K chunk is loaded and converted once for the 4 heads; the q values
    // are the same for the whole warp (broadcast reads).
    if ((tid >> 6) < nb) {
      const int k = tid >> 6, j = tid & 63;
      const int item = b0 + k, split = item % it.n_splits;
      const int nj = min(ST_CHUNK, ctx - split * ST_CHUNK);
      const uint32_t ks = smem_u32(stage(k));
      const uint32_t qb0 = smem_u32(sm.u.at.qs[item / it.n_splits - kv0][0]);
      constexpr uint32_t QROW = (HEAD_DIM + 4) * 4;            // bytes between the heads' q rows
      float dot[GQA][2];
#pragma unroll
      for (int h = 0; h < GQA; ++h) dot[h][0] = dot[h][1] = 0.f;
#pragma unroll
      for (int sl = 0; sl < 2; ++sl) {
#pragma unroll 2
        for (int i = 0; i < 8; ++i) {
          const uint4 kv = lds128_at(ks + kv_swz(j, sl * 64 + i * 8));
          const float k0 = bf16lo(kv.x), k1 = bf16hi(kv.x), k2 = bf16lo(kv.y), k3 = bf16hi(kv.y);
          const float k4 = bf16lo(kv.z), k5 = bf16hi(kv.z), k6 = bf16lo(kv.w), k7 = bf16hi(kv.w);
          const uint32_t qo = (sl * 64 + i * 8) * 4;
#pragma unroll
          for (int h = 0; h < GQA; ++h) {
            const uint4 qa = lds128_at(qb0 + h * QROW + qo);
            const uint4 qb = lds128_at(qb0 + h * QROW + qo + 16);
            float& dt = dot[h][sl];
            dt += __uint_as_float(qa.x) * k0;
            dt += __uint_as_float(qa.y) * k1;
            dt += __uint_as_float(qa.z) * k2;
            dt += __uint_as_float(qa.w) * k3;
            dt += __uint_as_float(qb.x) * k4;
            dt += __uint_as_float(qb.y) * k5;
            dt += __uint_as_float(qb.z) * k6;
            dt += __uint_as_float(qb.w) * k7;
          }
        }
      }
#pragma unroll
      for (int h = 0; h < GQA; ++h) {
        float sc = dot[h][0];
        sc += dot[h][1];
        sm.u.at.sc[k][h][j] = j < nj ? sc * p.attn_scale : -INFINITY;
      }
    }
    consumer_sync();
    if (tl) step_stamp(p, c.tl_phase, 11);
    // softmax over each (item, head) row, one warp per row
    for (int r = warp; r < nb * GQA; r += ST_WARPS) {
      float* row = sm.u.at.sc[r >> 2][r & 3];
      float pr[2];
      float m = -INFINITY;
#pragma unroll
      for (int i = 0; i < 2; ++i) { pr[i] = row[lane + 32 * i]; m = fmaxf(m, pr[i]); }
      m = warp_max(m);
      float lsum = 0.f;
#pragma unroll
      for (int i = 0; i < 2; ++i) { pr[i] = expf(pr[i] - m); lsum += pr[i]; row[lane + 32 * i] = pr[i]; }
      lsum = warp_sum(lsum);
      if (lane == 0) { sm.u.at.m_s[r >> 2][r & 3] = m; sm.u.at.l_s[r >> 2][r & 3] = lsum; }
    }
    consumer_sync();
    if (tl) step_stamp(p, c.tl_phase, 12);
    // P @ V: warps 2k, 2k+1 take item k; thread = dims d, d + 1 of all 4 heads; each output sums over the keys
    // in order (the reference's sequential loop). Keys go in groups of 8, for which the swizzled offsets of
    // this thread's dims are fixed (they depend on key & 7 only).
    if ((warp >> 1) < nb) {
      const int k = warp >> 1, item = b0 + k;
      const int kvh = item / it.n_splits, split = item - kvh * it.n_splits;
      const int nj = min(ST_CHUNK, ctx - split * ST_CHUNK);
      const int d = ((warp & 1) * 32 + lane) * 2;
      const uint8_t* Vs = stage(k) + ST_STAGE / 2;
      uint32_t off[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) off[r] = kv_swz(r, d);
      float acc[GQA][2];
#pragma unroll
      for (int h = 0; h < GQA; ++h) acc[h][0] = acc[h][1] = 0.f;
      const int n8 = nj >> 3;
#pragma unroll 2
      for (int t = 0; t < n8; ++t) {
        uint32_t v2[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) v2[r] = *reinterpret_cast<const uint32_t*>(Vs + t * 1024 + off[r]);
#pragma unroll
        for (int h = 0; h < GQA; ++h) {
          const float4 pa = *reinterpret_cast<const float4*>(&sm.u.at.sc[k][h][t * 8]);
          const float4 pb = *reinterpret_cast<const float4*>(&sm.u.at.sc[k][h][t * 8 + 4]);
          const float pj[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            acc[h][0] += pj[r] * bf16lo(v2[r]);
            acc[h][1] += pj[r] * bf16hi(v2[r]);
          }
        }
      }
      for (int j = n8 * 8; j < nj; ++j) {
        const uint32_t v2 = *reinterpret_cast<const uint32_t*>(Vs + kv_swz(j, d));
#pragma unroll
        for (int h = 0; h < GQA; ++h) {
          const float pj = sm.u.at.sc[k][h][j];
          acc[h][0] += pj * bf16lo(v2);
          acc[h][1] += pj * bf16hi(v2);
        }
      }
#pragma unroll
      for (int h = 0; h < GQA; ++h) {
        const size_t row = (size_t)(kvh * GQA + h) * p.max_splits + split;
        *reinterpret_cast<float2*>(p.o_part + row * HEAD_DIM + d) = make_float2(acc[h][0], acc[h][1]);
        if (d == 0) {
          p.ml_part[row * 2 + 0] = sm.u.at.m_s[k][h];
          p.ml_part[row * 2 + 1] = sm.u.at.l_s[k][h];
        }
      }
    }
    for (int k = 0; k < nb; ++k) c.release_stage((c.n + k) % ST_NSTAGE);
    c.n += nb;
    consumer_sync();
  }
}

// After its attention items, a CTA counts them on the per-KV-head counters (p.attn_counters: monotonic over the
// layers of a launch, reset by the launch's last CTA) with a release reduction; nothing waits for it here.
template <int NKV>
__device__ __forceinline__ void attention_arrive(const StepParams& p, int pos) {
  const AttnItems it = attn_items(pos, NKV);
  if (threadIdx.x != 0 || it.i1 <= it.i0) return;   // the consumer barrier before orders the CTA's partials
  const int g0 = it.i0 / it.n_splits, g1 = (it.i1 - 1) / it.n_splits;
  for (int g = g0; g <= g1; ++g) {
    const int mine = min(it.i1, (g + 1) * it.n_splits) - max(it.i0, g * it.n_splits);
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p.attn_counters + g), "r"(mine) : "memory");
  }
}

// Merge of the 64-key splits: CTA m < 4 * NQ produces dims 32*(m%4) .. +31 of query head m/4, once every split
// of that head's KV head is counted (bounded wait on its counter instead of a grid barrier). Warp 0 takes the
// maximum M of the split maxima and the weights w_s = exp(m_s - M) with their l-weighted sum (lane-strided over
// the splits, then a butterfly); all warps stage the partial rows in shared memory; threads 0-31 sum
// w_s * o_s[d] over the splits in order. The arithmetic of the attention op's merge (attn_merge_kernel), so
// the output is bit-identical to it.
template <int NQ>
__device__ void merge_phase(Consumer& c, int l, int pos) {
  StepSmem& sm = *c.sm;
  const StepParams& p = *c.p;
  if (blockIdx.x >= 4 * NQ) return;
  const int tid = threadIdx.x, lane = c.lane, warp = c.warp;
  const int qh = blockIdx.x >> 2, d0 = (blockIdx.x & 3) * 32;
  const int n_splits = (pos + 1 + ST_CHUNK - 1) / ST_CHUNK;
  const bool tl = p.tl != nullptr && tid == 0;
  if (tl) step_stamp(p, c.tl_phase, 13);
  if (tid == 0) {   // every split of the KV head has been counted (this layer: l + 1 rounds of n_splits)
    const unsigned* ctr = reinterpret_cast<const unsigned*>(p.attn_counters + qh / GQA);
    const unsigned target = (unsigned)((l + 1) * n_splits);
    if (ld_acquire_u32(ctr) < target) {
      const unsigned long long t0 = globaltimer();
      while (ld_acquire_u32(ctr) < target) {
        if (wait_failed()) break;
        if (globaltimer() - t0 > WAIT_LIMIT_NS) {
          atomicOr(&g_dev_error, DEVERR_GRID_TIMEOUT);
          break;
        }
      }
    }
  }
  consumer_sync();
  if (tl) step_stamp(p, c.tl_phase, 14);
  float* cw = sm.u.mg.w;
  if (warp == 0) {   // the split weights: one load of each (m_s, l_s) pair, kept in shared memory
    const float2* ml = reinterpret_cast<const float2*>(p.ml_part + (size_t)qh * p.max_splits * 2);
    float mloc = -INFINITY;
    for (int s = lane; s < n_splits; s += 32) {
      const float2 v = __ldcg(ml + s);
      cw[s] = v.x;
      sm.u.mg.l[s] = v.y;
      mloc = fmaxf(mloc, v.x);
    }
    const float M = warp_max(mloc);
    float lsum = 0.f;
    for (int s = lane; s < n_splits; s += 32) {   // each lane rereads only the entries it wrote
      const float wt = expf(cw[s] - M);
      cw[s] = wt;
      lsum += wt * sm.u.mg.l[s];
    }
    lsum = warp_sum(lsum);
    if (lane == 0) sm.u.mg.cl = lsum;
  }
  if (tl) step_stamp(p, c.tl_phase, 15);
  float o = 0.f;
  const float* op = p.o_part + (size_t)qh * p.max_splits * HEAD_DIM + d0;
  for (int s0 = 0; s0 < n_splits; s0 += ST_MERGE_ROUND) {
    const int ns = min(ST_MERGE_ROUND, n_splits - s0);
    // 8 x 16 bytes per split row of 32 dims; warps 1-7 load the first round while warp 0 computes the weights
    for (int i = s0 == 0 ? tid - 32 : tid; i < ns * 8; i += s0 == 0 ? ST_WARPS * 32 - 32 : ST_WARPS * 32) {
      if (i < 0) break;
      const int sr = i >> 3, f = i & 7;
      reinterpret_cast<uint4*>(sm.u.mg.o)[i] = ldcg_u4(op + (size_t)(s0 + sr) * HEAD_DIM + f * 4);
    }
    consumer_sync();
    if (tid < 32) {
      for (int sr = 0; sr < ns; ++sr) o += cw[s0 + sr] * sm.u.mg.o[sr * 32 + tid];
    }
    consumer_sync();
  }
  if (tid < 32) p.attn[qh * HEAD_DIM + d0 + tid] = __float2bfloat16_rn(o / sm.u.mg.cl);
}

// ---- tensor-parallel exchange -------------------------------------------------------------------------------------
// After a row-parallel GEMV phase (o_proj, down) every rank has stored its rows' fp32 partials, tagged, into
// every rank's TpArea. CTAs 0..31 each own 128 rows: a thread waits (bounded) until all tp words of its row
// carry this exchange's tag, sums them in rank order and writes the new residual row
// bf16(resid + bf16(sum)) to the other residual buffer. The grid barrier that follows publishes it to the
// next prologue (and keeps the GEMV scratch of the two phases apart).
__device__ __forceinline__ void tp_reduce(const StepParams& p, const bf16* resid, bf16* resid_next, int xbuf,
                                          unsigned tag) {
  constexpr int ROWS = 128;
  if (blockIdx.x >= HIDDEN / ROWS || threadIdx.x >= ROWS) return;
  const int row = blockIdx.x * ROWS + threadIdx.x;
  const unsigned long long* src = &p.areas[p.tp_rank]->recv[xbuf][0][row];
  float sum = 0.f;
  for (int r = 0; r < p.tp; ++r) {
    const unsigned long long* a = src + (size_t)r * HIDDEN;
    unsigned long long w = ld_relaxed_sys_u64(a);
    if ((unsigned)(w >> 32) != tag) {
      const long long c0 = clock64();
      while ((unsigned)((w = ld_relaxed_sys_u64(a)) >> 32) != tag && clock64() - c0 < 500000) {
      }
      if ((unsigned)(w >> 32) != tag) {
        const unsigned long long t0 = globaltimer();
        while ((unsigned)((w = ld_relaxed_sys_u64(a)) >> 32) != tag) {
          if (wait_failed()) break;
          if (globaltimer() - t0 > WAIT_LIMIT_NS) {
            atomicOr(&g_dev_error, DEVERR_GRID_TIMEOUT);
            break;
          }
        }
      }
    }
    const float v = __uint_as_float((unsigned)w);
    sum = r == 0 ? v : sum + v;
  }
  resid_next[row] = __float2bfloat16_rn(__bfloat162float(ldcg_bf16(resid + row)) + bf16r(sum));
}

// ---- bf16 lm_head (the reference checkpoint's format) -----------------------------------------------------------
// The CTA's rows [r0, r1) stream through the ring 4 rows (32 KiB) per stage; consumer warp w computes row w % 4 of
// every other stage (warps 0-3 the even stages, 4-7 the odd ones) and counts 2 of the stage's 8 releases. The
// arithmetic is the bf16 lm_head kernel's (csrc/gemv.cuh, lm_head_bf16_kernel): the final RMSNorm with the
// 256-thread strided sum of squares, and per row lane l summing elements (32 j + l) * 8 .. +7 for j = 0..15 in
// order, then a butterfly; so logits and the chosen token are bit-identical to it.
constexpr int ST_HEAD_ROWS = ST_STAGE / (HIDDEN * 2);   // bf16 rows per ring stage (4)
__device__ __forceinline__ SliceRange head_rows(int vocab) {
  const long long G = gridDim.x, c = blockIdx.x;
  return SliceRange{(int)(c * vocab / G), (int)((c + 1) * vocab / G)};
}
__device__ void head_bf16_phase(Consumer& c, const bf16* x, int row_offset) {
  StepSmem& sm = *c.sm;
  const StepParams& p = *c.p;
  const int tid = threadIdx.x, lane = c.lane, warp = c.warp;
  constexpr int K = HIDDEN;
  float* xn = reinterpret_cast<float*>(sm.xh);   // the normalised input, fp32 (16 KiB)
  float ss = 0.f;
  for (int i = tid; i < K; i += ST_WARPS * 32) {
    const float f = __bfloat162float(ldcg_bf16(x + i));
    xn[i] = f;
    ss += f * f;
  }
  ss = warp_sum(ss);
  if (lane == 0) sm.red[warp] = ss;
  consumer_sync();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < ST_WARPS; ++i) tot += sm.red[i];
  const float rstd = rsqrtf(tot / (float)K + p.eps);
  for (int i = tid; i < K; i += ST_WARPS * 32) xn[i] = bf16r(__bfloat162float(p.final_norm[i]) * bf16r(xn[i] * rstd));
  consumer_sync();
  const SliceRange r = head_rows(p.vocab);
  const int nst = (r.s1 - r.s0 + ST_HEAD_ROWS - 1) / ST_HEAD_ROWS;
  const int n0 = c.n;
  for (int s = warp / ST_HEAD_ROWS; s < nst; s += ST_WARPS / ST_HEAD_ROWS) {
    if (!c.wait_abs(n0 + s)) atomicOr(&g_dev_error, DEVERR_MBAR_TIMEOUT);
    const int row = r.s0 + s * ST_HEAD_ROWS + warp % ST_HEAD_ROWS;
    if (row < r.s1) {
      const uint8_t* wrow = sm.ring[(n0 + s) % ST_NSTAGE] + (warp % ST_HEAD_ROWS) * (K * 2);
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < K / 8 / 32; ++j) {
        const int k0 = (j * 32 + lane) * 8;
        const uint4 wv = lds128(wrow + (size_t)(j * 32 + lane) * 16);
        const uint32_t* q = reinterpret_cast<const uint32_t*>(&wv);
        const float4 x0 = *reinterpret_cast<const float4*>(&xn[k0]);
        const float4 x1 = *reinterpret_cast<const float4*>(&xn[k0 + 4]);
        acc += __uint_as_float(q[0] << 16) * x0.x + __uint_as_float(q[0] & 0xFFFF0000u) * x0.y;
        acc += __uint_as_float(q[1] << 16) * x0.z + __uint_as_float(q[1] & 0xFFFF0000u) * x0.w;
        acc += __uint_as_float(q[2] << 16) * x1.x + __uint_as_float(q[2] & 0xFFFF0000u) * x1.y;
        acc += __uint_as_float(q[3] << 16) * x1.z + __uint_as_float(q[3] & 0xFFFF0000u) * x1.w;
      }
      acc = warp_sum(acc);
      if (lane == 0) p.logits[row] = __float2bfloat16_rn(acc);
      const float lv = bf16r(acc);
      const int gid = row + row_offset;
      if (lv > c.best_v || (lv == c.best_v && gid < c.best_i)) {
        c.best_v = lv;
        c.best_i = gid;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_n(&sm.empty[(n0 + s) % ST_NSTAGE], ST_WARPS / ST_HEAD_ROWS);
  }
  c.n = n0 + nst;
}

// ---- the kernel -------------------------------------------------------------------------------------------------
// TP = 1: the whole model on one GPU. TP > 1: this rank's shard (query heads 32/TP, KV heads 8/TP, intermediate
// 12288/TP, vocabulary rows p.vocab from p.vocab_offset); o_proj and down produce fp32 partials that are
// exchanged (tp_reduce) and added to the residual, in rank order on every rank.
template <int SCALE, int TP, int HEAD_BF16>
__global__ void __launch_bounds__(ST_THREADS, 1) decode_step_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(1024) uint8_t smem_step[];
  StepSmem& sm = *reinterpret_cast<StepSmem*>(smem_step);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = p.state[0];
  if (pos < 0 || pos >= p.max_seq || (pos + ST_CHUNK) / ST_CHUNK > p.max_splits) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(&g_dev_error, DEVERR_BAD_STATE);
    return;   // every CTA returns: no barrier is entered
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST_NSTAGE; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], ST_WARPS);
    }
    sm.grab = 0;
    sm.plan[0] = make_plan(6144 / TP, HIDDEN / QB, 1);            // qkv
    sm.plan[1] = make_plan(HIDDEN, HIDDEN / TP / QB, 1);          // o_proj
    sm.plan[2] = make_plan(2 * 12288 / TP, HIDDEN / QB, 2);       // gate_up
    sm.plan[3] = make_plan(HIDDEN, 12288 / TP / QB, 1);           // down
    sm.plan[4] = make_plan(p.vocab, HIDDEN / QB, 1);              // lm_head (FP8)
    for (int i = 0; i < ST_BD_FLOATS / (4 * 16); ++i) sm.done[i] = 0;
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.tail_full[b], 32 * ST_FETCH_WARPS);   // every fetcher lane, after its words are in smem
      mbar_init(&sm.tail_empty[b], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  constexpr int H = HIDDEN, I = 12288 / TP, QKV_N = 6144 / TP, NKV = 8 / TP, NQ = 32 / TP, KO = HIDDEN / TP;
  // The step's GEMV phases in order: g = 4 l + k for layer l (k: 0 qkv, 1 o_proj, 2 gate_up, 3 down), then the
  // FP8 lm_head as g = 4 n_layers. Producer, tail fetcher and consumers walk this list with one call site each.
  const int n_gemv = 4 * p.n_layers + (HEAD_BF16 ? 0 : 1);
  auto gemv_timeline_phase = [&](int g) { return (g >> 2) == p.n_layers ? 5 * p.n_layers : 5 * (g >> 2) + ((g & 3) == 0 ? 0 : (g & 3) + 1); };
  if (warp >= ST_WARPS) {   // ---------------- producer ----------------
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(ST_PRODUCER_REGS) : "memory");
    if (warp == ST_WARPS && lane == 0) {
      Producer pr{&sm, 0, policy_evict_first(), true, 0};
      const AttnItems it = attn_items(pos, NKV);
      for (int g = 0; g < n_gemv; ++g) {
        const int l = g >> 2, k = g & 3, ph = gemv_timeline_phase(g);
        step_stamp(p, ph, 3);
        step_put(p, ph, 6, pr.wait_cycles);
        if (l == p.n_layers) {
          pr.gemv(p.w_head, (p.vocab / 16) * (H / QB));
          break;
        }
        const StepLayer& L = p.layers[l];
        const uint8_t* w = k == 0 ? L.w_qkv : k == 1 ? L.w_o : k == 2 ? L.w_gu : L.w_down;
        const int n_slices = k == 0 ? (QKV_N / 16) * (H / QB)
                             : k == 1 ? (H / 16) * (KO / QB)
                             : k == 2 ? (2 * I / 16) * (H / QB)
                                      : (H / 16) * (I / QB);
        pr.gemv(w, n_slices);
        if (k == 0) {   // the layer's attention items follow its qkv
          step_stamp(p, 5 * l + 1, 3);
          step_put(p, 5 * l + 1, 6, pr.wait_cycles);
          for (int item = it.i0; item < it.i1; ++item) {
            const int kvh = item / it.n_splits, split = item - kvh * it.n_splits;
            pr.push_kv(p, l, kvh, split * ST_CHUNK);
          }
        }
      }
      if (HEAD_BF16) {   // 4 bf16 rows per stage
        step_stamp(p, 5 * p.n_layers, 3);
        step_put(p, 5 * p.n_layers, 6, pr.wait_cycles);
        const SliceRange hr = head_rows(p.vocab);
        for (int row = hr.s0; row < hr.s1; row += ST_HEAD_ROWS)
          pr.push(p.w_head + (size_t)row * HIDDEN * 2, (uint32_t)(min(ST_HEAD_ROWS, hr.s1 - row) * HIDDEN * 2));
      }
    } else if (warp >= ST_WARPS + 1) {   // tail fetchers: the split units' remote block dots, phase by phase
      const int part = warp - (ST_WARPS + 1);   // this warp copies passes part, part + ST_FETCH_WARPS, ...
      const unsigned long long tb = tag_base(__ldcg(p.sync + 2), p.n_layers);
      int n = 0;
      for (int g = 0; g < n_gemv; ++g) {
        const int k = (g >> 2) == p.n_layers ? 0 : g & 3;
        const int KB = k == 1 ? KO / QB : k == 3 ? I / QB : H / QB;
        const int ph = gemv_timeline_phase(g);
        tail_fetch(sm, p, sm.plan[(g >> 2) == p.n_layers ? 4 : k], KB, k == 2 ? 2 : 1, ph, phase_tag(tb, ph), n, lane,
                   part);
      }
    }
    return;
  }
  // ---------------- consumers ----------------
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(ST_CONSUMER_REGS) : "memory");
  Consumer c{&sm, &p, 0, lane, warp, lane >> 2, lane & 3, -INFINITY, 0x7FFFFFFF, 0, 0};
  c.epoch = __ldcg(p.sync + 2);
  c.tag_base = tag_base(c.epoch, p.n_layers);
  unsigned nbar = 0;
  const int tok = p.token[0];
  const bool tok_ok = tok >= 0 && tok < p.vocab * TP;
  if (!tok_ok && threadIdx.x == 0 && blockIdx.x == 0) atomicOr(&g_dev_error, DEVERR_BAD_STATE);
  const bool tl = p.tl != nullptr && threadIdx.x == 0;
  // TP: exchanges so far (2 per layer per launch), read before this launch's last CTA advances the epoch
  const unsigned long long x_base = TP > 1 ? __ldcg(&p.areas[p.tp_rank]->epoch) * 2ull * p.n_layers : 0ull;
  unsigned xk = 0;                                  // exchange index within this launch
  // residual buffer k: exchange k reads rbuf(k) and writes rbuf(k + 1) (TP = 1: one buffer, updated in place)
  auto rbuf = [&](unsigned k) -> bf16* { return (TP > 1 && (k & 1)) ? p.resid_alt : p.resid; };
  for (int g = 0; g < n_gemv; ++g) {
    const int l = g >> 2, k = g & 3, ph = gemv_timeline_phase(g);
    const bool head = l == p.n_layers;
    const StepLayer& L = p.layers[head ? 0 : l];
    // the phase's input: QKV RMSNorm(resid) (layer 0: the token's embedding row, also copied into resid); O the
    // attention output; GU RMSNorm(resid); DOWN the SwiGLU output; HEAD the final RMSNorm of resid. TP: after a
    // row-parallel phase's exchange the residual lives in the other buffer.
    const bf16* x = k == 1 ? p.attn : k == 3 ? p.h : rbuf(xk);
    const bf16* nw = head ? p.final_norm : k == 0 ? L.ln1 : k == 2 ? L.ln2 : nullptr;
    bf16* embed_dst = nullptr;
    if (g == 0) {
      x = p.embed + (size_t)(tok_ok ? tok : 0) * H;
      embed_dst = p.resid;
    }
    const bool row_par = !head && (k == 1 || k == 3);   // o_proj, down: residual add (TP: fp32 partials)
    GemvPhase d{};
    d.K = k == 1 ? KO : k == 3 ? I : H;
    d.KB = d.K / QB;
    d.NG = !head && k == 2 ? 2 : 1;
    d.N = head ? p.vocab : k == 0 ? QKV_N : k == 2 ? 2 * I : H;
    d.ws = head ? p.s_head : k == 0 ? L.s_qkv : k == 1 ? L.s_o : k == 2 ? L.s_gu : L.s_down;
    d.scale_block = !head && SCALE == SCALE_BLOCK;
    d.epi = head ? EPI_ARGMAX : k == 0 ? EPI_STORE : k == 2 ? EPI_SWIGLU : (TP == 1 ? EPI_RESIDUAL : EPI_TP_PARTIAL);
    d.out = head ? p.logits : k == 0 ? p.qkv : k == 2 ? p.h : (TP == 1 ? p.resid : nullptr);
    d.part = p.part;
    d.row_offset = head ? p.vocab_offset : 0;
    d.xbuf = (int)(xk % 2);
    d.xtag = (unsigned)(x_base + xk + 1);
    if (tl) step_stamp(p, ph, 0);
    c.tl_phase = ph;
    step_prologue(c, x, nw, d.K, p.eps, embed_dst);
    if (tl) step_stamp(p, ph, 1);
    gemv_phase(c, d, sm.plan[head ? 4 : k]);
    if (tl) { step_put(p, ph, 4, c.wait_cycles); step_put(p, ph, 5, c.fold_cycles); }
    if (head) break;
    if (TP > 1 && row_par) {   // the tags tell a reducer when every rank's partial of its row has arrived
      tp_reduce(p, rbuf(xk), rbuf(xk + 1), (int)(xk % 2), (unsigned)(x_base + xk + 1));
      ++xk;
    }
    grid_barrier(p.sync, nbar++, step_word(p, ph, 2));
    if (k == 0) {   // ATTN: split partials (and the K/V rows at pos), then the merge into the attention output
      if (tl) step_stamp(p, ph + 1, 0);
      c.tl_phase = ph + 1;
      attention_phase<NKV>(c, L, l, pos);
      if (tl) step_stamp(p, ph + 1, 7);
      attention_arrive<NKV>(p, pos);
      merge_phase<NQ>(c, l, pos);
      if (tl) step_stamp(p, ph + 1, 1);
      if (tl) { step_put(p, ph + 1, 4, c.wait_cycles); step_put(p, ph + 1, 5, c.fold_cycles); }
      grid_barrier(p.sync, nbar++, step_word(p, ph + 1, 2));
    }
  }
  if (HEAD_BF16) {   // HEAD: the bf16 lm_head (reference checkpoint format) with the final RMSNorm
    if (tl) { step_stamp(p, 5 * p.n_layers, 0); step_stamp(p, 5 * p.n_layers, 1); }
    c.tl_phase = 5 * p.n_layers;
    head_bf16_phase(c, rbuf(xk), p.vocab_offset);
    if (tl) { step_put(p, 5 * p.n_layers, 4, c.wait_cycles); step_put(p, 5 * p.n_layers, 5, c.fold_cycles); }
  }
  if (tl) step_stamp(p, 5 * p.n_layers, 2);
  {
    unsigned long long key = (c.best_i == 0x7FFFFFFF) ? 0ull : argmax_key(c.best_v, c.best_i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
      key = other > key ? other : key;
    }
    if (lane == 0) sm.bestbuf[warp] = key;
    consumer_sync();
    if (threadIdx.x == 0) {
      unsigned long long b = 0;
      for (int i = 0; i < ST_WARPS; ++i) b = sm.bestbuf[i] > b ? sm.bestbuf[i] : b;
      if (b) atomicMax(p.best, b);
      __threadfence();
      // the last CTA to finish decodes the token and advances the state; no CTA waits on a barrier any more,
      // so it also resets the barrier counters for the next launch
      if (atomicAdd(p.sync + 1, 1u) == gridDim.x - 1) {
        __threadfence();
        unsigned long long k = atomicAdd(p.best, 0ull);
        if (TP > 1) {   // every rank's best key to every rank; all ranks then take the same maximum
          TpArea* own = p.areas[p.tp_rank];
          const unsigned long long ep = __ldcg(&own->epoch);
          for (int r = 0; r < TP; ++r) p.areas[r]->keys[p.tp_rank] = k;
          __threadfence_system();
          for (int r = 0; r < TP; ++r) red_add_release_sys(&p.areas[r]->key_ctr, 1ull);
          wait_sys_counter(&own->key_ctr, (ep + 1) * TP);
          for (int r = 0; r < TP; ++r) {
            const unsigned long long kr = __ldcg(&own->keys[r]);
            k = kr > k ? kr : k;
          }
          own->epoch = ep + 1;
        }
        const int next = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        p.token[0] = next;
        const int step = p.state[1];
        if (step >= 0 && step < p.out_len) p.out_tokens[step] = next;
        p.state[0] = pos + 1;
        p.state[1] = step + 1;
        *p.best = 0ull;
        for (int g = 0; g < NKV; ++g) p.attn_counters[g] = 0;
        p.sync[2] = c.epoch + 1;   // the next launch's block-dot tags
        p.sync[0] = 0;
        p.sync[1] = 0;
        __threadfence();
      }
    }
  }
}

}  // namespace qk
