// Persistent decode step: the whole batch-1 token (36 layers + lm_head + argmax + bookkeeping) in ONE launch.
//
// Why: at B200 bandwidth a layer's 193 MB of FP8 weights stream in ~30 us, while every kernel boundary costs
// several us (CTA turnover, the PDL wait, the activation prologue) during which DRAM idles. Here no boundary
// exists: every SM runs one CTA for the whole step and its weight stream never stops.
//
// Structure (grid = one CTA per SM, cooperative launch so all CTAs are resident):
//  * warp 8 (producer): lane 0 walks the CTA's static schedule of loads for the entire step and issues them
//    as bulk async copies into an 11 x 16 KiB shared-memory ring (full/empty mbarriers): for each layer its
//    slice range of W_qkv, the K and V chunks of its attention items, then its ranges of W_o, W_gu, W_down;
//    finally its range of the lm_head. Loads depend only on weights and on KV rows of earlier tokens, so the
//    producer runs ahead across phase boundaries and keeps DRAM busy while the consumers synchronise.
//  * warps 0-7 (consumers) execute the phases in order, separated by grid barriers (monotonic counter, bounded
//    spin): QKV, ATTN, O, GU, DOWN per layer, then HEAD. A GEMV phase gives each CTA a contiguous range of
//    2 KiB slices (16 rows x 128 k); the 8 warps take one slice each per stage, store the block dots in shared
//    memory, and one warp folds each finished 16-row unit in K order (units shared with a neighbouring CTA
//    go through global scratch and a last-arriver fold). The attention phase gives each CTA a range of
//    (kv head, 64-key split) items; the last CTA of a head merges its splits.
//  * The arithmetic is the per-op kernels' (csrc/gemv.cuh, csrc/attention.cuh), operation for operation, so
//    the step's outputs, logits and KV rows are bit-identical to the per-op path (and so to the reference).
// All data written by one CTA and read by another in a later phase is read with ld.global.cg (L2), never
// through L1, because L1 is not coherent across SMs.
#pragma once
#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"

namespace qk {

constexpr int ST_WARPS = 8;                        // consumer warps
constexpr int ST_THREADS = (ST_WARPS + 1) * 32;    // + one producer warp
constexpr int ST_STAGE = 16384;
constexpr int ST_SLICE = 2048;                     // 16 rows x 128 k of fp8
constexpr int ST_SLICES = ST_STAGE / ST_SLICE;     // 8 slices per stage, one per consumer warp
constexpr int ST_NSTAGE = 11;
constexpr int ST_MAX_K = 12288;
constexpr int ST_CHUNK = 64;                       // attention keys per item
constexpr int ST_MAX_SPLITS = 1024;                // contexts up to 64k

struct StepLayer {
  const uint8_t *w_qkv, *w_o, *w_gu, *w_down;      // model.pack_fp8 layout
  const float *s_qkv, *s_o, *s_gu, *s_down;        // scales (layout per the kernel's SCALE)
  const bf16 *ln1, *ln2, *q_norm, *k_norm;
  bf16 *k_cache, *v_cache;                         // [n_kv][max_seq][128] of this layer
};

struct StepParams {
  const StepLayer* layers;                         // device array [n_layers]
  int n_layers;
  const bf16* embed;                               // [vocab][4096]
  const bf16* final_norm;                          // [4096]
  const uint8_t* w_head;                           // packed fp8 [vocab x 4096]
  const float* s_head;                             // [vocab] per-channel
  int vocab;
  const bf16 *cos_tab, *sin_tab;                   // [max_seq][128]
  int* token;                                      // [1]
  int* state;                                      // [pos, step]
  int* out_tokens;
  int out_len;
  unsigned long long* best;                        // [1], zero between launches
  bf16 *resid, *qkv, *attn, *h, *logits;           // activations [4096], [6144], [4096], [12288], [vocab]
  float* part;                                     // GEMV boundary-unit block dots [max N*K/128]
  int* counters;                                   // [max N/16], zero between launches
  float *o_part, *ml_part;                         // attention partials [32][max_splits][128], [32][max_splits][2]
  int* attn_counters;                              // [8], zero between launches
  unsigned* sync;                                  // [2]: grid barrier counter, end counter; zero between launches
  int max_seq, max_splits;
  float eps, attn_scale;
};

struct StepSmem {
  uint8_t ring[ST_NSTAGE][ST_STAGE];
  uint32_t xh[ST_MAX_K / 2];                       // x as f16 MMA fragments (see gemv_prologue)
  float xscale[ST_MAX_K / QB];
  union {
    float bd[2][96 * 16];                          // block dots of the two 16-row units in flight
    bf16 xs[HIDDEN];                               // raw x during an RMSNorm prologue
    struct {
      float qs[GQA][HEAD_DIM + 4];                 // +4: conflict-free reads by 4 heads at once
      float sc[GQA][ST_CHUNK];
      float m_s[GQA], l_s[GQA], cl[GQA];
      float cw[GQA][ST_MAX_SPLITS];
    } at;
  } u;
  float red[8];
  unsigned long long bestbuf[ST_WARPS];
  uint64_t full[ST_NSTAGE], empty[ST_NSTAGE];
  int flag;
};

// ---- small helpers -------------------------------------------------------------------------------------------
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(ST_WARPS * 32) : "memory"); }
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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
__device__ __forceinline__ uint4 ldcg_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// Consumer-side grid barrier number `idx` (0-based) of this launch. Bounded: on timeout it records the error and
// lets the CTA continue (wrong results, but no hang).
__device__ __forceinline__ void grid_barrier(unsigned* ctr, unsigned idx) {
  consumer_sync();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(ctr, 1u);
    const unsigned target = (idx + 1) * gridDim.x;
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
    __threadfence();
  }
  consumer_sync();
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
  __device__ __forceinline__ void push(const void* src, uint32_t bytes) {
    if (!ok) return;
    const int s = n % ST_NSTAGE;
    if (n >= ST_NSTAGE && !mbar_wait(&sm->empty[s], (uint32_t)(((n / ST_NSTAGE) - 1) & 1))) {
      ok = false;
      return;
    }
    mbar_arrive_expect_tx(&sm->full[s], bytes);
    bulk_g2s(sm->ring[s], src, bytes, &sm->full[s], pol);
    ++n;
  }
  __device__ __forceinline__ void gemv(const uint8_t* w, int n_slices) {
    const SliceRange r = slice_range(n_slices);
    for (int q = r.s0; q < r.s1; q += ST_SLICES)
      push(w + (size_t)q * ST_SLICE, (uint32_t)(min(ST_SLICES, r.s1 - q) * ST_SLICE));
  }
};

// ---- consumer: GEMV phase ---------------------------------------------------------------------------------------
template <int EPI, int SCALE, int NG>
struct GemvPhase {
  const float* ws;
  int N, K;           // N = all rows (gate + up for NG = 2)
  bf16* out;          // STORE: qkv; RESIDUAL: resid; SWIGLU: h; ARGMAX: logits
  float* part;
  int* counters;
};

struct Consumer {
  StepSmem* sm;
  const StepParams* p;
  int n;              // stages consumed so far
  int lane, warp, g, t;
  float best_v;
  int best_i;

  __device__ __forceinline__ bool wait_stage(int s) {
    return __all_sync(0xffffffffu, mbar_wait(&sm->full[s], (uint32_t)((n / ST_NSTAGE) & 1)));
  }
  __device__ __forceinline__ void release_stage(int s) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm->empty[s]);
  }
};

// Weight scale of `row` at K block `kb` (both layouts).
template <int SCALE>
__device__ __forceinline__ float row_scale(const float* ws, int row, int kb, int KB) {
  return SCALE == SCALE_CHANNEL ? __ldg(ws + row) : __ldg(ws + (size_t)(row / QB) * KB + kb);
}

template <int EPI, int SCALE, int NG>
__device__ void gemv_phase(Consumer& c, const GemvPhase<EPI, SCALE, NG>& ph) {
  StepSmem& sm = *c.sm;
  const int KB = ph.K / QB;
  const int RPU = 16 * NG;                          // rows per unit
  const int spu = KB * NG;                          // slices per unit
  const int units = ph.N / RPU;
  const SliceRange r = slice_range(units * spu);
  const uint8_t* xh = reinterpret_cast<const uint8_t*>(sm.xh);
  for (int q0 = r.s0; q0 < r.s1; q0 += ST_SLICES) {
    const int s = c.n % ST_NSTAGE;
    if (!c.wait_stage(s)) atomicOr(&g_dev_error, DEVERR_MBAR_TIMEOUT);
    const int q = q0 + c.warp;
    if (q < r.s1) {
      const int tile = q / NG, gi = q - tile * NG;
      const int u = tile / KB, kb = tile - u * KB;
      const uint8_t* slice = sm.ring[s] + c.warp * ST_SLICE;
      const uint8_t* xk = xh + kb * 256 + c.t * 16;
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        const uint4 xb = lds128(xk + ch * 64);
        const uint4 w4 = lds128(slice + ch * 512 + c.lane * 16);
        float e[4];
        fp8_chunk_dot(w4, xb, e);
        d0 += e[0];
        d1 += e[2];
      }
      if (c.t == 0) {
        const bool interior = (u * spu >= r.s0) && ((u + 1) * spu <= r.s1);
        float* dst = interior ? &sm.u.bd[u & 1][kb * RPU + gi * 16 + c.g]
                              : ph.part + ((size_t)u * KB + kb) * RPU + gi * 16 + c.g;
        dst[0] = d0;
        dst[8] = d1;
      }
    }
    c.release_stage(s);
    ++c.n;
    consumer_sync();
    // fold the units whose last slice of this CTA's range is in this stage (at most two)
    const int q_end = min(q0 + ST_SLICES, r.s1) - 1;
    const int ua = q0 / NG / KB, ub = q_end / NG / KB;
    for (int u = ua; u <= ub; ++u) {
      const int last_q = min((u + 1) * spu, r.s1) - 1;
      if (last_q < q0 || last_q > q_end) continue;
      if (c.warp != (u & (ST_WARPS - 1))) continue;
      const bool interior = (u * spu >= r.s0) && ((u + 1) * spu <= r.s1);
      const float* src;
      size_t stride;
      bool do_fold = true;
      if (interior) {
        src = sm.u.bd[u & 1];
        stride = RPU;
      } else {
        __threadfence();
        int last = 0;
        if (c.lane == 0) {
          const int mine = last_q - max(u * spu, r.s0) + 1;
          last = (atomicAdd(&ph.counters[u], mine) + mine == spu);
        }
        do_fold = __shfl_sync(0xffffffffu, last, 0) != 0;
        if (do_fold) __threadfence();
        src = ph.part + (size_t)u * KB * RPU;
        stride = RPU;
      }
      if (do_fold && c.lane < 16) {
        const int rr = c.lane;
        const int row_a = (NG == 2) ? u * 16 + rr : u * 16 + rr;     // gate row (or the row)
        const int row_b = ph.N / 2 + u * 16 + rr;                     // up row (NG == 2)
        float a0 = 0.f, a1 = 0.f;
        const float swa_c = SCALE == SCALE_CHANNEL ? __ldg(ph.ws + row_a) : 0.f;
        const float swb_c = (SCALE == SCALE_CHANNEL && NG == 2) ? __ldg(ph.ws + row_b) : 0.f;
        for (int kb = 0; kb < KB; ++kb) {
          const float sx = sm.xscale[kb];
          const float da = interior ? src[kb * stride + rr] : __ldcg(src + kb * stride + rr);
          const float swa = SCALE == SCALE_CHANNEL ? swa_c : row_scale<SCALE>(ph.ws, row_a, kb, KB);
          a0 += da * sx * swa;
          if (NG == 2) {
            const float db = interior ? src[kb * stride + 16 + rr] : __ldcg(src + kb * stride + 16 + rr);
            const float swb = SCALE == SCALE_CHANNEL ? swb_c : row_scale<SCALE>(ph.ws, row_b, kb, KB);
            a1 += db * sx * swb;
          }
        }
        // epilogue for this row
        const int row = u * 16 + rr;
        if (EPI == EPI_STORE) {
          ph.out[row] = __float2bfloat16_rn(a0);
        } else if (EPI == EPI_RESIDUAL) {
          ph.out[row] = __float2bfloat16_rn(__bfloat162float(ldcg_bf16(ph.out + row)) + bf16r(a0));
        } else if (EPI == EPI_SWIGLU) {
          const float gt = bf16r(a0);
          const float up = bf16r(a1);
          const float act = bf16r(gt / (1.0f + expf(-gt)));
          ph.out[row] = __float2bfloat16_rn(act * up);
        } else {  // EPI_ARGMAX
          ph.out[row] = __float2bfloat16_rn(a0);
          const float lv = bf16r(a0);
          if (lv > c.best_v || (lv == c.best_v && row < c.best_i)) { c.best_v = lv; c.best_i = row; }
        }
      }
      if (!interior && do_fold && c.lane == 0) ph.counters[u] = 0;
    }
  }
}

// ---- consumer: activation prologue ---------------------------------------------------------------------------
// x (global, K values) -> optional RMSNorm (reference 128-thread reduction order) -> e4m3 per 128-group ->
// f16 fragments in sm.xh + scales in sm.xscale. `embed_row` (layer 0): x is that row of the embedding table
// and this CTA also writes its slice of it into the residual stream.
template <bool NORM>
__device__ void step_prologue(Consumer& c, const bf16* x, const bf16* norm_w, int K, float eps, bf16* resid_slice_dst) {
  StepSmem& sm = *c.sm;
  const int tid = threadIdx.x;
  float rstd = 0.f;
  if (NORM) {   // K == 4096: stage x in shared memory
    for (int i = tid; i < K / 8; i += ST_WARPS * 32)
      reinterpret_cast<uint4*>(sm.u.xs)[i] = ldcg_u4(x + i * 8);
    consumer_sync();
    if (resid_slice_dst) {
      const int per = (K / 8 + gridDim.x - 1) / gridDim.x;
      const int lo = blockIdx.x * per, hi = min(lo + per, K / 8);
      for (int i = lo + tid; i < hi; i += ST_WARPS * 32)
        reinterpret_cast<uint4*>(resid_slice_dst)[i] = reinterpret_cast<const uint4*>(sm.u.xs)[i];
    }
    if (tid < 128) {
      float ss = 0.f;
      for (int i = tid; i < K / 8; i += 128) {
        const uint4 v = reinterpret_cast<const uint4*>(sm.u.xs)[i];
        const bf16* e = reinterpret_cast<const bf16*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float f = __bfloat162float(e[j]);
          ss += f * f;
        }
      }
      ss = warp_sum(ss);
      if (c.lane == 0) sm.red[c.warp] = ss;
    }
    consumer_sync();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) tot += sm.red[i];
    rstd = rsqrtf(tot / (float)K + eps);
  }
  const int KB = K / QB;
  const int ch = c.lane >> 3, hi = (c.lane >> 2) & 1, t = c.lane & 3;
  for (int gq = c.warp; gq < KB; gq += ST_WARPS) {
    const int k0 = gq * QB + c.lane * 4;
    uint2 raw;
    if (NORM) raw = *reinterpret_cast<const uint2*>(sm.u.xs + k0);
    else raw = ldcg_u2(x + k0);
    const bf16* e = reinterpret_cast<const bf16*>(&raw);
    float v[4];
    if (NORM) {
      const uint2 nraw = *reinterpret_cast<const uint2*>(norm_w + k0);
      const bf16* we = reinterpret_cast<const bf16*>(&nraw);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = bf16r(__bfloat162float(we[j]) * bf16r(__bfloat162float(e[j]) * rstd));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = __bfloat162float(e[j]);
    }
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    amax = warp_max(amax);
    const float sc = div_full(amax, 448.0f);
    const uint32_t qv = quant4(v[0], v[1], v[2], v[3], sc);
    uint32_t* dst = sm.xh + ((gq * 4 + ch) * 4 + t) * 4;
    dst[hi] = e4m3x2_to_f16x2(qv);
    dst[2 + hi] = e4m3x2_to_f16x2(qv >> 16);
    if (c.lane == 0) sm.xscale[gq] = sc;
  }
  consumer_sync();
}

// ---- consumer: attention phase ---------------------------------------------------------------------------------
// Per-head RMSNorm + RoPE of 4 values per lane already in registers (the arithmetic of head_norm_rope).
__device__ __forceinline__ void norm_rope_regs(float (&v)[4], const bf16* nw, const bf16* cos_row, const bf16* sin_row,
                                               int lane, float eps, float (&o)[4]) {
  const int d0 = lane * 4;
  const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
  const float rstd = rsqrtf(ss / (float)HEAD_DIM + eps);
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = bf16r(__bfloat162float(nw[d0 + j]) * bf16r(v[j] * rstd));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float partner = __shfl_xor_sync(0xffffffffu, v[j], 16);
    const float rot = (lane < 16) ? -partner : partner;
    o[j] = bf16r(v[j] * __bfloat162float(cos_row[d0 + j])) + bf16r(rot * __bfloat162float(sin_row[d0 + j]));
  }
}

__device__ void attention_phase(Consumer& c, const StepLayer& L, int pos) {
  StepSmem& sm = *c.sm;
  const StepParams& p = *c.p;
  const int tid = threadIdx.x, lane = c.lane, warp = c.warp;
  constexpr int NKV = 8, NQ = 32;
  const AttnItems it = attn_items(pos, NKV);
  const int ctx = pos + 1;
  const bf16* cos_row = p.cos_tab + (size_t)pos * HEAD_DIM;
  const bf16* sin_row = p.sin_tab + (size_t)pos * HEAD_DIM;
  for (int item = it.i0; item < it.i1; ++item) {
    const int kvh = item / it.n_splits, split = item - kvh * it.n_splits;
    const int j0 = split * ST_CHUNK, nj = min(ST_CHUNK, ctx - j0);
    const bool owns_new = (split == it.n_splits - 1);
    const int jn = pos - j0;
    const int sk = c.n % ST_NSTAGE;
    const bool okk = c.wait_stage(sk);
    ++c.n;
    const int sv = c.n % ST_NSTAGE;
    const bool okv = c.wait_stage(sv);
    ++c.n;
    if (!(okk && okv)) atomicOr(&g_dev_error, DEVERR_MBAR_TIMEOUT);
    const bf16* Ks = reinterpret_cast<const bf16*>(sm.ring[sk]);
    const bf16* Vs = reinterpret_cast<const bf16*>(sm.ring[sv]);
    // q of the 4 heads (warps 0-3), new k (warp 4) and v (warp 5) of this kv head
    if (warp < 4) {
      const bf16* src = p.qkv + (kvh * GQA + warp) * HEAD_DIM + lane * 4;
      const uint2 raw = ldcg_u2(src);
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
      float v[4] = {__bfloat162float(e[0]), __bfloat162float(e[1]), __bfloat162float(e[2]), __bfloat162float(e[3])};
      float o[4];
      norm_rope_regs(v, L.q_norm, cos_row, sin_row, lane, p.eps, o);
#pragma unroll
      for (int j = 0; j < 4; ++j) sm.u.at.qs[warp][lane * 4 + j] = bf16r(o[j]);
    } else if (owns_new && warp == 4) {
      const uint2 raw = ldcg_u2(p.qkv + (NQ + kvh) * HEAD_DIM + lane * 4);
      const bf16* e = reinterpret_cast<const bf16*>(&raw);
      float v[4] = {__bfloat162float(e[0]), __bfloat162float(e[1]), __bfloat162float(e[2]), __bfloat162float(e[3])};
      float o[4];
      norm_rope_regs(v, L.k_norm, cos_row, sin_row, lane, p.eps, o);
      bf16* dst = L.k_cache + ((size_t)kvh * p.max_seq + pos) * HEAD_DIM + lane * 4;
      bf16* sdst = const_cast<bf16*>(Ks) + jn * HEAD_DIM + lane * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        dst[j] = __float2bfloat16_rn(o[j]);
        sdst[j] = __float2bfloat16_rn(o[j]);
      }
    } else if (owns_new && warp == 5) {
      const uint2 raw = ldcg_u2(p.qkv + (NQ + NKV + kvh) * HEAD_DIM + lane * 4);
      *reinterpret_cast<uint2*>(L.v_cache + ((size_t)kvh * p.max_seq + pos) * HEAD_DIM + lane * 4) = raw;
      *reinterpret_cast<uint2*>(const_cast<bf16*>(Vs) + jn * HEAD_DIM + lane * 4) = raw;
    }
    consumer_sync();
    // scores: thread (key j = tid/4, head h = tid%4): dims 0..63 then 64..127, each summed in order
    {
      const int j = tid >> 2, hh = tid & 3;
      float sfin = -INFINITY;
      if (j < nj) {
        float part[2];
#pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
          float dot = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 kv = lds128(Ks + j * HEAD_DIM + sl * 64 + i * 8);
            const bf16* e = reinterpret_cast<const bf16*>(&kv);
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) dot += sm.u.at.qs[hh][sl * 64 + i * 8 + jj] * __bfloat162float(e[jj]);
          }
          part[sl] = dot;
        }
        float s = part[0];
        s += part[1];
        sfin = s * p.attn_scale;
      }
      sm.u.at.sc[hh][j] = sfin;
    }
    consumer_sync();
    if (warp < 4) {  // softmax over the chunk, one warp per query head
      float pr[2];
      float m = -INFINITY;
#pragma unroll
      for (int i = 0; i < 2; ++i) { pr[i] = sm.u.at.sc[warp][lane + 32 * i]; m = fmaxf(m, pr[i]); }
      m = warp_max(m);
      float l = 0.f;
#pragma unroll
      for (int i = 0; i < 2; ++i) { pr[i] = expf(pr[i] - m); l += pr[i]; sm.u.at.sc[warp][lane + 32 * i] = pr[i]; }
      l = warp_sum(l);
      if (lane == 0) { sm.u.at.m_s[warp] = m; sm.u.at.l_s[warp] = l; }
    }
    consumer_sync();
    // P @ V: thread (d = tid % 128, heads 2*(tid/128) + {0,1})
    {
      const int d = tid & 127, h0 = (tid >> 7) * 2;
      float acc0 = 0.f, acc1 = 0.f;
      for (int j = 0; j < nj; ++j) {
        const float vf = __bfloat162float(Vs[j * HEAD_DIM + d]);
        acc0 += sm.u.at.sc[h0][j] * vf;
        acc1 += sm.u.at.sc[h0 + 1][j] * vf;
      }
      const size_t row0 = (size_t)(kvh * GQA + h0) * p.max_splits + split;
      const size_t row1 = row0 + p.max_splits;
      p.o_part[row0 * HEAD_DIM + d] = acc0;
      p.o_part[row1 * HEAD_DIM + d] = acc1;
      if (d == 0) {
        p.ml_part[row0 * 2 + 0] = sm.u.at.m_s[h0];
        p.ml_part[row0 * 2 + 1] = sm.u.at.l_s[h0];
        p.ml_part[row1 * 2 + 0] = sm.u.at.m_s[h0 + 1];
        p.ml_part[row1 * 2 + 1] = sm.u.at.l_s[h0 + 1];
      }
    }
    c.release_stage(sk);
    c.release_stage(sv);
    __threadfence();
    consumer_sync();
    if (tid == 0) sm.flag = (atomicAdd(p.attn_counters + kvh, 1) == it.n_splits - 1);
    consumer_sync();
    if (sm.flag) {  // the last item of this kv head merges its splits
      __threadfence();
      if (warp < 4) {
        const float* ml = p.ml_part + (size_t)(kvh * GQA + warp) * p.max_splits * 2;
        float mloc = -INFINITY;
        for (int s = lane; s < it.n_splits; s += 32) mloc = fmaxf(mloc, __ldcg(ml + 2 * s));
        const float M = warp_max(mloc);
        float lsum = 0.f;
        for (int s = lane; s < it.n_splits; s += 32) {
          const float wgt = expf(__ldcg(ml + 2 * s) - M);
          sm.u.at.cw[warp][s] = wgt;
          lsum += wgt * __ldcg(ml + 2 * s + 1);
        }
        lsum = warp_sum(lsum);
        if (lane == 0) sm.u.at.cl[warp] = lsum;
      }
      consumer_sync();
      const int d = tid & 127, h0 = (tid >> 7) * 2;
      float o0 = 0.f, o1 = 0.f;
      const float* op0 = p.o_part + (size_t)(kvh * GQA + h0) * p.max_splits * HEAD_DIM + d;
      const float* op1 = op0 + (size_t)p.max_splits * HEAD_DIM;
#pragma unroll 8
      for (int s = 0; s < it.n_splits; ++s) {
        o0 += sm.u.at.cw[h0][s] * __ldcg(op0 + (size_t)s * HEAD_DIM);
        o1 += sm.u.at.cw[h0 + 1][s] * __ldcg(op1 + (size_t)s * HEAD_DIM);
      }
      p.attn[(kvh * GQA + h0) * HEAD_DIM + d] = __float2bfloat16_rn(o0 / sm.u.at.cl[h0]);
      p.attn[(kvh * GQA + h0 + 1) * HEAD_DIM + d] = __float2bfloat16_rn(o1 / sm.u.at.cl[h0 + 1]);
      if (tid == 0) p.attn_counters[kvh] = 0;
    }
    consumer_sync();
  }
}

// ---- the kernel -------------------------------------------------------------------------------------------------
template <int SCALE>
__global__ void __launch_bounds__(ST_THREADS, 1) decode_step_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  StepSmem& sm = *reinterpret_cast<StepSmem*>(smem_raw);
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
    fence_mbar_init();
  }
  __syncthreads();
  constexpr int H = HIDDEN, I = 12288, QKV_N = 6144;
  if (warp == ST_WARPS) {   // ---------------- producer ----------------
    if (lane == 0) {
      Producer pr{&sm, 0, policy_evict_first(), true};
      const AttnItems it = attn_items(pos, 8);
      for (int l = 0; l < p.n_layers; ++l) {
        const StepLayer& L = p.layers[l];
        pr.gemv(L.w_qkv, (QKV_N / 16) * (H / QB));
        for (int item = it.i0; item < it.i1; ++item) {
          const int kvh = item / it.n_splits, split = item - kvh * it.n_splits;
          const int j0 = split * ST_CHUNK, nj = min(ST_CHUNK, pos + 1 - j0);
          const size_t off = ((size_t)kvh * p.max_seq + j0) * HEAD_DIM;
          pr.push(L.k_cache + off, (uint32_t)(nj * HEAD_DIM * 2));
          pr.push(L.v_cache + off, (uint32_t)(nj * HEAD_DIM * 2));
        }
        pr.gemv(L.w_o, (H / 16) * (H / QB));
        pr.gemv(L.w_gu, (2 * I / 16) * (H / QB));
        pr.gemv(L.w_down, (H / 16) * (I / QB));
      }
      pr.gemv(p.w_head, (p.vocab / 16) * (H / QB));
    }
    return;
  }
  // ---------------- consumers ----------------
  Consumer c{&sm, &p, 0, lane, warp, lane >> 2, lane & 3, -INFINITY, 0x7FFFFFFF};
  unsigned nbar = 0;
  const int tok = p.token[0];
  const bool tok_ok = tok >= 0 && tok < p.vocab;
  if (!tok_ok && threadIdx.x == 0 && blockIdx.x == 0) atomicOr(&g_dev_error, DEVERR_BAD_STATE);
  for (int l = 0; l < p.n_layers; ++l) {
    const StepLayer& L = p.layers[l];
    // QKV
    if (l == 0) step_prologue<true>(c, p.embed + (size_t)(tok_ok ? tok : 0) * H, L.ln1, H, p.eps, p.resid);
    else step_prologue<true>(c, p.resid, L.ln1, H, p.eps, nullptr);
    gemv_phase(c, GemvPhase<EPI_STORE, SCALE, 1>{L.s_qkv, QKV_N, H, p.qkv, p.part, p.counters});
    grid_barrier(p.sync, nbar++);
    // ATTN (writes K/V rows at pos and the merged attention output)
    attention_phase(c, L, pos);
    grid_barrier(p.sync, nbar++);
    // O: resid += W_o . quant(attn)
    step_prologue<false>(c, p.attn, nullptr, H, p.eps, nullptr);
    gemv_phase(c, GemvPhase<EPI_RESIDUAL, SCALE, 1>{L.s_o, H, H, p.resid, p.part, p.counters});
    grid_barrier(p.sync, nbar++);
    // GU: h = SwiGLU(W_gu . quant(RMSNorm(resid)))
    step_prologue<true>(c, p.resid, L.ln2, H, p.eps, nullptr);
    gemv_phase(c, GemvPhase<EPI_SWIGLU, SCALE, 2>{L.s_gu, 2 * I, H, p.h, p.part, p.counters});
    grid_barrier(p.sync, nbar++);
    // DOWN: resid += W_down . quant(h)
    step_prologue<false>(c, p.h, nullptr, I, p.eps, nullptr);
    gemv_phase(c, GemvPhase<EPI_RESIDUAL, SCALE, 1>{L.s_down, H, I, p.resid, p.part, p.counters});
    grid_barrier(p.sync, nbar++);
  }
  // HEAD: logits + greedy argmax (FP8 per-channel head)
  step_prologue<true>(c, p.resid, p.final_norm, H, p.eps, nullptr);
  gemv_phase(c, GemvPhase<EPI_ARGMAX, SCALE_CHANNEL, 1>{p.s_head, p.vocab, H, p.logits, p.part, p.counters});
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
        const unsigned long long k = atomicAdd(p.best, 0ull);
        const int next = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        p.token[0] = next;
        const int step = p.state[1];
        if (step >= 0 && step < p.out_len) p.out_tokens[step] = next;
        p.state[0] = pos + 1;
        p.state[1] = step + 1;
        *p.best = 0ull;
        p.sync[0] = 0;
        p.sync[1] = 0;
        __threadfence();
      }
    }
  }
}

}  // namespace qk
