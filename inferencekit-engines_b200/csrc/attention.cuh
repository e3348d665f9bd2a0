// Decode attention for one new token per sequence: q/k RMSNorm + RoPE, KV-cache append, GQA split-KV
// attention over a bf16 cache, split merge. Two kernels per call (the second launched with programmatic
// dependent launch):
//
//  attn_partials_kernel<CHUNK>   grid (n_kv * key blocks, batch), 256 threads. A CTA owns one block of 128
//    consecutive keys of one (sequence, KV head): 128/CHUNK reference splits. Its K and V rows arrive by four
//    TMA box loads ({64 dims, 128 keys}, 128-byte swizzle, issued before griddepcontrol.wait: they are earlier
//    tokens' rows) so that 8 keys read at the same dims hit 8 different bank groups. After the wait the four
//    query heads of the KV head are normalised and rotated (one warp each); the CTA whose block holds `pos`
//    also writes the new K (normalised + rotated) and V rows to the cache and into its shared copy. Then
//    thread = (key, pair of query heads) computes the scores, one warp per (split, head) row takes the
//    softmax (fp32 probabilities), thread = (dim, pair of heads) computes P @ V for every split, and each
//    split's unnormalised partial (m, l, o[128]) goes to o_part / ml_part.
//  attn_merge_kernel             grid (2 * n_q, batch), 128 threads: CTA (query head, 64-dim half) combines
//    that head's split partials: M = max m_s, w_s = exp(m_s - M), out = bf16(sum_s w_s o_s / sum_s w_s l_s).
//
// Numerics: for CHUNK in {32, 64, 128} every sum runs in the order of the reference decode kernel
// (Q/kernels/decode.cu:343-360 head norm + RoPE, :462-527 scores / softmax / P@V per CHUNK-key split,
// :537-567 merge): a score is the in-order dot over each CHUNK-wide slice of the head dims, slices added left
// to right; probabilities and sums stay fp32; the merge sums over splits in split order. Cache rows and outputs
// are therefore bit-identical to the reference kernel's for the same CHUNK. The number of splits is bounded
// only by the caller's o_part (max_splits), not by a compile-time constant.
#pragma once
#include <cuda.h>   // CUtensorMap
#include "common.cuh"

namespace qk {

constexpr int ATT_KEYS = 128;          // keys per partials CTA (the rows of one TMA box)
constexpr int ATT_THREADS = 256;      // partials: thread = (key or dim, pair of query heads)
constexpr int ATT_MERGE_THREADS = 128;
constexpr int ATT_MERGE_ROUND = 128;   // splits staged per round of the merge

struct AttnParams {
  CUtensorMap tm_k, tm_v;    // K / V cache of the layer: bf16 {128 dims, max_seq, n_kv, batch}, box {64, 128}
  const bf16* qkv;           // [B][qkv_stride]: q heads | k heads | v heads, 128 each
  const bf16* q_norm_w;      // [128]
  const bf16* k_norm_w;      // [128]
  const bf16* cos_tab;       // [max_seq, 128]
  const bf16* sin_tab;
  const int* state;          // per sequence: state[b * state_stride] = pos
  bf16* k_cache;             // [B][n_kv][max_seq][128] (one layer)
  bf16* v_cache;
  float* o_part;             // [B][n_q][max_splits][128]
  float* ml_part;            // [B][n_q][max_splits][2]
  bf16* out;                 // [B][n_q * 128]
  int n_kv, max_seq, max_splits, qkv_stride, state_stride, chunk;
  float scale, eps;
  int tl_slot;               // timeline region of this call, -1 when off (words 0-2 partials, 3-4 merge)
};

// Byte offset of (key r, dim d) in a swizzled K or V block: dims 0-63 in the first 16 KiB box, 64-127 in the
// second; 16-byte chunk c of a 128-byte row r sits at chunk c ^ (r % 8).
__device__ __forceinline__ uint32_t att_off(int r, int d) {
  return (uint32_t)((d >> 6) * (ATT_KEYS * 128) + r * 128 + ((((d & 63) >> 3) ^ (r & 7)) << 4) + (d & 7) * 2);
}

// Per-head RMSNorm (eps) + RoPE of one head held as 4 values per lane (dims 4*lane .. 4*lane+3): the sum of
// squares over the warp, each step rounded to bf16 as the reference forward does (Q/model.py:121-130, :265-266),
// the rotation partner of dim d being d +- 64 (lane ^ 16). Shared with the fused step.
__device__ __forceinline__ void head_norm_rope(float (&v)[4], const bf16* nw, const bf16* cos_row, const bf16* sin_row,
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
// The same from 4 bf16 values at `src` (global memory written by an earlier kernel or phase, read through L2).
__device__ __forceinline__ void head_norm_rope_from(const bf16* src, const bf16* nw, const bf16* cos_row,
                                                    const bf16* sin_row, int lane, float eps, float (&o)[4]) {
  uint2 raw;
  asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(raw.x), "=r"(raw.y) : "l"(src + lane * 4));
  float v[4] = {bf16lo(raw.x), bf16hi(raw.x), bf16lo(raw.y), bf16hi(raw.y)};
  head_norm_rope(v, nw, cos_row, sin_row, lane, eps, o);
}

struct AttnSmem {
  uint8_t k[2 * ATT_KEYS * 128];         // swizzled K block (two 16 KiB boxes)
  uint8_t v[2 * ATT_KEYS * 128];         // swizzled V block
  float q[GQA][HEAD_DIM];                // the 4 query heads after norm + RoPE (bf16 values)
  float p[GQA][ATT_KEYS];                // scores, then probabilities, per head and key of the block
  float m[ATT_KEYS / 32][GQA], l[ATT_KEYS / 32][GQA];   // per (split of the block, head)
  uint64_t bar;
};

template <int CHUNK>
__global__ void __launch_bounds__(ATT_THREADS) attn_partials_kernel(const __grid_constant__ AttnParams p) {
  constexpr int NSPLIT = ATT_KEYS / CHUNK;         // reference splits per block
  constexpr int PER_LANE = CHUNK / 32;             // softmax values per lane
  extern __shared__ __align__(1024) uint8_t att_smem[];
  AttnSmem& sm = *reinterpret_cast<AttnSmem*>(att_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_blocks = (p.max_seq + ATT_KEYS - 1) / ATT_KEYS;
  const int kvh = blockIdx.x / n_blocks, blk = blockIdx.x - kvh * n_blocks, b = blockIdx.y;
  const int n_q = p.n_kv * GQA;
  const int pos = p.state[(size_t)b * p.state_stride];   // written by the previous step's finalize
  if (pos < 0 || pos >= p.max_seq) {
    if (tid == 0 && blk == 0 && kvh == 0) atomicOr(&g_dev_error, DEVERR_BAD_STATE);
    return;
  }
  const int ctx = pos + 1, key0 = blk * ATT_KEYS;
  if (key0 >= ctx) return;    // a block past the context (the grid covers max_seq): nothing to do
  if (tid == 0) {
    tl_stamp(p.tl_slot, 0);
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&sm.bar, 4 * ATT_KEYS * 128);
    tma_load_4d(sm.k, &p.tm_k, 0, key0, kvh, b, &sm.bar);
    tma_load_4d(sm.k + ATT_KEYS * 128, &p.tm_k, 64, key0, kvh, b, &sm.bar);
    tma_load_4d(sm.v, &p.tm_v, 0, key0, kvh, b, &sm.bar);
    tma_load_4d(sm.v + ATT_KEYS * 128, &p.tm_v, 64, key0, kvh, b, &sm.bar);
  }
  __syncthreads();            // the barrier's initialisation is visible to every thread
  grid_dep_wait();            // qkv comes from the kernel before
  if (tid == 0) tl_stamp(p.tl_slot, 1);
  const bf16* qkv = p.qkv + (size_t)b * p.qkv_stride;
  const bf16* cos_row = p.cos_tab + (size_t)pos * HEAD_DIM;
  const bf16* sin_row = p.sin_tab + (size_t)pos * HEAD_DIM;
  const bool owns_new = pos - key0 < ATT_KEYS;
  bool ok = true;
  if (warp < GQA) {           // warp h: query head 4*kvh + h
    float o[4];
    head_norm_rope_from(qkv + (size_t)(kvh * GQA + warp) * HEAD_DIM, p.q_norm_w, cos_row, sin_row, lane, p.eps, o);
#pragma unroll
    for (int j = 0; j < 4; ++j) sm.q[warp][lane * 4 + j] = bf16r(o[j]);
  } else if (owns_new && warp < GQA + 2) {
    // the new token's K (warp 4: normalised + rotated) and V (warp 5) rows: cache slot `pos`, and the copy here
    // once the block's TMA load has landed
    const int r = pos - key0;
    const size_t row = (((size_t)b * p.n_kv + kvh) * p.max_seq + pos) * HEAD_DIM + lane * 4;
    if (warp == GQA) {
      float o[4];
      head_norm_rope_from(qkv + (size_t)(n_q + kvh) * HEAD_DIM, p.k_norm_w, cos_row, sin_row, lane, p.eps, o);
      bf16 kb[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) kb[j] = __float2bfloat16_rn(o[j]);
      *reinterpret_cast<uint2*>(p.k_cache + row) = *reinterpret_cast<const uint2*>(kb);
      ok = mbar_wait(&sm.bar, 0);
      *reinterpret_cast<uint2*>(sm.k + att_off(r, lane * 4)) = *reinterpret_cast<const uint2*>(kb);
    } else {
      uint2 raw;
      const bf16* src = qkv + (size_t)(n_q + p.n_kv + kvh) * HEAD_DIM + lane * 4;
      asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(raw.x), "=r"(raw.y) : "l"(src));
      *reinterpret_cast<uint2*>(p.v_cache + row) = raw;
      ok = mbar_wait(&sm.bar, 0);
      *reinterpret_cast<uint2*>(sm.v + att_off(r, lane * 4)) = raw;
    }
  }
  ok = mbar_wait(&sm.bar, 0) && ok;
  __syncthreads();

  // scores: thread = (key j of the block, query heads 2*hp, 2*hp+1); per head the CHUNK-dim slices summed in
  // order, then added left to right
  {
    const int j = tid & (ATT_KEYS - 1), hp = tid / ATT_KEYS, sp = j / CHUNK, split = key0 / CHUNK + sp;
    const bool valid = j - sp * CHUNK < min(CHUNK, ctx - split * CHUNK);
    float total[2];
#pragma unroll
    for (int sl = 0; sl < HEAD_DIM / CHUNK; ++sl) {
      float d[2] = {0.f, 0.f};
#pragma unroll 4
      for (int i = 0; i < CHUNK / 8; ++i) {
        const int d0 = sl * CHUNK + i * 8;
        const uint4 kv = lds128(sm.k + att_off(j, d0));
        const float kf[8] = {bf16lo(kv.x), bf16hi(kv.x), bf16lo(kv.y), bf16hi(kv.y),
                             bf16lo(kv.z), bf16hi(kv.z), bf16lo(kv.w), bf16hi(kv.w)};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float4 qa = *reinterpret_cast<const float4*>(&sm.q[2 * hp + h][d0]);
          const float4 qb = *reinterpret_cast<const float4*>(&sm.q[2 * hp + h][d0 + 4]);
          d[h] += qa.x * kf[0];
          d[h] += qa.y * kf[1];
          d[h] += qa.z * kf[2];
          d[h] += qa.w * kf[3];
          d[h] += qb.x * kf[4];
          d[h] += qb.y * kf[5];
          d[h] += qb.z * kf[6];
          d[h] += qb.w * kf[7];
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) total[h] = sl == 0 ? d[h] : total[h] + d[h];
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) sm.p[2 * hp + h][j] = valid ? total[h] * p.scale : -INFINITY;
  }
  __syncthreads();
  // softmax: one warp per (split, head) row of CHUNK scores
  const int n_splits = (ctx + CHUNK - 1) / CHUNK;
  for (int r = warp; r < NSPLIT * GQA; r += ATT_THREADS / 32) {
    const int sp = r / GQA, h = r - sp * GQA;
    if (key0 / CHUNK + sp >= n_splits) continue;
    float* row = &sm.p[h][sp * CHUNK];
    float pr[PER_LANE];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      pr[i] = row[lane + 32 * i];
      mx = fmaxf(mx, pr[i]);
    }
    mx = warp_max(mx);
    float ls = 0.f;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      pr[i] = expf(pr[i] - mx);
      ls += pr[i];
      row[lane + 32 * i] = pr[i];
    }
    ls = warp_sum(ls);
    if (lane == 0) {
      sm.m[sp][h] = mx;
      sm.l[sp][h] = ls;
    }
  }
  __syncthreads();
  // P @ V: thread = (output dim d, query heads 2*hp, 2*hp+1), every split of the block; keys in order
  {
    const int d = tid & (HEAD_DIM - 1), hp = tid / HEAD_DIM;
#pragma unroll
    for (int sp = 0; sp < NSPLIT; ++sp) {
      const int split = key0 / CHUNK + sp;
      if (split >= n_splits) break;
      const int nj = min(CHUNK, ctx - split * CHUNK);
      float acc[2] = {0.f, 0.f};
      for (int j = 0; j < nj; ++j) {
        const int r = sp * CHUNK + j;
        const float vf = __bfloat162float(*reinterpret_cast<const bf16*>(sm.v + att_off(r, d)));
#pragma unroll
        for (int h = 0; h < 2; ++h) acc[h] += sm.p[2 * hp + h][r] * vf;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const size_t row = ((size_t)b * n_q + kvh * GQA + 2 * hp + h) * p.max_splits + split;
        p.o_part[row * HEAD_DIM + d] = acc[h];
        if (d == 0) {
          p.ml_part[row * 2 + 0] = sm.m[sp][2 * hp + h];
          p.ml_part[row * 2 + 1] = sm.l[sp][2 * hp + h];
        }
      }
    }
  }
  if (!ok && tid == 0) atomicOr(&g_dev_error, DEVERR_MBAR_TIMEOUT);
  if (tid == 0) tl_stamp(p.tl_slot, 2);
  grid_dep_launch();          // the merge kernel may start; it waits for this grid's completion and writes
}

// Merge of one query head's split partials, dims [64 * half, 64 * half + 64): warp 0 takes the max of the
// split maxima and the weights w_s = exp(m_s - M) and their l-weighted sum (lane-strided over the splits, then a
// butterfly, as the reference); all warps stage the partial rows in shared memory (cp.async, rounds of
// ATT_MERGE_ROUND splits) and threads 0-63 sum w_s * o_s[d] over the splits in order.
struct MergeSmem {
  float o[ATT_MERGE_ROUND * 64];
  float cl;
  // followed by w[max_splits] (dynamic)
};

__global__ void __launch_bounds__(ATT_MERGE_THREADS) attn_merge_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) uint8_t mg_smem[];
  MergeSmem& sm = *reinterpret_cast<MergeSmem*>(mg_smem);
  float* w = reinterpret_cast<float*>(mg_smem + sizeof(MergeSmem));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qh = blockIdx.x >> 1, half = blockIdx.x & 1, b = blockIdx.y;
  const int n_q = p.n_kv * GQA;
  const int pos = p.state[(size_t)b * p.state_stride];
  grid_dep_wait();            // every partial of this call is written
  grid_dep_launch();
  if (pos < 0 || pos >= p.max_seq) return;   // reported by the partials kernel
  if (tid == 0 && qh == 0 && half == 0) tl_stamp(p.tl_slot, 3);
  const int n_splits = (pos + p.chunk) / p.chunk;
  const size_t hrow = ((size_t)b * n_q + qh) * p.max_splits;
  if (warp == 0) {
    const float* ml = p.ml_part + hrow * 2;
    float mloc = -INFINITY;
    for (int s = lane; s < n_splits; s += 32) mloc = fmaxf(mloc, __ldcg(ml + 2 * s));
    const float M = warp_max(mloc);
    float lsum = 0.f;
    for (int s = lane; s < n_splits; s += 32) {
      const float wt = expf(__ldcg(ml + 2 * s) - M);
      w[s] = wt;
      lsum += wt * __ldcg(ml + 2 * s + 1);
    }
    lsum = warp_sum(lsum);
    if (lane == 0) sm.cl = lsum;
  }
  const float* op = p.o_part + hrow * HEAD_DIM + half * 64;
  float acc = 0.f;
  for (int s0 = 0; s0 < n_splits; s0 += ATT_MERGE_ROUND) {
    const int ns = min(ATT_MERGE_ROUND, n_splits - s0);
    for (int i = tid; i < ns * 16; i += ATT_MERGE_THREADS) {   // 16 x 16 bytes per split row of 64 dims
      const int s = i >> 4, f = i & 15;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(&sm.o[s * 64 + f * 4])),
                   "l"(op + (size_t)(s0 + s) * HEAD_DIM + f * 4)
                   : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    if (tid < 64) {
      for (int s = 0; s < ns; ++s) acc += w[s0 + s] * sm.o[s * 64 + tid];
    }
    __syncthreads();
  }
  if (tid < 64) p.out[(size_t)b * n_q * HEAD_DIM + qh * HEAD_DIM + half * 64 + tid] = __float2bfloat16_rn(acc / sm.cl);
  if (tid == 0 && qh == 0 && half == 0) tl_stamp(p.tl_slot, 4);
}

inline size_t attn_partials_smem_bytes() { return sizeof(AttnSmem); }
inline size_t attn_merge_smem_bytes(int max_splits) { return sizeof(MergeSmem) + (size_t)max_splits * 4; }

// ---- step bookkeeping ----------------------------------------------------------------------------------------
// resid[b] = table[token[b]]   (512 threads x 16 bytes = one 4096-wide bf16 row per sequence)
__global__ void __launch_bounds__(512) embed_kernel(const int* __restrict__ token, const bf16* __restrict__ table,
                                                    bf16* __restrict__ resid, int vocab) {
  grid_dep_wait();
  grid_dep_launch();
  int tok = token[blockIdx.x];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) atomicOr(&g_dev_error, DEVERR_BAD_STATE);
    tok = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)tok * HIDDEN);
  reinterpret_cast<uint4*>(resid + (size_t)blockIdx.x * HIDDEN)[threadIdx.x] = src[threadIdx.x];
}

// Decode the argmax key into the next token, record it, advance the step state [pos, step], clear the key.
// resid[i] = bf16(resid[i] + bf16(sum[i])): the residual update of a row-parallel layer after its all-reduce
// (the same rounding as the in-place residual epilogue, decode.cu:320-323).
__global__ void residual_add_kernel(bf16* __restrict__ resid, const float* __restrict__ sum, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) resid[i] = __float2bfloat16_rn(__bfloat162float(resid[i]) + bf16r(sum[i]));
}

// Flip the top bit of packed argmax keys: unsigned key order <-> signed 64-bit order, so a signed MAX
// reduction (NCCL int64) picks the same key as the unsigned atomicMax.
__global__ void key_flip_kernel(unsigned long long* __restrict__ keys, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) keys[i] ^= 0x8000000000000000ull;
}

__global__ void finalize_kernel(unsigned long long* __restrict__ best, int* __restrict__ token,
                                int* __restrict__ out_tokens, int* __restrict__ state, int out_len) {
  grid_dep_wait();
  grid_dep_launch();
  const int b = blockIdx.x;
  const unsigned long long k = best[b];
  const int tok = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
  token[b] = tok;
  const int step = state[2 * b + 1];
  if (step >= 0 && step < out_len) out_tokens[(size_t)b * out_len + step] = tok;
  state[2 * b + 0] += 1;
  state[2 * b + 1] += 1;
  best[b] = 0ull;
}

}  // namespace qk
