// Decode attention for one token per sequence: q/k RMSNorm + RoPE, KV-cache append, GQA split-KV
// ("flash-decoding") attention, in-kernel merge of the splits.
//
// Grid (kv_head, split, sequence), 128 threads. A CTA owns CHUNK keys of one KV head and its 4 query heads.
//  * Before griddepcontrol.wait (the qkv GEMV may still be running) the CTA loads its cached keys into
//    registers (16-byte loads, one key per CHUNK threads' slice) and issues one bulk async copy of its
//    cached values into shared memory. Those rows were written by earlier steps.
//  * After the wait: 4 warps RMS-normalise + rotate the 4 query heads; the CTA whose chunk holds the new
//    position normalises + rotates the new key and writes K and V into the cache slot `pos` (exactly one
//    slot per KV head per token), and patches its shared copies.
//  * fp32 scores, softmax over the chunk (probabilities stay fp32), P @ V, and the unnormalised partial
//    (m, l, o) per query head to `o_part` / `ml_part`. The last CTA of a KV head (atomic counter) merges
//    the splits and resets the counter.
// The arithmetic is in the same order as the reference decode kernel (decode.cu:343-360, :462-567) for
// the same CHUNK, so cache rows and outputs are bit-identical to it; the number of splits is not bounded
// by a compile-time constant (long contexts), only by `max_splits` of the scratch the caller passes.
#pragma once
#include "common.cuh"

namespace qk {

struct AttnParams {
  const bf16* qkv;           // [B][qkv_stride]: q heads | k heads | v heads of this rank, 128 each
  const bf16* q_norm_w;      // [128]
  const bf16* k_norm_w;      // [128]
  const bf16* cos_tab;       // [max_seq, 128]
  const bf16* sin_tab;
  const int* state;          // per sequence: state[b * state_stride] = pos
  bf16* k_cache;             // [B][n_kv][max_seq][128] (one layer)
  bf16* v_cache;
  float* o_part;             // [B][n_q][max_splits][128]
  float* ml_part;            // [B][n_q][max_splits][2]
  int* counters;             // [B][n_kv], zero between launches
  bf16* out;                 // [B][n_q * 128]
  int max_seq, max_splits, qkv_stride, state_stride;
  float scale, eps;
  int tl_slot;               // timeline region of this launch, -1 when off
};

// Per-head RMSNorm (eps) + RoPE (rotate_half pairs d and d+64 = lane l and l^16), one warp, 4 dims per
// lane, each step rounded to bf16 as in the reference forward (model.py:121-125, :265-266).
__device__ __forceinline__ void head_norm_rope(const bf16* __restrict__ src, const bf16* __restrict__ nw,
                                               const bf16* __restrict__ cos_row, const bf16* __restrict__ sin_row,
                                               int lane, float eps, float (&o)[4]) {
  const int d0 = lane * 4;
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = __bfloat162float(src[d0 + j]);
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

template <int CHUNK>
struct AttnSmem {
  static constexpr int TPK = HEAD_DIM / CHUNK;
  float qs[GQA][HEAD_DIM];
  float sc[GQA][CHUNK];
  float part[TPK > 1 ? TPK - 1 : 1][GQA][CHUNK];
  __align__(16) bf16 vs[CHUNK][HEAD_DIM];
  __align__(16) bf16 knew[HEAD_DIM];
  float m_s[GQA], l_s[GQA], cl[GQA];
  uint64_t vbar;
  int is_last;
  // followed by cw[GQA][max_splits] floats (dynamic)
};

template <int CHUNK>
__global__ void __launch_bounds__(128) attention_kernel(const __grid_constant__ AttnParams p) {
  constexpr int TPK = HEAD_DIM / CHUNK;    // threads per key
  constexpr int DPT = HEAD_DIM / TPK;      // dims per thread in the score dot
  constexpr int PER_LANE = CHUNK / 32;     // softmax values per lane
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem<CHUNK>& sm = *reinterpret_cast<AttnSmem<CHUNK>*>(smem_raw);
  float* cw = reinterpret_cast<float*>(smem_raw + ((sizeof(AttnSmem<CHUNK>) + 15) / 16) * 16);

  const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
  const int n_kv = gridDim.x, n_q = n_kv * GQA;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = p.state[b * p.state_stride];   // written by the previous step's last kernel
  if (pos < 0 || pos >= p.max_seq) {
    if (tid == 0 && split == 0) atomicOr(&g_dev_error, DEVERR_BAD_STATE);
    return;
  }
  const int ctx = pos + 1;
  const int n_splits = (ctx + CHUNK - 1) / CHUNK;
  if (split >= n_splits) return;
  const int j0 = split * CHUNK;
  const int nj = min(CHUNK, ctx - j0);
  const bool owns_new = (split == n_splits - 1);
  const int jn = pos - j0;

  const size_t head_base = ((size_t)b * n_kv + kvh) * p.max_seq;
  const bf16* kb = p.k_cache + (head_base + j0) * HEAD_DIM;
  const bf16* vb = p.v_cache + (head_base + j0) * HEAD_DIM;
  const int key = tid % CHUNK, slice = tid / CHUNK;
  const bool is_new = owns_new && key == jn;

  // ---- 1. cached K -> registers, cached V -> shared memory (bulk copy), before the wait ----
  uint4 kr[DPT / 8];
  if (key < nj && !is_new) {
#pragma unroll
    for (int i = 0; i < DPT / 8; ++i) kr[i] = ldg_stream(kb + key * HEAD_DIM + slice * DPT + i * 8);
  }
  if (tid == 0) {
    tl_stamp(p.tl_slot, 0);
    mbar_init(&sm.vbar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&sm.vbar, (uint32_t)(nj * HEAD_DIM * 2));
    bulk_g2s(&sm.vs[0][0], vb, (uint32_t)(nj * HEAD_DIM * 2), &sm.vbar);
  }
  grid_dep_wait();
  grid_dep_launch();
  if (tid == 0) tl_stamp(p.tl_slot, 1);
  __syncthreads();                          // barrier init visible to all threads
  const bool v_ok = mbar_wait(&sm.vbar, 0); // the copy must land before the new row is patched in

  // ---- 2. q (and the new k, v): norm + RoPE; KV append ----
  const bf16* qkv = p.qkv + (size_t)b * p.qkv_stride;
  const bf16* cos_row = p.cos_tab + (size_t)pos * HEAD_DIM;
  const bf16* sin_row = p.sin_tab + (size_t)pos * HEAD_DIM;
  {
    float o[4];
    head_norm_rope(qkv + (kvh * GQA + warp) * HEAD_DIM, p.q_norm_w, cos_row, sin_row, lane, p.eps, o);
#pragma unroll
    for (int j = 0; j < 4; ++j) sm.qs[warp][lane * 4 + j] = bf16r(o[j]);
  }
  if (owns_new && warp == 0) {
    float o[4];
    head_norm_rope(qkv + (n_q + kvh) * HEAD_DIM, p.k_norm_w, cos_row, sin_row, lane, p.eps, o);
    bf16* dst = p.k_cache + (head_base + pos) * HEAD_DIM + lane * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      dst[j] = __float2bfloat16_rn(o[j]);
      sm.knew[lane * 4 + j] = __float2bfloat16_rn(o[j]);
    }
  } else if (owns_new && warp == 1) {
    const bf16* src = qkv + (n_q + n_kv + kvh) * HEAD_DIM + lane * 4;
    bf16* dst = p.v_cache + (head_base + pos) * HEAD_DIM + lane * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      dst[j] = src[j];
      sm.vs[jn][lane * 4 + j] = src[j];
    }
  }
  __syncthreads();

  // ---- 3. scores: thread (key, slice) sums DPT dims in order for all 4 heads ----
  float dot[GQA] = {0.f, 0.f, 0.f, 0.f};
  if (key < nj) {
    if (is_new) {
#pragma unroll
      for (int i = 0; i < DPT / 8; ++i) kr[i] = *reinterpret_cast<const uint4*>(sm.knew + slice * DPT + i * 8);
    }
#pragma unroll
    for (int i = 0; i < DPT / 8; ++i) {
      const bf16* e = reinterpret_cast<const bf16*>(&kr[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float kf = __bfloat162float(e[j]);
#pragma unroll
        for (int h = 0; h < GQA; ++h) dot[h] += sm.qs[h][slice * DPT + i * 8 + j] * kf;
      }
    }
  }
  if (TPK > 1 && slice > 0) {
#pragma unroll
    for (int h = 0; h < GQA; ++h) sm.part[slice - 1][h][key] = dot[h];
  }
  if (TPK > 1) __syncthreads();
  if (slice == 0) {
#pragma unroll
    for (int h = 0; h < GQA; ++h) {
      float s = dot[h];
#pragma unroll
      for (int q = 0; q + 1 < TPK; ++q) s += sm.part[q][h][key];
      sm.sc[h][key] = (key < nj) ? s * p.scale : -INFINITY;
    }
  }
  __syncthreads();

  {  // softmax over the chunk, one warp per query head
    float pr[PER_LANE];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) { pr[i] = sm.sc[warp][lane + 32 * i]; m = fmaxf(m, pr[i]); }
    m = warp_max(m);
    float l = 0.f;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) { pr[i] = expf(pr[i] - m); l += pr[i]; sm.sc[warp][lane + 32 * i] = pr[i]; }
    l = warp_sum(l);
    if (lane == 0) { sm.m_s[warp] = m; sm.l_s[warp] = l; }
  }
  __syncthreads();

  // ---- P @ V: thread d owns output dim d for the 4 heads ----
  const int d = tid;
  float acc[GQA] = {0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < nj; ++j) {
    const float vf = __bfloat162float(sm.vs[j][d]);
#pragma unroll
    for (int h = 0; h < GQA; ++h) acc[h] += sm.sc[h][j] * vf;
  }
  const size_t qbase = (size_t)b * n_q;
#pragma unroll
  for (int h = 0; h < GQA; ++h) {
    const size_t row = (qbase + kvh * GQA + h) * p.max_splits + split;
    p.o_part[row * HEAD_DIM + d] = acc[h];
    if (tid == 0) {
      p.ml_part[row * 2 + 0] = sm.m_s[h];
      p.ml_part[row * 2 + 1] = sm.l_s[h];
    }
  }
  if (!v_ok) atomicOr(&g_dev_error, DEVERR_MBAR_TIMEOUT);

  // ---- 4. the last CTA of this KV head merges all splits ----
  __threadfence();
  __syncthreads();
  int* counter = p.counters + (size_t)b * n_kv + kvh;
  if (tid == 0) {
    tl_stamp(p.tl_slot, 2);
    sm.is_last = (atomicAdd(counter, 1) == n_splits - 1);
  }
  __syncthreads();
  if (!sm.is_last) return;
  __threadfence();
  {
    const int qh = kvh * GQA + warp;
    const float* ml = p.ml_part + (qbase + qh) * p.max_splits * 2;
    float mloc = -INFINITY;
    for (int s = lane; s < n_splits; s += 32) mloc = fmaxf(mloc, __ldcg(ml + 2 * s));
    const float M = warp_max(mloc);
    float lsum = 0.f;
    for (int s = lane; s < n_splits; s += 32) {
      const float wgt = expf(__ldcg(ml + 2 * s) - M);
      cw[warp * p.max_splits + s] = wgt;
      lsum += wgt * __ldcg(ml + 2 * s + 1);
    }
    lsum = warp_sum(lsum);
    if (lane == 0) sm.cl[warp] = lsum;
  }
  __syncthreads();
  float o[GQA] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
  for (int s = 0; s < n_splits; ++s) {
#pragma unroll
    for (int h = 0; h < GQA; ++h)
      o[h] += cw[h * p.max_splits + s] *
              __ldcg(p.o_part + ((qbase + kvh * GQA + h) * p.max_splits + s) * HEAD_DIM + d);
  }
#pragma unroll
  for (int h = 0; h < GQA; ++h)
    p.out[(qbase + kvh * GQA + h) * HEAD_DIM + d] = __float2bfloat16_rn(o[h] / sm.cl[h]);
  if (tid == 0) {
    *counter = 0;
    tl_stamp(p.tl_slot, 3);
  }
}

template <int CHUNK>
inline size_t attention_smem_bytes(int max_splits) {
  return ((sizeof(AttnSmem<CHUNK>) + 15) / 16) * 16 + (size_t)GQA * max_splits * 4;
}

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
