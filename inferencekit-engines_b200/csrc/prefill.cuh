// Chunked prefill: a prompt chunk of up to 128 positions through the decoder layers, with the tcgen05 batched
// linear (gemm_tc.cuh) for the four projections and these row-wise kernels around it:
//
//   resid[M]    = embed rows of the chunk's tokens                              embed_rows_kernel
//   qkv[M]      = W_qkv . fp8quant(RMSNorm(resid, ln1))                         qk_fp8_gemm_rows (norm fused)
//   q[M], K/V   = per-head RMSNorm + RoPE of q and k at p0 + m; K and V rows     prefill_qkv_kernel
//                 appended to the cache
//   attn[M]     = causal GQA attention of q over keys 0 .. p0 + m               prefill_attention_kernel
//   resid      += bf16(W_o . fp8quant(attn))                                    qk_fp8_gemm_rows + add_rows_kernel
//   gu[M]       = W_gu . fp8quant(RMSNorm(resid, ln2))                          qk_fp8_gemm_rows (norm fused)
//   h[M]        = bf16(bf16(silu(g)) * u)                                       swiglu_rows_kernel
//   resid      += bf16(W_down . fp8quant(h))                                    qk_fp8_gemm_rows + add_rows_kernel
//
// This is the reference's batched forward (Q/model.py:243-281 with Q/kernels/prefill.py's W8A8 linear) for a
// chunk of positions. The row-wise arithmetic is the decode step's:
//  * q/k RMSNorm + RoPE: head_norm_rope (attention.cuh), the same bf16 roundings, so the K/V rows written are the
//    values the decode step writes for that position given the same qkv row;
//  * SwiGLU and the residual add round exactly as the decode epilogues.
// The attention is fp32 throughout (scores, softmax probabilities, P.V) with one online-softmax pass over 64-key
// chunks, 4 rows of a KV head per CTA. Its sums run in a different order from the decode path's
// split-and-merge, so it matches an fp32 reference to rounding, not the decode step bit for bit.
#pragma once
#include "attention.cuh"
#include "common.cuh"

namespace qk {

// out[m][:] = table[tokens[m]][:] (H values, 16-byte copies). A token outside [0, vocab) sets the error word
// and copies row 0.
__global__ void __launch_bounds__(256) embed_rows_kernel(const int* __restrict__ tokens, int vocab,
                                                         const bf16* __restrict__ table, int H,
                                                         bf16* __restrict__ out) {
  const int m = blockIdx.x;
  int tok = tokens[m];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) atomicOr(&g_dev_error, DEVERR_BAD_STATE);
    tok = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)tok * H);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)m * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// Row m of the chunk sits at position p0 + m. Warp w of CTA (m, part) handles task part * 8 + w of the row's
// n_q + 2 n_kv head tasks: query head t (RMSNorm + RoPE into q_out), key head (RMSNorm + RoPE, into the cache),
// value head (copied into the cache). The K/V cache of the layer is [n_kv][max_seq][128].
__global__ void __launch_bounds__(256) prefill_qkv_kernel(const bf16* __restrict__ qkv, int p0, int n_q, int n_kv,
                                                          const bf16* __restrict__ q_norm,
                                                          const bf16* __restrict__ k_norm,
                                                          const bf16* __restrict__ cos_tab,
                                                          const bf16* __restrict__ sin_tab, float eps,
                                                          bf16* __restrict__ k_cache, bf16* __restrict__ v_cache,
                                                          int max_seq, bf16* __restrict__ q_out) {
  const int m = blockIdx.x, lane = threadIdx.x & 31;
  const int t = blockIdx.y * 8 + (threadIdx.x >> 5);
  if (t >= n_q + 2 * n_kv) return;
  const int pos = p0 + m;
  const int qkv_stride = (n_q + 2 * n_kv) * HEAD_DIM;
  const bf16* row = qkv + (size_t)m * qkv_stride;
  const bf16* cos_row = cos_tab + (size_t)pos * HEAD_DIM;
  const bf16* sin_row = sin_tab + (size_t)pos * HEAD_DIM;
  if (t < n_q + n_kv) {   // a query or key head: RMSNorm + RoPE
    float o[4];
    head_norm_rope_from(row + (size_t)t * HEAD_DIM, t < n_q ? q_norm : k_norm, cos_row, sin_row, lane, eps, o);
    bf16* dst = t < n_q ? q_out + ((size_t)m * n_q + t) * HEAD_DIM
                        : k_cache + ((size_t)(t - n_q) * max_seq + pos) * HEAD_DIM;
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[lane * 4 + j] = __float2bfloat16_rn(o[j]);
  } else {                 // a value head: the row as it is
    const int g = t - n_q - n_kv;
    *reinterpret_cast<uint2*>(v_cache + ((size_t)g * max_seq + pos) * HEAD_DIM + lane * 4) =
        *reinterpret_cast<const uint2*>(row + (size_t)t * HEAD_DIM + lane * 4);
  }
}

// Causal GQA attention of the chunk's queries. CTA (row block, g): PA_ROWS = 4 consecutive rows m0 .. m0 + 3
// (positions p0 + m) and KV head g, i.e. PA_Q = 16 query vectors (head h = 4 g + qi / 4 of row m0 + qi % 4),
// over keys 0 .. p0 + m in chunks of PF_KEYS; 256 threads. The chunk's K and V rows arrive in shared memory by
// 16-byte cp.async copies, double-buffered (the next chunk loads while this one is computed), so each K/V row
// crosses L2 once per 4 rows instead of once per row. Per chunk, all fp32:
//  * scores s = (q . k) * scale, thread = (2 queries, keys j and j + 32), each dot summed over the dims in order;
//    keys past a query's position are -inf;
//  * a running softmax per query (one warp per 2 queries): the chunk's max, the rescale of the old sums by
//    exp(m_old - m_new), the exponentials and their sum;
//  * P.V with thread = (1 query, 8 dims), the chunk's keys in order, after rescaling the accumulators.
// The output is bf16(acc / l). Every query has key 0 in its first chunk, so no running max stays -inf.
constexpr int PF_KEYS = 64;
constexpr int PF_THREADS = 256;
constexpr int PA_ROWS = 4;            // rows per CTA: a 128-row chunk gives 32 x 8 = 256 CTAs
constexpr int PA_Q = PA_ROWS * GQA;   // 16 query vectors per CTA
constexpr int PA_QPW = PA_Q / 8;      // scores and softmax: queries per warp
constexpr int PA_QPT = PA_Q / 16;     // P.V: queries per thread (16 thread groups of 16 dims x 8)
struct PrefillAttnSmem {
  bf16 k[2][PF_KEYS][HEAD_DIM + 8];   // +8: consecutive rows start 16 bytes apart in bank order
  bf16 v[2][PF_KEYS][HEAD_DIM];
  float q[PA_Q][HEAD_DIM + 4];
  float p[PA_Q][PF_KEYS + 4];
  float m_run[PA_Q], l_run[PA_Q], scale_old[PA_Q];
};
__device__ __forceinline__ void pf_cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__global__ void __launch_bounds__(PF_THREADS) prefill_attention_kernel(const bf16* __restrict__ q, int M, int p0,
                                                                       int n_q, const bf16* __restrict__ k_cache,
                                                                       const bf16* __restrict__ v_cache, int max_seq,
                                                                       float scale, bf16* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t pf_smem[];
  PrefillAttnSmem& sm = *reinterpret_cast<PrefillAttnSmem*>(pf_smem);
  const int g = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m0 = blockIdx.x * PA_ROWS, rows = min(PA_ROWS, M - m0);
  const int ctx = p0 + m0 + rows;                        // keys 0 .. ctx - 1 cover the block's last row
  const bf16* kc = k_cache + (size_t)g * max_seq * HEAD_DIM;
  const bf16* vc = v_cache + (size_t)g * max_seq * HEAD_DIM;
  auto load_chunk = [&](int buf, int j0) {               // 2 x 64 rows x 16 pieces of 16 bytes, 8 per thread
    const int nj = min(PF_KEYS, ctx - j0);
    for (int i = tid; i < nj * (HEAD_DIM / 8); i += PF_THREADS) {
      const int r = i / (HEAD_DIM / 8), c8 = (i % (HEAD_DIM / 8)) * 8;
      pf_cp_async16(&sm.k[buf][r][c8], kc + (size_t)(j0 + r) * HEAD_DIM + c8);
      pf_cp_async16(&sm.v[buf][r][c8], vc + (size_t)(j0 + r) * HEAD_DIM + c8);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_chunk(0, 0);
  for (int i = tid; i < PA_Q * HEAD_DIM; i += PF_THREADS) {   // query qi = h * PA_ROWS + r, h = 0..3 in the group
    const int qi = i / HEAD_DIM, d = i % HEAD_DIM, r = qi % PA_ROWS, h = qi / PA_ROWS;
    sm.q[qi][d] = r < rows ? __bfloat162float(q[((size_t)(m0 + r) * n_q + g * GQA + h) * HEAD_DIM + d]) : 0.f;
  }
  if (tid < PA_Q) {
    sm.m_run[tid] = -INFINITY;
    sm.l_run[tid] = 0.f;
  }
  // P.V ownership: queries PA_QPT * (tid / 16) .. +PA_QPT-1, dims 8 * (tid % 16) .. +7
  const int pq = (tid >> 4) * PA_QPT, pd = (tid & 15) * 8;
  float acc[PA_QPT][8];
#pragma unroll
  for (int a = 0; a < PA_QPT; ++a)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[a][e] = 0.f;
  // score ownership: queries PA_QPW * warp .. +PA_QPW-1, keys lane and lane + 32
  const int sq = warp * PA_QPW;
  int buf = 0;
  for (int j0 = 0; j0 < ctx; j0 += PF_KEYS, buf ^= 1) {
    const int nj = min(PF_KEYS, ctx - j0);
    if (j0 + PF_KEYS < ctx) {
      load_chunk(buf ^ 1, j0 + PF_KEYS);   // the buffer freed by the previous chunk's final barrier
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    {   // scores
      float s[PA_QPW][2];
#pragma unroll
      for (int a = 0; a < PA_QPW; ++a) s[a][0] = s[a][1] = 0.f;
      const int ja = lane, jb = lane + 32;
      for (int d = 0; d < HEAD_DIM; d += 8) {
        const uint4 ka = *reinterpret_cast<const uint4*>(&sm.k[buf][ja][d]);
        const uint4 kb = *reinterpret_cast<const uint4*>(&sm.k[buf][jb][d]);
        const float fa[8] = {bf16lo(ka.x), bf16hi(ka.x), bf16lo(ka.y), bf16hi(ka.y),
                             bf16lo(ka.z), bf16hi(ka.z), bf16lo(ka.w), bf16hi(ka.w)};
        const float fb[8] = {bf16lo(kb.x), bf16hi(kb.x), bf16lo(kb.y), bf16hi(kb.y),
                             bf16lo(kb.z), bf16hi(kb.z), bf16lo(kb.w), bf16hi(kb.w)};
#pragma unroll
        for (int a = 0; a < PA_QPW; ++a) {
          const float4 q0 = *reinterpret_cast<const float4*>(&sm.q[sq + a][d]);
          const float4 q1 = *reinterpret_cast<const float4*>(&sm.q[sq + a][d + 4]);
          const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            s[a][0] += qv[e] * fa[e];
            s[a][1] += qv[e] * fb[e];
          }
        }
      }
#pragma unroll
      for (int a = 0; a < PA_QPW; ++a) {
        const int pos = p0 + m0 + (sq + a) % PA_ROWS;
        sm.p[sq + a][ja] = (ja < nj && j0 + ja <= pos) ? s[a][0] * scale : -INFINITY;
        sm.p[sq + a][jb] = (jb < nj && j0 + jb <= pos) ? s[a][1] * scale : -INFINITY;
      }
    }
    __syncwarp();
    // running softmax: warp w owns queries PA_QPW w .. +PA_QPW-1, exactly the rows its lanes just scored
#pragma unroll
    for (int a = 0; a < PA_QPW; ++a) {
      const int qi = sq + a;
      const float x0 = sm.p[qi][lane], x1 = sm.p[qi][lane + 32];
      const float cmax = warp_max(fmaxf(x0, x1));
      const float m_old = sm.m_run[qi], m_new = fmaxf(m_old, cmax);
      const float e0 = expf(x0 - m_new), e1 = expf(x1 - m_new);
      sm.p[qi][lane] = e0;
      sm.p[qi][lane + 32] = e1;
      const float csum = warp_sum(e0 + e1);
      if (lane == 0) {
        const float r = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        sm.scale_old[qi] = r;
        sm.l_run[qi] = sm.l_run[qi] * r + csum;
        sm.m_run[qi] = m_new;
      }
    }
    __syncthreads();
    {   // P.V
#pragma unroll
      for (int a = 0; a < PA_QPT; ++a) {
        const float r = sm.scale_old[pq + a];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[a][e] *= r;
      }
      for (int j = 0; j < nj; ++j) {
        const uint4 vv = *reinterpret_cast<const uint4*>(&sm.v[buf][j][pd]);
        const float vf[8] = {bf16lo(vv.x), bf16hi(vv.x), bf16lo(vv.y), bf16hi(vv.y),
                             bf16lo(vv.z), bf16hi(vv.z), bf16lo(vv.w), bf16hi(vv.w)};
#pragma unroll
        for (int a = 0; a < PA_QPT; ++a) {
          const float w = sm.p[pq + a][j];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[a][e] += w * vf[e];
        }
      }
    }
    __syncthreads();   // this chunk's K/V buffer and p are free for the next load and scores
  }
#pragma unroll
  for (int a = 0; a < PA_QPT; ++a) {
    const int qi = pq + a, r = qi % PA_ROWS, h = qi / PA_ROWS;
    if (r >= rows) continue;
    const float inv_l = 1.f / sm.l_run[qi];
    bf16 o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __float2bfloat16_rn(acc[a][e] * inv_l);
    *reinterpret_cast<uint4*>(out + ((size_t)(m0 + r) * n_q + g * GQA + h) * HEAD_DIM + pd) =
        *reinterpret_cast<const uint4*>(o);
  }
}

// resid[i] = bf16(resid[i] + y[i]) for y = bf16(W . x): the decode step's residual epilogue, bf16(resid + bf16(a)).
__global__ void add_rows_kernel(bf16* __restrict__ resid, const bf16* __restrict__ y, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    resid[i] = __float2bfloat16_rn(__bfloat162float(resid[i]) + __bfloat162float(y[i]));
}

// h[m][i] = bf16(bf16(silu(g)) * u) with g = gu[m][i], u = gu[m][I + i] (both already bf16): the decode step's
// SwiGLU epilogue (silu as g / (1 + expf(-g)), IEEE division).
__global__ void swiglu_rows_kernel(const bf16* __restrict__ gu, int M, int I, bf16* __restrict__ h) {
  const long long n = (long long)M * I;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long m = idx / I, i = idx - m * I;
    const float gt = __bfloat162float(gu[m * 2 * I + i]);
    const float up = __bfloat162float(gu[m * 2 * I + I + i]);
    const float act = bf16r(gt / (1.0f + expf(-gt)));
    h[idx] = __float2bfloat16_rn(act * up);
  }
}

// Greedy argmax of each row of bf16 logits [rows][V] (ties to the lowest index), as the packed u64 key of the
// decode step's lm_head (argmax_key), written to best[row]; finalize_kernel decodes it. One CTA of 1024 threads
// per row.
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const bf16* __restrict__ logits, int V,
                                                           unsigned long long* __restrict__ best) {
  __shared__ unsigned long long red[32];
  const int row = blockIdx.x, tid = threadIdx.x;
  const bf16* x = logits + (size_t)row * V;
  unsigned long long key = 0ull;
  for (int i = tid; i < V; i += 1024) {
    const unsigned long long k = argmax_key(__bfloat162float(x[i]), i);
    key = k > key ? k : key;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
    key = other > key ? other : key;
  }
  if ((tid & 31) == 0) red[tid >> 5] = key;
  __syncthreads();
  if (tid < 32) {
    key = red[tid];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
      key = other > key ? other : key;
    }
    if (tid == 0) best[row] = key;
  }
}

}  // namespace qk
