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
// chunks. Its sums run in a different order from the decode path's split-and-merge, so it matches an fp32
// reference to rounding, not the decode step bit for bit.
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

// Causal GQA attention of the chunk's queries. CTA (m, g): row m (position p0 + m), KV head g and its GQA = 4
// query heads, over keys 0 .. p0 + m in chunks of PF_KEYS; 128 threads. Per chunk: K and V rows into shared
// memory, scores s = (q . k) * scale (thread = key, two heads; each dot summed over the dims in order), a running
// softmax per head (max, rescale by exp(m_old - m_new), sum of exponentials), and P.V with thread = dim, 4 heads.
// The output is bf16(acc / l). All fp32.
constexpr int PF_KEYS = 64;
constexpr int PF_THREADS = 128;
struct PrefillAttnSmem {
  float q[GQA][HEAD_DIM];
  bf16 k[PF_KEYS][HEAD_DIM + 8];   // +8: consecutive rows start 16 bytes apart in bank order
  bf16 v[PF_KEYS][HEAD_DIM];
  float p[GQA][PF_KEYS];
  float m_run[GQA], l_run[GQA], scale_old[GQA];
};
__global__ void __launch_bounds__(PF_THREADS) prefill_attention_kernel(const bf16* __restrict__ q, int p0, int n_q,
                                                                       const bf16* __restrict__ k_cache,
                                                                       const bf16* __restrict__ v_cache, int max_seq,
                                                                       float scale, bf16* __restrict__ out) {
  __shared__ __align__(16) PrefillAttnSmem sm;
  const int m = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ctx = p0 + m + 1;
  for (int i = tid; i < GQA * HEAD_DIM; i += PF_THREADS)
    sm.q[i / HEAD_DIM][i % HEAD_DIM] = __bfloat162float(q[((size_t)m * n_q + g * GQA) * HEAD_DIM + i]);
  if (tid < GQA) {
    sm.m_run[tid] = -INFINITY;
    sm.l_run[tid] = 0.f;
  }
  const bf16* kc = k_cache + (size_t)g * max_seq * HEAD_DIM;
  const bf16* vc = v_cache + (size_t)g * max_seq * HEAD_DIM;
  float acc[GQA] = {0.f, 0.f, 0.f, 0.f};   // thread = dim tid, the 4 heads
  __syncthreads();
  for (int j0 = 0; j0 < ctx; j0 += PF_KEYS) {
    const int nj = min(PF_KEYS, ctx - j0);
    for (int i = tid; i < nj * (HEAD_DIM / 8); i += PF_THREADS) {   // 16-byte pieces of the chunk's K and V rows
      const int r = i / (HEAD_DIM / 8), c8 = i % (HEAD_DIM / 8);
      *reinterpret_cast<uint4*>(&sm.k[r][c8 * 8]) =
          *reinterpret_cast<const uint4*>(kc + (size_t)(j0 + r) * HEAD_DIM + c8 * 8);
      *reinterpret_cast<uint4*>(&sm.v[r][c8 * 8]) =
          *reinterpret_cast<const uint4*>(vc + (size_t)(j0 + r) * HEAD_DIM + c8 * 8);
    }
    __syncthreads();
    {   // scores: thread = (key tid % 64, heads 2 (tid / 64) .. +1)
      const int j = tid & (PF_KEYS - 1), h0 = (tid >> 6) * 2;
      float d0 = 0.f, d1 = 0.f;
      if (j < nj) {
        for (int d = 0; d < HEAD_DIM; d += 8) {
          const uint4 kv = *reinterpret_cast<const uint4*>(&sm.k[j][d]);
          const float kf[8] = {bf16lo(kv.x), bf16hi(kv.x), bf16lo(kv.y), bf16hi(kv.y),
                               bf16lo(kv.z), bf16hi(kv.z), bf16lo(kv.w), bf16hi(kv.w)};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            d0 += sm.q[h0][d + e] * kf[e];
            d1 += sm.q[h0 + 1][d + e] * kf[e];
          }
        }
      }
      sm.p[h0][j] = j < nj ? d0 * scale : -INFINITY;
      sm.p[h0 + 1][j] = j < nj ? d1 * scale : -INFINITY;
    }
    __syncthreads();
    {   // running softmax, warp h takes head h: the chunk's max, the rescale of the old sums, the exponentials
      const int h = warp;
      const float a = sm.p[h][lane], b = sm.p[h][lane + 32];
      const float cmax = warp_max(fmaxf(a, b));
      const float m_old = sm.m_run[h], m_new = fmaxf(m_old, cmax);
      const float ea = expf(a - m_new), eb = expf(b - m_new);
      sm.p[h][lane] = ea;
      sm.p[h][lane + 32] = eb;
      const float csum = warp_sum(ea + eb);
      __syncwarp();
      if (lane == 0) {
        const float r = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        sm.scale_old[h] = r;
        sm.l_run[h] = sm.l_run[h] * r + csum;
        sm.m_run[h] = m_new;
      }
    }
    __syncthreads();
    {   // P.V: thread = dim tid, the 4 heads, the chunk's keys in order
#pragma unroll
      for (int h = 0; h < GQA; ++h) acc[h] *= sm.scale_old[h];
      for (int j = 0; j < nj; ++j) {
        const float v = __bfloat162float(sm.v[j][tid]);
#pragma unroll
        for (int h = 0; h < GQA; ++h) acc[h] += sm.p[h][j] * v;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int h = 0; h < GQA; ++h)
    out[((size_t)m * n_q + g * GQA + h) * HEAD_DIM + tid] = __float2bfloat16_rn(acc[h] / sm.l_run[h]);
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

}  // namespace qk
