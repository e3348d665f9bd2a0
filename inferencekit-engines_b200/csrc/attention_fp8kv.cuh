// Decode attention over an FP8 KV cache: each cached K and V row (one sequence, KV head and position: 128
// dims) is stored as 128 e4m3 bytes plus one fp32 scale, 264 bytes per key and head against 512 for bf16.
// The reference has no such cache (it lists one as future work: it halves long-context KV bytes but changes
// numerics); its contract here:
//
//   row quantization   s = amax(|x|) / 448 (div.full, as the activation quantizer), q = e4m3(x / s) round to
//                      nearest even, saturating; s = 0 gives q = 0. x is the bf16 value the bf16 cache would
//                      hold: the normalised and rotated K row, or the V row as projected.
//   scores             s_j = (sum_d q_h[d] * k8_j[d]: dims 0-63 and 64-127 each in order, then added) * s_kj * scale
//   softmax            per split of 128, 256 or 512 keys (1, 2 or 4 blocks, by max_seq: below 4096, below
//                      16384, above), over its 128-key blocks in order: the running maximum m, the
//                      sums rescaled by exp(m_old - m_new), p_j = exp(s_j - m), l = sum p_j (fp32)
//   P.V                o[d] = sum_j (p_j * s_vj) * v8_j[d], rescaled with the running maximum; within a block 4
//                      groups of 32 keys, each in order; the groups added in order at the end
//   merge              the bf16 path's merge kernel over the splits (attn_merge_kernel)
//
// attn_fp8kv_partials_kernel: grid (n_kv * splits, batch), 256 threads, ~86 KB of shared memory. A CTA takes
// one split of one (sequence, KV head): up to 4 blocks of 128 keys, each block's rows and scales copied
// by cp.async into one of two buffers while the previous block is computed (flash-decoding within the split).
// The first block is requested before griddepcontrol.wait (earlier tokens' rows). Warps 0-3 normalise and
// rotate the 4 query heads; in the split holding `pos`, warps 4 and 5 quantize the new K and V rows into the
// cache and a staging copy that replaces the stale slot once the last block has landed. Scores: thread = (key,
// half of the dims), the 4 heads, halves added by a shuffle. Softmax: one warp per head. P.V: thread = (2 dims,
// 32 keys of the block), the 4 heads. Every e4m3 byte is decoded once. Each split's (m, l, o[128]) goes to
// o_part / ml_part in the layout of the bf16 kernel; its merge kernel finishes the call.
#pragma once
#include "attention.cuh"
#include "common.cuh"

namespace qk {

constexpr int KV8_KEYS = 128;      // keys per block (one cp.async batch)
constexpr int KV8_MAX_BLOCKS = 4;  // blocks per split (a CTA's keys, one partial per head): 1 or 4, by max_seq
constexpr int KV8_THREADS = 256;

struct Kv8Params {
  const bf16* qkv;           // [B][qkv_stride]: q heads | k heads | v heads, 128 each
  const bf16* q_norm_w;      // [128]
  const bf16* k_norm_w;      // [128]
  const bf16* cos_tab;       // [max_seq, 128]
  const bf16* sin_tab;
  const int* state;          // per sequence: state[b * state_stride] = pos
  uint8_t* k_cache;          // [B][n_kv][max_seq][128] e4m3 (one layer)
  uint8_t* v_cache;
  float* k_scale;            // [B][n_kv][max_seq]
  float* v_scale;
  float* o_part;             // [B][n_q][max_splits][128]
  float* ml_part;            // [B][n_q][max_splits][2]
  int n_kv, max_seq, max_splits, qkv_stride, state_stride;
  int blocks;                // 128-key blocks per split (the merge's chunk is 128 * blocks)
  float scale, eps;
};

struct Kv8Buf {
  uint8_t k[KV8_KEYS][HEAD_DIM + 16];   // rows 144 bytes apart: a warp's 16-byte row reads spread over the banks
  uint8_t v[KV8_KEYS][HEAD_DIM];
  float ks[KV8_KEYS], vs[KV8_KEYS];
};
struct Kv8Smem {
  Kv8Buf buf[2];                          // double-buffered blocks
  float4 q[HEAD_DIM];                     // q[d] = the 4 query heads' values at dim d
  float s[GQA][KV8_KEYS];                 // scores of the block per head
  float4 pv[KV8_KEYS];                    // p_j * s_vj of the 4 heads
  float o4[4][GQA][HEAD_DIM];             // P.V sums of the 4 key quarters, combined at the end
  float m_run[GQA], l_run[GQA], scale_old[GQA];
  uint32_t new_k[HEAD_DIM / 4], new_v[HEAD_DIM / 4];   // the quantized new rows (split holding `pos`)
  float new_ks, new_vs;
};
inline size_t kv8_smem_bytes() { return sizeof(Kv8Smem); }

__device__ __forceinline__ void kv8_cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// two e4m3 bytes (the low 16 bits of `two`, low byte first) as two floats; exact
__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t two) {
  const uint32_t h = e4m3x2_to_f16x2(two & 0xFFFFu);
  __half2 hh;
  memcpy(&hh, &h, 4);
  return __half22float2(hh);
}
// one e4m3 byte (the low byte of `b`) as a float; exact
__device__ __forceinline__ float e4m3_to_float(uint32_t b) {
  const uint32_t h2 = e4m3x2_to_f16x2(b & 0xFFu);
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
}

__device__ __forceinline__ void kv8_cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__global__ void __launch_bounds__(KV8_THREADS) attn_fp8kv_partials_kernel(const __grid_constant__ Kv8Params p) {
  extern __shared__ __align__(16) uint8_t kv8_smem[];
  Kv8Smem& sm = *reinterpret_cast<Kv8Smem*>(kv8_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split_keys = KV8_KEYS * p.blocks;
  const int n_sp = (p.max_seq + split_keys - 1) / split_keys;
  const int kvh = blockIdx.x / n_sp, sp = blockIdx.x - kvh * n_sp, b = blockIdx.y;
  const int n_q = p.n_kv * GQA;
  const int pos = p.state[(size_t)b * p.state_stride];   // written by the previous step's finalize
  if (pos < 0 || pos >= p.max_seq) {
    if (tid == 0 && sp == 0 && kvh == 0) atomicOr(&g_dev_error, DEVERR_BAD_STATE);
    return;
  }
  const int key_lo = sp * split_keys;
  if (key_lo > pos) return;                                       // a split past the context
  const int n_keys = min(split_keys, pos + 1 - key_lo);           // `pos` included
  const int nblk = (n_keys + KV8_KEYS - 1) / KV8_KEYS;
  const size_t slab = ((size_t)b * p.n_kv + kvh) * p.max_seq;     // row of position 0
  auto load_block = [&](int i) {   // block i's rows and scales (keys below n_keys only) into buf[i % 2]
    Kv8Buf& B = sm.buf[i & 1];
    const int k0 = key_lo + i * KV8_KEYS, nk = min(KV8_KEYS, n_keys - i * KV8_KEYS);
    for (int e = tid; e < nk * 8; e += KV8_THREADS) {             // 8 pieces of 16 bytes per row
      const int r = e >> 3, c = (e & 7) * 16;
      kv8_cp_async16(&B.k[r][c], p.k_cache + (slab + k0 + r) * HEAD_DIM + c);
      kv8_cp_async16(&B.v[r][c], p.v_cache + (slab + k0 + r) * HEAD_DIM + c);
    }
    for (int e = tid; e < nk; e += KV8_THREADS) {
      kv8_cp_async4(&B.ks[e], p.k_scale + slab + k0 + e);
      kv8_cp_async4(&B.vs[e], p.v_scale + slab + k0 + e);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_block(0);               // earlier tokens' rows: before the wait for the kernel that writes qkv
  grid_dep_wait();
  grid_dep_launch();
  const bf16* qkv = p.qkv + (size_t)b * p.qkv_stride;
  const bf16* cos_row = p.cos_tab + (size_t)pos * HEAD_DIM;
  const bf16* sin_row = p.sin_tab + (size_t)pos * HEAD_DIM;
  const bool owns_new = pos < key_lo + split_keys;                // this split holds `pos` (its last block)
  if (warp < GQA) {            // warp h: query head 4 * kvh + h
    float o[4];
    head_norm_rope_from(qkv + (size_t)(kvh * GQA + warp) * HEAD_DIM, p.q_norm_w, cos_row, sin_row, lane, p.eps, o);
#pragma unroll
    for (int j = 0; j < 4; ++j) reinterpret_cast<float*>(&sm.q[lane * 4 + j])[warp] = bf16r(o[j]);
    if (lane == 0) {
      sm.m_run[warp] = -INFINITY;
      sm.l_run[warp] = 0.f;
    }
  } else if (owns_new && warp < GQA + 2) {   // the new K (warp 4) and V (warp 5) rows: quantized, into the cache
    float x[4];
    if (warp == GQA) {
      float o[4];
      head_norm_rope_from(qkv + (size_t)(n_q + kvh) * HEAD_DIM, p.k_norm_w, cos_row, sin_row, lane, p.eps, o);
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = bf16r(o[j]);
    } else {
      uint2 raw;
      const bf16* src = qkv + (size_t)(n_q + p.n_kv + kvh) * HEAD_DIM + lane * 4;
      asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(raw.x), "=r"(raw.y) : "l"(src));
      x[0] = bf16lo(raw.x), x[1] = bf16hi(raw.x), x[2] = bf16lo(raw.y), x[3] = bf16hi(raw.y);
    }
    const float amax = warp_max(fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3]))));
    const float sc = div_full(amax, 448.0f);
    const uint32_t q4 = quant4(x[0], x[1], x[2], x[3], sc);
    *reinterpret_cast<uint32_t*>((warp == GQA ? p.k_cache : p.v_cache) + (slab + pos) * HEAD_DIM + lane * 4) = q4;
    (warp == GQA ? sm.new_k : sm.new_v)[lane] = q4;
    if (lane == 0) {
      (warp == GQA ? p.k_scale : p.v_scale)[slab + pos] = sc;
      (warp == GQA ? sm.new_ks : sm.new_vs) = sc;
    }
  }
  const int dp = (tid & 63) * 2, kq = tid >> 6;   // P.V: dims dp, dp + 1; keys 32 kq .. +31 of each block
  float o[GQA][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
  for (int i = 0; i < nblk; ++i) {
    const int nk = min(KV8_KEYS, n_keys - i * KV8_KEYS);
    Kv8Buf& B = sm.buf[i & 1];
    if (i + 1 < nblk) {
      load_block(i + 1);       // buf[(i + 1) % 2] was released by block i - 1's final barrier
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    if (owns_new && i == nblk - 1) {   // the slot of `pos` holds what the cache had: the new rows instead
      const int r = pos - (key_lo + i * KV8_KEYS);
      if (tid < 32) *reinterpret_cast<uint32_t*>(&B.k[r][tid * 4]) = sm.new_k[tid];
      else if (tid < 64) *reinterpret_cast<uint32_t*>(&B.v[r][(tid - 32) * 4]) = sm.new_v[tid - 32];
      else if (tid == 64) {
        B.ks[r] = sm.new_ks;
        B.vs[r] = sm.new_vs;
      }
      __syncthreads();
    }
    {   // scores: thread = (key j = tid / 2, dims 64 * (tid % 2) .. +63), the 4 heads; each byte decoded once
      const int j = tid >> 1, half = tid & 1;
      float acc[GQA] = {0.f, 0.f, 0.f, 0.f};
      if (j < nk) {
#pragma unroll 2
        for (int d = half * 64; d < half * 64 + 64; d += 16) {
          const uint4 kw = *reinterpret_cast<const uint4*>(&B.k[j][d]);
          const uint32_t w[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float2 lo = e4m3x2_to_float2(w[t]), hi = e4m3x2_to_float2(w[t] >> 16);
            const float kv[4] = {lo.x, lo.y, hi.x, hi.y};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float4 q4 = sm.q[d + 4 * t + e];
              acc[0] += q4.x * kv[e];
              acc[1] += q4.y * kv[e];
              acc[2] += q4.z * kv[e];
              acc[3] += q4.w * kv[e];
            }
          }
        }
      }
#pragma unroll
      for (int h = 0; h < GQA; ++h) acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 1);   // dims 0-63 + 64-127
      if (half == 0) {
        const float ks = j < nk ? B.ks[j] : 0.f;
#pragma unroll
        for (int h = 0; h < GQA; ++h) sm.s[h][j] = j < nk ? acc[h] * ks * p.scale : -INFINITY;
      }
    }
    __syncthreads();
    if (warp < GQA) {   // running softmax of head h = warp over the block's 128 keys (4 per lane)
      const int h = warp;
      float x[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) x[e] = sm.s[h][lane + 32 * e];
      const float cmax = warp_max(fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3])));
      const float m_old = sm.m_run[h], m_new = fmaxf(m_old, cmax);   // finite: every block has a key in context
      float csum = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = lane + 32 * e;
        const float pe = expf(x[e] - m_new);
        csum += pe;
        reinterpret_cast<float*>(&sm.pv[j])[h] = j < nk ? pe * B.vs[j] : 0.f;
      }
      csum = warp_sum(csum);
      if (lane == 0) {
        const float r = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        sm.scale_old[h] = r;
        sm.l_run[h] = sm.l_run[h] * r + csum;
        sm.m_run[h] = m_new;
      }
    }
    __syncthreads();
    {   // P.V: the thread's 32 keys of the block, after rescaling its sums to the new running maxima
#pragma unroll
      for (int h = 0; h < GQA; ++h) {
        const float r = sm.scale_old[h];
        o[h][0] *= r;
        o[h][1] *= r;
      }
      const int ja = kq * 32, jb = min(nk, ja + 32);
      for (int j = ja; j < jb; ++j) {
        const float2 v2 = e4m3x2_to_float2(*reinterpret_cast<const uint16_t*>(&B.v[j][dp]));
        const float4 w = sm.pv[j];
        o[0][0] += w.x * v2.x;
        o[0][1] += w.x * v2.y;
        o[1][0] += w.y * v2.x;
        o[1][1] += w.y * v2.y;
        o[2][0] += w.z * v2.x;
        o[2][1] += w.z * v2.y;
        o[3][0] += w.w * v2.x;
        o[3][1] += w.w * v2.y;
      }
    }
    __syncthreads();   // this block's buffer, scores and weights are free for the next block
  }
#pragma unroll
  for (int h = 0; h < GQA; ++h) *reinterpret_cast<float2*>(&sm.o4[kq][h][dp]) = make_float2(o[h][0], o[h][1]);
  __syncthreads();
  {   // thread = (head tid / 64, dims dp, dp + 1): the 4 key quarters in order, then the split's partial
    const int h = tid >> 6;
    float2 r = make_float2(0.f, 0.f);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 x = *reinterpret_cast<const float2*>(&sm.o4[q][h][dp]);
      r.x += x.x;
      r.y += x.y;
    }
    const size_t row = ((size_t)b * n_q + kvh * GQA + h) * p.max_splits + sp;
    *reinterpret_cast<float2*>(p.o_part + row * HEAD_DIM + dp) = r;
    if (dp == 0) {
      p.ml_part[row * 2] = sm.m_run[h];
      p.ml_part[row * 2 + 1] = sm.l_run[h];
    }
  }
}

}  // namespace qk
