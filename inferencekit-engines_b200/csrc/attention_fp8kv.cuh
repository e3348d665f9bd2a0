// Decode attention over an FP8 KV cache: each cached K and V row (one sequence, KV head and position: 128
// dims) is stored as 128 e4m3 bytes plus one fp32 scale, 264 bytes per key and head against 512 for bf16.
// The reference has no such cache (it lists one as future work: it halves long-context KV bytes but changes
// numerics); its contract here:
//
//   row quantization   s = amax(|x|) / 448 (div.full, as the activation quantizer), q = e4m3(x / s) round to
//                      nearest even, saturating; s = 0 gives q = 0. x is the bf16 value the bf16 cache would
//                      hold: the normalised and rotated K row, or the V row as projected.
//   scores             s_j = (sum_d q_h[d] * k8_j[d], dims in order) * s_kj * scale
//   softmax            per 64-key split: m = max s_j, p_j = exp(s_j - m), l = sum p_j (fp32)
//   P.V                o[d] = sum_j (p_j * s_vj) * v8_j[d], keys in order
//   merge              the bf16 path's merge kernel over the 64-key splits (attn_merge_kernel)
//
// attn_fp8kv_partials_kernel: grid (n_kv * 128-key blocks, batch), 256 threads. A CTA takes one block of 128
// keys of one (sequence, KV head): two 64-key splits. The block's earlier rows and scales are copied to shared
// memory with 16-byte cp.async before griddepcontrol.wait (they are earlier tokens' rows). Then warps 0-3
// normalise and rotate the 4 query heads; in the block holding `pos`, warps 4 and 5 quantize the new K and V
// rows into the cache and into the shared copy. Scores: thread = (key, pair of heads). Softmax: one warp per
// (split, head). P.V: thread = (dim, pair of heads). Each split's (m, l, o[128]) goes to o_part / ml_part in
// the layout of the bf16 kernel, so the same merge kernel finishes the call.
#pragma once
#include "attention.cuh"
#include "common.cuh"

namespace qk {

constexpr int KV8_KEYS = 128;      // keys per partials CTA
constexpr int KV8_SPLIT = 64;      // keys per split (the merge's chunk)
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
  float scale, eps;
};

struct Kv8Smem {
  uint8_t k[KV8_KEYS][HEAD_DIM + 16];   // rows 144 bytes apart: a warp's 16-byte row reads spread over the banks
  uint8_t v[KV8_KEYS][HEAD_DIM];
  float ks[KV8_KEYS], vs[KV8_KEYS];
  float q[GQA][HEAD_DIM];
  float p[2][GQA][KV8_SPLIT];           // per (split, head): scores, then p_j * s_vj
  float m[2][GQA], l[2][GQA];
};

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

__global__ void __launch_bounds__(KV8_THREADS) attn_fp8kv_partials_kernel(const __grid_constant__ Kv8Params p) {
  __shared__ __align__(16) Kv8Smem sm;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_blocks = (p.max_seq + KV8_KEYS - 1) / KV8_KEYS;
  const int kvh = blockIdx.x / n_blocks, blk = blockIdx.x - kvh * n_blocks, b = blockIdx.y;
  const int n_q = p.n_kv * GQA;
  const int pos = p.state[(size_t)b * p.state_stride];   // written by the previous step's finalize
  if (pos < 0 || pos >= p.max_seq) {
    if (tid == 0 && blk == 0 && kvh == 0) atomicOr(&g_dev_error, DEVERR_BAD_STATE);
    return;
  }
  const int key0 = blk * KV8_KEYS;
  if (key0 > pos) return;                                 // a block past the context
  const int nk = min(KV8_KEYS, pos + 1 - key0);           // keys key0 .. key0 + nk - 1, `pos` included
  const size_t row0 = ((size_t)b * p.n_kv + kvh) * p.max_seq + key0;
  for (int i = tid; i < nk * 8; i += KV8_THREADS) {       // 8 pieces of 16 bytes per row
    const int r = i >> 3, c = (i & 7) * 16;
    kv8_cp_async16(&sm.k[r][c], p.k_cache + (row0 + r) * HEAD_DIM + c);
    kv8_cp_async16(&sm.v[r][c], p.v_cache + (row0 + r) * HEAD_DIM + c);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int i = tid; i < nk; i += KV8_THREADS) {
    sm.ks[i] = p.k_scale[row0 + i];
    sm.vs[i] = p.v_scale[row0 + i];
  }
  grid_dep_wait();            // qkv comes from the kernel before
  grid_dep_launch();
  const bf16* qkv = p.qkv + (size_t)b * p.qkv_stride;
  const bf16* cos_row = p.cos_tab + (size_t)pos * HEAD_DIM;
  const bf16* sin_row = p.sin_tab + (size_t)pos * HEAD_DIM;
  if (warp < GQA) {           // warp h: query head 4 * kvh + h
    float o[4];
    head_norm_rope_from(qkv + (size_t)(kvh * GQA + warp) * HEAD_DIM, p.q_norm_w, cos_row, sin_row, lane, p.eps, o);
#pragma unroll
    for (int j = 0; j < 4; ++j) sm.q[warp][lane * 4 + j] = bf16r(o[j]);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();            // earlier rows landed (the slot of `pos` holds whatever the cache had)
  if (pos - key0 < KV8_KEYS && (warp == GQA || warp == GQA + 1)) {   // the new K (warp 4) and V (warp 5) rows
    const int n_q_heads = n_q;
    float x[4];
    if (warp == GQA) {
      float o[4];
      head_norm_rope_from(qkv + (size_t)(n_q_heads + kvh) * HEAD_DIM, p.k_norm_w, cos_row, sin_row, lane, p.eps, o);
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = bf16r(o[j]);
    } else {
      uint2 raw;
      const bf16* src = qkv + (size_t)(n_q_heads + p.n_kv + kvh) * HEAD_DIM + lane * 4;
      asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(raw.x), "=r"(raw.y) : "l"(src));
      x[0] = bf16lo(raw.x), x[1] = bf16hi(raw.x), x[2] = bf16lo(raw.y), x[3] = bf16hi(raw.y);
    }
    const float amax = warp_max(fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3]))));
    const float s = div_full(amax, 448.0f);
    const uint32_t q4 = quant4(x[0], x[1], x[2], x[3], s);
    const int r = pos - key0;
    uint8_t* cache = warp == GQA ? p.k_cache : p.v_cache;
    *reinterpret_cast<uint32_t*>(cache + (row0 + r) * HEAD_DIM + lane * 4) = q4;
    *reinterpret_cast<uint32_t*>((warp == GQA ? &sm.k[r][0] : &sm.v[r][0]) + lane * 4) = q4;
    if (lane == 0) {
      (warp == GQA ? p.k_scale : p.v_scale)[row0 + r] = s;
      (warp == GQA ? sm.ks : sm.vs)[r] = s;
    }
  }
  __syncthreads();
  {   // scores: thread = (key j, heads h0 and h0 + 1); keys past nk are -inf
    const int j = tid & (KV8_KEYS - 1), h0 = (tid >> 7) * 2;
    float d0 = 0.f, d1 = 0.f;
    if (j < nk) {
#pragma unroll 2
      for (int d = 0; d < HEAD_DIM; d += 16) {
        const uint4 kw = *reinterpret_cast<const uint4*>(&sm.k[j][d]);
        const uint32_t w[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 lo = e4m3x2_to_float2(w[t]), hi = e4m3x2_to_float2(w[t] >> 16);
          const int dd = d + 4 * t;
          d0 += sm.q[h0][dd] * lo.x;
          d0 += sm.q[h0][dd + 1] * lo.y;
          d0 += sm.q[h0][dd + 2] * hi.x;
          d0 += sm.q[h0][dd + 3] * hi.y;
          d1 += sm.q[h0 + 1][dd] * lo.x;
          d1 += sm.q[h0 + 1][dd + 1] * lo.y;
          d1 += sm.q[h0 + 1][dd + 2] * hi.x;
          d1 += sm.q[h0 + 1][dd + 3] * hi.y;
        }
      }
    }
    const float ks = j < nk ? sm.ks[j] : 0.f;
    sm.p[j >> 6][h0][j & 63] = j < nk ? d0 * ks * p.scale : -INFINITY;
    sm.p[j >> 6][h0 + 1][j & 63] = j < nk ? d1 * ks * p.scale : -INFINITY;
  }
  __syncthreads();
  {   // softmax: warp = (split warp / 4, head warp % 4); a split past the context has no keys and is skipped
    const int sp = warp >> 2, h = warp & 3;
    if (sp * KV8_SPLIT < nk) {
      const float a = sm.p[sp][h][lane], c = sm.p[sp][h][lane + 32];
      const float m = warp_max(fmaxf(a, c));        // finite: the split's first key is in the context
      const float ea = expf(a - m), ec = expf(c - m);
      const float l = warp_sum(ea + ec);
      const int ja = sp * KV8_SPLIT + lane, jc = ja + 32;
      sm.p[sp][h][lane] = ja < nk ? ea * sm.vs[ja] : 0.f;
      sm.p[sp][h][lane + 32] = jc < nk ? ec * sm.vs[jc] : 0.f;
      if (lane == 0) {
        sm.m[sp][h] = m;
        sm.l[sp][h] = l;
      }
    }
  }
  __syncthreads();
  {   // P.V: thread = (dim d, heads h0 and h0 + 1), keys of each split in order
    const int d = tid & (HEAD_DIM - 1), h0 = (tid >> 7) * 2;
    for (int sp = 0; sp < 2; ++sp) {
      const int j0 = sp * KV8_SPLIT;
      if (j0 >= nk) break;
      const int nj = min(KV8_SPLIT, nk - j0);
      float a0 = 0.f, a1 = 0.f;
      for (int j = 0; j < nj; ++j) {
        const float v = e4m3_to_float(sm.v[j0 + j][d]);
        a0 += sm.p[sp][h0][j] * v;
        a1 += sm.p[sp][h0 + 1][j] * v;
      }
      const int split = blk * (KV8_KEYS / KV8_SPLIT) + sp;
      const size_t r0 = ((size_t)b * n_q + kvh * GQA + h0) * p.max_splits + split;
      const size_t r1 = r0 + p.max_splits;
      p.o_part[r0 * HEAD_DIM + d] = a0;
      p.o_part[r1 * HEAD_DIM + d] = a1;
      if (d == 0) {
        p.ml_part[r0 * 2] = sm.m[sp][h0];
        p.ml_part[r0 * 2 + 1] = sm.l[sp][h0];
        p.ml_part[r1 * 2] = sm.m[sp][h0 + 1];
        p.ml_part[r1 * 2 + 1] = sm.l[sp][h0 + 1];
      }
    }
  }
}

}  // namespace qk
