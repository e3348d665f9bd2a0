// FP8 W8A8 GEMV for the batch-1 decode step: y[N] = W[N, K] . quant(x[K]), block- or channel-scaled.
//
// Design (B200):
//  * Work split. The weights are a stream of tiles ordered [unit][kb] (unit = 16 output rows, or 16 gate
//    + 16 up rows for SwiGLU; kb = 128-wide K block; a tile is 2 KiB per 16 rows), see model.pack_fp8.
//    Every warp of the grid takes an equal, contiguous range of that stream, so each SM reads the same
//    number of bytes whatever N is.
//  * Data movement. Each warp runs its own shared-memory ring: lane 0 issues bulk async copies
//    (cp.async.bulk, L2 evict-first) of `stage_tiles` tiles per stage and the warp waits on the stage's
//    mbarrier. The first `pre` stages are requested before griddepcontrol.wait, so under programmatic
//    dependent launch a kernel streams its weights while the previous kernel finishes.
//  * Math. The prologue RMS-normalises x (optional), quantizes it to e4m3 per 128-group exactly as the
//    reference, and stores it as f16 MMA fragments in shared memory. Per 32-wide K chunk a lane reads 16
//    weight bytes (rows r and r+8 of the unit), converts them to f16 and issues two m16n8k16 MMAs with the
//    weights as the A operand (see fp8_chunk_dot): 16 rows x 32 k per two MMAs and 8 conversions.
//    Per K block: acc += d * s_x * s_w (fp32), in K order.
//  * Exactness. The chunk dot is bit-identical to the reference decode kernel's fp8 mma, the chunks and
//    blocks are accumulated in the same order, so outputs are bit-identical to it. A unit whose K range is
//    split between two warps stores its raw block dots in `part`; the warp that completes the unit
//    (atomic counter, last-arriver) replays the same in-order accumulation, so splitting changes no bit.
//  * Epilogues: bf16 store (qkv), residual add in place (o_proj, down), SwiGLU (gate_up), logits +
//    greedy argmax (lm_head), fp32 partial store (tensor-parallel row shards).
#pragma once
#include "common.cuh"

namespace qk {

enum { PRO_QUANT = 0, PRO_RMSNORM_QUANT = 1, PRO_RESADD_RMSNORM_QUANT = 2 };
enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3, EPI_F32 = 4 };
enum { SCALE_BLOCK = 0, SCALE_CHANNEL = 1 };
constexpr int GEMV_UNIT_ROWS = 16;
constexpr int GEMV_TILE_BYTES = GEMV_UNIT_ROWS * QB;   // 2 KiB per 16 rows x 128 k

struct GemvParams {
  const uint8_t* w;          // packed fp8 tiles (model.pack_fp8)
  const float* ws;           // scales: [N/128][K/128] (block) or [N] (channel)
  const bf16* x;             // input [K]; for RESADD the residual stream [K]
  const bf16* norm_w;        // RMSNorm weight [K] (RMSNORM / RESADD prologues)
  const float* resadd;       // RESADD: fp32 sums to add to the residual first [K]
  bf16* resid_out;           // RESADD: the updated residual (each CTA writes a slice)
  bf16* out;                 // STORE [N] | RESIDUAL [N] in place | SWIGLU [N/2] | ARGMAX logits [N]
  float* out_f32;            // F32 [N]
  float* part;               // split-K block dots [units][KB][16*NG]
  int* counters;             // [units], zero between launches (the kernel leaves them zero)
  unsigned long long* best;  // ARGMAX: packed (value, index) key, zero before the launch
  int N, K;
  int row_offset;            // ARGMAX: vocabulary index of local row 0
  float eps;
  int stages, stage_tiles, pre;
  int tl_slot;               // timeline region of this launch, -1 when off
};

// Shared-memory carve-up, computed identically on host and device.
struct GemvSmem {
  int xs, xh, xscale, red, bestbuf, bars, ring, total;
};
__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }
__host__ __device__ inline GemvSmem gemv_smem(int K, int warps, int stages, int stage_bytes) {
  GemvSmem L;
  L.xs = 0;                                      // raw bf16 input, K*2
  L.xh = align_up(L.xs + K * 2, 128);            // quantized input as f16 MMA fragments, K*2
  L.xscale = align_up(L.xh + K * 2, 16);         // K/128 floats
  L.red = align_up(L.xscale + (K / QB) * 4, 16); // 32 floats
  L.bestbuf = L.red + 32 * 4;                    // 32 u64
  L.bars = align_up(L.bestbuf + 32 * 8, 16);     // warps*stages mbarriers
  L.ring = align_up(L.bars + warps * stages * 8, 1024);
  L.total = L.ring + warps * stages * stage_bytes;
  return L;
}

// ---- prologue: x -> (residual add) -> (RMSNorm) -> e4m3 per 128-group -> f16 fragments in shared memory -----
// Fragment order: 16 bytes at ((kb*4 + c)*4 + t)*16 hold x(32c + 4t, +1), x(32c + 16 + 4t, +1),
// x(32c + 4t + 2, +3), x(32c + 16 + 4t + 2, +3) of block kb as f16x2: the B operands of the two MMAs of
// chunk c for every lane with that t.
template <int PRO>
__device__ __forceinline__ void gemv_prologue(const GemvParams& p, uint8_t* smem, const GemvSmem& L) {
  const int K = p.K, KB = K / QB;
  const int nthr = blockDim.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = nthr >> 5;
  bf16* xs = reinterpret_cast<bf16*>(smem + L.xs);
  if (PRO == PRO_RESADD_RMSNORM_QUANT) {
    // resid = bf16(resid + bf16(sum)), the same rounding as the in-place residual epilogue
    for (int i = threadIdx.x; i < K / 2; i += nthr) {
      const __nv_bfloat162 r = reinterpret_cast<const __nv_bfloat162*>(p.x)[i];
      const float2 a = reinterpret_cast<const float2*>(p.resadd)[i];
      reinterpret_cast<__nv_bfloat162*>(xs)[i] =
          __floats2bfloat162_rn(__low2float(r) + bf16r(a.x), __high2float(r) + bf16r(a.y));
    }
    __syncthreads();
    const int per = (K / 2 + gridDim.x - 1) / gridDim.x;
    const int lo = blockIdx.x * per, hi = min(lo + per, K / 2);
    for (int i = lo + threadIdx.x; i < hi; i += nthr)
      reinterpret_cast<__nv_bfloat162*>(p.resid_out)[i] = reinterpret_cast<const __nv_bfloat162*>(xs)[i];
  } else {
    for (int i = threadIdx.x; i < K / 8; i += nthr)
      reinterpret_cast<uint4*>(xs)[i] = reinterpret_cast<const uint4*>(p.x)[i];
  }
  __syncthreads();
  float rstd = 0.f;
  if (PRO != PRO_QUANT) {
    // Sum of squares in the reference's order for its 4-warp CTA (decode.cu:213-228): thread i of 128
    // adds 8-element chunks i, i+128, ... in order, then a warp butterfly, then the 4 warp sums in order.
    float* red = reinterpret_cast<float*>(smem + L.red);
    if (threadIdx.x < 128) {
      float ss = 0.f;
      for (int i = threadIdx.x; i < K / 8; i += 128) {
        const uint4 v = reinterpret_cast<const uint4*>(xs)[i];
        const bf16* e = reinterpret_cast<const bf16*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float f = __bfloat162float(e[j]);
          ss += f * f;
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
    }
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) tot += red[i];
    rstd = rsqrtf(tot / (float)K + p.eps);
  }
  uint32_t* xh = reinterpret_cast<uint32_t*>(smem + L.xh);
  float* xsc = reinterpret_cast<float*>(smem + L.xscale);
  const int c = lane >> 3, hi = (lane >> 2) & 1, t = lane & 3;
  for (int g = warp; g < KB; g += warps) {
    const int k0 = g * QB + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(xs + k0);
    const bf16* e = reinterpret_cast<const bf16*>(&raw);
    float v[4];
    if (PRO != PRO_QUANT) {
      const uint2 nraw = *reinterpret_cast<const uint2*>(p.norm_w + k0);
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
    const uint32_t q = quant4(v[0], v[1], v[2], v[3], sc);   // x(32c + 16hi + 4t + 0..3)
    uint32_t* dst = xh + ((g * 4 + c) * 4 + t) * 4;
    dst[hi] = e4m3x2_to_f16x2(q);
    dst[2 + hi] = e4m3x2_to_f16x2(q >> 16);
    if (lane == 0) xsc[g] = sc;
  }
  __syncthreads();
}

// ---- main kernel -------------------------------------------------------------------------------------------
template <int PRO, int EPI, int SCALE, int NG>
__global__ void __launch_bounds__(512) fp8_gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int UB = GEMV_TILE_BYTES * NG;       // bytes per tile
  constexpr int RPU = GEMV_UNIT_ROWS * NG;       // rows per unit
  const int K = p.K, KB = K / QB, N = p.N;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int S = p.stages, ST = p.stage_tiles;
  const GemvSmem L = gemv_smem(K, warps, S, ST * UB);
  const int units = N / RPU;
  const long long T = (long long)units * KB;
  const long long TW = (long long)gridDim.x * warps;
  const long long gw = (long long)blockIdx.x * warps + warp;
  const int t0 = (int)(gw * T / TW), t1 = (int)((gw + 1) * T / TW);
  const int nchunks = (t1 - t0 + ST - 1) / ST;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bars) + warp * S;
  uint8_t* ring = smem + L.ring + (size_t)warp * S * ST * UB;
  const uint64_t pol = policy_evict_first();

  if (threadIdx.x == 0) tl_stamp(p.tl_slot, 0);
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  auto issue = [&](int ch) {  // lane 0: chunk ch of this warp's range into stage ch % S
    const int s = ch % S, ta = t0 + ch * ST, n = min(ST, t1 - ta);
    mbar_arrive_expect_tx(&bar[s], (uint32_t)(n * UB));
    bulk_g2s(ring + (size_t)s * ST * UB, p.w + (size_t)ta * UB, (uint32_t)(n * UB), &bar[s], pol);
  };
  const int first = min(S, nchunks);
  if (lane == 0)
    for (int ch = 0; ch < min(p.pre, first); ++ch) issue(ch);
  grid_dep_wait();
  grid_dep_launch();
  if (threadIdx.x == 0) tl_stamp(p.tl_slot, 1);
  if (lane == 0)
    for (int ch = min(p.pre, first); ch < first; ++ch) issue(ch);

  gemv_prologue<PRO>(p, smem, L);
  if (threadIdx.x == 0) tl_stamp(p.tl_slot, 2);
  const uint8_t* xh = smem + L.xh;
  const float* xsc = reinterpret_cast<const float*>(smem + L.xscale);

  float acc[NG][2];   // rows r = g and r = g + 8 of each 16-row sub-unit
  float swc[NG][2];   // channel scales of those rows
  float swb[NG][3];   // block scales of the unit's row block: lane l holds kb = l, l+32, l+64
  bool full = false;
  float best_v = -INFINITY;
  int best_i = 0x7FFFFFFF;

  auto row0 = [&](int u, int gi) { return (NG == 2 && gi == 1) ? N / 2 + u * 16 : u * 16; };
  auto block_scale = [&](int gi, int kb) {   // warp-uniform kb; all lanes must call
    const float v = kb < 32 ? swb[gi][0] : (kb < 64 ? swb[gi][1] : swb[gi][2]);
    return __shfl_sync(0xffffffffu, v, kb & 31);
  };
  auto begin_unit = [&](int u) {
    full = (u * KB >= t0) && ((u + 1) * KB <= t1);
#pragma unroll
    for (int gi = 0; gi < NG; ++gi) {
      acc[gi][0] = acc[gi][1] = 0.f;
      if (SCALE == SCALE_CHANNEL) {
        swc[gi][0] = __ldg(p.ws + row0(u, gi) + g);
        swc[gi][1] = __ldg(p.ws + row0(u, gi) + g + 8);
      } else {
        const float* srow = p.ws + (size_t)(row0(u, gi) / QB) * KB;
#pragma unroll
        for (int i = 0; i < 3; ++i) swb[gi][i] = (lane + 32 * i < KB) ? __ldg(srow + lane + 32 * i) : 0.f;
      }
    }
  };
  auto epilogue = [&](int u) {   // lanes with t == 0 own rows u*16 + g and + 8
    if (t != 0) return;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = u * 16 + g + 8 * j;
      if (EPI == EPI_STORE) {
        p.out[n] = __float2bfloat16_rn(acc[0][j]);
      } else if (EPI == EPI_ARGMAX) {
        p.out[n] = __float2bfloat16_rn(acc[0][j]);
        const float lv = bf16r(acc[0][j]);
        const int idx = p.row_offset + n;
        if (lv > best_v || (lv == best_v && idx < best_i)) { best_v = lv; best_i = idx; }
      } else if (EPI == EPI_RESIDUAL) {
        p.out[n] = __float2bfloat16_rn(__bfloat162float(p.out[n]) + bf16r(acc[0][j]));
      } else if (EPI == EPI_SWIGLU) {
        const float gt = bf16r(acc[0][j]);
        const float up = bf16r(acc[NG - 1][j]);
        const float act = bf16r(gt / (1.0f + expf(-gt)));
        p.out[n] = __float2bfloat16_rn(act * up);
      } else {  // EPI_F32
        p.out_f32[n] = acc[0][j];
      }
    }
  };

  int tt = t0, u = t0 / KB, kb = t0 - (t0 / KB) * KB;
  if (t0 < t1) begin_unit(u);
  int ch = 0;
  bool ok = true;
  for (; ch < nchunks; ++ch) {
    const int s = ch % S;
    if (!__all_sync(0xffffffffu, mbar_wait(&bar[s], (uint32_t)((ch / S) & 1)))) { ok = false; break; }
    if (ch == 0 && lane == 0) tl_stamp_max(p.tl_slot, 3);
    const uint8_t* buf = ring + (size_t)s * ST * UB;
    const int n_here = min(ST, t1 - tt);
    for (int i = 0; i < n_here; ++i, ++tt) {
      const uint8_t* tile = buf + (size_t)i * UB;
      const uint8_t* xk = xh + kb * 256 + t * 16;
      float dk[NG][2];
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) dk[gi][0] = dk[gi][1] = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 xb = lds128(xk + c * 64);
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          const uint4 w4 = lds128(tile + gi * GEMV_TILE_BYTES + c * 512 + lane * 16);
          float e[4];
          fp8_chunk_dot(w4, xb, e);
          dk[gi][0] += e[0];
          dk[gi][1] += e[2];
        }
      }
      if (full) {
        const float sx = xsc[kb];
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          float sw0, sw1;
          if (SCALE == SCALE_CHANNEL) { sw0 = swc[gi][0]; sw1 = swc[gi][1]; }
          else { sw0 = sw1 = block_scale(gi, kb); }
          acc[gi][0] += dk[gi][0] * sx * sw0;
          acc[gi][1] += dk[gi][1] * sx * sw1;
        }
      } else if (t == 0) {
        float* dst = p.part + ((size_t)u * KB + kb) * RPU + g;
#pragma unroll
        for (int gi = 0; gi < NG; ++gi) {
          dst[gi * 16] = dk[gi][0];
          dst[gi * 16 + 8] = dk[gi][1];
        }
      }
      if (kb == KB - 1 || tt == t1 - 1) {   // this warp's last tile of unit u
        if (full) {
          epilogue(u);
        } else {
          __threadfence();
          int last = 0;
          if (lane == 0) {
            const int mine = tt - max(t0, u * KB) + 1;
            last = (atomicAdd(&p.counters[u], mine) + mine == KB);
          }
          last = __shfl_sync(0xffffffffu, last, 0);
          if (last) {
            __threadfence();
            const float* src = p.part + (size_t)u * KB * RPU + g;
#pragma unroll
            for (int gi = 0; gi < NG; ++gi) acc[gi][0] = acc[gi][1] = 0.f;
            for (int k2 = 0; k2 < KB; ++k2) {
              const float sx = xsc[k2];
#pragma unroll
              for (int gi = 0; gi < NG; ++gi) {
                const float d0 = __ldcg(src + (size_t)k2 * RPU + gi * 16);
                const float d1 = __ldcg(src + (size_t)k2 * RPU + gi * 16 + 8);
                float sw0, sw1;
                if (SCALE == SCALE_CHANNEL) { sw0 = swc[gi][0]; sw1 = swc[gi][1]; }
                else { sw0 = sw1 = block_scale(gi, k2); }
                acc[gi][0] += d0 * sx * sw0;
                acc[gi][1] += d1 * sx * sw1;
              }
            }
            epilogue(u);
            if (lane == 0) p.counters[u] = 0;
          }
        }
      }
      if (++kb == KB) {
        kb = 0;
        ++u;
        if (tt + 1 < t1) begin_unit(u);
      }
    }
    __syncwarp();
    if (lane == 0 && ch + S < nchunks) {
      fence_proxy_async_smem();
      issue(ch + S);
    }
  }
  if (lane == 0) tl_stamp_max(p.tl_slot, 4);
  if (!ok) {  // a stage never arrived: wait (bounded) for this warp's copies still in flight, then stop
    for (int c2 = ch; c2 < min(ch + S, nchunks); ++c2) mbar_wait(&bar[c2 % S], (uint32_t)((c2 / S) & 1), 100000000ull);
  }

  if (EPI == EPI_ARGMAX) {
    unsigned long long key = (best_i == 0x7FFFFFFF) ? 0ull : argmax_key(best_v, best_i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
      key = other > key ? other : key;
    }
    unsigned long long* bb = reinterpret_cast<unsigned long long*>(smem + L.bestbuf);
    if (lane == 0) bb[warp] = key;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = 0;
      for (int i = 0; i < warps; ++i) b = bb[i] > b ? bb[i] : b;
      if (b) atomicMax(p.best, b);
    }
  }
}

// ---- bf16 lm_head (reference checkpoint format) with final RMSNorm and greedy argmax -------------------------
// Rows are split into equal contiguous ranges per warp and streamed one 8 KiB row per ring stage.
// Arithmetic order as the reference lm_head kernel (decode.cu:610-652) so logits are bit-identical:
// 256-thread strided sum of squares; per row lane l owns elements (32i + l)*8 .. +7, i = 0..15.
struct HeadParams {
  const bf16* w;             // [V, 4096] row-major
  const bf16* x;             // residual [4096]
  const bf16* norm_w;        // [4096]
  bf16* logits;              // [V]
  unsigned long long* best;  // packed key, zero before the launch
  int V;
  int row_offset;
  float eps;
  int stages, pre;
  int tl_slot;
};
constexpr int HEAD_WARPS = 8;
constexpr int HEAD_ROW_BYTES = HIDDEN * 2;
__host__ __device__ inline int head_smem_ring(int stages) { return align_up(HIDDEN * 4 + 8 * 4 + 8 * 8 + HEAD_WARPS * stages * 8, 1024); }
__host__ __device__ inline int head_smem_total(int stages) { return head_smem_ring(stages) + HEAD_WARPS * stages * HEAD_ROW_BYTES; }

__global__ void __launch_bounds__(HEAD_WARPS * 32) lm_head_bf16_kernel(const __grid_constant__ HeadParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int K = HIDDEN;
  float* xn = reinterpret_cast<float*>(smem);
  float* red = xn + K;
  unsigned long long* bb = reinterpret_cast<unsigned long long*>(red + 8);
  const int S = p.stages;
  uint64_t* bar = reinterpret_cast<uint64_t*>(bb + 8);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  bar += warp * S;
  uint8_t* ring = smem + head_smem_ring(S) + (size_t)warp * S * HEAD_ROW_BYTES;
  const long long TW = (long long)gridDim.x * HEAD_WARPS, gw = (long long)blockIdx.x * HEAD_WARPS + warp;
  const int r0 = (int)(gw * p.V / TW), r1 = (int)((gw + 1) * p.V / TW);
  const int nrows = r1 - r0;
  const uint64_t pol = policy_evict_first();
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  auto issue = [&](int i) {
    const int s = i % S;
    mbar_arrive_expect_tx(&bar[s], HEAD_ROW_BYTES);
    bulk_g2s(ring + (size_t)s * HEAD_ROW_BYTES, p.w + (size_t)(r0 + i) * K, HEAD_ROW_BYTES, &bar[s], pol);
  };
  const int first = min(S, nrows);
  if (threadIdx.x == 0) tl_stamp(p.tl_slot, 0);
  if (lane == 0)
    for (int i = 0; i < min(p.pre, first); ++i) issue(i);
  grid_dep_wait();
  grid_dep_launch();
  if (threadIdx.x == 0) tl_stamp(p.tl_slot, 1);
  if (lane == 0)
    for (int i = min(p.pre, first); i < first; ++i) issue(i);

  float ss = 0.f;
  for (int i = threadIdx.x; i < K; i += HEAD_WARPS * 32) {
    const float f = __bfloat162float(p.x[i]);
    xn[i] = f;
    ss += f * f;
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < HEAD_WARPS; ++i) tot += red[i];
  const float rstd = rsqrtf(tot / (float)K + p.eps);
  __syncthreads();
  for (int i = threadIdx.x; i < K; i += HEAD_WARPS * 32) xn[i] = bf16r(__bfloat162float(p.norm_w[i]) * bf16r(xn[i] * rstd));
  __syncthreads();

  float best_v = -INFINITY;
  int best_i = 0x7FFFFFFF;
  int i = 0;
  bool ok = true;
  for (; i < nrows; ++i) {
    const int s = i % S;
    if (!__all_sync(0xffffffffu, mbar_wait(&bar[s], (uint32_t)((i / S) & 1)))) { ok = false; break; }
    const uint8_t* wrow = ring + (size_t)s * HEAD_ROW_BYTES;
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
    __syncwarp();
    if (lane == 0 && i + S < nrows) {
      fence_proxy_async_smem();
      issue(i + S);
    }
    acc = warp_sum(acc);
    const int row = r0 + i;
    const float lv = bf16r(acc);
    if (lane == 0) p.logits[row] = __float2bfloat16_rn(acc);
    const int gidx = p.row_offset + row;
    if (lv > best_v || (lv == best_v && gidx < best_i)) { best_v = lv; best_i = gidx; }
  }
  if (!ok) {
    for (int c2 = i; c2 < min(i + S, nrows); ++c2) mbar_wait(&bar[c2 % S], (uint32_t)((c2 / S) & 1), 100000000ull);
  }
  if (lane == 0) tl_stamp_max(p.tl_slot, 4);
  if (lane == 0) bb[warp] = (best_i == 0x7FFFFFFF) ? 0ull : argmax_key(best_v, best_i);
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < HEAD_WARPS; ++w) b = bb[w] > b ? bb[w] : b;
    if (b) atomicMax(p.best, b);
  }
}

}  // namespace qk
