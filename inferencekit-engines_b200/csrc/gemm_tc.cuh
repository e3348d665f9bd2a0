// Batched FP8 W8A8 linear on the 5th-generation tensor cores (tcgen05), for a few activation rows at a time
// (decode batches of 2..128 sequences, or a prefill chunk of up to 128 positions):
//
//   Y[m, n] = bf16( sum over K blocks kb, in order, of  D_kb[m, n] * s_x[m, kb] * s_w[n (, kb)] ),
//   D_kb[m, n] = the fp32 dot of the e4m3 activations and weights over the 128 k of block kb,
//
// the reference recipe of its batched path (Q/kernels/prefill.py:44-73 `_fp8_block_matmul_kernel`,
// :121-156 `fp8_matmul`, activations quantized per 128-group by :23-41 `act_quant`).
//
// Work split: the (weight tile of 128 rows, K block) pairs, tile-major, are dealt in equal contiguous ranges to
// one CTA per SM, whatever N is. Per CTA (320 threads):
//  * warp 0, one lane: TMA loads, per pair, the weight box {128 k-bytes, 128 rows} and the activation box
//    {128 k-bytes, MP rows} (rows past M zero-filled), both with the 128-byte swizzle, into a ring of
//    tc_stages<MP>() stages;
//  * warp 1 owns the tensor memory (tc_naccs<MP>() accumulators of MP fp32 columns: the MMAs of later pairs run
//    while the epilogue still reads earlier ones) and one lane issues, per pair, four
//    tcgen05.mma.kind::f8f6f4 (M 128 = weight rows, N = MP = activation rows, K 32 each, the first from zero)
//    reading both operands straight from shared memory, then commits to the stage's `empty` barrier and to
//    the accumulator's `dfull` barrier;
//  * warps 2-9 (TMEM lane quarters 2, 3, 0, 1, twice: warps 2-5 take activation rows [0, MP/2), warps 6-9 the
//    rest) read each K block's dots with tcgen05.ld, free the accumulator, and fold them into fp32 registers in
//    K order: acc[m] += (D * s_x[m, kb]) * s_w[n, kb] for block scales; for per-channel scales, which do not
//    change with kb, acc[m] += D * s_x[m, kb] and the CTA's piece of the tile is multiplied by s_w[n] once
//    (the activation scales staged in shared memory once, K-block major, the weight scales per CTA).
// A tile whose pairs lie in one CTA is stored directly (bf16). A tile split between consecutive CTAs: every
// piece stores its fp32 partial in `part` (slot 0 for a CTA's first tile, 1 for its last) and counts itself on
// the tile's counter; the CTA that completes the count adds the pieces in CTA order and stores the tile.
// Deterministic for a given grid; the K-block sum is split at CTA boundaries, so results match the oracle's
// in-order sum to rounding (the parity bar of this path is 1e-2 rel-L2, not bit-identity).
#pragma once
#include <cuda.h>   // CUtensorMap
#include "common.cuh"

namespace qk {

constexpr int TC_TILE = 128;          // weight rows per tile (the UMMA M)
constexpr int TC_BK = 128;            // K per pair: one activation quant group, one weight scale block
constexpr int TC_EPI_WARPS = 8;       // two per TMEM lane quarter, each folding half of the activation rows
constexpr int TC_THREADS = (2 + TC_EPI_WARPS) * 32;   // warp 0 producer, warp 1 MMA issuer and TMEM owner
constexpr int TC_MAX_ROWS = 128;
constexpr int TC_MAX_KB = 16384 / TC_BK;
constexpr int TC_MAX_KB_128 = 12288 / TC_BK;   // 128 padded rows: K up to 12,288 (the activation scales' room)
constexpr int TC_MAX_TILES = 8192;    // the tile counters' fixed region: N up to 1,048,576 rows
constexpr int TC_SW_MAX = 2048;       // weight scales staged in shared memory per CTA (16 tiles' channels)

struct TcGemmParams {
  CUtensorMap tm_w;     // weights fp8 [N][K] row-major: box {128, 128}, 128-byte swizzle
  CUtensorMap tm_x;     // activations fp8 [M][K]: box {128, MP}, 128-byte swizzle, rows >= M read as zero
  // Tile-packed operands (both set, or both null for the tensor maps above): the weights as
  // [N/128][K/128] tiles of 16 KiB and the activations as [K/128] tiles of MP x 128 B, each tile already in
  // the 128-byte-swizzle K-major image the MMAs read, so one bulk copy per operand and pair fills a stage
  // and a CTA's weight range is one contiguous stream.
  const uint8_t* w_tiles;
  const uint8_t* x_tiles;
  const float* sx;      // activation scales [M][K/128]
  const float* sw;      // weight scales [N] (per channel) or [N/128][K/128] (block)
  bf16* out;            // [M][N]
  float* part;          // split-tile partials [gridDim.x][2][128][MP]
  int* counters;        // [N/128], zero between launches (left zero)
  int M, N, K;
  int scale_block;
};

// Ring depth and accumulator count per padded row count: the ring fills 160-200 KiB of shared memory, the
// accumulators at most 512 TMEM columns (128 rows: four of 128 columns).
template <int MP>
__host__ __device__ constexpr int tc_stages() {
  return MP >= 128 ? 5 : (MP >= 64 ? 7 : (MP >= 32 ? 8 : 9));
}
template <int MP>
__host__ __device__ constexpr int tc_max_kb() {
  return MP >= 128 ? TC_MAX_KB_128 : TC_MAX_KB;
}
template <int MP>
__host__ __device__ constexpr int tc_naccs() {
  return MP >= 64 ? 4 : 8;
}

template <int MP>
struct TcSmem {
  static constexpr int S = tc_stages<MP>(), A = tc_naccs<MP>();
  uint8_t w[S][TC_TILE * TC_BK];   // 16 KiB per stage (1024-byte aligned: the swizzle atom)
  uint8_t x[S][MP * TC_BK];        // MP * 128 B per stage (a multiple of 1024 for MP % 8 == 0)
  uint64_t full[S], empty[S];
  uint64_t dfull[A], dempty[A];
  uint32_t tmem_base;
  int last;
  alignas(16) float sxs[tc_max_kb<MP>() * MP];   // the activation scales, K-block major: sxs[kb * MP + m] (0 for m >= M)
  float sws[TC_SW_MAX];   // the CTA's weight scales: per channel, its tiles' rows; per block, one per pair
};

// Instruction descriptor of tcgen05.mma.kind::f8f6f4: D fp32, A and B e4m3, both K-major, M = 128, N = MP.
template <int MP>
__host__ __device__ constexpr uint32_t tc_idesc() {
  return (1u << 4)                              // D format: F32
         | (0u << 7) | (0u << 10)               // A, B format: E4M3
         | (0u << 15) | (0u << 16)              // A, B K-major
         | ((uint32_t)(MP >> 3) << 17)          // N / 8
         | ((uint32_t)(TC_TILE >> 4) << 24);    // M / 16
}
// Shared-memory matrix descriptor of a K-major operand in the 128-byte-swizzle canonical layout (rows of 128 bytes,
// 8-row groups 1024 bytes apart; the leading offset is unused for this layout and set to 1).
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF)     // start address / 16
         | ((uint64_t)1 << 16)                  // leading byte offset / 16
         | ((uint64_t)(1024 >> 4) << 32)        // stride byte offset / 16
         | ((uint64_t)1 << 46)                  // descriptor version (sm_100)
         | ((uint64_t)2 << 61);                 // layout: 128-byte swizzle
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  const uint32_t z = 0;   // no output lane disabled
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 8 consecutive fp32 columns of this warp's 32 TMEM lanes (one lane per thread); tc_wait_ld before use
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// The CTA whose range of pairs holds pair u, for ranges [c * P / G, (c + 1) * P / G).
__host__ __device__ __forceinline__ int tc_owner(long long u, long long P, int G) {
  return (int)(((u + 1) * G - 1) / P);
}

template <int MP>
__global__ void __launch_bounds__(TC_THREADS, 1) fp8_gemm_tc_kernel(const __grid_constant__ TcGemmParams p) {
  extern __shared__ __align__(1024) uint8_t tc_smem[];
  TcSmem<MP>& sm = *reinterpret_cast<TcSmem<MP>*>(tc_smem);
  constexpr int S = TcSmem<MP>::S, A = TcSmem<MP>::A;
  constexpr uint32_t NCOLS = A * MP < 32 ? 32 : A * MP;   // TMEM columns (a power of 2)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = p.K / TC_BK, n_tiles = p.N / TC_TILE;
  const long long P = (long long)n_tiles * KB;
  const int G = gridDim.x, c = blockIdx.x;
  const int u0 = (int)(c * P / G), u1 = (int)((c + 1) * P / G);
  const int nu = u1 - u0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < A; ++b) {
      mbar_init(&sm.dfull[b], 1);
      mbar_init(&sm.dempty[b], TC_EPI_WARPS);
    }
    fence_mbar_init();
    // the weights are no output of an earlier kernel: the first stages' weight boxes are requested before
    // griddepcontrol.wait, so under programmatic dependent launch they stream while the quantizer still runs
    for (int i = 0; i < min(S, nu); ++i) {
      const int u = u0 + i, t = u / KB, kb = u - t * KB;
      mbar_arrive_expect_tx(&sm.full[i], TC_TILE * TC_BK + MP * TC_BK);
      if (p.w_tiles)
        bulk_g2s(sm.w[i], p.w_tiles + (size_t)u * (TC_TILE * TC_BK), TC_TILE * TC_BK, &sm.full[i], policy_evict_first());
      else
        tma_load_2d(sm.w[i], &p.tm_w, kb * TC_BK, t * TC_TILE, &sm.full[i]);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                 "r"(NCOLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // The weight scales of the CTA's pairs go to shared memory before the wait (like the weights, they are no
  // earlier kernel's output), so the epilogue's fold never waits on a global load. Ranges too long to stage
  // (more than 16 tiles per CTA) read them from global memory.
  const int t_first = u0 / KB, t_last = nu > 0 ? (u1 - 1) / KB : t_first;
  const int n_sw = p.scale_block ? nu : (t_last - t_first + 1) * TC_TILE;
  const bool sw_staged = n_sw <= TC_SW_MAX;
  if (sw_staged)
    for (int i = threadIdx.x; i < n_sw; i += TC_THREADS)
      sm.sws[i] = p.scale_block ? __ldg(p.sw + u0 + i) : __ldg(p.sw + (size_t)t_first * TC_TILE + i);
  grid_dep_wait();   // the quantized activations, their scales and the output buffer are the previous kernels'
  for (int i = threadIdx.x; i < MP * KB; i += TC_THREADS) {
    const int kb = i / MP, m = i - kb * MP;
    sm.sxs[i] = m < p.M ? p.sx[m * KB + kb] : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;

  if (warp == 0) {
    if (lane == 0) {   // producer
      const uint64_t pol = policy_evict_first();
      auto load_x = [&](int s, int kb) {
        if (p.x_tiles)
          bulk_g2s(sm.x[s], p.x_tiles + (size_t)kb * (MP * TC_BK), MP * TC_BK, &sm.full[s]);
        else
          tma_load_2d(sm.x[s], &p.tm_x, kb * TC_BK, 0, &sm.full[s]);
      };
      for (int i = 0; i < min(S, nu); ++i) load_x(i, (u0 + i) % KB);
      for (int i = S; i < nu; ++i) {
        const int s = i % S;
        if (i >= S && !mbar_wait(&sm.empty[s], (uint32_t)(((i / S) - 1) & 1))) break;
        const int u = u0 + i, t = u / KB, kb = u - t * KB;
        mbar_arrive_expect_tx(&sm.full[s], TC_TILE * TC_BK + MP * TC_BK);
        if (p.w_tiles)
          bulk_g2s(sm.w[s], p.w_tiles + (size_t)u * (TC_TILE * TC_BK), TC_TILE * TC_BK, &sm.full[s], pol);
        else
          tma_load_2d(sm.w[s], &p.tm_w, kb * TC_BK, t * TC_TILE, &sm.full[s]);
        load_x(s, kb);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {   // MMA issuer
      constexpr uint32_t idesc = tc_idesc<MP>();
      for (int i = 0; i < nu; ++i) {
        const int s = i % S, b = i % A;
        if (!mbar_wait(&sm.full[s], (uint32_t)((i / S) & 1))) break;
        if (i >= A && !mbar_wait(&sm.dempty[b], (uint32_t)(((i / A) - 1) & 1))) break;
        tc_fence_after();
        const uint32_t wa = smem_u32(sm.w[s]), xa = smem_u32(sm.x[s]);
#pragma unroll
        for (int k = 0; k < TC_BK / 32; ++k)
          tc_mma(tbase + (uint32_t)(b * MP), tc_desc_sw128(wa + 32 * k), tc_desc_sw128(xa + 32 * k), idesc, k > 0);
        tc_commit(&sm.empty[s]);   // the stage's shared memory is free once these MMAs have read it
        tc_commit(&sm.dfull[b]);   // accumulator b holds pair i's block dots
      }
    }
  } else {   // epilogue warps 2-9: TMEM lanes 32 q .. 32 q + 31 (q = warp % 4) = this thread's weight rows,
             // activation rows [h * MP / 2, (h + 1) * MP / 2) with h = (warp - 2) / 4
    constexpr int HM = MP / 2;
    const int q = warp & 3, r = 32 * q + lane, h = (warp - 2) / 4, m0 = h * HM;
    auto w_scale = [&](int u) {   // block scales [N/128][K/128]: pair u = t * KB + kb is element u
      if (sw_staged) return p.scale_block ? sm.sws[u - u0] : sm.sws[(u / KB - t_first) * TC_TILE + r];
      return p.scale_block ? __ldg(p.sw + u) : __ldg(p.sw + (u / KB) * TC_TILE + r);
    };
    float acc[HM];
#pragma unroll
    for (int m = 0; m < HM; ++m) acc[m] = 0.f;
    float sw_next = nu > 0 ? w_scale(u0) : 0.f;
    bool ok = true;   // a failed wait is recorded, but every epilogue warp keeps the same control flow (they meet at
                      // named barriers); once a wait has timed out, later waits give up at once
    for (int i = 0; i < nu; ++i) {
      const int b = i % A, u = u0 + i, t = u / KB, kb = u - t * KB;
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.dfull[b], (uint32_t)((i / A) & 1))) && ok;
      tc_fence_after();
      uint32_t d[HM / 8][8];
#pragma unroll
      for (int j = 0; j < HM / 8; ++j) tc_ld8(tbase + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * MP + m0 + 8 * j), d[j]);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.dempty[b]);
      const int n = t * TC_TILE + r;
      const float swv = sw_next;
      if (i + 1 < nu) sw_next = w_scale(u + 1);
      const float* sxk = sm.sxs + kb * MP + m0;
      // rows past M fold zeros (their scale is 0) and are never stored
      if (p.scale_block) {   // the block's weight scale varies with kb: acc += (D * s_x) * s_w per block
#pragma unroll
        for (int mm = 0; mm < HM; mm += 4) {
          const float4 sx4 = *reinterpret_cast<const float4*>(sxk + mm);
          acc[mm] += (__uint_as_float(d[mm / 8][mm % 8]) * sx4.x) * swv;
          acc[mm + 1] += (__uint_as_float(d[mm / 8][mm % 8 + 1]) * sx4.y) * swv;
          acc[mm + 2] += (__uint_as_float(d[mm / 8][mm % 8 + 2]) * sx4.z) * swv;
          acc[mm + 3] += (__uint_as_float(d[mm / 8][mm % 8 + 3]) * sx4.w) * swv;
        }
      } else {               // one weight scale per row: acc += D * s_x, times s_w once the piece is summed
#pragma unroll
        for (int mm = 0; mm < HM; mm += 4) {
          const float4 sx4 = *reinterpret_cast<const float4*>(sxk + mm);
          acc[mm] = fmaf(__uint_as_float(d[mm / 8][mm % 8]), sx4.x, acc[mm]);
          acc[mm + 1] = fmaf(__uint_as_float(d[mm / 8][mm % 8 + 1]), sx4.y, acc[mm + 1]);
          acc[mm + 2] = fmaf(__uint_as_float(d[mm / 8][mm % 8 + 2]), sx4.z, acc[mm + 2]);
          acc[mm + 3] = fmaf(__uint_as_float(d[mm / 8][mm % 8 + 3]), sx4.w, acc[mm + 3]);
        }
      }
      if (kb != KB - 1 && i != nu - 1) continue;
      if (!p.scale_block) {
#pragma unroll
        for (int mm = 0; mm < HM; ++mm) acc[mm] *= swv;
      }
      // the end of this CTA's piece of tile t
      const bool whole = max(u0, t * KB) == t * KB && u == t * KB + KB - 1;
      if (whole) {
#pragma unroll
        for (int mm = 0; mm < HM; ++mm)
          if (m0 + mm < p.M) p.out[(size_t)(m0 + mm) * p.N + n] = __float2bfloat16_rn(acc[mm]);
      } else {
        const int slot = t == t_first ? 0 : 1;
        float* mine = p.part + ((size_t)(c * 2 + slot) * TC_TILE + r) * MP + m0;
#pragma unroll
        for (int mm = 0; mm < HM; mm += 4)
          *reinterpret_cast<float4*>(mine + mm) = make_float4(acc[mm], acc[mm + 1], acc[mm + 2], acc[mm + 3]);
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"n"(TC_EPI_WARPS * 32) : "memory");   // the epilogue warps
        const int c_first = tc_owner((long long)t * KB, P, G), c_last = tc_owner((long long)t * KB + KB - 1, P, G);
        if (warp == 2 && lane == 0) {
          const int before = atomicAdd(p.counters + t, 1);
          sm.last = before == c_last - c_first;
          if (sm.last) {
            __threadfence();
            p.counters[t] = 0;
          }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(TC_EPI_WARPS * 32) : "memory");
        if (sm.last) {   // add the pieces in CTA order (into acc: this piece's own values are in `part` too)
#pragma unroll
          for (int mm = 0; mm < HM; ++mm) acc[mm] = 0.f;
          for (int cc = c_first; cc <= c_last; ++cc) {
            const int sl = t == (int)((long long)cc * P / G) / KB ? 0 : 1;   // t is cc's first tile, or its last
            const float* pc = p.part + ((size_t)(cc * 2 + sl) * TC_TILE + r) * MP + m0;
#pragma unroll
            for (int mm = 0; mm < HM; mm += 4) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(pc + mm));
              acc[mm] += v.x;
              acc[mm + 1] += v.y;
              acc[mm + 2] += v.z;
              acc[mm + 3] += v.w;
            }
          }
#pragma unroll
          for (int mm = 0; mm < HM; ++mm)
            if (m0 + mm < p.M) p.out[(size_t)(m0 + mm) * p.N + n] = __float2bfloat16_rn(acc[mm]);
        }
      }
#pragma unroll
      for (int mm = 0; mm < HM; ++mm) acc[mm] = 0.f;
    }
    if (!ok && lane == 0) atomicOr(&g_dev_error, DEVERR_MBAR_TIMEOUT);
  }
  // every tcgen05 operation of the CTA is complete before the allocating warp frees the tensor memory
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(NCOLS) : "memory");
  }
}

// x bf16 [M][K] -> optional RMSNorm per row (as the GEMV prologue: bf16(w * bf16(x * rstd))) -> e4m3 per 128-group
// (s = amax / 448 with div.full, round to nearest even, saturating; a zero group gives zeros) -> qx, sx [M][K/128].
// qx is row-major [M][K] (tiled_mp = 0), or tiles [K/128][tiled_mp][128 B] in the 128-byte-swizzle image (16-byte
// chunk c of row m at chunk c ^ (m % 8)), rows M .. tiled_mp - 1 zero. One CTA of 256 threads per row (grid M, or
// tiled_mp when tiled).
__global__ void __launch_bounds__(256) quantize_rows_kernel(const bf16* __restrict__ x, const bf16* __restrict__ norm_w,
                                                            int M, int K, float eps, uint8_t* __restrict__ qx,
                                                            float* __restrict__ sx, int tiled_mp) {
  __shared__ float red[8];
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  grid_dep_wait();     // x is the previous kernel's output
  grid_dep_launch();   // the GEMM may start its weight stream now; it waits for this grid before reading qx
  // byte offset of k (a multiple of 4) of this row in qx
  auto qx_at = [&](int k) -> size_t {
    if (!tiled_mp) return (size_t)row * K + k;
    const int kb = k / QB, c = (k % QB) / 16;
    return ((size_t)kb * tiled_mp + row) * QB + ((c ^ (row & 7)) * 16) + (k & 15);
  };
  if (row >= M) {   // a padding row of the tiled layout
    for (int k = tid * 4; k < K; k += 256 * 4) *reinterpret_cast<uint32_t*>(qx + qx_at(k)) = 0u;
    return;
  }
  const bf16* xr = x + (size_t)row * K;
  float rstd = 1.f;
  if (norm_w) {
    float ss = 0.f;
    for (int i = tid; i < K; i += 256) {
      const float f = __bfloat162float(xr[i]);
      ss += f * f;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    rstd = rsqrtf(tot / (float)K + eps);
  }
  const int KB = K / QB;
  for (int g = warp; g < KB; g += 8) {
    const int k0 = g * QB + lane * 4;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float f = __bfloat162float(xr[k0 + j]);
      v[j] = norm_w ? bf16r(__bfloat162float(norm_w[k0 + j]) * bf16r(f * rstd)) : f;
    }
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    amax = warp_max(amax);
    const float s = div_full(amax, 448.0f);
    *reinterpret_cast<uint32_t*>(qx + qx_at(k0)) = quant4(v[0], v[1], v[2], v[3], s);
    if (lane == 0) sx[(size_t)row * KB + g] = s;
  }
}

template <int MP>
inline size_t tc_smem_bytes() { return sizeof(TcSmem<MP>); }

}  // namespace qk
