// Shared device helpers for the Qwen3-8B FP8 decode kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace qk {

using bf16 = __nv_bfloat16;

constexpr int HIDDEN = 4096;
constexpr int HEAD_DIM = 128;
constexpr int GQA = 4;          // query heads per KV head
constexpr int QB = 128;         // quantization block (weights and activations)

// Device-side error word: bounded waits that give up set a bit here instead of hanging; the host reads
// and clears it with qk_get_device_error().
enum : int { DEVERR_MBAR_TIMEOUT = 1, DEVERR_BAD_STATE = 2, DEVERR_GRID_TIMEOUT = 4 };
// Once a wait has timed out anywhere, every later wait gives up at once instead of waiting its own limit,
// so a failure ends the launch quickly (the host reads and clears the word with qk_get_device_error).
constexpr int DEVERR_WAIT_FAILED = DEVERR_MBAR_TIMEOUT | DEVERR_GRID_TIMEOUT;
__device__ int g_dev_error = 0;
__device__ __forceinline__ bool wait_failed() {
  return (*reinterpret_cast<volatile int*>(&g_dev_error) & DEVERR_WAIT_FAILED) != 0;
}

// Optional profiling timeline (qk_set_timeline): a caller buffer of `g_timeline_slots` regions of
// TL_SLOT_WORDS u64; launch number `slot` (assigned by the host in launch order) owns region `slot`, and CTA c
// (c < TL_MAX_CTAS) writes %globaltimer stamps into words c*TL_CTA_WORDS + i. Null when disabled.
constexpr int TL_CTA_WORDS = 8;
constexpr int TL_MAX_CTAS = 256;
constexpr int TL_SLOT_WORDS = TL_CTA_WORDS * TL_MAX_CTAS;
__device__ unsigned long long* g_timeline = nullptr;
__device__ int g_timeline_slots = 0;

// A bounded wait gives up after this many nanoseconds of %globaltimer.
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
// The low / high bf16 of a 32-bit word as f32 (exact: a bf16 is the high half of an f32).
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned long long* tl_cta(int slot) {
  unsigned long long* tl = g_timeline;
  const int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  if (tl == nullptr || slot < 0 || slot >= g_timeline_slots || cta >= TL_MAX_CTAS) return nullptr;
  return tl + (size_t)slot * TL_SLOT_WORDS + (size_t)cta * TL_CTA_WORDS;
}
__device__ __forceinline__ void tl_stamp(int slot, int i) {
  unsigned long long* t = tl_cta(slot);
  if (t) t[i] = globaltimer();
}
__device__ __forceinline__ void tl_stamp_max(int slot, int i) {
  unsigned long long* t = tl_cta(slot);
  if (t) atomicMax(t + i, globaltimer());
}

// ---- programmatic dependent launch ------------------------------------------------------------------------
// grid_dep_wait blocks until the preceding kernel in the stream has completed and its writes are visible;
// grid_dep_launch allows the next kernel to be scheduled. Every kernel here calls grid_dep_launch only
// after grid_dep_wait, so while kernel i runs, kernel i-2 has completed: code before grid_dep_wait may
// read data written two or more launches earlier (KV rows of earlier tokens, the step state) but nothing
// the immediately preceding kernel writes. Both are no-ops without the launch attribute.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- shared memory, mbarriers, bulk async copies -----------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking: has the phase with this parity completed? (acquire, like try_wait)
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_n(uint64_t* bar, uint32_t n) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(n) : "memory");
}

// Wait for phase `parity` of an mbarrier, at most `limit_ns`; on timeout set the device error word.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned long long limit_ns = WAIT_LIMIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  // Short waits poll only the barrier (clock64 is a local register); after ~0.25 ms the loop also checks
  // the wall clock and the device error word, both of which cost a global round trip.
  const long long c0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - c0 > 500000) break;
  }
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (wait_failed()) return false;
    if (globaltimer() - t0 > limit_ns) {
      atomicOr(&g_dev_error, DEVERR_MBAR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// L2 policy for data read exactly once per token (weights): evict first, so the small activations,
// KV rows of the current chunk and scratch stay in L2.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Bulk (non-tensor) async copy global -> shared, completion counted on an mbarrier in transaction bytes.
// dst, src 16-byte aligned, bytes a multiple of 16. Destination: this CTA only.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Tiled TMA load of one box of a 4-D tensor map into this CTA's shared memory, completion counted on an
// mbarrier in transaction bytes. x (innermost) * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, int x, int y, int z, int w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint4 lds128_at(uint32_t a) {   // a: shared-memory address
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
  return r;
}
__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(smem_u32(p)));
  return r;
}

// 16-byte global load of data read once per token: no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---- FP8 arithmetic ----------------------------------------------------------------------------------------
// Two e4m3 values (low byte -> low half) to an f16x2 register; exact (every e4m3 value is an f16 value).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((uint16_t)two_bytes));
  return r;
}

// Tensor-core D[16x8] += A[16x16] * B[16x8], f16 operands, fp32 accumulate (legacy warp-level mma).
__device__ __forceinline__ void hmma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm(   // a pure register computation: not volatile, so independent MMAs can be interleaved
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 32-wide K chunk of an fp8 dot for two weight rows (r and r+8 of a 16-row unit), x in every B column.
// w4 = this lane's 16 weight bytes of the chunk: {row r: k 4t..4t+3, row r+8: k 4t.., row r: k 16+4t..,
// row r+8: k 16+4t..}; xb = the matching x fragments as f16x2 {x(4t,4t+1), x(16+4t,+1), x(4t+2,+3),
// x(16+4t+2,+3)}. Returns the chunk dots of rows r (e[0]) and r+8 (e[2]).
// Operand placement and chaining: the pairs (4t,4t+1) and (16+4t,16+4t+1) go through one k16 MMA from zero,
// the pairs (4t+2,4t+3) and (16+4t+2,..) through a second one accumulating onto it. This is bit-identical to
// sm_100's `mma.sync.m16n8k32 ... e4m3.e4m3` (verified on 131k random chunks, both operand orientations),
// which the reference decode kernel uses as its dot engine, while costing only the 8 weight conversions.
__device__ __forceinline__ void fp8_chunk_dot(const uint4 w4, const uint4 xb, float (&e)[4]) {
  e[0] = e[1] = e[2] = e[3] = 0.f;
  hmma16816(e, e4m3x2_to_f16x2(w4.x), e4m3x2_to_f16x2(w4.y), e4m3x2_to_f16x2(w4.z), e4m3x2_to_f16x2(w4.w), xb.x, xb.y);
  hmma16816(e, e4m3x2_to_f16x2(w4.x >> 16), e4m3x2_to_f16x2(w4.y >> 16), e4m3x2_to_f16x2(w4.z >> 16),
            e4m3x2_to_f16x2(w4.w >> 16), xb.z, xb.w);
}

// The reference quantizer divides with the approximate `div.full.f32` (what Triton emits for fp32 `/`).
// Activations and their max are bf16, so x/s often lands on a rounding tie between two fp8 values; using
// the same instruction keeps the quantized activations identical to the reference.
__device__ __forceinline__ float div_full(float a, float b) {
  float r;
  asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// 4 floats -> 4 packed e4m3 bytes (round to nearest even, saturating); scale 0 gives 0.
__device__ __forceinline__ uint32_t quant4(float a, float b, float c, float d, float s) {
  const bool nz = s > 0.f;
  const float qa = nz ? div_full(a, s) : 0.f, qb = nz ? div_full(b, s) : 0.f;
  const float qc = nz ? div_full(c, s) : 0.f, qd = nz ? div_full(d, s) : 0.f;
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(qa, qb), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(qc, qd), __NV_SATFINITE, __NV_E4M3);
  return (uint32_t)lo | ((uint32_t)hi << 16);
}

// Greedy argmax key: order-preserving float bits in the high word, (~index) in the low word, so the u64
// maximum is the largest value and, among equal values, the smallest index.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)idx);
}

}  // namespace qk
