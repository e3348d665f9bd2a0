// C ABI of the B200 decode kernels: argument checks, launch shapes, PDL launches. One translation unit so
// the device symbols (error word) are shared by every kernel without relocatable device code.
#include <cudaTypedefs.h>   // PFN_cuTensorMapEncodeTiled

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/qwen3_b200.h"
#include "attention.cuh"
#include "attention_fp8kv.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "prefill.cuh"
#include "step.cuh"

static_assert(sizeof(qk_layer_t) == sizeof(qk::StepLayer), "qk_layer_t must mirror StepLayer");

using namespace qk;

namespace {

thread_local char g_msg[512] = "";
bool g_pdl = false;
int g_tl_next = -1;        // next timeline slot (launch number since qk_set_timeline), -1 when off
bool g_tl_ever = false;    // a timeline buffer was set at some point

int next_tl_slot() { return g_tl_next >= 0 ? g_tl_next++ : -1; }

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  return fail(QK_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// TMA map of a K or V cache: bf16 {128 dims, max_seq keys, n_kv heads, n_outer} (n_outer = layers for the fused
// step, sequences for the attention op), box {64, box_rows, 1, 1}, 128-byte swizzle, rows past max_seq
// zero-filled. outer_stride_bytes: distance between consecutive outer indices.
int encode_cache_map(CUtensorMap* map, void* base, int max_seq, int n_kv, int n_outer, long long outer_stride_bytes,
                     int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(QK_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[4] = {HEAD_DIM, (cuuint64_t)max_seq, (cuuint64_t)n_kv, (cuuint64_t)n_outer};
  const cuuint64_t strides[3] = {HEAD_DIM * 2, (cuuint64_t)max_seq * HEAD_DIM * 2, (cuuint64_t)outer_stride_bytes};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QK_EINVAL, "cuTensorMapEncodeTiled failed for a KV cache (CUresult %d)", (int)r);
  return QK_OK;
}
int encode_kv_map(CUtensorMap* map, void* base, int max_seq, int n_kv, int n_layers, long long layer_stride_bytes) {
  return encode_cache_map(map, base, max_seq, n_kv, n_layers, layer_stride_bytes, 64);
}

// TMA map of a row-major fp8 matrix [rows][cols] (cols bytes per row), box {128 bytes, box_rows}, 128-byte
// swizzle, rows past the end zero-filled.
int encode_fp8_rows_map(CUtensorMap* map, const void* base, long long rows, long long cols, int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(QK_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols};
  const cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QK_EINVAL, "cuTensorMapEncodeTiled failed for an fp8 matrix (CUresult %d)", (int)r);
  return QK_OK;
}

int device_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// Raise a kernel's dynamic shared-memory limit once per (kernel, device); done on the first (eager) call,
// so nothing but launches happen while a stream is being captured.
int ensure_smem(const void* fn, int bytes) {
  static std::mutex mu;
  static const void* fns[256];
  static int devs[256], limit[256];
  static int n = 0;
  if (bytes <= 48 * 1024) return QK_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < n; ++i)
    if (fns[i] == fn && devs[i] == dev && limit[i] >= bytes) return QK_OK;
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (bytes > optin) return fail(QK_EINVAL, "needs %d bytes of shared memory per CTA, device allows %d", bytes, optin);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  if (n < 256) { fns[n] = fn; devs[n] = dev; limit[n] = optin; ++n; }
  return QK_OK;
}

template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return QK_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// The failure path of the bounded waits, on purpose: thread 0 waits, with the given limit, either for phase 0
// of a fresh mbarrier that nothing arrives on (mode 0, the ring's wait) or for a counter that nothing adds to
// (mode 1, the cross-GPU counter wait). Both give up, set the device error word and return.
__global__ void wait_probe_kernel(int mode, const unsigned long long* counter, unsigned long long limit_ns,
                                  int* gave_up) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  bool ok;
  if (mode == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    ok = mbar_wait(&bar, 0u, limit_ns);
  } else {
    wait_sys_counter(counter, 1ull, limit_ns);
    ok = ld_acquire_sys_u64(counter) >= 1ull;
  }
  *gave_up = ok ? 0 : 1;
}

struct GemvShape { int warps, stages, stage_tiles, pre, ctas; };

GemvShape gemv_defaults(int kind) {
  // 8 warps x 4 stages x 4 KiB ring per warp (128 KiB per CTA), one CTA per SM
  const bool pairs = (kind == QK_GEMV_GATE_UP || kind == QK_GEMV_GATE_UP_RESADD);
  return GemvShape{8, 4, pairs ? 1 : 2, 4, 1};
}

template <int PRO, int EPI, int NG>
int launch_gemv_scaled(int scale_mode, const GemvParams& p, const GemvShape& sh, cudaStream_t stream) {
  const int smem = gemv_smem(p.K, sh.warps, sh.stages, sh.stage_tiles * GEMV_TILE_BYTES * NG).total;
  const dim3 grid(device_sms() * sh.ctas), block(sh.warps * 32);
  if (scale_mode == QK_SCALE_CHANNEL) {
    auto k = fp8_gemv_kernel<PRO, EPI, SCALE_CHANNEL, NG>;
    if (int r = ensure_smem((const void*)k, smem)) return r;
    return launch(k, grid, block, smem, stream, p);
  }
  auto k = fp8_gemv_kernel<PRO, EPI, SCALE_BLOCK, NG>;
  if (int r = ensure_smem((const void*)k, smem)) return r;
  return launch(k, grid, block, smem, stream, p);
}


// Every argument check of qk_fp8_gemv, before anything is enqueued (also run by qk_fp8_gemv_noalloc ahead of
// its counter reset, so a rejected call leaves nothing on the stream).
int gemv_check(int kind, const void* w, const float* w_scale, int scale_mode, const void* x, const void* norm_w,
               const float* resadd, const void* resid_out, const void* out, int N, int K, const float* part,
               const int* counters, const GemvShape& sh, bool library_scratch = false) {
  if (sh.warps < 4 || sh.warps > 16) return fail(QK_EINVAL, "warps must be in [4, 16], got %d", sh.warps);
  if (sh.stages < 1 || sh.stages > 16 || sh.stage_tiles < 1 || sh.stage_tiles > 64 || sh.ctas < 1 || sh.ctas > 8)
    return fail(QK_EINVAL, "bad launch shape stages=%d stage_tiles=%d ctas_per_sm=%d", sh.stages, sh.stage_tiles, sh.ctas);
  if (!w || !w_scale || !x || !out || (!library_scratch && (!part || !counters)))
    return fail(QK_EINVAL, "null pointer argument");
  if (scale_mode != QK_SCALE_BLOCK128 && scale_mode != QK_SCALE_CHANNEL) return fail(QK_EINVAL, "bad scale_mode %d", scale_mode);
  if (K <= 0 || K % QB || K > 16384) return fail(QK_EINVAL, "K=%d must be a positive multiple of 128, at most 16384", K);
  const bool pairs = (kind == QK_GEMV_GATE_UP || kind == QK_GEMV_GATE_UP_RESADD);
  if (N <= 0 || N % (pairs ? 32 : 16)) return fail(QK_EINVAL, "N=%d must be a positive multiple of %d", N, pairs ? 32 : 16);
  if (scale_mode == QK_SCALE_BLOCK128 && N % QB) return fail(QK_EINVAL, "block-128 scales need N %% 128 == 0 (N=%d)", N);
  const bool norm = (kind == QK_GEMV_QKV || kind == QK_GEMV_GATE_UP || kind == QK_GEMV_QKV_RESADD || kind == QK_GEMV_GATE_UP_RESADD);
  const bool resadd_k = (kind == QK_GEMV_QKV_RESADD || kind == QK_GEMV_GATE_UP_RESADD);
  const bool known = norm || kind == QK_GEMV_O || kind == QK_GEMV_DOWN || kind == QK_GEMV_PARTIAL;
  if (!known) return fail(QK_EINVAL, "unknown gemv kind %d", kind);
  if (norm && !norm_w) return fail(QK_EINVAL, "kind %d needs norm_w", kind);
  if (resadd_k && (!resadd || !resid_out)) return fail(QK_EINVAL, "kind %d needs resadd and resid_out", kind);
  if (!aligned(w, 16) || !aligned(x, 16) || !aligned(out, 16) || !aligned(w_scale, 8) ||
      (!library_scratch && !aligned(part, 16)) || (norm_w && !aligned(norm_w, 16)) || (resadd && !aligned(resadd, 16)) ||
      (resid_out && !aligned(resid_out, 16)))
    return fail(QK_EINVAL, "tensor pointers must be 16-byte aligned");
  return QK_OK;
}
}  // namespace

extern "C" {

int qk_version(void) { return 100; }
const char* qk_last_error(void) { return g_msg; }

int qk_set_pdl(int on) {
  g_pdl = on != 0;
  return QK_OK;
}

int qk_set_timeline(uint64_t* buf, int n_slots) {
  if (buf == nullptr) {
    g_tl_next = -1;
    if (!g_tl_ever) return QK_OK;   // never enabled: nothing on the device to clear
    n_slots = 0;
  } else {
    if (n_slots <= 0) return fail(QK_EINVAL, "n_slots must be positive");
    if (reinterpret_cast<uintptr_t>(buf) % 8) return fail(QK_EINVAL, "timeline buffer must be 8-byte aligned");
    g_tl_ever = true;
  }
  unsigned long long* p = reinterpret_cast<unsigned long long*>(buf);
  cudaError_t e = cudaMemcpyToSymbol(g_timeline, &p, sizeof(p));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_timeline_slots, &n_slots, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "setting the timeline buffer");
  g_tl_next = buf ? 0 : -1;
  return QK_OK;
}

int qk_get_device_error(int* err, qk_stream_t stream) {
  if (!err) return fail(QK_EINVAL, "err is NULL");
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(err, g_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_dev_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  return QK_OK;
}

int qk_wait_probe(int mode, void* counter, unsigned long long limit_ns, int* gave_up, qk_stream_t stream) {
  if (mode != 0 && mode != 1) return fail(QK_EINVAL, "mode must be 0 (mbarrier) or 1 (counter)");
  if (!gave_up || (mode == 1 && !counter)) return fail(QK_EINVAL, "null pointer argument");
  if (!aligned(gave_up, 4) || (counter && !aligned(counter, 8))) return fail(QK_EINVAL, "misaligned pointer");
  if (limit_ns == 0 || limit_ns > 1000000000ull) return fail(QK_EINVAL, "limit_ns must be in (0, 1e9]");
  return launch(wait_probe_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), mode,
                static_cast<const unsigned long long*>(counter), limit_ns, gave_up);
}

int qk_fp8_gemv(int kind, const void* w, const float* w_scale, int scale_mode, const void* x, const void* norm_w,
                const float* resadd, void* resid_out, void* out, int N, int K, float eps, float* part, int* counters,
                int warps, int stages, int stage_tiles, int pre, int ctas_per_sm, qk_stream_t stream) {
  GemvShape sh = gemv_defaults(kind);
  if (warps) sh.warps = warps;
  if (stages) sh.stages = stages;
  if (stage_tiles) sh.stage_tiles = stage_tiles;
  if (pre >= 0) sh.pre = pre;
  if (ctas_per_sm) sh.ctas = ctas_per_sm;
  if (int r = gemv_check(kind, w, w_scale, scale_mode, x, norm_w, resadd, resid_out, out, N, K, part, counters, sh))
    return r;
  GemvParams p = {};
  p.w = static_cast<const uint8_t*>(w);
  p.ws = w_scale;
  p.x = static_cast<const bf16*>(x);
  p.norm_w = static_cast<const bf16*>(norm_w);
  p.resadd = resadd;
  p.resid_out = static_cast<bf16*>(resid_out);
  p.out = static_cast<bf16*>(out);
  p.out_f32 = static_cast<float*>(out);
  p.part = part;
  p.counters = counters;
  p.best = nullptr;
  p.N = N;
  p.K = K;
  p.row_offset = 0;
  p.eps = eps;
  p.stages = sh.stages;
  p.stage_tiles = sh.stage_tiles;
  p.pre = sh.pre;
  p.tl_slot = next_tl_slot();
  switch (kind) {
    case QK_GEMV_QKV: return launch_gemv_scaled<PRO_RMSNORM_QUANT, EPI_STORE, 1>(scale_mode, p, sh, stream);
    case QK_GEMV_O:
    case QK_GEMV_DOWN: return launch_gemv_scaled<PRO_QUANT, EPI_RESIDUAL, 1>(scale_mode, p, sh, stream);
    case QK_GEMV_GATE_UP: return launch_gemv_scaled<PRO_RMSNORM_QUANT, EPI_SWIGLU, 2>(scale_mode, p, sh, stream);
    case QK_GEMV_PARTIAL: return launch_gemv_scaled<PRO_QUANT, EPI_F32, 1>(scale_mode, p, sh, stream);
    case QK_GEMV_QKV_RESADD: return launch_gemv_scaled<PRO_RESADD_RMSNORM_QUANT, EPI_STORE, 1>(scale_mode, p, sh, stream);
    case QK_GEMV_GATE_UP_RESADD: return launch_gemv_scaled<PRO_RESADD_RMSNORM_QUANT, EPI_SWIGLU, 2>(scale_mode, p, sh, stream);
    default: return fail(QK_EINVAL, "unknown gemv kind %d", kind);
  }
}

int qk_attention(const void* qkv, const void* q_norm_w, const void* k_norm_w, const void* cos_tab,
                 const void* sin_tab, const int* state, void* k_cache, void* v_cache, float* o_part,
                 float* ml_part, int* counters, void* out, int batch, int n_kv, int max_seq, int max_splits,
                 int qkv_stride, int state_stride, float scale, float eps, int chunk, qk_stream_t stream) {
  if (!qkv || !q_norm_w || !k_norm_w || !cos_tab || !sin_tab || !state || !k_cache || !v_cache || !o_part ||
      !ml_part || !counters || !out)
    return fail(QK_EINVAL, "null pointer argument");
  if (batch < 1 || batch > 65535 || n_kv < 1 || n_kv > 64 || max_seq < 1) return fail(QK_EINVAL, "bad batch/n_kv/max_seq");
  if (chunk != 32 && chunk != 64 && chunk != 128) return fail(QK_EINVAL, "chunk must be 32, 64 or 128, got %d", chunk);
  if ((long long)max_splits * chunk < max_seq) return fail(QK_EINVAL, "o_part too small: max_splits*chunk < max_seq");
  if (max_splits > 4096) return fail(QK_EINVAL, "max_splits %d > 4096", max_splits);
  if (qkv_stride < n_kv * 6 * HEAD_DIM || state_stride < 1) return fail(QK_EINVAL, "bad qkv_stride/state_stride");
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(qkv, 16) || !aligned(o_part, 16))
    return fail(QK_EINVAL, "caches, qkv and o_part must be 16-byte aligned");
  if ((long long)n_kv * ((max_seq + ATT_KEYS - 1) / ATT_KEYS) > 0x7fffffff) return fail(QK_EINVAL, "max_seq too large");
  AttnParams p = {};
  // the layer's caches as 4-D tensors {128 dims, max_seq keys, n_kv heads, batch}
  if (int r = encode_cache_map(&p.tm_k, k_cache, max_seq, n_kv, batch, (long long)n_kv * max_seq * HEAD_DIM * 2,
                               ATT_KEYS))
    return r;
  if (int r = encode_cache_map(&p.tm_v, v_cache, max_seq, n_kv, batch, (long long)n_kv * max_seq * HEAD_DIM * 2,
                               ATT_KEYS))
    return r;
  p.qkv = static_cast<const bf16*>(qkv);
  p.q_norm_w = static_cast<const bf16*>(q_norm_w);
  p.k_norm_w = static_cast<const bf16*>(k_norm_w);
  p.cos_tab = static_cast<const bf16*>(cos_tab);
  p.sin_tab = static_cast<const bf16*>(sin_tab);
  p.state = state;
  p.k_cache = static_cast<bf16*>(k_cache);
  p.v_cache = static_cast<bf16*>(v_cache);
  p.o_part = o_part;
  p.ml_part = ml_part;
  p.out = static_cast<bf16*>(out);
  p.n_kv = n_kv;
  p.max_seq = max_seq;
  p.max_splits = max_splits;
  p.qkv_stride = qkv_stride;
  p.state_stride = state_stride;
  p.chunk = chunk;
  p.scale = scale;
  p.eps = eps;
  p.tl_slot = next_tl_slot();
  (void)counters;   // the reference's last-CTA merge counters: the separate merge kernel needs none
  const dim3 grid(n_kv * ((max_seq + ATT_KEYS - 1) / ATT_KEYS), batch);
  auto partials = chunk == 32 ? attn_partials_kernel<32> : chunk == 64 ? attn_partials_kernel<64> : attn_partials_kernel<128>;
  const int smem_p = (int)attn_partials_smem_bytes();
  if (int r = ensure_smem((const void*)partials, smem_p)) return r;
  if (int r = launch(partials, grid, dim3(ATT_THREADS), smem_p, stream, p)) return r;
  const int smem_m = (int)attn_merge_smem_bytes(max_splits);
  if (int r = ensure_smem((const void*)attn_merge_kernel, smem_m)) return r;
  return launch(attn_merge_kernel, dim3(2 * n_kv * GQA, batch), dim3(ATT_MERGE_THREADS), smem_m, stream, p);
}

int qk_lm_head_argmax(const void* w, const float* w_scale, int head_fp8, const void* x, const void* norm_w,
                      void* logits, unsigned long long* best, int V, int row_offset, float eps, float* part,
                      int* counters, int ctas, qk_stream_t stream) {
  if (!w || !x || !norm_w || !logits || !best) return fail(QK_EINVAL, "null pointer argument");
  if (V <= 0 || V % (head_fp8 ? 16 : 8)) return fail(QK_EINVAL, "V=%d must be a positive multiple of %d", V, head_fp8 ? 16 : 8);
  if (!aligned(w, 16) || !aligned(x, 16) || !aligned(norm_w, 16) || !aligned(logits, 16))
    return fail(QK_EINVAL, "tensor pointers must be 16-byte aligned");
  const int sms = device_sms();
  if (head_fp8) {
    if (!w_scale || !part || !counters) return fail(QK_EINVAL, "fp8 head needs w_scale, part and counters");
    GemvShape sh = gemv_defaults(4);
    if (ctas > 0) sh.ctas = (ctas + sms - 1) / sms;
    GemvParams p = {};
    p.w = static_cast<const uint8_t*>(w);
    p.ws = w_scale;
    p.x = static_cast<const bf16*>(x);
    p.norm_w = static_cast<const bf16*>(norm_w);
    p.out = static_cast<bf16*>(logits);
    p.part = part;
    p.counters = counters;
    p.best = best;
    p.N = V;
    p.K = HIDDEN;
    p.row_offset = row_offset;
    p.eps = eps;
    p.stages = sh.stages;
    p.stage_tiles = sh.stage_tiles;
    p.pre = sh.pre;
    p.tl_slot = next_tl_slot();
    return launch_gemv_scaled<PRO_RMSNORM_QUANT, EPI_ARGMAX, 1>(QK_SCALE_CHANNEL, p, sh, stream);
  }
  HeadParams p = {};
  p.w = static_cast<const bf16*>(w);
  p.x = static_cast<const bf16*>(x);
  p.norm_w = static_cast<const bf16*>(norm_w);
  p.logits = static_cast<bf16*>(logits);
  p.best = best;
  p.V = V;
  p.row_offset = row_offset;
  p.eps = eps;
  p.stages = 3;
  p.pre = 3;
  p.tl_slot = next_tl_slot();
  const int smem = head_smem_total(p.stages);
  if (int r = ensure_smem((const void*)lm_head_bf16_kernel, smem)) return r;
  return launch(lm_head_bf16_kernel, dim3(ctas > 0 ? ctas : sms), dim3(HEAD_WARPS * 32), smem, stream, p);
}

// Scratch of the fused step: the tagged block dots (one u64 = two floats each) of the GEMV units shared by two
// CTAs, indexed by unit, so sized for the largest N*K/128 (gate|up: 24576*4096/128, or the head: vocab*32); and
// the unit counters, sized for the most units (gate|up pairs: 768, or the head: vocab/16).
long long qk_decode_step_part_floats(int vocab) {
  const long long gu = 24576LL * 4096 / 128, down = 4096LL * 12288 / 128, head = (long long)vocab * 4096 / 128;
  long long m = gu > down ? gu : down;
  return 2 * (m > head ? m : head);
}
int qk_decode_step_counters(int vocab) {
  const int head = vocab / 16;
  return head > 768 ? head : 768;
}

}  // extern "C"

namespace {
// Shared by qk_decode_step (tp = 1) and qk_decode_step_tp (tp > 1: this rank's shard, see StepParams).
int launch_decode_step(const qk_layer_t* layers, int n_layers, void* k_cache, void* v_cache, long long kv_layer_stride,
                       const void* embed, const void* final_norm, const void* w_head, const float* s_head, int vocab,
                       const void* cos_tab, const void* sin_tab, int* token, int* state, int* out_tokens, int out_len,
                       unsigned long long* best, void* resid, void* qkv, void* attn, void* h, void* logits,
                       float* part, long long part_floats, int* counters, int n_counters, float* o_part,
                       float* ml_part, int* attn_counters, unsigned* sync, int max_seq, int max_splits, float eps,
                       int scale_mode, uint64_t* timeline, int tp, int rank, void* resid_alt, int vocab_offset,
                       void* const* areas, cudaStream_t stream) {
  if (!layers || n_layers < 1 || !k_cache || !v_cache || !embed || !final_norm || !w_head || !cos_tab ||
      !sin_tab || !token || !state || !out_tokens || !best || !resid || !qkv || !attn || !h || !logits || !part ||
      !counters || !o_part || !ml_part || !attn_counters || !sync)
    return fail(QK_EINVAL, "null pointer argument");
  if (max_seq < 1) return fail(QK_EINVAL, "bad max_seq");
  const int n_kv = 8 / tp;
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || kv_layer_stride % 16 ||
      kv_layer_stride < (long long)n_kv * max_seq * HEAD_DIM * 2)
    return fail(QK_EINVAL, "KV caches must be 16-byte aligned with a layer stride (bytes) that is a multiple of 16 "
                           "and at least n_kv * max_seq * 256");
  if (vocab <= 0 || vocab % 16 || out_len < 1) return fail(QK_EINVAL, "bad vocab/out_len");
  if (part_floats < qk_decode_step_part_floats(vocab) || n_counters < qk_decode_step_counters(vocab))
    return fail(QK_EINVAL, "scratch too small: part needs %lld floats, counters %d ints",
                qk_decode_step_part_floats(vocab), qk_decode_step_counters(vocab));
  if (max_splits < (max_seq + ST_CHUNK - 1) / ST_CHUNK || max_splits > ST_MAX_SPLITS)
    return fail(QK_EINVAL, "max_splits must cover max_seq/64 and be at most %d", ST_MAX_SPLITS);
  if (scale_mode != QK_SCALE_BLOCK128 && scale_mode != QK_SCALE_CHANNEL) return fail(QK_EINVAL, "bad scale_mode");
  const bool head_bf16 = s_head == nullptr;   // the reference checkpoint's bf16 lm_head
  if (head_bf16 && tp != 1) return fail(QK_EINVAL, "the tensor-parallel step needs the FP8 head (s_head)");
  if (!aligned(w_head, 16)) return fail(QK_EINVAL, "w_head must be 16-byte aligned");
  StepParams p = {};
  if (int r = encode_kv_map(&p.tm_k, k_cache, max_seq, n_kv, n_layers, kv_layer_stride)) return r;
  if (int r = encode_kv_map(&p.tm_v, v_cache, max_seq, n_kv, n_layers, kv_layer_stride)) return r;
  p.k_cache = static_cast<bf16*>(k_cache);
  p.v_cache = static_cast<bf16*>(v_cache);
  p.kv_layer_elems = kv_layer_stride / 2;
  p.layers = reinterpret_cast<const StepLayer*>(layers);
  p.n_layers = n_layers;
  p.embed = static_cast<const bf16*>(embed);
  p.final_norm = static_cast<const bf16*>(final_norm);
  p.w_head = static_cast<const uint8_t*>(w_head);
  p.s_head = s_head;
  p.vocab = vocab;
  p.cos_tab = static_cast<const bf16*>(cos_tab);
  p.sin_tab = static_cast<const bf16*>(sin_tab);
  p.token = token;
  p.state = state;
  p.out_tokens = out_tokens;
  p.out_len = out_len;
  p.best = best;
  p.resid = static_cast<bf16*>(resid);
  p.qkv = static_cast<bf16*>(qkv);
  p.attn = static_cast<bf16*>(attn);
  p.h = static_cast<bf16*>(h);
  p.logits = static_cast<bf16*>(logits);
  p.part = part;
  p.counters = counters;
  p.o_part = o_part;
  p.ml_part = ml_part;
  p.attn_counters = attn_counters;
  p.sync = sync;
  p.max_seq = max_seq;
  p.max_splits = max_splits;
  p.eps = eps;
  p.attn_scale = 0.08838834764831845f;   // 128 ** -0.5
  p.tl = reinterpret_cast<unsigned long long*>(timeline);
  p.tp = tp;
  p.tp_rank = rank;
  p.vocab_offset = vocab_offset;
  p.resid_alt = static_cast<bf16*>(resid_alt);
  p.areas = reinterpret_cast<TpArea* const*>(areas);
  void (*kernel)(const StepParams) = nullptr;
  if (tp == 1) {
    if (scale_mode == QK_SCALE_CHANNEL)
      kernel = head_bf16 ? decode_step_kernel<SCALE_CHANNEL, 1, 1> : decode_step_kernel<SCALE_CHANNEL, 1, 0>;
    else
      kernel = head_bf16 ? decode_step_kernel<SCALE_BLOCK, 1, 1> : decode_step_kernel<SCALE_BLOCK, 1, 0>;
  } else if (tp == 2) kernel = decode_step_kernel<SCALE_CHANNEL, 2, 0>;
  else if (tp == 4) kernel = decode_step_kernel<SCALE_CHANNEL, 4, 0>;
  else if (tp == 8) kernel = decode_step_kernel<SCALE_CHANNEL, 8, 0>;
  const int smem = (int)sizeof(StepSmem);
  if (int r = ensure_smem((const void*)kernel, smem)) return r;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(device_sms());
  cfg.blockDim = dim3(ST_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;   // all CTAs resident: the grid barriers rely on it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) return cuda_fail(e, "decode step launch");
  return QK_OK;
}
}  // namespace

extern "C" {

int qk_decode_step(const qk_layer_t* layers, int n_layers, void* k_cache, void* v_cache, long long kv_layer_stride,
                   const void* embed, const void* final_norm, const void* w_head, const float* s_head, int vocab,
                   const void* cos_tab, const void* sin_tab, int* token, int* state, int* out_tokens, int out_len,
                   unsigned long long* best, void* resid, void* qkv, void* attn, void* h, void* logits, float* part,
                   long long part_floats, int* counters, int n_counters, float* o_part, float* ml_part,
                   int* attn_counters, unsigned* sync, int max_seq, int max_splits, float eps, int scale_mode,
                   uint64_t* timeline, qk_stream_t stream) {
  return launch_decode_step(layers, n_layers, k_cache, v_cache, kv_layer_stride, embed, final_norm, w_head, s_head,
                            vocab, cos_tab, sin_tab, token, state, out_tokens, out_len, best, resid, qkv, attn, h,
                            logits, part, part_floats, counters, n_counters, o_part, ml_part, attn_counters, sync,
                            max_seq, max_splits, eps, scale_mode, timeline, 1, 0, nullptr, 0, nullptr, stream);
}

long long qk_tp_area_bytes(void) { return (long long)sizeof(TpArea); }

int qk_tp_area_alloc(void** area, void* ipc_handle) {
  if (!area || !ipc_handle) return fail(QK_EINVAL, "null pointer argument");
  void* a = nullptr;
  cudaError_t e = cudaMalloc(&a, sizeof(TpArea));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (TP area)");
  e = cudaMemset(a, 0, sizeof(TpArea));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), a);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(a);
    return cuda_fail(e, "TP area setup");
  }
  *area = a;
  return QK_OK;
}

int qk_tp_area_open(const void* ipc_handle, void** peer_area) {
  if (!ipc_handle || !peer_area) return fail(QK_EINVAL, "null pointer argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(peer_area, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? QK_OK : cuda_fail(e, "cudaIpcOpenMemHandle (peer TP area)");
}

int qk_tp_area_close(void* peer_area) {
  if (!peer_area) return fail(QK_EINVAL, "null pointer argument");
  const cudaError_t e = cudaIpcCloseMemHandle(peer_area);
  return e == cudaSuccess ? QK_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int qk_tp_area_free(void* area) {
  if (!area) return fail(QK_EINVAL, "null pointer argument");
  const cudaError_t e = cudaFree(area);
  return e == cudaSuccess ? QK_OK : cuda_fail(e, "cudaFree (TP area)");
}

int qk_tp_area_reset(void* area, qk_stream_t stream) {
  if (!area) return fail(QK_EINVAL, "null pointer argument");
  const cudaError_t e = cudaMemsetAsync(area, 0, sizeof(TpArea), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? QK_OK : cuda_fail(e, "cudaMemsetAsync (TP area reset)");
}

int qk_decode_step_tp(const qk_layer_t* layers, int n_layers, void* k_cache, void* v_cache, long long kv_layer_stride,
                      const void* embed, const void* final_norm, const void* w_head, const float* s_head, int vocab,
                      const void* cos_tab, const void* sin_tab, int* token, int* state, int* out_tokens,
                      int out_len, unsigned long long* best, void* resid, void* qkv, void* attn, void* h,
                      void* logits, float* part, long long part_floats, int* counters, int n_counters,
                      float* o_part, float* ml_part, int* attn_counters, unsigned* sync, int max_seq,
                      int max_splits, float eps, uint64_t* timeline, void* resid_alt, int vocab_offset,
                      const qk_tp_comm_t* comm, qk_stream_t stream) {
  if (!comm || !comm->areas || !resid_alt) return fail(QK_EINVAL, "null pointer argument");
  if (comm->tp != 2 && comm->tp != 4 && comm->tp != 8) return fail(QK_EINVAL, "tp must be 2, 4 or 8");
  if (comm->rank < 0 || comm->rank >= comm->tp) return fail(QK_EINVAL, "bad rank");
  if (vocab_offset < 0 || vocab_offset % 16) return fail(QK_EINVAL, "bad vocab_offset");
  return launch_decode_step(layers, n_layers, k_cache, v_cache, kv_layer_stride, embed, final_norm, w_head, s_head,
                            vocab, cos_tab, sin_tab, token, state, out_tokens, out_len, best, resid, qkv, attn, h,
                            logits, part, part_floats, counters, n_counters, o_part, ml_part, attn_counters, sync,
                            max_seq, max_splits, eps, QK_SCALE_CHANNEL, timeline, comm->tp, comm->rank, resid_alt,
                            vocab_offset, comm->areas, stream);
}

int qk_embed(const int* token, const void* table, void* resid, int vocab, int batch, qk_stream_t stream) {
  if (!token || !table || !resid || vocab <= 0 || batch < 1) return fail(QK_EINVAL, "bad embed arguments");
  if (!aligned(table, 16) || !aligned(resid, 16)) return fail(QK_EINVAL, "table/resid must be 16-byte aligned");
  return launch(embed_kernel, dim3(batch), dim3(HIDDEN / 8), 0, stream, token, static_cast<const bf16*>(table),
                static_cast<bf16*>(resid), vocab);
}

int qk_finalize(unsigned long long* best, int* token, int* out_tokens, int* state, int out_len, int batch,
                qk_stream_t stream) {
  if (!best || !token || !out_tokens || !state || out_len < 1 || batch < 1) return fail(QK_EINVAL, "bad finalize arguments");
  return launch(finalize_kernel, dim3(batch), dim3(1), 0, stream, best, token, out_tokens, state, out_len);
}

int qk_residual_add(void* resid, const float* sum, int n, qk_stream_t stream) {
  if (!resid || !sum || n < 1) return fail(QK_EINVAL, "bad residual_add arguments");
  const int threads = 256;
  residual_add_kernel<<<(n + threads - 1) / threads, threads, 0, stream>>>(static_cast<bf16*>(resid), sum, n);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? QK_OK : cuda_fail(e, "residual_add launch");
}

int qk_argmax_key_flip(unsigned long long* keys, int n, qk_stream_t stream) {
  if (!keys || n < 1) return fail(QK_EINVAL, "bad argmax_key_flip arguments");
  key_flip_kernel<<<(n + 255) / 256, 256, 0, stream>>>(keys, n);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? QK_OK : cuda_fail(e, "argmax_key_flip launch");
}

}  // extern "C"

// ---- batched FP8 linear on the tcgen05 tensor cores ----------------------------------------------------------
namespace {
int gemm_rows_pad(int M) { return M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128)); }
struct GemmScratch { size_t qx, sx, part, counters, total; };
// The tile counters come first, in a region of fixed size, so that they stay zero from call to call whatever
// the shapes (every call leaves them zero); the quantized activations, their scales and the split-tile partials
// follow and need no initial value.
GemmScratch gemm_scratch_layout(int M, int N, int K, int grid) {
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  GemmScratch L;
  (void)N;
  L.counters = 0;
  L.qx = up((size_t)TC_MAX_TILES * 4);
  L.sx = L.qx + up((size_t)gemm_rows_pad(M) * K);   // room for the tiled layout's padding rows
  L.part = L.sx + up((size_t)M * (K / QB) * 4);
  L.total = L.part + up((size_t)grid * 2 * TC_TILE * gemm_rows_pad(M) * 4);
  return L;
}
}  // namespace

extern "C" long long qk_fp8_gemm_rows_scratch_bytes(int M, int N, int K) {
  if (M < 1 || M > TC_MAX_ROWS || N < TC_TILE || N % TC_TILE || N / TC_TILE > TC_MAX_TILES || K < TC_BK ||
      K % TC_BK || K > (M > 64 ? 12288 : 16384))
    return -1;
  return (long long)gemm_scratch_layout(M, N, K, device_sms()).total;
}

namespace {
// The batched linear with row-major operands through tensor maps (tiles == false) or tile-packed operands
// through bulk copies (tiles == true).
int gemm_rows_impl(bool tiles, const void* x, const void* norm_w, int M, int K, const void* w, const float* w_scale,
                   int scale_mode, int N, float eps, void* out, void* scratch, long long scratch_bytes,
                   qk_stream_t stream) {
  if (!x || !w || !w_scale || !out || !scratch) return fail(QK_EINVAL, "null pointer argument");
  if (M < 1 || M > TC_MAX_ROWS) return fail(QK_EINVAL, "M=%d rows: 1..%d per call", M, TC_MAX_ROWS);
  if (N < TC_TILE || N % TC_TILE || N / TC_TILE > TC_MAX_TILES || K < TC_BK || K % TC_BK || K > (M > 64 ? 12288 : 16384))
    return fail(QK_EINVAL, "N=%d, K=%d: both multiples of 128 (N at most %d, K at most 16384, or 12288 above 64 rows)", N,
                K, TC_MAX_TILES * TC_TILE);
  if (scale_mode != QK_SCALE_BLOCK128 && scale_mode != QK_SCALE_CHANNEL) return fail(QK_EINVAL, "bad scale_mode %d", scale_mode);
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(out, 16) || !aligned(scratch, 256) || (norm_w && !aligned(norm_w, 16)))
    return fail(QK_EINVAL, "x, w and out must be 16-byte aligned, scratch 256-byte aligned");
  const int sms = device_sms();
  const long long pairs = (long long)(N / TC_TILE) * (K / TC_BK);
  const int grid = (int)(pairs < sms ? pairs : sms);
  const GemmScratch L = gemm_scratch_layout(M, N, K, sms);
  if (scratch_bytes < (long long)L.total)
    return fail(QK_EINVAL, "scratch too small: %lld bytes, need qk_fp8_gemm_rows_scratch_bytes = %zu", scratch_bytes, L.total);
  unsigned char* sc = static_cast<unsigned char*>(scratch);
  TcGemmParams p = {};
  const int mp = gemm_rows_pad(M);
  if (tiles) {
    p.w_tiles = static_cast<const uint8_t*>(w);
    p.x_tiles = sc + L.qx;
  } else {
    if (int r = encode_fp8_rows_map(&p.tm_w, w, N, K, TC_TILE)) return r;
    if (int r = encode_fp8_rows_map(&p.tm_x, sc + L.qx, M, K, mp)) return r;
  }
  p.sx = reinterpret_cast<const float*>(sc + L.sx);
  p.sw = w_scale;
  p.out = static_cast<bf16*>(out);
  p.part = reinterpret_cast<float*>(sc + L.part);
  p.counters = reinterpret_cast<int*>(sc + L.counters);
  p.M = M;
  p.N = N;
  p.K = K;
  p.scale_block = scale_mode == QK_SCALE_BLOCK128;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int r = launch(quantize_rows_kernel, dim3(tiles ? mp : M), dim3(256), 0, st, static_cast<const bf16*>(x),
                     static_cast<const bf16*>(norm_w), M, K, eps, sc + L.qx, reinterpret_cast<float*>(sc + L.sx),
                     tiles ? mp : 0))
    return r;
  auto run = [&](auto kernel, size_t smem) -> int {
    if (int r = ensure_smem((const void*)kernel, (int)smem)) return r;
    return launch(kernel, dim3(grid), dim3(TC_THREADS), smem, st, p);
  };
  if (mp == 16) return run(fp8_gemm_tc_kernel<16>, tc_smem_bytes<16>());
  if (mp == 32) return run(fp8_gemm_tc_kernel<32>, tc_smem_bytes<32>());
  if (mp == 64) return run(fp8_gemm_tc_kernel<64>, tc_smem_bytes<64>());
  return run(fp8_gemm_tc_kernel<128>, tc_smem_bytes<128>());
}
}  // namespace

extern "C" int qk_fp8_gemm_rows(const void* x, const void* norm_w, int M, int K, const void* w, const float* w_scale,
                                int scale_mode, int N, float eps, void* out, void* scratch, long long scratch_bytes,
                                qk_stream_t stream) {
  return gemm_rows_impl(false, x, norm_w, M, K, w, w_scale, scale_mode, N, eps, out, scratch, scratch_bytes, stream);
}

extern "C" int qk_fp8_gemm_tiles(const void* x, const void* norm_w, int M, int K, const void* w_tiles,
                                 const float* w_scale, int scale_mode, int N, float eps, void* out, void* scratch,
                                 long long scratch_bytes, qk_stream_t stream) {
  return gemm_rows_impl(true, x, norm_w, M, K, w_tiles, w_scale, scale_mode, N, eps, out, scratch, scratch_bytes,
                        stream);
}

// ---- GEMV without caller-provided scratch --------------------------------------------------------------------
// qk_fp8_gemv needs two scratch buffers from its caller (the split-K block dots and the per-unit counters).
// Some callers cannot allocate device memory at all: code that runs inside an allocator-free host runtime,
// plugins that only receive the tensors of one op call, or a process whose device memory is fully reserved
// up front. For them, qk_fp8_gemv_noalloc runs the same GEMV with its scratch in the fixed device array
// below, which the library owns. It is sized for the largest per-layer GEMV of Qwen3-8B (gate|up:
// N*K/128 = 24576*4096/128 block dots); every GPU that loads this library holds these 3 MiB + 16 KiB until
// the process exits.
namespace {
constexpr size_t NOALLOC_PART_FLOATS = 786432;     // max N*K/128
constexpr size_t NOALLOC_COUNTERS = 4096;          // max N/16
constexpr size_t NOALLOC_BYTES = NOALLOC_PART_FLOATS * 4 + NOALLOC_COUNTERS * 4;
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

// The array's name in host code is only a host-side stand-in: its device address is looked up with the
// device current. The lookup is repeated on every call (it is cheap and allocates nothing), so the address
// stays right after a cudaDeviceReset reloads the module at another address. The first call on a device
// loads the library's module there, so make it before any stream capture.
int noalloc_scratch(unsigned char** out) {
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress of the no-alloc scratch");
  *out = static_cast<unsigned char*>(ptr);
  return QK_OK;
}
}  // namespace

extern "C" int qk_fp8_gemv_noalloc(int kind, const void* w, const float* w_scale, int scale_mode, const void* x,
                                   const void* norm_w, const float* resadd, void* resid_out, void* out, int N,
                                   int K, float eps, qk_stream_t stream) {
  if (N <= 0 || K <= 0 || K % QB) return fail(QK_EINVAL, "N=%d K=%d: K must be a positive multiple of 128", N, K);
  const size_t part = (size_t)N * (K / QB), units = (size_t)N / GEMV_UNIT_ROWS;
  if (part > NOALLOC_PART_FLOATS || units > NOALLOC_COUNTERS)
    return fail(QK_EINVAL, "N=%d K=%d exceeds the no-alloc scratch (N*K/128 <= %zu, N/16 <= %zu); use qk_fp8_gemv",
                N, K, NOALLOC_PART_FLOATS, NOALLOC_COUNTERS);
  // every check of qk_fp8_gemv first, so that a rejected call enqueues nothing (not even the counter reset)
  if (int r = gemv_check(kind, w, w_scale, scale_mode, x, norm_w, resadd, resid_out, out, N, K, nullptr, nullptr,
                         gemv_defaults(kind), true))
    return r;
  unsigned char* base = nullptr;
  if (int r = noalloc_scratch(&base)) return r;
  float* part_ptr = reinterpret_cast<float*>(base);
  int* counters = reinterpret_cast<int*>(base + NOALLOC_PART_FLOATS * 4);
  // The array keeps whatever the previous call left; the counters must start at zero.
  cudaError_t e = cudaMemsetAsync(counters, 0, units * sizeof(int), stream);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the no-alloc counters");
  return qk_fp8_gemv(kind, w, w_scale, scale_mode, x, norm_w, resadd, resid_out, out, N, K, eps, part_ptr, counters,
                     0, 0, 0, -1, 0, stream);
}

// ---- chunked prefill: the row-wise kernels around the batched linear ------------------------------------------
namespace {
int plain_launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? QK_OK : cuda_fail(e, what);
}
int elementwise_blocks(long long n) { return (int)std::min<long long>((n + 255) / 256, 4096); }
}  // namespace

extern "C" {

int qk_embed_rows(const int* tokens, int M, const void* table, int vocab, void* out, qk_stream_t stream) {
  if (!tokens || !table || !out || M < 1 || vocab < 1) return fail(QK_EINVAL, "bad embed_rows arguments");
  if (!aligned(table, 16) || !aligned(out, 16)) return fail(QK_EINVAL, "table/out must be 16-byte aligned");
  embed_rows_kernel<<<M, 256, 0, static_cast<cudaStream_t>(stream)>>>(tokens, vocab, static_cast<const bf16*>(table),
                                                                      HIDDEN, static_cast<bf16*>(out));
  return plain_launch_status("embed_rows launch");
}

int qk_prefill_qkv(const void* qkv, int M, int p0, int n_q, int n_kv, const void* q_norm, const void* k_norm,
                   const void* cos_tab, const void* sin_tab, float eps, void* k_cache, void* v_cache, int max_seq,
                   void* q_out, qk_stream_t stream) {
  if (!qkv || !q_norm || !k_norm || !cos_tab || !sin_tab || !k_cache || !v_cache || !q_out)
    return fail(QK_EINVAL, "null pointer argument");
  if (M < 1 || p0 < 0 || n_kv < 1 || n_q != GQA * n_kv) return fail(QK_EINVAL, "M=%d p0=%d n_q=%d n_kv=%d", M, p0, n_q, n_kv);
  if ((long long)p0 + M > max_seq) return fail(QK_EINVAL, "positions %d..%d past max_seq %d", p0, p0 + M - 1, max_seq);
  if (!aligned(qkv, 8) || !aligned(k_cache, 8) || !aligned(v_cache, 8) || !aligned(q_out, 8))
    return fail(QK_EINVAL, "qkv, caches and q_out must be 8-byte aligned");
  const dim3 grid(M, (n_q + 2 * n_kv + 7) / 8);
  prefill_qkv_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const bf16*>(qkv), p0, n_q, n_kv, static_cast<const bf16*>(q_norm), static_cast<const bf16*>(k_norm),
      static_cast<const bf16*>(cos_tab), static_cast<const bf16*>(sin_tab), eps, static_cast<bf16*>(k_cache),
      static_cast<bf16*>(v_cache), max_seq, static_cast<bf16*>(q_out));
  return plain_launch_status("prefill_qkv launch");
}

int qk_prefill_attention(const void* q, int M, int p0, int n_q, int n_kv, const void* k_cache, const void* v_cache,
                         int max_seq, float scale, void* out, qk_stream_t stream) {
  if (!q || !k_cache || !v_cache || !out) return fail(QK_EINVAL, "null pointer argument");
  if (M < 1 || p0 < 0 || n_kv < 1 || n_q != GQA * n_kv) return fail(QK_EINVAL, "M=%d p0=%d n_q=%d n_kv=%d", M, p0, n_q, n_kv);
  if ((long long)p0 + M > max_seq) return fail(QK_EINVAL, "positions %d..%d past max_seq %d", p0, p0 + M - 1, max_seq);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(out, 16))
    return fail(QK_EINVAL, "caches and out must be 16-byte aligned");
  const int smem = (int)sizeof(PrefillAttnSmem);
  if (int r = ensure_smem((const void*)prefill_attention_kernel, smem)) return r;
  prefill_attention_kernel<<<dim3((M + PA_ROWS - 1) / PA_ROWS, n_kv), PF_THREADS, smem,
                             static_cast<cudaStream_t>(stream)>>>(
      static_cast<const bf16*>(q), M, p0, n_q, static_cast<const bf16*>(k_cache), static_cast<const bf16*>(v_cache),
      max_seq, scale, static_cast<bf16*>(out));
  return plain_launch_status("prefill_attention launch");
}

int qk_add_rows(void* resid, const void* y, long long n, qk_stream_t stream) {
  if (!resid || !y || n < 1) return fail(QK_EINVAL, "bad add_rows arguments");
  add_rows_kernel<<<elementwise_blocks(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<bf16*>(resid), static_cast<const bf16*>(y), n);
  return plain_launch_status("add_rows launch");
}

int qk_argmax_rows(const void* logits, int rows, int V, unsigned long long* best, qk_stream_t stream) {
  if (!logits || !best || rows < 1 || V < 1) return fail(QK_EINVAL, "bad argmax_rows arguments");
  argmax_rows_kernel<<<rows, 1024, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const bf16*>(logits), V, best);
  return plain_launch_status("argmax_rows launch");
}

int qk_swiglu_rows(const void* gu, int M, int I, void* h, qk_stream_t stream) {
  if (!gu || !h || M < 1 || I < 1) return fail(QK_EINVAL, "bad swiglu_rows arguments");
  swiglu_rows_kernel<<<elementwise_blocks((long long)M * I), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const bf16*>(gu), M, I, static_cast<bf16*>(h));
  return plain_launch_status("swiglu_rows launch");
}

}  // extern "C"

// ---- decode attention over an FP8 KV cache ---------------------------------------------------------------------
extern "C" int qk_attention_fp8kv(const void* qkv, const void* q_norm_w, const void* k_norm_w, const void* cos_tab,
                                  const void* sin_tab, const int* state, void* k_cache, float* k_scale, void* v_cache,
                                  float* v_scale, float* o_part, float* ml_part, void* out, int batch, int n_kv,
                                  int max_seq, int max_splits, int qkv_stride, int state_stride, float scale,
                                  float eps, qk_stream_t stream) {
  if (!qkv || !q_norm_w || !k_norm_w || !cos_tab || !sin_tab || !state || !k_cache || !k_scale || !v_cache ||
      !v_scale || !o_part || !ml_part || !out)
    return fail(QK_EINVAL, "null pointer argument");
  if (batch < 1 || batch > 65535 || n_kv < 1 || n_kv > 64 || max_seq < 1) return fail(QK_EINVAL, "bad batch/n_kv/max_seq");
  // long contexts: 4 blocks (512 keys) per split, each CTA streaming them double-buffered; medium ones 2,
  // short ones 1, for enough CTAs
  const int blocks = max_seq >= 16384 ? KV8_MAX_BLOCKS : (max_seq >= 4096 ? 2 : 1), split_keys = KV8_KEYS * blocks;
  if ((long long)max_splits * split_keys < max_seq) return fail(QK_EINVAL, "o_part too small: max_splits*%d < max_seq", split_keys);
  if (max_splits > 4096) return fail(QK_EINVAL, "max_splits %d > 4096", max_splits);
  if (qkv_stride < n_kv * 6 * HEAD_DIM || state_stride < 1) return fail(QK_EINVAL, "bad qkv_stride/state_stride");
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(qkv, 8) || !aligned(k_scale, 4) || !aligned(v_scale, 4))
    return fail(QK_EINVAL, "caches must be 16-byte aligned, qkv 8-byte");
  if ((long long)n_kv * ((max_seq + split_keys - 1) / split_keys) > 0x7fffffff) return fail(QK_EINVAL, "max_seq too large");
  Kv8Params p = {};
  p.qkv = static_cast<const bf16*>(qkv);
  p.q_norm_w = static_cast<const bf16*>(q_norm_w);
  p.k_norm_w = static_cast<const bf16*>(k_norm_w);
  p.cos_tab = static_cast<const bf16*>(cos_tab);
  p.sin_tab = static_cast<const bf16*>(sin_tab);
  p.state = state;
  p.k_cache = static_cast<uint8_t*>(k_cache);
  p.v_cache = static_cast<uint8_t*>(v_cache);
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.o_part = o_part;
  p.ml_part = ml_part;
  p.n_kv = n_kv;
  p.max_seq = max_seq;
  p.max_splits = max_splits;
  p.qkv_stride = qkv_stride;
  p.state_stride = state_stride;
  p.blocks = blocks;
  p.scale = scale;
  p.eps = eps;
  const dim3 grid(n_kv * ((max_seq + split_keys - 1) / split_keys), batch);
  const int smem_p = (int)kv8_smem_bytes();
  if (int r = ensure_smem((const void*)attn_fp8kv_partials_kernel, smem_p)) return r;
  if (int r = launch(attn_fp8kv_partials_kernel, grid, dim3(KV8_THREADS), smem_p, stream, p)) return r;
  AttnParams m = {};   // the merge reads the partials in the bf16 kernel's layout, one per split
  m.state = state;
  m.o_part = o_part;
  m.ml_part = ml_part;
  m.out = static_cast<bf16*>(out);
  m.n_kv = n_kv;
  m.max_seq = max_seq;
  m.max_splits = max_splits;
  m.state_stride = state_stride;
  m.chunk = split_keys;
  m.tl_slot = -1;
  const int smem_m = (int)attn_merge_smem_bytes(max_splits);
  if (int r = ensure_smem((const void*)attn_merge_kernel, smem_m)) return r;
  return launch(attn_merge_kernel, dim3(2 * n_kv * GQA, batch), dim3(ATT_MERGE_THREADS), smem_m, stream, m);
}

