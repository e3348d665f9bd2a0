/*
 * qwen3_b200.h - C ABI of the B200 (sm_100a) Qwen3-8B FP8 decode-step kernels.
 *
 * Drop-in replacement for the pybind11 ops of the reference engine
 * (KittenML/inferencekit-engines, qwen3-8b-fp8_rtx-5090/kernels/decode.cu:822-830, loaded by
 * kernels/__init__.py:11-24 and called from generate.py:102-119). Each reference op maps to one entry point
 * below; the citations give the reference function each one replaces.
 *
 * Conventions
 *   - All tensor arguments are DEVICE pointers owned by the caller; nothing is allocated by any entry point.
 *     Scratch (`part`, `counters`, `o_part`, `ml_part`) is caller-provided; counters must be zero before the
 *     first launch and are left zero by every kernel that uses them.
 *   - Every launch goes to `stream` (a cudaStream_t) with no host synchronisation, so the calls can be
 *     captured into a CUDA graph.
 *   - Return value: QK_OK, or an error code with a message from qk_last_error() (thread-local). Bad
 *     arguments are rejected before anything is launched.
 *   - bf16 tensors are passed as void* (__nv_bfloat16 in device code); fp8 weights are e4m3 bytes in the
 *     packed layout of model.pack_fp8 (2 KiB tiles of 16 rows x 128 k in MMA fragment order).
 *   - Process-global state, as in the reference: the PDL switch (qk_set_pdl). Not thread-safe to change
 *     while another thread launches.
 */
#ifndef QWEN3_B200_H
#define QWEN3_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* qk_stream_t; /* == cudaStream_t */

enum {
  QK_OK = 0,
  QK_EINVAL = 1,  /* bad argument (message in qk_last_error) */
  QK_ECUDA = 2    /* CUDA runtime error (message in qk_last_error) */
};

/* GEMV kinds. 0-3 are the reference's kinds (decode.cu:734-746); 5-8 are the tensor-parallel variants. */
enum {
  QK_GEMV_QKV = 0,          /* RMSNorm(x, norm_w) -> quant -> bf16 store                       */
  QK_GEMV_O = 1,            /* quant(x) -> out[n] = bf16(out[n] + bf16(y[n]))  (residual, in place) */
  QK_GEMV_GATE_UP = 2,      /* RMSNorm -> quant -> SwiGLU(gate rows, up rows) -> bf16 [N/2]      */
  QK_GEMV_DOWN = 3,         /* like O with K = 12288 (K is an argument here)                      */
  QK_GEMV_PARTIAL = 5,      /* quant(x) -> fp32 store (row-parallel shard before the all-reduce)  */
  QK_GEMV_QKV_RESADD = 6,   /* x = bf16(resid + bf16(resadd)) first (written back), then as QKV   */
  QK_GEMV_GATE_UP_RESADD = 7 /* the same residual update, then as GATE_UP                         */
};

enum { QK_SCALE_BLOCK128 = 0, QK_SCALE_CHANNEL = 1 };

/* Library version (major*10000 + minor*100 + patch) and the last error message of this thread. */
int qk_version(void);
const char* qk_last_error(void);

/* Programmatic dependent launch on/off for subsequent launches (reference decode.cu:713 set_pdl). */
int qk_set_pdl(int on);

/* Profiling timeline (reference decode.cu:56-62, :716 set_timeline): `buf` is a zeroed device buffer of
 * n_slots * 2048 u64. Launch number i after this call (any kernel but embed/finalize) writes %globaltimer
 * stamps of its first 256 CTAs into slot i: CTA c uses words c*8 + j. GEMV and lm_head: j=0 entry, 1 after
 * the wait on the previous kernel, 2 after the prologue (GEMV), 3 max over warps of the first weight stage
 * landing (GEMV), 4 max over warps of the end of the weight loop. Attention: 0 entry, 1 after the wait,
 * 2 partial results written, 3 merge done (merging CTA only). NULL disables. Synchronous; not while
 * capturing a graph (the slots are fixed into a graph at capture). */
int qk_set_timeline(uint64_t* buf, int n_slots);

/* Read and clear the device-side error word (bit 1: a bounded wait gave up; bit 2: bad step state or
 * token id). Synchronises `stream`. No counterpart in the reference (its waits are unbounded). */
int qk_get_device_error(int* err, qk_stream_t stream);

/* Exercise the failure path of the bounded waits (no counterpart in the reference, whose waits are unbounded):
 * one thread waits, at most limit_ns (<= 1 s), for something that never happens — phase 0 of an mbarrier nothing
 * arrives on (mode 0, as a ring stage that never lands) or *counter >= 1 for a zeroed u64 counter nothing adds to
 * (mode 1, as a peer rank that stopped). The wait gives up, writes 1 to the device int *gave_up, sets the device
 * error word (bit 1 for mode 0, bit 4 for mode 1; read with qk_get_device_error) and the context stays usable.
 * Waits skip ahead while the error word already holds a timeout, so read it (which clears it) first. */
int qk_wait_probe(int mode, void* counter, unsigned long long limit_ns, int* gave_up, qk_stream_t stream);

/*
 * FP8 W8A8 GEMV (reference decode.cu:765-774 fp8_gemv, kernels :128-335).
 *   w          packed fp8 [N x K] (model.pack_fp8; gate|up units interleaved for kind 2/7)
 *   w_scale    fp32 scales, [N/128][K/128] (QK_SCALE_BLOCK128) or [N] (QK_SCALE_CHANNEL)
 *   x          bf16 [K] input (kinds 6/7: the residual stream, updated in place through resid_out)
 *   norm_w     bf16 [K] RMSNorm weight (kinds 0, 2, 6, 7), else may be NULL
 *   resadd     fp32 [K] sums added to the residual (kinds 6, 7), else NULL
 *   resid_out  bf16 [K] destination of the updated residual (kinds 6, 7; may equal x), else NULL
 *   out        bf16 output: [N] (0, 6), residual [N] in place (1, 3), [N/2] (2, 7); fp32 [N] for kind 5
 *   part       fp32 scratch of N*K/128 floats; counters: int scratch of N/16 ints, zeroed once
 *   warps/stages/stage_tiles/pre/ctas_per_sm: launch shape (0 = default). pre = ring stages issued
 *              before waiting on the previous kernel; stage_tiles = tiles per ring stage (a tile is
 *              16 rows x 128 k = 2 KiB; 4 KiB for the gate|up kinds 2/7).
 */
int qk_fp8_gemv(int kind, const void* w, const float* w_scale, int scale_mode, const void* x, const void* norm_w,
                const float* resadd, void* resid_out, void* out, int N, int K, float eps, float* part, int* counters,
                int warps, int stages, int stage_tiles, int pre, int ctas_per_sm, qk_stream_t stream);

/*
 * qk_fp8_gemv for callers that cannot allocate device memory (no counterpart in the reference, whose ops take
 * caller tensors only). Same arguments minus the scratch and the launch shape (defaults are used): the
 * split-K scratch lives in a fixed 3 MiB + 16 KiB device array inside the library, present on every GPU that
 * loads it until the process exits. Limit: N*K/128 <= 786432 and N/16 <= 4096 (every per-layer GEMV of
 * Qwen3-8B fits; the 151936-row lm_head does not), else QK_EINVAL. Nothing is allocated: the first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) with that device current, so make that
 * first call before any stream capture. Each call clears the counters with cudaMemsetAsync on `stream`. All
 * calls share the one array, so calls that may overlap on the GPU (different streams, or concurrent host
 * threads) race on it; serialise them.
 */
int qk_fp8_gemv_noalloc(int kind, const void* w, const float* w_scale, int scale_mode, const void* x,
                        const void* norm_w, const float* resadd, void* resid_out, void* out, int N, int K, float eps,
                        qk_stream_t stream);

/*
 * Fused q/k RMSNorm + RoPE + KV append + GQA split-KV decode attention
 * (reference decode.cu:776-800 attention, kernel :379-570).
 *   qkv        bf16 [batch][qkv_stride]: n_q = 4*n_kv query heads, then n_kv k heads, n_kv v heads (128 each)
 *   state      int32, per sequence b: state[b*state_stride] = position of the new token
 *   k_cache/v_cache  bf16 [batch][n_kv][max_seq][128] of ONE layer; slot `pos` of each head is written
 *   o_part     fp32 [batch][n_q][max_splits][128]; ml_part fp32 [batch][n_q][max_splits][2]
 *   counters   int32 [batch][n_kv], zero before the first launch (left zero)
 *   out        bf16 [batch][n_q*128]
 *   chunk      keys per CTA: 32, 64 or 128; requires max_splits*chunk >= max_seq
 */
int qk_attention(const void* qkv, const void* q_norm_w, const void* k_norm_w, const void* cos_tab,
                 const void* sin_tab, const int* state, void* k_cache, void* v_cache, float* o_part,
                 float* ml_part, int* counters, void* out, int batch, int n_kv, int max_seq, int max_splits,
                 int qkv_stride, int state_stride, float scale, float eps, int chunk, qk_stream_t stream);

/*
 * Final RMSNorm + lm_head GEMV + greedy argmax (reference decode.cu:802-810 lm_head_argmax, :584-661).
 * bf16 head (reference format): w bf16 [V][4096] row-major, w_scale NULL.
 * fp8 head (per-channel): w packed fp8 [V x 4096], w_scale fp32 [V], part/counters as qk_fp8_gemv.
 * logits bf16 [V]; best: packed (value, ~index) u64, zero before the launch (qk_finalize clears it).
 * row_offset: vocabulary index of row 0 (vocab-parallel shards). ctas: CTAs (0 = one per SM).
 */
int qk_lm_head_argmax(const void* w, const float* w_scale, int head_fp8, const void* x, const void* norm_w,
                      void* logits, unsigned long long* best, int V, int row_offset, float eps, float* part,
                      int* counters, int ctas, qk_stream_t stream);

/* Device pointers of one decoder layer, as laid out in the device array given to qk_decode_step. */
typedef struct {
  const void *w_qkv, *w_o, *w_gu, *w_down;       /* packed fp8 (model.pack_fp8; gate|up interleaved) */
  const float *s_qkv, *s_o, *s_gu, *s_down;      /* scales, layout per scale_mode */
  const void *ln1, *ln2, *q_norm, *k_norm;       /* bf16 */
} qk_layer_t;

/*
 * The whole batch-1 decode step in one launch: embed -> n_layers x (qkv GEMV, attention with KV append,
 * o_proj, gate_up, down) -> lm_head + greedy argmax -> token/state update. Replaces the reference's 183-launch
 * `Engine.decode_step` (generate.py:102-119) with bit-identical results; the ops it fuses are the entry points
 * above. Cooperative launch of one CTA per SM (graph-capturable).
 *   layers      DEVICE array of n_layers qk_layer_t
 *   w_head/s_head  FP8 per-channel head: packed fp8 [vocab x 4096] and fp32 scales [vocab]; or, with s_head
 *               NULL, the reference checkpoint's bf16 head, row-major [vocab][4096] (tp = 1 only)
 *   k_cache/v_cache  bf16 KV caches of all layers: layer l at byte offset l * kv_layer_stride, each
 *               [8][max_seq][128] (16-byte aligned, stride a multiple of 16); read through TMA tensor maps
 *   state       [pos, step]; token [1]; out_tokens [out_len]; best u64 [1] zero before the first launch
 *   resid/qkv/attn/h/logits  bf16 activations [4096]/[6144]/[4096]/[12288]/[vocab]
 *   part        scratch of part_floats >= qk_decode_step_part_floats(vocab) floats (tagged block dots of the
 *               GEMV units two CTAs share), zeroed once before the first launch; counters int
 *               [n_counters >= qk_decode_step_counters(vocab)], zero before the first launch
 *   o_part/ml_part  fp32 [32][max_splits][128] / [32][max_splits][2]; attn_counters int [8] zero
 *   sync        unsigned [4] zeroed once before the first launch: [0], [1] barrier counters (left zero), [2] the
 *               launches completed (tags of the shared block dots; zero it only together with `part`)
 *   max_splits  >= ceil(max_seq/64), <= 1024
 *   timeline    NULL, or a device buffer of (#SMs) x (5*n_layers + 1) x 32 u64: per CTA and phase (layer l:
 *               qkv, attn, o, gu, down = 5l+0..4; lm_head = 5*n_layers) the %globaltimer of 0 consumers start,
 *               1 prologue done (attention: arrivals counted and, on merging CTAs, the merge done), 2 the whole
 *               CTA done (inside the grid barrier), 3 producer issues the phase's first load, 7 consumer warp 0
 *               leaves the stage loop (attention: partials done), 9-15 consumer warps 1-7 leave it; cumulative
 *               clock64 cycles: 4 consumer warp 0 waiting for data, 5 consumer warp 0 folding units, 6 producer
 *               waiting for free ring stages, 8 consumer warp 0 waiting for other warps' slices of a unit it
 *               folds, 16 consumer warp 0 computing slice pairs, 17 taking and counting them; 18 pairs it took.
 */
int qk_decode_step(const qk_layer_t* layers, int n_layers, void* k_cache, void* v_cache, long long kv_layer_stride,
                   const void* embed, const void* final_norm, const void* w_head, const float* s_head, int vocab,
                   const void* cos_tab, const void* sin_tab, int* token, int* state, int* out_tokens, int out_len,
                   unsigned long long* best, void* resid, void* qkv, void* attn, void* h, void* logits, float* part,
                   long long part_floats, int* counters, int n_counters, float* o_part, float* ml_part,
                   int* attn_counters, unsigned* sync, int max_seq, int max_splits, float eps, int scale_mode,
                   uint64_t* timeline, qk_stream_t stream);

/*
 * Tensor-parallel fused step (no counterpart in the reference, whose engine is single-GPU; this is the TP
 * `comm` handle entry point its scope allows). Every rank runs qk_decode_step_tp on its shard, one process per
 * GPU: query heads 32/tp, KV heads 8/tp (KV caches [n_layers][8/tp][max_seq][128]), gate|up rows 2*12288/tp,
 * o_proj and down columns 4096/tp and 12288/tp, lm_head rows `vocab` (this rank's) from global id
 * `vocab_offset`. o_proj and down produce fp32 partials that the kernel exchanges itself: it stores them into
 * every rank's TP area over NVLink (plain stores to peer memory mapped with CUDA IPC), each as one 64-bit word
 * that carries the value and the exchange's tag, and waits (bounded) until every rank's word of a row carries
 * the current tag; each rank adds the partials to its residual in rank order, so all ranks hold the same
 * residual. The argmax keys go to every rank's area behind a system-scope counter, and every rank writes the
 * same token. Results equal
 * the single-GPU step up to the order of the fp32 partial sums. Per-channel scales only.
 *   areas      DEVICE array [tp] of every rank's TP area as mapped in this process ([rank] = its own):
 *              qk_tp_area_alloc on each rank, the 64-byte IPC handles exchanged by the caller, then
 *              qk_tp_area_open on each peer's handle. Areas start zeroed and must not be reset between launches.
 *   resid_alt  a second bf16 [4096] residual buffer
 * All ranks must launch the same number of steps; a rank that stops makes the others' bounded waits time out
 * and set the device error word (qk_get_device_error). After such a timeout the ranks' launch epochs differ
 * and every later step would time out as well: every rank then resets its own area with qk_tp_area_reset
 * (and zeroes its step scratch counters, sync and best), between two host barriers with no launch in flight.
 */
typedef struct {
  int tp;                   /* ranks: 2, 4 or 8 */
  int rank;                 /* this rank */
  void* const* areas;       /* DEVICE array [tp] of TP area pointers */
} qk_tp_comm_t;

long long qk_tp_area_bytes(void);
int qk_tp_area_alloc(void** area, void* ipc_handle /* 64 bytes out */);
int qk_tp_area_open(const void* ipc_handle, void** peer_area);
int qk_tp_area_close(void* peer_area);
int qk_tp_area_free(void* area);
/* Zero this rank's own TP area (receive words, key counter, epoch) on `stream`: recovery after a failed step. */
int qk_tp_area_reset(void* area, qk_stream_t stream);
int qk_decode_step_tp(const qk_layer_t* layers, int n_layers, void* k_cache, void* v_cache, long long kv_layer_stride,
                      const void* embed, const void* final_norm, const void* w_head, const float* s_head, int vocab,
                      const void* cos_tab, const void* sin_tab, int* token, int* state, int* out_tokens,
                      int out_len, unsigned long long* best, void* resid, void* qkv, void* attn, void* h,
                      void* logits, float* part, long long part_floats, int* counters, int n_counters,
                      float* o_part, float* ml_part, int* attn_counters, unsigned* sync, int max_seq,
                      int max_splits, float eps, uint64_t* timeline, void* resid_alt, int vocab_offset,
                      const qk_tp_comm_t* comm, qk_stream_t stream);

/* Minimum scratch sizes of qk_decode_step for a vocabulary size (no GPU needed). */
long long qk_decode_step_part_floats(int vocab);
int qk_decode_step_counters(int vocab);

/* resid[b] = table[token[b]] for b < batch (reference decode.cu:812 embed, :667-673). */
int qk_embed(const int* token, const void* table, void* resid, int vocab, int batch, qk_stream_t stream);

/* token = argmax key, out_tokens[step] = token, pos++, step++, best = 0; state = [pos, step] per sequence
 * (reference decode.cu:817 finalize, :676-687). out_len: capacity of out_tokens per sequence. */
int qk_finalize(unsigned long long* best, int* token, int* out_tokens, int* state, int out_len, int batch,
                qk_stream_t stream);

/* Batched FP8 W8A8 linear on the tcgen05 tensor cores (1-128 rows: the batched GEMV rows and prefill chunks; the
 * reference's batched path is its Triton fp8_matmul, prefill.py:121-156, with act_quant :23-41): out[m][n] = bf16(sum over K blocks
 * kb of dot_kb(q(x[m]), w[n]) * s_x[m][kb] * s_w[n][kb]) for M = 1..128 rows (per-channel scales: the sum of
 * dot_kb * s_x[m][kb], times s_w[n]), where q() is the per-128-group e4m3
 * quantizer of the GEMV (optionally after RMSNorm with norm_w). x bf16 [M][K]; w fp8 row-major [N][K] (plain
 * matrix, TMA boxes; not the GEMV's packed layout); w_scale fp32 [N] (QK_SCALE_CHANNEL) or [N/128][K/128];
 * out bf16 [M][N]; N and K multiples of 128, N <= 1,048,576, K <= 16384 (12288 above 64 rows). scratch: at least
 * qk_fp8_gemm_rows_scratch_bytes(M, N, K) bytes, 256-byte aligned, zeroed once before the first call (its first
 * 32 KiB hold the tile counters, which every call leaves zero, so one buffer serves calls of any shape). Results match the oracle's
 * recipe to rounding (split-K boundaries reorder the fp32 sum), not bit for bit. */
long long qk_fp8_gemm_rows_scratch_bytes(int M, int N, int K);
int qk_fp8_gemm_rows(const void* x, const void* norm_w, int M, int K, const void* w, const float* w_scale,
                     int scale_mode, int N, float eps, void* out, void* scratch, long long scratch_bytes,
                     qk_stream_t stream);
/* The same linear with the weights tile-packed (no tensor maps): w_tiles is [N/128][K/128] tiles of 128 rows x
 * 128 k, 16,384 bytes each, row r of a tile at byte 128 r and its 16-byte chunk c at chunk c ^ (r % 8) (the
 * image a 128-byte-swizzled TMA box would leave in shared memory; `model.pack_fp8_tiles` builds it). Each CTA's
 * weight range is then one contiguous stream of bulk copies. Same arguments, scratch and results otherwise. */
int qk_fp8_gemm_tiles(const void* x, const void* norm_w, int M, int K, const void* w_tiles, const float* w_scale,
                      int scale_mode, int N, float eps, void* out, void* scratch, long long scratch_bytes,
                      qk_stream_t stream);

/* Decode attention over an FP8 KV cache (no counterpart in the reference, which lists one as future work:
 * fewer long-context KV bytes, different numerics). Each cached K and V row (sequence, KV head, position) is 128
 * e4m3 bytes plus one fp32 scale: s = amax/448 (div.full), q = e4m3(x / s) round-to-nearest-even, saturating,
 * s = 0 -> 0, where x is the bf16 row the bf16 cache would hold (K normalised and rotated, V as projected).
 * Scores s_j = (q . k8_j) * ks_j * scale; per split (128, 256 or 512 keys by max_seq) a running
 * softmax over 128-key blocks (m, l, p = exp(s - m)) and o = sum_j (p_j * vs_j) * v8_j; the splits merge as in
 * qk_attention. Appends the new K and V rows (and scales) at pos. k_cache/v_cache: [batch][n_kv][max_seq][128]
 * bytes, k_scale/v_scale: [batch][n_kv][max_seq] fp32; o_part, ml_part, state and out as qk_attention
 * (max_splits * 128 >= max_seq suffices). */
int qk_attention_fp8kv(const void* qkv, const void* q_norm_w, const void* k_norm_w, const void* cos_tab,
                       const void* sin_tab, const int* state, void* k_cache, float* k_scale, void* v_cache,
                       float* v_scale, float* o_part, float* ml_part, void* out, int batch, int n_kv, int max_seq,
                       int max_splits, int qkv_stride, int state_stride, float scale, float eps,
                       qk_stream_t stream);

/* Chunked prefill: the row-wise steps of the reference's batched forward (Q/model.py:243-281, with the fused
 * prefill kernels of Q/kernels/prefill_fused.py:57-183), run on a chunk of M prompt positions p0 .. p0+M-1
 * around four qk_fp8_gemm_rows calls per layer. All tensors bf16, row-major, on the device.
 *
 * qk_embed_rows: out[m] = table[tokens[m]] (HIDDEN values) for m < M; a token outside [0, vocab) sets the
 *   error word's bad-state bit and copies row 0.
 * qk_prefill_qkv: from qkv [M][(n_q + 2 n_kv) * 128] (the qkv projection of the chunk), per row m at position
 *   p0 + m: q_out[m][h] = RoPE(RMSNorm(q_h, q_norm)), k_cache[g][p0+m] = RoPE(RMSNorm(k_g, k_norm)),
 *   v_cache[g][p0+m] = v_g, with the decode step's bf16 roundings (the rows written equal what the decode step
 *   writes for that position from the same qkv row). k_cache/v_cache: one layer, [n_kv][max_seq][128];
 *   cos_tab/sin_tab: [max_seq][128]. n_q = 4 n_kv; p0 + M <= max_seq.
 * qk_prefill_attention: out[m][h] = softmax(q[m][h] . K[g][0..p0+m] * scale) . V[g][0..p0+m] with g = h / 4
 *   (causal GQA); fp32 scores, probabilities and sums, one online-softmax pass; matches an fp32 reference to
 *   rounding. q and out: [M][n_q * 128]; the caches as above, rows 0 .. p0+M-1 written.
 * qk_add_rows: resid[i] = bf16(resid[i] + y[i]) for i < n (the decode step's residual epilogue).
 * qk_swiglu_rows: h[m][i] = bf16(bf16(silu(gu[m][i])) * gu[m][I + i]) for gu [M][2I], h [M][I] (the decode
 *   step's SwiGLU epilogue). */
int qk_embed_rows(const int* tokens, int M, const void* table, int vocab, void* out, qk_stream_t stream);
int qk_prefill_qkv(const void* qkv, int M, int p0, int n_q, int n_kv, const void* q_norm, const void* k_norm,
                   const void* cos_tab, const void* sin_tab, float eps, void* k_cache, void* v_cache, int max_seq,
                   void* q_out, qk_stream_t stream);
int qk_prefill_attention(const void* q, int M, int p0, int n_q, int n_kv, const void* k_cache, const void* v_cache,
                         int max_seq, float scale, void* out, qk_stream_t stream);
int qk_add_rows(void* resid, const void* y, long long n, qk_stream_t stream);
int qk_swiglu_rows(const void* gu, int M, int I, void* h, qk_stream_t stream);
/* best[r] = the packed argmax key (the lm_head's: order-preserving value bits, then ~index, so ties go to the
 * lowest index) of bf16 logits row r of [rows][V]; qk_finalize decodes it. The batched decode step's argmax. */
int qk_argmax_rows(const void* logits, int rows, int V, unsigned long long* best, qk_stream_t stream);

/* Tensor-parallel helpers (no counterpart in the single-GPU reference; the TP plan of its decode step):
 * resid[i] = bf16(resid[i] + bf16(sum[i])) for the fp32 all-reduced partial of a row-parallel GEMV (the
 * rounding of the reference's residual epilogue, decode.cu:320-323); and the top-bit flip of packed argmax
 * keys, which maps their unsigned order onto signed int64 order for an NCCL int64 MAX all-reduce. */
int qk_residual_add(void* resid, const float* sum, int n, qk_stream_t stream);
int qk_argmax_key_flip(unsigned long long* keys, int n, qk_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* QWEN3_B200_H */
