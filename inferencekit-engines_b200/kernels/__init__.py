"""Loads the B200 decode kernels (C ABI, libqwen3_b200.so) and exposes them under the reference's op names.

Drop-in for the reference's `kernels.ops()` (qwen3-8b-fp8_rtx-5090/kernels/__init__.py:11-24), whose pybind11
module exports fp8_gemv, attention, lm_head_argmax, embed, finalize, set_pdl and set_timeline
(kernels/decode.cu:822-830). The methods below take the same positional arguments in the same order and
launch on torch's current CUDA stream without a host sync, so `Engine.decode_step` can be captured into a
CUDA graph exactly as before. There is no fallback: if the library is missing or the device is not an
sm_100 GPU, `ops()` raises.

Differences a caller must know:
  * FP8 weights must be in `model.pack_fp8` layout (the B200 kernels' tile order). `pack_fp8` returns a
    `PackedFP8` tensor (`PackedFP8Pairs` for gate|up); `fp8_gemv` and the FP8 `lm_head_argmax` raise
    RuntimeError for any other tensor, e.g. weights in the reference's `tile_fp8` layout (convert those
    with `model.pack_reference_tiled`). `depth` maps to ring stages per warp, `warps` to warps per CTA,
    `pre` to ring stages issued before waiting on the previous kernel. `kmajor` must be 0 or 1 and `trig`
    must be -1 or a K block in [0, K/128), as in the reference; neither changes anything here (the layout
    is fixed by the tag, and every kernel lets its successor launch right after its own wait).
  * Scales may be 128x128 blocks [N/128, K/128] or per output channel [N]; the layout is read off the
    tensor's shape.
  * `lm_head_argmax` also takes an FP8 head: pass `w_scale=` (fp32 [V]) with packed fp8 weights.
  * The split-K scratch of the GEMV is owned by this object (allocated on first use per device, before any
    graph capture when the engine warms up eagerly).
"""
from __future__ import annotations

import ctypes
import os

import torch

_here = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_here, "libqwen3_b200.so")

GEMV_QKV, GEMV_O, GEMV_GATE_UP, GEMV_DOWN = 0, 1, 2, 3
GEMV_PARTIAL, GEMV_QKV_RESADD, GEMV_GATE_UP_RESADD = 5, 6, 7
SCALE_BLOCK128, SCALE_CHANNEL = 0, 1

_VP, _I, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
_SIGS = {
    "qk_version": ([], _I),
    "qk_last_error": ([], ctypes.c_char_p),
    "qk_set_pdl": ([_I], _I),
    "qk_set_timeline": ([_VP, _I], _I),
    "qk_get_device_error": ([ctypes.POINTER(_I), _VP], _I),
    "qk_wait_probe": ([_I, _VP, ctypes.c_ulonglong, _VP, _VP], _I),
    "qk_fp8_gemv": ([_I, _VP, _VP, _I, _VP, _VP, _VP, _VP, _VP, _I, _I, _F, _VP, _VP, _I, _I, _I, _I, _I, _VP], _I),
    "qk_attention": ([_VP] * 12 + [_I, _I, _I, _I, _I, _I, _F, _F, _I, _VP], _I),
    "qk_lm_head_argmax": ([_VP, _VP, _I, _VP, _VP, _VP, _VP, _I, _I, _F, _VP, _VP, _I, _VP], _I),
    "qk_embed": ([_VP, _VP, _VP, _I, _I, _VP], _I),
    "qk_decode_step": ([_VP, _I, _VP, _VP, ctypes.c_longlong, _VP, _VP, _VP, _VP, _I, _VP, _VP, _VP, _VP, _VP, _I,
                        _VP, _VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_longlong, _VP, _I, _VP, _VP, _VP, _VP, _I, _I,
                        _F, _I, _VP, _VP], _I),
    "qk_decode_step_tp": ([_VP, _I, _VP, _VP, ctypes.c_longlong, _VP, _VP, _VP, _VP, _I, _VP, _VP, _VP, _VP, _VP,
                           _I, _VP, _VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_longlong, _VP, _I, _VP, _VP, _VP, _VP,
                           _I, _I, _F, _VP, _VP, _I, _VP, _VP], _I),
    "qk_tp_area_bytes": ([], ctypes.c_longlong),
    "qk_tp_area_alloc": ([ctypes.POINTER(_VP), _VP], _I),
    "qk_tp_area_open": ([_VP, ctypes.POINTER(_VP)], _I),
    "qk_tp_area_close": ([_VP], _I),
    "qk_tp_area_free": ([_VP], _I),
    "qk_tp_area_reset": ([_VP, _VP], _I),
    "qk_residual_add": ([_VP, _VP, _I, _VP], _I),
    "qk_argmax_key_flip": ([_VP, _I, _VP], _I),
    "qk_decode_step_part_floats": ([_I], ctypes.c_longlong),
    "qk_decode_step_counters": ([_I], _I),
    "qk_fp8_gemv_noalloc": ([_I, _VP, _VP, _I, _VP, _VP, _VP, _VP, _VP, _I, _I, _F, _VP], _I),
    "qk_finalize": ([_VP, _VP, _VP, _VP, _I, _I, _VP], _I),
    "qk_fp8_gemm_rows_scratch_bytes": ([_I, _I, _I], ctypes.c_longlong),
    "qk_fp8_gemm_rows": ([_VP, _VP, _I, _I, _VP, _VP, _I, _I, _F, _VP, _VP, ctypes.c_longlong, _VP], _I),
    "qk_fp8_gemm_tiles": ([_VP, _VP, _I, _I, _VP, _VP, _I, _I, _F, _VP, _VP, ctypes.c_longlong, _VP], _I),
    "qk_attention_fp8kv": ([_VP] * 13 + [_I, _I, _I, _I, _I, _I, _F, _F, _VP], _I),
    "qk_embed_rows": ([_VP, _I, _VP, _I, _VP, _VP], _I),
    "qk_prefill_qkv": ([_VP, _I, _I, _I, _I, _VP, _VP, _VP, _VP, _F, _VP, _VP, _I, _VP, _VP], _I),
    "qk_prefill_attention": ([_VP, _I, _I, _I, _I, _VP, _VP, _I, _F, _VP, _VP], _I),
    "qk_add_rows": ([_VP, _VP, ctypes.c_longlong, _VP], _I),
    "qk_swiglu_rows": ([_VP, _I, _I, _VP, _VP], _I),
    "qk_argmax_rows": ([_VP, _I, _I, _VP, _VP], _I),
}


class PackedFP8(torch.Tensor):
    """uint8 weights in the `model.pack_fp8` layout (16-row units of 2 KiB tiles). The type survives
    `.to()`, `.cuda()`, views and slicing, so the ops can tell packed weights from any other fp8/uint8
    tensor of the same size."""


class PackedTiles(torch.Tensor):
    """fp8 [N, K] weights in the `model.pack_fp8_tiles` layout: 128 x 128 tiles, each in the 128-byte-swizzle
    image the tcgen05 linear's MMAs read, tile-major. Keeps its type through `.to()` and views."""


class PackedFP8Pairs(PackedFP8):
    """gate|up weights packed as 16 gate rows + the matching 16 up rows per unit (`pack_fp8(w, pairs=True)`)."""


def check_packed(w, pairs: bool, what: str):
    """Raise RuntimeError unless `w` is a pack_fp8 tensor of the right kind (gate|up pairs or plain)."""
    if not isinstance(w, PackedFP8) or isinstance(w, PackedFP8Pairs) != pairs:
        want = "pack_fp8(w, pairs=True)" if pairs else "pack_fp8(w)"
        got = type(w).__name__ if isinstance(w, PackedFP8) else f"an untagged {getattr(w, 'dtype', type(w))} tensor"
        raise RuntimeError(f"{what}: weights must be in the model.{want} layout, got {got} (weights in the "
                           "reference's tile_fp8 layout convert with model.pack_reference_tiled)")


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `make -C {os.path.dirname(_here)}` "
                           "(or __graft_entry__.build())")
    lib = ctypes.CDLL(path)
    for name, (args, res) in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


class QkTpComm(ctypes.Structure):
    """qk_tp_comm_t"""
    _fields_ = [("tp", ctypes.c_int), ("rank", ctypes.c_int), ("areas", ctypes.c_void_p)]


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class DecodeOps:
    """The reference's op set over the C ABI (see module docstring)."""

    TL_SLOT_WORDS = 2048     # u64 words per launch in a timeline buffer (256 CTAs x 8 stamps)

    def __init__(self, lib: ctypes.CDLL):
        self.lib = lib
        self._scratch = {}
        self.timeline_names = None   # launch names in timeline-slot order while a timeline is set

    # ---- helpers ------------------------------------------------------------------------------------------
    def _check(self, status: int, what: str):
        if status != 0:
            raise RuntimeError(f"{what}: {self.lib.qk_last_error().decode()}")

    def scratch(self, device: torch.device, part_floats: int, units: int):
        """Split-K scratch for the GEMV on `device` (grown, never shrunk; counters start at zero)."""
        key = device.index if device.index is not None else torch.cuda.current_device()
        part, counters = self._scratch.get(key, (None, None))
        if part is None or part.numel() < part_floats or counters.numel() < units:
            n_part = max(part_floats, 0 if part is None else part.numel())
            n_cnt = max(units, 0 if counters is None else counters.numel())
            part = torch.empty(n_part, dtype=torch.float32, device=device)
            counters = torch.zeros(n_cnt, dtype=torch.int32, device=device)
            self._scratch[key] = (part, counters)
        return part, counters

    def device_error(self) -> int:
        """Read and clear the device error word (bounded waits that gave up, bad state)."""
        v = ctypes.c_int(0)
        self._check(self.lib.qk_get_device_error(ctypes.byref(v), _stream()), "qk_get_device_error")
        return v.value

    # ---- the reference's ops -----------------------------------------------------------------------------
    def set_pdl(self, on: bool):
        self._check(self.lib.qk_set_pdl(int(bool(on))), "set_pdl")

    def set_timeline(self, buf=None):
        """buf: zeroed int64 CUDA tensor of n_slots * 2048 words, or None to disable. Launch i after this
        call stamps slot i (layout in include/qwen3_b200.h); `timeline_names[i]` names it."""
        n = 0 if buf is None else buf.numel() // self.TL_SLOT_WORDS
        self._check(self.lib.qk_set_timeline(_p(buf), n), "set_timeline")
        self.timeline_names = None if buf is None else []

    def _tl(self, name):
        if self.timeline_names is not None:
            self.timeline_names.append(name)

    def fp8_gemv(self, kind, w, ws, x, norm_w, out, N, eps, depth=0, warps=0, pre=-1, trig=-1, kmajor=1,
                 resadd=None, resid_out=None, stage_tiles=0, ctas_per_sm=0):
        N = int(N)
        check_packed(w, int(kind) in (GEMV_GATE_UP, GEMV_GATE_UP_RESADD), "fp8_gemv")
        K = w.numel() // N
        if int(kmajor) not in (0, 1):
            raise RuntimeError(f"fp8_gemv: kmajor must be 0 or 1, got {kmajor}")
        if int(trig) != -1 and not 0 <= int(trig) < K // 128:
            raise RuntimeError(f"fp8_gemv: trig must be -1 or a K block in [0, {K // 128}), got {trig}")
        scale_mode = SCALE_CHANNEL if ws.dim() == 1 else SCALE_BLOCK128
        part, counters = self.scratch(w.device, N * K // 128, N // 8)
        st = self.lib.qk_fp8_gemv(int(kind), _p(w), _p(ws), scale_mode, _p(x), _p(norm_w), _p(resadd),
                                  _p(resid_out), _p(out), N, K, float(eps), _p(part), _p(counters),
                                  int(warps), int(depth), int(stage_tiles), int(pre), int(ctas_per_sm), _stream())
        self._check(st, "fp8_gemv")
        self._tl(f"gemv{int(kind)}")

    def attention(self, qkv, q_norm_w, k_norm_w, cos_tab, sin_tab, state, k_cache, v_cache, o_part, ml_part,
                  counters, out, scale, eps, late_trigger=0, chunk=64, batch=None, state_stride=2):
        """k_cache/v_cache: one layer, [n_kv, max_seq, 128] (batch 1, as the reference) or
        [batch, n_kv, max_seq, 128]."""
        if k_cache.dim() == 3:
            b, n_kv, max_seq = 1, k_cache.shape[0], k_cache.shape[1]
        else:
            b, n_kv, max_seq = k_cache.shape[0], k_cache.shape[1], k_cache.shape[2]
        if batch is not None:
            b = batch
        max_splits = o_part.shape[-2]
        qkv_stride = qkv.shape[-1] if qkv.dim() > 1 else qkv.numel()
        st = self.lib.qk_attention(_p(qkv), _p(q_norm_w), _p(k_norm_w), _p(cos_tab), _p(sin_tab), _p(state),
                                   _p(k_cache), _p(v_cache), _p(o_part), _p(ml_part), _p(counters), _p(out),
                                   b, n_kv, max_seq, max_splits, qkv_stride, int(state_stride), float(scale),
                                   float(eps), int(chunk), _stream())
        self._check(st, "attention")
        self._tl("attention")

    def attention_fp8kv(self, qkv, q_norm_w, k_norm_w, cos_tab, sin_tab, state, k_cache, k_scale, v_cache, v_scale,
                        o_part, ml_part, out, scale, eps, batch=None, state_stride=2):
        """Decode attention over an FP8 KV cache (e4m3 rows + one fp32 scale per row), 64-key splits.
        k_cache/v_cache: one layer, uint8 or float8_e4m3fn [n_kv, max_seq, 128] (batch 1) or
        [batch, n_kv, max_seq, 128]; k_scale/v_scale: fp32 [n_kv, max_seq] or [batch, n_kv, max_seq]."""
        if k_cache.dim() == 3:
            b, n_kv, max_seq = 1, k_cache.shape[0], k_cache.shape[1]
        else:
            b, n_kv, max_seq = k_cache.shape[0], k_cache.shape[1], k_cache.shape[2]
        if batch is not None:
            b = batch
        if k_cache.element_size() != 1 or v_cache.element_size() != 1 or k_scale.dtype != torch.float32:
            raise RuntimeError("attention_fp8kv: caches must be 1-byte e4m3 rows, scales fp32")
        max_splits = o_part.shape[-2]
        qkv_stride = qkv.shape[-1] if qkv.dim() > 1 else qkv.numel()
        st = self.lib.qk_attention_fp8kv(_p(qkv), _p(q_norm_w), _p(k_norm_w), _p(cos_tab), _p(sin_tab), _p(state),
                                         _p(k_cache), _p(k_scale), _p(v_cache), _p(v_scale), _p(o_part), _p(ml_part),
                                         _p(out), b, n_kv, max_seq, max_splits, qkv_stride, int(state_stride),
                                         float(scale), float(eps), _stream())
        self._check(st, "attention_fp8kv")

    def lm_head_argmax(self, w, x, norm_w, logits, best, eps, ctas=0, w_scale=None, row_offset=0):
        V = logits.numel()
        fp8 = w_scale is not None
        part = counters = None
        if fp8:
            check_packed(w, False, "lm_head_argmax")
            part, counters = self.scratch(w.device, V * 4096 // 128, V // 8)
        elif w.dtype != torch.bfloat16 or isinstance(w, PackedFP8):
            raise RuntimeError("lm_head_argmax: a bf16 [V, 4096] head, or packed fp8 weights with w_scale=")
        st = self.lib.qk_lm_head_argmax(_p(w), _p(w_scale), int(fp8), _p(x), _p(norm_w), _p(logits), _p(best), V,
                                        int(row_offset), float(eps), _p(part), _p(counters), int(ctas), _stream())
        self._check(st, "lm_head_argmax")
        self._tl("lm_head")

    def decode_step(self, layer_table, n_layers, k_cache, v_cache, embed, final_norm, w_head, s_head, cos_tab,
                    sin_tab, token, state, out_tokens, best, resid, qkv, attn, h, logits, part, counters, o_part,
                    ml_part, attn_counters, sync, max_seq, eps, scale_mode, timeline=None):
        """The fused decode step (qk_decode_step): one launch per token. layer_table: int64 CUDA tensor
        [n_layers, 12] of device pointers in qk_layer_t order; k_cache/v_cache: bf16 [n_layers, 1, 8, max_seq, 128]
        (a layer stride of any multiple of 16 bytes); timeline: optional int64 CUDA tensor of
        #SMs * (5*n_layers + 1) * 24 words (layout in include/qwen3_b200.h)."""
        if k_cache.stride() != v_cache.stride() or k_cache.shape[-2] != max_seq or k_cache.shape[-1] != 128:
            raise ValueError("k_cache/v_cache must be [layers, 1, 8, max_seq, 128] with equal strides")
        if s_head is not None:
            check_packed(w_head, False, "decode_step")
        elif w_head.dtype != torch.bfloat16:
            raise RuntimeError("decode_step: without s_head the head must be bf16 [vocab, 4096]")
        stride = k_cache.stride(0) * k_cache.element_size()
        st = self.lib.qk_decode_step(_p(layer_table), int(n_layers), _p(k_cache), _p(v_cache), stride, _p(embed),
                                     _p(final_norm), _p(w_head),
                                     _p(s_head), embed.shape[0], _p(cos_tab), _p(sin_tab), _p(token), _p(state),
                                     _p(out_tokens), out_tokens.numel(), _p(best), _p(resid), _p(qkv), _p(attn), _p(h),
                                     _p(logits), _p(part), part.numel(), _p(counters), counters.numel(), _p(o_part),
                                     _p(ml_part), _p(attn_counters), _p(sync), int(max_seq), o_part.shape[-2],
                                     float(eps), int(scale_mode), _p(timeline), _stream())
        self._check(st, "decode_step")

    def decode_step_tp(self, layer_table, n_layers, k_cache, v_cache, embed, final_norm, w_head, s_head, cos_tab,
                       sin_tab, token, state, out_tokens, best, resid, qkv, attn, h, logits, part, counters, o_part,
                       ml_part, attn_counters, sync, max_seq, eps, resid_alt, vocab_offset, comm, timeline=None):
        """The fused tensor-parallel step of one rank (qk_decode_step_tp); comm: a `TPComm` (areas exchanged)."""
        stride = k_cache.stride(0) * k_cache.element_size()
        st = self.lib.qk_decode_step_tp(_p(layer_table), int(n_layers), _p(k_cache), _p(v_cache), stride, _p(embed),
                                        _p(final_norm), _p(w_head), _p(s_head), logits.numel(), _p(cos_tab),
                                        _p(sin_tab), _p(token), _p(state), _p(out_tokens), out_tokens.numel(),
                                        _p(best), _p(resid), _p(qkv), _p(attn), _p(h), _p(logits), _p(part),
                                        part.numel(), _p(counters), counters.numel(), _p(o_part), _p(ml_part),
                                        _p(attn_counters), _p(sync), int(max_seq), o_part.shape[-2], float(eps),
                                        _p(timeline), _p(resid_alt), int(vocab_offset), ctypes.byref(comm),
                                        _stream())
        self._check(st, "decode_step_tp")

    def tp_area_alloc(self):
        """A zeroed TP area on the current device and its 64-byte CUDA IPC handle (bytes)."""
        area = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        self._check(self.lib.qk_tp_area_alloc(ctypes.byref(area), handle), "tp_area_alloc")
        return area.value, handle.raw

    def tp_area_open(self, handle: bytes):
        peer = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(handle, 64)
        self._check(self.lib.qk_tp_area_open(buf, ctypes.byref(peer)), "tp_area_open")
        return peer.value

    def tp_area_close(self, peer):
        self._check(self.lib.qk_tp_area_close(ctypes.c_void_p(peer)), "tp_area_close")

    def tp_area_free(self, area):
        self._check(self.lib.qk_tp_area_free(ctypes.c_void_p(area)), "tp_area_free")

    def tp_area_reset(self, area):
        """Zero this rank's own TP area on the current stream (recovery after a failed step)."""
        self._check(self.lib.qk_tp_area_reset(ctypes.c_void_p(area), _stream()), "tp_area_reset")

    def residual_add(self, resid, sum_f32):
        """resid = bf16(resid + bf16(sum)) (after the all-reduce of a row-parallel partial)."""
        self._check(self.lib.qk_residual_add(_p(resid), _p(sum_f32), resid.numel(), _stream()), "residual_add")

    def argmax_key_flip(self, keys):
        """Unsigned <-> signed order of packed argmax keys (int64 tensor), in place."""
        self._check(self.lib.qk_argmax_key_flip(_p(keys), keys.numel(), _stream()), "argmax_key_flip")

    def embed(self, token, table, resid):
        b = token.numel()
        self._check(self.lib.qk_embed(_p(token), _p(table), _p(resid), table.shape[0], b, _stream()), "embed")

    def fp8_gemm_rows(self, x, w, w_scale, out, norm_w=None, eps=1e-6):
        """Batched FP8 linear on the tcgen05 tensor cores: out[m] = bf16 W8A8 linear of x[m] (optionally
        RMS-normalised with norm_w first), for M = 1..128 rows (K <= 12288 above 64). x bf16 [M, K]; w fp8 [N, K],
        either a plain row-major matrix (read through TMA boxes) or a `PackedTiles` tensor from
        `model.pack_fp8_tiles` (read as contiguous tiles; not the GEMV's pack_fp8 layout); w_scale fp32 [N] or
        [N/128, K/128]; out bf16 [M, N]. Scratch is owned by this object (zeroed once per size and device)."""
        tiles = isinstance(w, PackedTiles)
        if (isinstance(w, PackedFP8) or w.dtype != torch.float8_e4m3fn or w.dim() != 2 or not w.is_contiguous()):
            raise RuntimeError("fp8_gemm_rows: w must be a row-major float8_e4m3fn [N, K] matrix or "
                               "model.pack_fp8_tiles(w) (not pack_fp8)")
        M, K = x.shape
        N = w.shape[0]
        nbytes = self.lib.qk_fp8_gemm_rows_scratch_bytes(M, N, K)
        if nbytes < 0:
            raise RuntimeError(f"fp8_gemm_rows: unsupported shape M={M} N={N} K={K} (M 1..128; N, K multiples of "
                               "128; K at most 16384, or 12288 above 64 rows)")
        key = ("gemm", x.device.index if x.device.index is not None else torch.cuda.current_device())
        sc = self._scratch.get(key)
        if sc is None or sc.numel() < nbytes:
            sc = torch.zeros(nbytes, dtype=torch.uint8, device=x.device)
            self._scratch[key] = sc
        scale_mode = SCALE_CHANNEL if w_scale.dim() == 1 else SCALE_BLOCK128
        fn = self.lib.qk_fp8_gemm_tiles if tiles else self.lib.qk_fp8_gemm_rows
        st = fn(_p(x), _p(norm_w), M, K, _p(w), _p(w_scale), scale_mode, N, float(eps), _p(out), _p(sc), sc.numel(),
                _stream())
        self._check(st, "fp8_gemm_rows")

    def embed_rows(self, tokens, table, out):
        """out[m] = table[tokens[m]] for the chunk's int32 tokens [M]; out bf16 [M, H]."""
        M = tokens.numel()
        self._check(self.lib.qk_embed_rows(_p(tokens), M, _p(table), table.shape[0], _p(out), _stream()),
                    "embed_rows")

    def prefill_qkv(self, qkv, p0, q_norm, k_norm, cos, sin, eps, k_cache, v_cache, q_out):
        """Per-head RMSNorm + RoPE of the chunk's q and k rows (positions p0 .. p0+M-1), K and V appended to
        one layer's cache [n_kv, max_seq, 128]; q_out bf16 [M, n_q, 128]."""
        M = qkv.shape[0]
        n_kv, max_seq = k_cache.shape[0], k_cache.shape[1]
        n_q = q_out.shape[1]
        st = self.lib.qk_prefill_qkv(_p(qkv), M, int(p0), n_q, n_kv, _p(q_norm), _p(k_norm), _p(cos), _p(sin),
                                     float(eps), _p(k_cache), _p(v_cache), max_seq, _p(q_out), _stream())
        self._check(st, "prefill_qkv")

    def prefill_attention(self, q, p0, k_cache, v_cache, scale, out):
        """Causal GQA attention of the chunk's queries q [M, n_q, 128] over cache rows 0 .. p0+m; out bf16
        [M, n_q * 128] (or [M, n_q, 128])."""
        M, n_q = q.shape[0], q.shape[1]
        n_kv, max_seq = k_cache.shape[0], k_cache.shape[1]
        st = self.lib.qk_prefill_attention(_p(q), M, int(p0), n_q, n_kv, _p(k_cache), _p(v_cache), max_seq,
                                           float(scale), _p(out), _stream())
        self._check(st, "prefill_attention")

    def add_rows(self, resid, y):
        """resid = bf16(resid + y), elementwise."""
        self._check(self.lib.qk_add_rows(_p(resid), _p(y), resid.numel(), _stream()), "add_rows")

    def swiglu_rows(self, gu, h):
        """h[m] = bf16(bf16(silu(gate)) * up) for gu = [gate | up] rows [M, 2I]; h [M, I]."""
        M, I = h.shape
        self._check(self.lib.qk_swiglu_rows(_p(gu), M, I, _p(h), _stream()), "swiglu_rows")

    def argmax_rows(self, logits, best):
        """best[r] = packed argmax key of bf16 logits row r ([rows, V]; ties to the lowest index)."""
        rows, V = logits.shape
        self._check(self.lib.qk_argmax_rows(_p(logits), rows, V, _p(best), _stream()), "argmax_rows")

    def finalize(self, best, token, out_tokens, state):
        b = token.numel()
        out_len = out_tokens.shape[-1]
        self._check(self.lib.qk_finalize(_p(best), _p(token), _p(out_tokens), _p(state), out_len, b, _stream()),
                    "finalize")


_ops = None


def ops() -> DecodeOps:
    """The decode ops (loads libqwen3_b200.so once). Raises if the library or an sm_100 GPU is missing."""
    global _ops
    if _ops is None:
        lib = load_library()
        if not torch.cuda.is_available():
            raise RuntimeError("the B200 decode kernels need a CUDA device")
        major, minor = torch.cuda.get_device_capability()
        if (major, minor) != (10, 0):
            raise RuntimeError(f"libqwen3_b200.so is built for sm_100a; this device is sm_{major}{minor}")
        _ops = DecodeOps(lib)
    return _ops
