"""Batch-1 greedy decode engine on the B200 kernels: one CUDA graph per decode step.

Mirrors the reference engine (qwen3-8b-fp8_rtx-5090/generate.py:39-197): device-resident step state
`[pos, step]`, static activation buffers, `decode_step()` (the hot path, 183 launches), `capture()` into one
CUDA graph, and `generate()`, which replays the graph without a host sync per token.

Prompt processing, two ways:
* `prefill()` feeds the prompt through the decode graph one position at a time (teacher forcing), which
  writes the KV rows and leaves the first generated token in `token`;
* `prefill_chunked()` runs the reference's batched forward (qwen3-8b-fp8_rtx-5090/model.py:243-281) on chunks
  of up to 128 positions: the tcgen05 batched FP8 linear for the projections, the row-wise prefill kernels
  (csrc/prefill.cuh) around it. It reads every weight once per chunk instead of once per position.
Synthetic long-context setups instead fill the cache directly (`Qwen3FP8Decode.fill_cache_random`).
"""
from __future__ import annotations

import torch

from kernels import ops
from model import Qwen3FP8Decode, Linear, pack_fp8_tiles, unpack_fp8

# Per-kind GEMV launch shape: ring stages per warp, warps per CTA, stages issued before the wait,
# tiles per stage (2 KiB = 16 rows x 128 k; 4 KiB for gate|up), CTAs per SM. Kinds: qkv, o_proj, gate_up, down.
DEFAULT_GEMV_SHAPE = {
    0: dict(depth=4, warps=8, pre=4, stage_tiles=2, ctas=1),
    1: dict(depth=4, warps=8, pre=4, stage_tiles=2, ctas=1),
    2: dict(depth=4, warps=8, pre=4, stage_tiles=1, ctas=1),
    3: dict(depth=4, warps=8, pre=4, stage_tiles=2, ctas=1),
}


class Engine:
    """fused=True runs each token as ONE persistent kernel (qk_decode_step, csrc/step.cuh) instead of the
    reference's 183 launches; results are bit-identical. It takes either head format (FP8 per-channel or the
    reference's bf16 head) and needs 64-key attention splits; fused=False is the op-by-op path with the
    reference's drop-in ops."""

    def __init__(self, model: Qwen3FP8Decode, pdl: bool = True, attn_chunk: int = 64, lm_head_ctas: int = 0,
                 gemv_shape: dict | None = None, fused: bool = False):
        self.m = m = model
        self.k = ops()
        self.pdl = pdl
        self.k.set_pdl(pdl)
        cfg = m.cfg
        dev = m.device
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.max_seq = m.max_seq
        self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)        # [pos, step]
        self.out_tokens = torch.zeros(m.max_seq, dtype=torch.int32, device=dev)
        self.best = torch.zeros(1, dtype=torch.int64, device=dev)
        self.resid = torch.zeros(cfg.hidden, **bf)
        self.qkv = torch.zeros((cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim, **bf)
        self.attn = torch.zeros(cfg.n_heads * cfg.head_dim, **bf)
        self.h = torch.zeros(cfg.inter, **bf)
        self.logits = torch.zeros(cfg.vocab, **bf)
        self.max_splits = (m.max_seq + attn_chunk - 1) // attn_chunk   # fused: 64-key splits, up to 64k context
        self.o_part = torch.zeros(cfg.n_heads, self.max_splits, cfg.head_dim, dtype=torch.float32, device=dev)
        self.ml_part = torch.zeros(cfg.n_heads, self.max_splits, 2, dtype=torch.float32, device=dev)
        self.counters = torch.zeros(cfg.n_kv_heads, dtype=torch.int32, device=dev)
        self.attn_chunk = attn_chunk
        self.gemv_shape = {k: dict(v) for k, v in DEFAULT_GEMV_SHAPE.items()}
        if gemv_shape:
            for k, v in gemv_shape.items():
                self.gemv_shape[k].update(v)
        self.lm_head_ctas = lm_head_ctas
        self.graph = None
        self.fused = fused
        self.step_timeline = None     # fused step only: int64 [#SMs, 5*layers+1, 32] stamps (include/qwen3_b200.h)
        if m.kv_dtype == "fp8" and (fused or attn_chunk != 64):
            raise ValueError("an FP8 KV cache runs on the op path (fused=False) with 64-key splits")
        if fused:
            if attn_chunk != 64 or m.batch != 1:
                raise ValueError("the fused step needs 64-key attention splits and batch 1")
            ptrs = []
            for li, L in enumerate(m.layers):
                ptrs.append([L.qkv.packed.data_ptr(), L.o.packed.data_ptr(), L.gu.packed.data_ptr(),
                             L.down.packed.data_ptr(), L.qkv.scale.data_ptr(), L.o.scale.data_ptr(),
                             L.gu.scale.data_ptr(), L.down.scale.data_ptr(), L.ln1.data_ptr(), L.ln2.data_ptr(),
                             L.q_norm.data_ptr(), L.k_norm.data_ptr()])
            self.layer_table = torch.tensor(ptrs, dtype=torch.int64, device=dev)
            lib = self.k.lib
            # the shared block dots carry (launch, phase) tags: part starts zeroed, sync[2] counts the launches
            self.part = torch.zeros(lib.qk_decode_step_part_floats(cfg.vocab), dtype=torch.float32, device=dev)
            self.gemv_counters = torch.zeros(lib.qk_decode_step_counters(cfg.vocab), dtype=torch.int32, device=dev)
            self.sync = torch.zeros(4, dtype=torch.int32, device=dev)
            self.scale_mode = 1 if m.scale_mode == "channel" else 0

    def settings(self) -> dict:
        return {"pdl": self.pdl, "decode_graph": True, "attn_chunk": self.attn_chunk, "gemv_shape": self.gemv_shape,
                "lm_head_ctas": self.lm_head_ctas, "max_seq": self.max_seq, "scale_mode": self.m.scale_mode,
                "head_dtype": self.m.head_dtype}

    def _gemv(self, kind: int, lin: Linear, x, norm_w, out):
        s = self.gemv_shape[kind]
        self.k.fp8_gemv(kind, lin.packed, lin.scale, x, norm_w, out, lin.N, self.m.cfg.eps, s["depth"], s["warps"],
                        s["pre"], -1, 1, stage_tiles=s["stage_tiles"], ctas_per_sm=s["ctas"])

    # ------------------------------------------------------------------------------------------------------
    def decode_step(self):
        """Launch one decode step (eager). Also what gets captured into the graph."""
        m, k, cfg = self.m, self.k, self.m.cfg
        if self.fused:
            fp8_head = isinstance(m.lm_head, Linear)
            k.decode_step(self.layer_table, len(m.layers), m.k_cache, m.v_cache, m.embed, m.norm,
                          m.lm_head.packed if fp8_head else m.lm_head, m.lm_head.scale if fp8_head else None, m.cos, m.sin, self.token, self.state, self.out_tokens, self.best,
                          self.resid, self.qkv, self.attn, self.h, self.logits, self.part, self.gemv_counters,
                          self.o_part, self.ml_part, self.counters, self.sync, m.max_seq, cfg.eps, self.scale_mode,
                          self.step_timeline)
            return
        k.embed(self.token, m.embed, self.resid)
        for li, L in enumerate(m.layers):
            self._gemv(0, L.qkv, self.resid, L.ln1, self.qkv)
            if m.kv_dtype == "fp8":
                k.attention_fp8kv(self.qkv, L.q_norm, L.k_norm, m.cos, m.sin, self.state, m.k_cache[li],
                                  m.k_scale[li], m.v_cache[li], m.v_scale[li], self.o_part, self.ml_part, self.attn,
                                  cfg.head_dim ** -0.5, cfg.eps)
            else:
                k.attention(self.qkv, L.q_norm, L.k_norm, m.cos, m.sin, self.state, m.k_cache[li], m.v_cache[li],
                            self.o_part, self.ml_part, self.counters, self.attn, cfg.head_dim ** -0.5, cfg.eps, 0,
                            self.attn_chunk)
            self._gemv(1, L.o, self.attn, None, self.resid)
            self._gemv(2, L.gu, self.resid, L.ln2, self.h)
            self._gemv(3, L.down, self.h, None, self.resid)
        if isinstance(m.lm_head, Linear):
            k.lm_head_argmax(m.lm_head.packed, self.resid, m.norm, self.logits, self.best, cfg.eps,
                             self.lm_head_ctas, w_scale=m.lm_head.scale)
        else:
            k.lm_head_argmax(m.lm_head, self.resid, m.norm, self.logits, self.best, cfg.eps, self.lm_head_ctas)
        k.finalize(self.best, self.token, self.out_tokens, self.state)

    def capture(self):
        """Record one decode step into a CUDA graph (needs a valid state). The warm-up steps rewrite the KV
        slot at the current position with identical values, so only token and state are restored."""
        token, state = self.token.clone(), self.state.clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self.token.copy_(token)
                self.state.copy_(state)
                self.decode_step()
        torch.cuda.current_stream().wait_stream(s)
        self.token.copy_(token)
        self.state.copy_(state)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.decode_step()
        torch.cuda.synchronize()

    def step(self, n: int = 1, use_graph: bool = True):
        for _ in range(n):
            if use_graph:
                self.graph.replay()
            else:
                self.decode_step()

    # ------------------------------------------------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, prompt_ids, use_graph: bool = True) -> torch.Tensor:
        """Feed the prompt through the decode step at positions 0..P-1. Leaves state = [P, 0] and the first
        generated token in `token`; returns it as a device tensor (no host sync)."""
        ids = torch.as_tensor(prompt_ids, dtype=torch.int32, device=self.m.device)
        P = ids.numel()
        assert 0 < P < self.max_seq
        self.state.zero_()
        self.best.zero_()
        self.token.copy_(ids[:1])
        if use_graph and self.graph is None:
            self.capture()
        for i in range(P):
            if i:
                self.token.copy_(ids[i:i + 1])
            self.step(1, use_graph)
        self.state[1].fill_(0)
        return self.token.clone()

    def prefill_weights(self):
        """Per layer, the (qkv, o, gate_up, down) weights in the batched linear's tile-packed layout
        (`pack_fp8_tiles`: 16 KiB tiles a CTA streams contiguously), built once from the decode layout and
        cached: 7.0 GB more device memory for Qwen3-8B, as the reference's prefill keeps its own row-major copy
        (model.py `rowmajor_copy`)."""
        if getattr(self, "_prefill_w", None) is None:
            self._prefill_w = [tuple(pack_fp8_tiles(unpack_fp8(lin.packed, lin.N, lin.K, lin.pairs))
                                     for lin in (L.qkv, L.o, L.gu, L.down)) for L in self.m.layers]
        return self._prefill_w

    @torch.no_grad()
    def prefill_chunked(self, prompt_ids, chunk: int = 128) -> torch.Tensor:
        """Prompt positions 0..P-1 through the batched forward, `chunk` (<= 128) positions per pass: per layer
        qkv = W_qkv . q(RMSNorm(h)), per-head norm + RoPE with K/V appended to the cache, causal attention over
        the cache, h += W_o . q(attn), h += W_down . q(SwiGLU(W_gu . q(RMSNorm(h)))). The last position's
        hidden row then goes through the head and argmax. Leaves state = [P, 0] and the first generated token
        in `token`, like `prefill()`, and returns it as a device tensor (no host sync)."""
        m, k, cfg = self.m, self.k, self.m.cfg
        if m.batch != 1 or m.kv_dtype != "bf16":
            raise ValueError("prefill_chunked runs batch 1 over a bf16 KV cache (an FP8 cache prefills through "
                             "the decode step: prefill())")
        if not 1 <= chunk <= 128:
            raise ValueError("chunk must be 1..128 positions")
        ids = torch.as_tensor(prompt_ids, dtype=torch.int32, device=m.device)
        P = ids.numel()
        assert 0 < P < self.max_seq
        nq, nkv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        bf = dict(dtype=torch.bfloat16, device=m.device)
        if getattr(self, "_pf", None) is None or self._pf["resid"].shape[0] < chunk:
            self._pf = dict(resid=torch.empty(chunk, cfg.hidden, **bf),
                            qkv=torch.empty(chunk, (nq + 2 * nkv) * hd, **bf),
                            q=torch.empty(chunk, nq, hd, **bf), attn=torch.empty(chunk, nq * hd, **bf),
                            y=torch.empty(chunk, cfg.hidden, **bf), gu=torch.empty(chunk, 2 * cfg.inter, **bf),
                            h=torch.empty(chunk, cfg.inter, **bf))
        b = self._pf
        weights = self.prefill_weights()
        for p0 in range(0, P, chunk):
            M = min(chunk, P - p0)
            resid, qkv, q, attn = b["resid"][:M], b["qkv"][:M], b["q"][:M], b["attn"][:M]
            y, gu, h = b["y"][:M], b["gu"][:M], b["h"][:M]
            k.embed_rows(ids[p0:p0 + M], m.embed, resid)
            for li, L in enumerate(m.layers):
                wq, wo, wgu, wd = weights[li]
                kc, vc = m.k_cache[li, 0], m.v_cache[li, 0]
                k.fp8_gemm_rows(resid, wq, L.qkv.scale, qkv, norm_w=L.ln1, eps=cfg.eps)
                k.prefill_qkv(qkv, p0, L.q_norm, L.k_norm, m.cos, m.sin, cfg.eps, kc, vc, q)
                k.prefill_attention(q, p0, kc, vc, hd ** -0.5, attn)
                k.fp8_gemm_rows(attn, wo, L.o.scale, y)
                k.add_rows(resid, y)
                k.fp8_gemm_rows(resid, wgu, L.gu.scale, gu, norm_w=L.ln2, eps=cfg.eps)
                k.swiglu_rows(gu, h)
                k.fp8_gemm_rows(h, wd, L.down.scale, y)
                k.add_rows(resid, y)
        last = b["resid"][(P - 1) % chunk]
        self.best.zero_()
        if isinstance(m.lm_head, Linear):
            k.lm_head_argmax(m.lm_head.packed, last, m.norm, self.logits, self.best, cfg.eps, self.lm_head_ctas,
                             w_scale=m.lm_head.scale)
        else:
            k.lm_head_argmax(m.lm_head, last, m.norm, self.logits, self.best, cfg.eps, self.lm_head_ctas)
        self.state[0] = P - 1
        self.state[1] = 0
        k.finalize(self.best, self.token, self.out_tokens, self.state)
        self.state[1] = 0
        return self.token.clone()

    def check(self):
        """Raise RuntimeError if a kernel recorded a device error since the last check: a bounded wait that
        gave up (its step's outputs are not valid) or a position / token id out of range. Reads and clears
        the error word (a host sync). After a wait has timed out, every later wait gives up at once until
        this read clears the word, so a caller that sees the error should stop and rebuild its state."""
        err = self.k.device_error()
        if err:
            raise RuntimeError(f"decode step failed on the device (error word {err:#x}: 1 = a ring wait timed out, "
                               "2 = bad position or token, 4 = a grid or peer wait timed out)")

    def recover(self):
        """Reset the step's scratch counters after a failed step (a wait that gave up leaves them mid-count):
        the fused step's grid-barrier, GEMV-unit and attention counters and the argmax key, or the op path's
        counters. Call it between steps, with no launch in flight; clears the device error word."""
        torch.cuda.synchronize()
        for t in (self.counters, self.best) + ((self.sync, self.gemv_counters, self.part) if self.fused else ()):
            t.zero_()
        if not self.fused:
            for key, val in self.k._scratch.items():
                if isinstance(val, tuple):   # the GEMV's (block dots, unit counters)
                    val[1].zero_()
        torch.cuda.synchronize()
        self.k.device_error()

    @torch.no_grad()
    def generate(self, prompt_ids, gen_len: int, use_graph: bool = True):
        """Greedy generation of exactly gen_len tokens (no early stop). Returns a list of ids; raises
        RuntimeError if any step recorded a device error (see `check`)."""
        assert len(prompt_ids) + gen_len <= self.max_seq
        first = self.prefill(prompt_ids, use_graph)
        if gen_len > 1:
            self.step(gen_len - 1, use_graph)
        out = [int(first.item())]
        out += self.out_tokens[: gen_len - 1].tolist()
        self.check()
        return out


class BatchEngine:
    """Greedy decode of B sequences per step (the batch-16 case of the tensor-parallel configuration, here on one
    GPU), the reference engine's step structure with batched ops: per layer the qkv, o_proj, gate_up and down
    projections through the tcgen05 batched linear (B activation rows; each weight byte streams once per step
    for all B sequences), the attention op over each sequence's own cache and position (bf16 or FP8 KV), the
    residual and SwiGLU row kernels; then the final RMSNorm + FP8 lm_head as one more batched linear, the row
    argmax and finalize. `state` is [B, 2] ([pos, step] per sequence), `token` [B]; one CUDA graph per step.
    Needs the FP8 (per-channel) head: the batched linear takes FP8 weights only."""

    def __init__(self, model: Qwen3FP8Decode, pdl: bool = True):
        m = self.m = model
        if not isinstance(m.lm_head, Linear):
            raise ValueError("BatchEngine needs the FP8 lm_head (the batched linear takes FP8 weights)")
        self.k = ops()
        self.k.set_pdl(pdl)
        cfg, dev, B = m.cfg, m.device, m.batch
        self.B, self.max_seq = B, m.max_seq
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.token = torch.zeros(B, dtype=torch.int32, device=dev)
        self.state = torch.zeros(B, 2, dtype=torch.int32, device=dev)
        self.out_tokens = torch.zeros(B, m.max_seq, dtype=torch.int32, device=dev)
        self.best = torch.zeros(B, dtype=torch.int64, device=dev)
        nq, nkv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        self.resid = torch.zeros(B, cfg.hidden, **bf)
        self.qkv = torch.zeros(B, (nq + 2 * nkv) * hd, **bf)
        self.attn = torch.zeros(B, nq * hd, **bf)
        self.y = torch.zeros(B, cfg.hidden, **bf)
        self.gu = torch.zeros(B, 2 * cfg.inter, **bf)
        self.h = torch.zeros(B, cfg.inter, **bf)
        self.logits = torch.zeros(B, cfg.vocab, **bf)
        self.max_splits = (m.max_seq + 63) // 64
        self.o_part = torch.zeros(B, nq, self.max_splits, hd, dtype=torch.float32, device=dev)
        self.ml_part = torch.zeros(B, nq, self.max_splits, 2, dtype=torch.float32, device=dev)
        self.counters = torch.zeros(B, nkv, dtype=torch.int32, device=dev)
        self.w = [tuple(pack_fp8_tiles(unpack_fp8(lin.packed, lin.N, lin.K, lin.pairs))
                        for lin in (L.qkv, L.o, L.gu, L.down)) for L in m.layers]
        self.head_w = pack_fp8_tiles(unpack_fp8(m.lm_head.packed, m.lm_head.N, m.lm_head.K))
        self.graph = None

    def decode_step(self):
        m, k, cfg = self.m, self.k, self.m.cfg
        k.embed(self.token, m.embed, self.resid)
        for li, L in enumerate(m.layers):
            wq, wo, wgu, wd = self.w[li]
            k.fp8_gemm_rows(self.resid, wq, L.qkv.scale, self.qkv, norm_w=L.ln1, eps=cfg.eps)
            if m.kv_dtype == "fp8":
                k.attention_fp8kv(self.qkv, L.q_norm, L.k_norm, m.cos, m.sin, self.state, m.k_cache[li],
                                  m.k_scale[li], m.v_cache[li], m.v_scale[li], self.o_part, self.ml_part, self.attn,
                                  cfg.head_dim ** -0.5, cfg.eps, batch=self.B)
            else:
                k.attention(self.qkv, L.q_norm, L.k_norm, m.cos, m.sin, self.state, m.k_cache[li], m.v_cache[li],
                            self.o_part, self.ml_part, self.counters, self.attn, cfg.head_dim ** -0.5, cfg.eps, 0, 64,
                            batch=self.B)
            k.fp8_gemm_rows(self.attn, wo, L.o.scale, self.y)
            k.add_rows(self.resid, self.y)
            k.fp8_gemm_rows(self.resid, wgu, L.gu.scale, self.gu, norm_w=L.ln2, eps=cfg.eps)
            k.swiglu_rows(self.gu, self.h)
            k.fp8_gemm_rows(self.h, wd, L.down.scale, self.y)
            k.add_rows(self.resid, self.y)
        k.fp8_gemm_rows(self.resid, self.head_w, m.lm_head.scale, self.logits, norm_w=m.norm, eps=cfg.eps)
        k.argmax_rows(self.logits, self.best)
        k.finalize(self.best, self.token, self.out_tokens, self.state)

    def capture(self):
        """One decode step into a CUDA graph (needs a valid state; the warm-up steps rewrite the KV rows at the
        current positions with identical values, so only token and state are restored)."""
        token, state = self.token.clone(), self.state.clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self.token.copy_(token)
                self.state.copy_(state)
                self.decode_step()
        torch.cuda.current_stream().wait_stream(s)
        self.token.copy_(token)
        self.state.copy_(state)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.decode_step()
        torch.cuda.synchronize()

    def step(self, n: int = 1, use_graph: bool = True):
        for _ in range(n):
            if use_graph:
                self.graph.replay()
            else:
                self.decode_step()

    def check(self):
        err = self.k.device_error()
        if err:
            raise RuntimeError(f"batched decode step failed on the device (error word {err:#x})")
