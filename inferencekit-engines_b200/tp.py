"""Tensor-parallel decode: one process per GPU, two exchanges per layer.

Two engines share the partition below: `TPEngine` runs the single-GPU ops on each shard with NCCL
all-reduces (torch.distributed) between them; `FusedTPEngine` runs the whole token in one persistent kernel
per rank (qk_decode_step_tp) that exchanges the partials itself over NVLink.

The partition is Megatron-style and follows the reference's 128-blocks, so every rank runs the same kernels
as the single-GPU engine on its shard:

* qkv: column-parallel by KV group. Rank r holds query heads [r*32/TP, (r+1)*32/TP) and KV heads
  [r*8/TP, (r+1)*8/TP): its local qkv is q|k|v of those heads, the layout the attention op expects.
* attention and the KV cache: local (the cache holds only the rank's KV heads).
* o_proj: row-parallel over its K = the rank's query-head dims. The activation is quantized in 128-groups,
  one group per head, so each rank's block dots equal the TP=1 block dots; the rank's fp32 partial
  (GEMV kind 5) is all-reduced (fp32, 16 KiB).
* gate_up: column-parallel with matching gate and up rows, so SwiGLU stays local.
* down: row-parallel over K = 12288/TP (group-aligned), fp32 partial, all-reduce.
* residual: replicated. The all-reduced sum is added as bf16(resid + bf16(sum)) inside the next GEMV's
  prologue (kinds 6/7) or by qk_residual_add before the lm_head.
* lm_head: vocab-parallel (rows [r*V/TP, (r+1)*V/TP), row_offset gives global ids); the packed argmax keys
  are reduced with an int64 MAX all-reduce (after qk_argmax_key_flip maps their unsigned order to signed).

Results equal TP=1 up to the order of the fp32 partial sums (o_proj, down). Synthetic shards are generated
from the same seeded full matrices as `Qwen3FP8Decode.synthetic`, then sliced.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import torch

import model as M


@dataclass(frozen=True)
class Partition:
    tp: int
    rank: int
    cfg: M.Config

    def __post_init__(self):
        c, tp = self.cfg, self.tp
        if tp < 1 or not 0 <= self.rank < tp:
            raise ValueError(f"bad rank {self.rank} of {tp}")
        if c.n_kv_heads % tp or c.n_heads % tp:
            raise ValueError(f"TP={tp} must divide the {c.n_kv_heads} KV heads")
        if c.inter % (M.QBLOCK * tp):
            raise ValueError(f"TP={tp}: the intermediate size {c.inter} must split into 128-aligned shards")
        if c.vocab % (16 * tp):
            raise ValueError(f"TP={tp}: the vocabulary {c.vocab} must split into 16-row shards")

    def span(self, n: int) -> tuple[int, int]:
        return n * self.rank // self.tp, n * (self.rank + 1) // self.tp

    @property
    def q_rows(self):          # rows of q_proj (= columns of o_proj) held by this rank
        a, b = self.span(self.cfg.n_heads)
        return a * self.cfg.head_dim, b * self.cfg.head_dim

    @property
    def kv_rows(self):         # rows of k_proj / v_proj
        a, b = self.span(self.cfg.n_kv_heads)
        return a * self.cfg.head_dim, b * self.cfg.head_dim

    @property
    def inter_rows(self):      # rows of gate_proj / up_proj (= columns of down_proj)
        return self.span(self.cfg.inter)

    @property
    def vocab_rows(self):
        return self.span(self.cfg.vocab)

    def local_cfg(self) -> M.Config:
        c, tp = self.cfg, self.tp
        return replace(c, n_heads=c.n_heads // tp, n_kv_heads=c.n_kv_heads // tp, inter=c.inter // tp,
                       vocab=c.vocab // tp)


def slice_rows(q: torch.Tensor, s: torch.Tensor, a: int, b: int):
    """Rows [a, b) of an fp8 matrix and its scales (per-row [N] or 128x128 blocks [N/128, K/128])."""
    if s.dim() == 1:
        return q[a:b].contiguous(), s[a:b].contiguous()
    assert a % M.QBLOCK == 0 and b % M.QBLOCK == 0
    return q[a:b].contiguous(), s[a // M.QBLOCK:b // M.QBLOCK].contiguous()


def slice_cols(q: torch.Tensor, s: torch.Tensor, a: int, b: int):
    """Columns [a, b) (K range) of an fp8 matrix and its scales."""
    assert a % M.QBLOCK == 0 and b % M.QBLOCK == 0
    if s.dim() == 1:
        return q[:, a:b].contiguous(), s.clone()
    return q[:, a:b].contiguous(), s[:, a // M.QBLOCK:b // M.QBLOCK].contiguous()


def layer_shard(part: Partition, seed: int, li: int, scale_mode: str, device) -> dict:
    """Row-major fp8 shards (and scales) of layer li for this rank: qkv, o_proj, gate_up (gate rows then up
    rows), down_proj. The full matrices are generated from the same seeds as `Qwen3FP8Decode.synthetic`."""
    c = part.cfg
    H, I, hd = c.hidden, c.inter, c.head_dim
    p = f"layers.{li}."

    def full(name, N, K):
        return M.synth_linear(seed, p + name, N, K, scale_mode, device)

    qa, qb = part.q_rows
    ka, kb = part.kv_rows
    ia, ib = part.inter_rows
    q = slice_rows(*full("q_proj", c.n_heads * hd, H), qa, qb)
    k = slice_rows(*full("k_proj", c.n_kv_heads * hd, H), ka, kb)
    v = slice_rows(*full("v_proj", c.n_kv_heads * hd, H), ka, kb)
    g = slice_rows(*full("gate_proj", I, H), ia, ib)
    u = slice_rows(*full("up_proj", I, H), ia, ib)
    cat = lambda *ts: (torch.cat([t[0] for t in ts], 0), torch.cat([t[1] for t in ts], 0).contiguous())
    return {
        "qkv": cat(q, k, v),
        "o_proj": slice_cols(*full("o_proj", H, c.n_heads * hd), qa, qb),
        "gate_up": cat(g, u),
        "down_proj": slice_cols(*full("down_proj", H, I), ia, ib),
    }


def head_shard(part: Partition, seed: int, head_dtype: str, device):
    """This rank's rows of the lm_head: (fp8 rows, fp32 per-row scales) or (bf16 rows, None)."""
    c = part.cfg
    a, b = part.vocab_rows
    w = M.randn((c.vocab, c.hidden), seed, "lm_head", device, 0.02)
    if head_dtype == "fp8":
        q, s = M.quantize_fp8(w, "channel")
        return q[a:b].contiguous(), s[a:b].contiguous()
    return w.to(torch.bfloat16)[a:b].contiguous(), None


def synthetic_shard(cfg: M.Config, tp: int, rank: int, max_seq: int = 4096, device: str = "cuda", seed: int = 0,
                    scale_mode: str = "channel", head_dtype: str = "fp8", norm_init: str = "ones",
                    n_layers: int | None = None) -> M.Qwen3FP8Decode:
    """This rank's shard of `Qwen3FP8Decode.synthetic(cfg, ...)`: a decode model of the local head / row
    counts (its `cfg`), plus the full embedding table and the vocabulary offset of its lm_head rows."""
    cfg.check()
    part = Partition(tp, rank, cfg)
    lc = part.local_cfg()
    m = M.Qwen3FP8Decode(lc, max_seq, device, scale_mode, head_dtype)
    H, hd = cfg.hidden, cfg.head_dim
    m.embed = M.randn((cfg.vocab, H), seed, "embed", device, 0.02).to(torch.bfloat16)
    m.norm = M.synth_norm(seed, "norm", H, norm_init, device)
    for li in range(cfg.layers if n_layers is None else n_layers):
        p = f"layers.{li}."
        L = M.Layer()
        L.ln1 = M.synth_norm(seed, p + "ln1", H, norm_init, device)
        L.ln2 = M.synth_norm(seed, p + "ln2", H, norm_init, device)
        L.q_norm = M.synth_norm(seed, p + "q_norm", hd, norm_init, device)
        L.k_norm = M.synth_norm(seed, p + "k_norm", hd, norm_init, device)
        L.rowmajor = {}
        sh = layer_shard(part, seed, li, scale_mode, device)
        for attr, name, pairs in (("qkv", "qkv", False), ("o", "o_proj", False), ("gu", "gate_up", True),
                                  ("down", "down_proj", False)):
            w, s = sh[name]
            setattr(L, attr, M.Linear(M.pack_fp8(w, pairs), s, w.shape[0], w.shape[1], pairs))
        m.layers.append(L)
    w, s = head_shard(part, seed, head_dtype, device)
    m.lm_head = M.Linear(M.pack_fp8(w), s, w.shape[0], w.shape[1]) if s is not None else w
    m.lm_head_rowmajor = None
    m.vocab_offset = part.vocab_rows[0]
    m.partition = part
    m.alloc_cache()
    return m


class TPEngine:
    """Batch-1 greedy decode on one rank of a TP group: the single-GPU engine's ops on the local shard plus
    NCCL all-reduces (fp32 partial sums after o_proj and down, the argmax key after the lm_head), one CUDA
    graph per step. `group`: the torch.distributed process group (backend nccl)."""

    def __init__(self, m: M.Qwen3FP8Decode, group=None, attn_chunk: int = 64):
        import torch.distributed as dist
        from kernels import ops
        self.dist = dist
        self.group = group
        self.m = m
        self.k = ops()
        self.k.set_pdl(True)
        self.part = m.partition
        cfg, dev = m.cfg, m.device
        H = self.part.cfg.hidden
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.max_seq = m.max_seq
        self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.out_tokens = torch.zeros(m.max_seq, dtype=torch.int32, device=dev)
        self.best = torch.zeros(1, dtype=torch.int64, device=dev)
        # the residual stream alternates between two buffers: a residual-add GEMV reads one and writes the other
        self.resid = [torch.zeros(H, **bf), torch.zeros(H, **bf)]
        self.qkv = torch.zeros((cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim, **bf)
        self.attn = torch.zeros(cfg.n_heads * cfg.head_dim, **bf)
        self.h = torch.zeros(cfg.inter, **bf)
        self.sum = torch.zeros(H, dtype=torch.float32, device=dev)
        self.logits = torch.zeros(cfg.vocab, **bf)
        self.max_splits = (m.max_seq + 31) // 32
        self.o_part = torch.zeros(cfg.n_heads, self.max_splits, cfg.head_dim, dtype=torch.float32, device=dev)
        self.ml_part = torch.zeros(cfg.n_heads, self.max_splits, 2, dtype=torch.float32, device=dev)
        self.counters = torch.zeros(cfg.n_kv_heads, dtype=torch.int32, device=dev)
        self.attn_chunk = attn_chunk
        self.graph = None

    def _allreduce(self, t, op=None):
        self.dist.all_reduce(t, op=op or self.dist.ReduceOp.SUM, group=self.group)

    def decode_step(self):
        m, k, eps = self.m, self.k, self.m.cfg.eps
        H = self.part.cfg.hidden
        cur = 0
        k.embed(self.token, m.embed, self.resid[cur])
        for li, L in enumerate(m.layers):
            if li == 0:
                k.fp8_gemv(0, L.qkv.packed, L.qkv.scale, self.resid[cur], L.ln1, self.qkv, L.qkv.N, eps)
            else:   # residual += the all-reduced down partial, then RMSNorm -> quant -> qkv
                k.fp8_gemv(6, L.qkv.packed, L.qkv.scale, self.resid[cur], L.ln1, self.qkv, L.qkv.N, eps,
                           resadd=self.sum, resid_out=self.resid[1 - cur])
                cur = 1 - cur
            k.attention(self.qkv, L.q_norm, L.k_norm, m.cos, m.sin, self.state, m.k_cache[li, 0], m.v_cache[li, 0],
                        self.o_part, self.ml_part, self.counters, self.attn, m.cfg.head_dim ** -0.5, eps, 0,
                        self.attn_chunk)
            k.fp8_gemv(5, L.o.packed, L.o.scale, self.attn, None, self.sum, H, eps)
            self._allreduce(self.sum)
            k.fp8_gemv(7, L.gu.packed, L.gu.scale, self.resid[cur], L.ln2, self.h, L.gu.N, eps,
                       resadd=self.sum, resid_out=self.resid[1 - cur])
            cur = 1 - cur
            k.fp8_gemv(5, L.down.packed, L.down.scale, self.h, None, self.sum, H, eps)
            self._allreduce(self.sum)
        k.residual_add(self.resid[cur], self.sum)
        if isinstance(m.lm_head, M.Linear):
            k.lm_head_argmax(m.lm_head.packed, self.resid[cur], m.norm, self.logits, self.best, eps,
                             w_scale=m.lm_head.scale, row_offset=m.vocab_offset)
        else:
            k.lm_head_argmax(m.lm_head, self.resid[cur], m.norm, self.logits, self.best, eps,
                             row_offset=m.vocab_offset)
        k.argmax_key_flip(self.best)
        self._allreduce(self.best, self.dist.ReduceOp.MAX)
        k.argmax_key_flip(self.best)
        k.finalize(self.best, self.token, self.out_tokens, self.state)

    def capture(self):
        """One decode step into a CUDA graph (NCCL collectives included); warm-up steps rewrite the current KV
        slot with the same values, so only token and state are restored."""
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
        torch.cuda.synchronize()
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
        """Raise RuntimeError if a kernel of this rank recorded a device error (reads and clears the word)."""
        err = self.k.device_error()
        if err:
            raise RuntimeError(f"rank {self.part.rank}: decode step failed on the device (error word {err:#x})")

    def release(self):
        """Drop the graph (it holds NCCL work) before the process group is destroyed."""
        self.graph = None
        torch.cuda.synchronize()


class FusedTPEngine:
    """One rank of the fused tensor-parallel step: the whole token in one persistent launch per GPU
    (qk_decode_step_tp), the o_proj/down partials and the argmax keys exchanged inside the kernel over NVLink
    (each rank's TP area is mapped into every other rank with CUDA IPC). One CUDA graph per step, no NCCL in
    the step. `group`: the torch.distributed process group, used only to exchange the IPC handles."""

    def __init__(self, m: M.Qwen3FP8Decode, group=None):
        import ctypes
        import torch.distributed as dist
        from kernels import ops, QkTpComm
        self.dist, self.group = dist, group
        self.m = m
        self.k = k = ops()
        self.part_ = part = m.partition
        if not isinstance(m.lm_head, M.Linear) or m.scale_mode != "channel":
            raise ValueError("the fused TP step needs per-channel scales and an FP8 lm_head")
        cfg, dev = m.cfg, m.device
        H = part.cfg.hidden
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.max_seq = m.max_seq
        self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.out_tokens = torch.zeros(m.max_seq, dtype=torch.int32, device=dev)
        self.best = torch.zeros(1, dtype=torch.int64, device=dev)
        self.resid = torch.zeros(H, **bf)
        self.resid_alt = torch.zeros(H, **bf)
        self.qkv = torch.zeros((cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim, **bf)
        self.attn = torch.zeros(cfg.n_heads * cfg.head_dim, **bf)
        self.h = torch.zeros(cfg.inter, **bf)
        self.logits = torch.zeros(cfg.vocab, **bf)
        self.max_splits = (m.max_seq + 63) // 64   # 64-key splits: contexts up to 64k
        self.o_part = torch.zeros(cfg.n_heads, self.max_splits, cfg.head_dim, dtype=torch.float32, device=dev)
        self.ml_part = torch.zeros(cfg.n_heads, self.max_splits, 2, dtype=torch.float32, device=dev)
        self.counters = torch.zeros(cfg.n_kv_heads, dtype=torch.int32, device=dev)
        lib = k.lib
        self.scratch = torch.zeros(lib.qk_decode_step_part_floats(cfg.vocab), dtype=torch.float32, device=dev)
        self.gemv_counters = torch.zeros(lib.qk_decode_step_counters(cfg.vocab), dtype=torch.int32, device=dev)
        self.sync = torch.zeros(4, dtype=torch.int32, device=dev)
        self.layer_table = torch.tensor([[L.qkv.packed.data_ptr(), L.o.packed.data_ptr(), L.gu.packed.data_ptr(),
                                          L.down.packed.data_ptr(), L.qkv.scale.data_ptr(), L.o.scale.data_ptr(),
                                          L.gu.scale.data_ptr(), L.down.scale.data_ptr(), L.ln1.data_ptr(),
                                          L.ln2.data_ptr(), L.q_norm.data_ptr(), L.k_norm.data_ptr()]
                                         for L in m.layers], dtype=torch.int64, device=dev)
        # TP areas: allocate, exchange IPC handles, map the peers'
        torch.cuda.synchronize()
        self.area, handle = k.tp_area_alloc()
        handles = [None] * part.tp
        dist.all_gather_object(handles, handle, group=group)
        self.peers = [self.area if r == part.rank else k.tp_area_open(handles[r]) for r in range(part.tp)]
        self.areas = torch.tensor(self.peers, dtype=torch.int64, device=dev)
        self.comm = QkTpComm(part.tp, part.rank, self.areas.data_ptr())
        torch.cuda.synchronize()
        dist.barrier(group=group)          # every area is zeroed and mapped before any rank launches
        self.graph = None
        self.step_timeline = None

    def decode_step(self):
        m, k = self.m, self.k
        k.decode_step_tp(self.layer_table, len(m.layers), m.k_cache, m.v_cache, m.embed, m.norm, m.lm_head.packed,
                         m.lm_head.scale, m.cos, m.sin, self.token, self.state, self.out_tokens, self.best,
                         self.resid, self.qkv, self.attn, self.h, self.logits, self.scratch, self.gemv_counters,
                         self.o_part, self.ml_part, self.counters, self.sync, m.max_seq, m.cfg.eps, self.resid_alt,
                         m.vocab_offset, self.comm, self.step_timeline)

    def capture(self):
        """One step into a CUDA graph. Every rank must capture (the warm-up steps exchange with the peers)."""
        token, state = self.token.clone(), self.state.clone()
        for _ in range(2):
            self.token.copy_(token)
            self.state.copy_(state)
            self.decode_step()
        torch.cuda.synchronize()
        self.token.copy_(token)
        self.state.copy_(state)
        self.graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(self.graph, stream=s):
                self.decode_step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()

    def step(self, n: int = 1, use_graph: bool = True):
        for _ in range(n):
            if use_graph:
                self.graph.replay()
            else:
                self.decode_step()

    def check(self):
        """Raise RuntimeError if this rank's kernel recorded a device error (reads and clears the word). A
        timed-out exchange (a peer that did not run the step) leaves the ranks' launch epochs apart, so
        every later step would time out too: call `recover()` on every rank before stepping again."""
        err = self.k.device_error()
        if err:
            raise RuntimeError(f"rank {self.part_.rank}: fused TP step failed on the device (error word {err:#x}); "
                               "call recover() on every rank before the next step")

    def recover(self):
        """Bring every rank back to a clean exchange state after a failed step. Collective: every rank calls
        it, between steps, with no launch in flight. Each rank zeroes its own TP area (receive words, key
        counter, epoch) and its step scratch counters between two barriers, so no peer store of the failed
        step can land after the reset and all ranks restart from epoch 0."""
        torch.cuda.synchronize()
        self.dist.barrier(group=self.group)
        self.k.tp_area_reset(self.area)
        for t in (self.gemv_counters, self.counters, self.sync, self.best, self.scratch):
            t.zero_()
        torch.cuda.synchronize()
        self.k.device_error()
        self.dist.barrier(group=self.group)

    def release(self):
        """Unmap the peers' areas and free this rank's (after every rank has finished its launches)."""
        self.graph = None
        torch.cuda.synchronize()
        self.dist.barrier(group=self.group)
        for r, ptr in enumerate(self.peers):
            if r != self.part_.rank:
                self.k.tp_area_close(ptr)
        self.dist.barrier(group=self.group)
        self.k.tp_area_free(self.area)
        self.peers, self.area = [], None
