"""The reference's own decode kernels on the GPU, as a checker. TEST INFRASTRUCTURE ONLY.

oracle/_ref/ref_decode.so is the reference's kernels/decode.cu (qwen3-8b-fp8_rtx-5090) compiled for sm_100a by
oracle/build_ref.py. This module loads it and restates the two pieces of reference Python needed to drive it:

* `ref_tile_fp8`  the weight layout its GEMV reads (Q/model.py:92-104); it has to be the same permutation,
                  since it defines the kernel's input format.
* `RefEngine`     the reference decode step (Q/generate.py:102-119) with its shipped launch knobs
                  (Q/generate.py:78-83: depth [4,8,4,8], warps 4, pre [2,8,2,2], trig [24,20,30,88], kmajor,
                  attention chunk 64, lm_head CTAs = SM count), block-128 scales and a bf16 lm_head.
Only tests/ use it, to check the B200 kernels bit for bit against the reference's kernels on the same GPU.
"""
from __future__ import annotations

import importlib.util
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "ref_decode.so")
FP8 = torch.float8_e4m3fn


def available() -> bool:
    return os.path.exists(REF_SO)


_mod = None


def ref_ops():
    global _mod
    if _mod is None:
        spec = importlib.util.spec_from_file_location("ref_decode", REF_SO)
        _mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(_mod)
    return _mod


def ref_tile_fp8(w: torch.Tensor, kmajor: bool = True) -> torch.Tensor:
    """Row-major fp8 [N, K] -> the reference GEMV's tile order (Q/model.py:92-104)."""
    N, K = w.shape
    v = w.view(torch.uint8).view(N // 8, 8, K // 64, 4, 4, 4)
    order = (2, 0, 1, 4, 3, 5) if kmajor else (0, 2, 1, 4, 3, 5)
    return v.permute(*order).contiguous().view(FP8).view(N, K)


class RefEngine:
    """The reference decode step over the reference kernels (batch 1, block-128 scales, bf16 lm_head).

    `layers`: list of dicts with row-major fp8 'qkv', 'o_proj', 'gate_up', 'down_proj' as (w, block scale)
    plus bf16 'ln1', 'ln2', 'q_norm', 'k_norm'; all on the GPU."""

    DEPTH, WARPS, PRE, TRIG = [4, 8, 4, 8], [4, 4, 4, 4], [2, 8, 2, 2], [24, 20, 30, 88]

    def __init__(self, layers, embed, norm, lm_head, cos, sin, max_seq, pdl=True):
        self.k = ref_ops()
        self.k.set_pdl(pdl)
        dev = embed.device
        self.layers = []
        for d in layers:
            t = dict(d)
            for name in ("qkv", "o_proj", "gate_up", "down_proj"):
                w, s = d[name]
                t[name] = (ref_tile_fp8(w, True), s)
            self.layers.append(t)
        self.embed, self.norm, self.lm_head, self.cos, self.sin = embed, norm, lm_head, cos, sin
        self.max_seq = max_seq
        L = len(layers)
        self.k_cache = torch.zeros(L, 8, max_seq, 128, dtype=torch.bfloat16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.out_tokens = torch.zeros(max_seq, dtype=torch.int32, device=dev)
        self.best = torch.zeros(1, dtype=torch.int64, device=dev)
        self.resid = torch.zeros(4096, **bf)
        self.qkv = torch.zeros(6144, **bf)
        self.attn = torch.zeros(4096, **bf)
        self.h = torch.zeros(12288, **bf)
        self.logits = torch.zeros(lm_head.shape[0], **bf)
        ms = (max_seq + 31) // 32
        self.o_part = torch.zeros(32, ms, 128, dtype=torch.float32, device=dev)
        self.ml_part = torch.zeros(32, ms, 2, dtype=torch.float32, device=dev)
        self.counters = torch.zeros(8, dtype=torch.int32, device=dev)
        self.lm_head_ctas = torch.cuda.get_device_properties(dev).multi_processor_count

    def gemv(self, kind, lin, x, norm_w, out, eps=1e-6):
        w, s = lin
        i = kind
        self.k.fp8_gemv(kind, w, s, x, norm_w, out, w.shape[0], eps, self.DEPTH[i], self.WARPS[i], self.PRE[i],
                        self.TRIG[i], 1)

    def attention(self, li, eps=1e-6, chunk=64):
        L = self.layers[li]
        self.k.attention(self.qkv, L["q_norm"], L["k_norm"], self.cos, self.sin, self.state, self.k_cache[li],
                         self.v_cache[li], self.o_part, self.ml_part, self.counters, self.attn, 128 ** -0.5, eps, 0,
                         chunk)

    def decode_step(self, eps=1e-6):
        k = self.k
        k.embed(self.token, self.embed, self.resid)
        for li, L in enumerate(self.layers):
            self.gemv(0, L["qkv"], self.resid, L["ln1"], self.qkv)
            self.attention(li)
            self.gemv(1, L["o_proj"], self.attn, None, self.resid)
            self.gemv(2, L["gate_up"], self.resid, L["ln2"], self.h)
            self.gemv(3, L["down_proj"], self.h, None, self.resid)
        k.lm_head_argmax(self.lm_head, self.resid, self.norm, self.logits, self.best, eps, self.lm_head_ctas)
        k.finalize(self.best, self.token, self.out_tokens, self.state)

    def capture(self):
        """One decode step into a CUDA graph, as the reference engine does (Q/generate.py:121-137): two eager
        warm-up steps on a side stream (token and state restored after each), then the capture."""
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

    @torch.no_grad()
    def generate(self, prompt, gen_len):
        """Prompt through the decode step (teacher forcing, as the B200 engine does), then greedy."""
        ids = torch.as_tensor(prompt, dtype=torch.int32, device=self.token.device)
        self.state.zero_()
        self.best.zero_()
        for i in range(ids.numel()):
            self.token.copy_(ids[i:i + 1])
            self.decode_step()
        self.state[1].fill_(0)
        first = int(self.token.item())
        for _ in range(gen_len - 1):
            self.decode_step()
        return [first] + self.out_tokens[: gen_len - 1].tolist()
