"""CPU oracle for the Qwen3-8B FP8 decode step. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module, and only as
the checker (or as the timed CPU baseline). The product path never calls it and has no CPU fallback.

It restates, in plain torch CPU ops, the arithmetic of the reference engine
(KittenML/inferencekit-engines, folder qwen3-8b-fp8_rtx-5090, abbreviated Q/ below):

* `act_quant`      Q/kernels/prefill.py:23-32 (Triton) and Q/kernels/decode.cu:92-110, :257-259:
                   per 128-wide group s = max|x| / 448, q = fp8_e4m3(x / s) round-to-nearest-even,
                   saturated to +-448; a group with s == 0 quantizes to 0 (decode.cu:105).
* `fp8_linear`     Q/kernels/prefill.py:44-73, :115-118: per 128-wide K block, the fp32 dot of the fp8
                   operands times s_x times s_w, accumulated over K blocks in order, rounded to bf16.
                   Scales are 128x128 blocks [N/128, K/128] (the reference checkpoint) or one per output
                   row [N] (the north-star format; the reference indexes scales per 128 rows, this is the
                   same expression with s_w[n] broadcast over K).
* `rms_norm`       Q/model.py:121-125.  `rotate_half` Q/model.py:128-130.  RoPE Q/model.py:265-266.
* `decode_layer`   Q/model.py:259-279 for one token (M = 1, start = pos), with the KV write at `pos`
                   (model.py:267-268). Attention is the decode kernel's arithmetic (Q/kernels/decode.cu:
                   462-567): fp32 scores, fp32 softmax with the probabilities kept in fp32, fp32 P @ V,
                   rounded to bf16 once. `attn_impl="sdpa"` instead uses torch SDPA exactly as
                   model.py:271-272 does (bf16 probabilities), which is what the golden fixtures pin.
* `prefill_layer`  Q/model.py:255-279 for M prompt positions at once (start..start+M-1): the same layer with
                   the KV rows written for every position and causal attention (row m sees cache rows
                   0..start+m), fp32 scores and probabilities, rounded to bf16 once; `attn_impl="sdpa"`
                   calls SDPA as model.py:271-273 does, which tests/golden/prefill_block.npz pins bit for bit
                   against the reference's own forward(tokens, 0).
* `quant_kv_rows`, `attention_fp8kv_f32`: the FP8 KV cache's contract (an extension with no reference
                   counterpart): e4m3 rows with one fp32 scale each, scores and probabilities in fp32.
* `lm_head_argmax` Q/model.py:280-281 (final RMSNorm + linear) and Q/kernels/decode.cu:572-661: greedy
                   argmax over bf16 logits, ties to the lowest index.

Parity pinning: tests/golden/ holds outputs of the reference's own `Qwen3FP8.forward` (Q/model.py:243-281),
run on CPU in the build container with its Triton `fp8_linear` replaced by `fp8_linear` below (the
Triton interpreter's fp8 cast is wrong, so the Triton kernel itself cannot run on CPU). The fixtures
therefore pin the layer structure, norms, RoPE, KV slots, residuals, SwiGLU and lm_head; the FP8 linear
arithmetic is pinned on the B200 by bitwise comparison with the reference's decode.cu (oracle/_ref).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

FP8 = torch.float8_e4m3fn
FP8_MAX = 448.0
QBLOCK = 128


def act_quant(x: torch.Tensor):
    """x [..., K] bf16 -> (q fp8 [..., K], s fp32 [..., K/128])."""
    xf = x.float()
    shp = xf.shape
    g = xf.reshape(*shp[:-1], shp[-1] // QBLOCK, QBLOCK)
    s = g.abs().amax(-1) / FP8_MAX
    safe = torch.where(s > 0, s, torch.ones_like(s))
    q = torch.where(s[..., None] > 0, g / safe[..., None], torch.zeros_like(g))
    q = q.clamp(-FP8_MAX, FP8_MAX).to(FP8).reshape(shp)
    return q, s


def block_dots(q: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Per-128-block fp32 dots: q fp8 [M, K], w fp8 [N, K] -> [M, N, K/128]."""
    M, K = q.shape
    N = w.shape[0]
    KB = K // QBLOCK
    qf = q.float().view(M, KB, QBLOCK).permute(1, 0, 2)            # [KB, M, 128]
    wf = w.float().view(N, KB, QBLOCK).permute(1, 2, 0)            # [KB, 128, N]
    return torch.bmm(qf, wf).permute(1, 2, 0)                      # [M, N, KB]


def scale_rows(w_scale: torch.Tensor, N: int, KB: int) -> torch.Tensor:
    """Weight scale per (row, K block) as [N, KB] for either scale layout."""
    if w_scale.dim() == 1:
        return w_scale.float()[:, None].expand(N, KB)
    return w_scale.float().repeat_interleave(QBLOCK, 0)[:N]


def fp8_linear_f32(x: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor) -> torch.Tensor:
    """x bf16 [M, K], w fp8 [N, K] row-major, scales -> fp32 [M, N] (before the bf16 rounding)."""
    q, s = act_quant(x)
    M, K = x.shape
    N = w.shape[0]
    KB = K // QBLOCK
    d = block_dots(q, w)                                           # [M, N, KB]
    terms = d * s[:, None, :] * scale_rows(w_scale, N, KB)[None]
    acc = torch.zeros(M, N, dtype=torch.float32, device=x.device)
    for kb in range(KB):                                           # in K order, like the kernels
        acc = acc + terms[..., kb]
    return acc


def fp8_linear(x: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor) -> torch.Tensor:
    return fp8_linear_f32(x, w, w_scale).to(torch.bfloat16)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * xf.to(x.dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def norm_rope(x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, eps: float):
    """Per-head RMSNorm then RoPE; x [heads, 128] bf16, cos/sin [128] bf16."""
    x = rms_norm(x, w, eps)
    return (x * cos) + (rotate_half(x) * sin)


def attention_f32(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float) -> torch.Tensor:
    """GQA decode attention in fp32 (probabilities kept in fp32). q [32, 128], K/V [8, ctx, 128] -> [32*128] bf16."""
    nq, hd = q.shape
    nkv = K.shape[0]
    qf = q.float().view(nkv, nq // nkv, hd)
    s = torch.einsum("ghd,gjd->ghj", qf, K.float()) * scale
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("ghj,gjd->ghd", p, V.float())
    return o.reshape(nq * hd).to(torch.bfloat16)


def quant_kv_rows(x: torch.Tensor):
    """The FP8 KV cache's row format (this engine's extension; the reference keeps bf16 rows): bf16 [..., 128]
    -> (e4m3 [..., 128], fp32 [...]) with s = amax / 448, q = e4m3(x / s) round to nearest even, saturating,
    s = 0 -> 0. IEEE division here; the kernels use div.full, so a quotient on a tie may round one step apart."""
    xf = x.float()
    s = xf.abs().amax(-1) / FP8_MAX
    safe = torch.where(s > 0, s, torch.ones_like(s))
    q = torch.where(s[..., None] > 0, xf / safe[..., None], torch.zeros_like(xf))
    return q.clamp(-FP8_MAX, FP8_MAX).to(FP8), s


def attention_fp8kv_f32(q: torch.Tensor, K8: torch.Tensor, ks: torch.Tensor, V8: torch.Tensor, vs: torch.Tensor,
                        scale: float) -> torch.Tensor:
    """GQA decode attention over an FP8 KV cache in fp32: q [32, 128] (bf16 values), K8/V8 e4m3 [8, ctx, 128],
    ks/vs fp32 [8, ctx]. Scores (q . k8_j) * ks_j * scale, softmax, sum_j (p_j * vs_j) * v8_j -> bf16 [32*128]."""
    nq, hd = q.shape
    nkv = K8.shape[0]
    qf = q.float().view(nkv, nq // nkv, hd)
    s = torch.einsum("ghd,gjd->ghj", qf, K8.float()) * ks.float()[:, None, :] * scale
    p = torch.softmax(s, dim=-1) * vs.float()[:, None, :]
    o = torch.einsum("ghj,gjd->ghd", p, V8.float())
    return o.reshape(nq * hd).to(torch.bfloat16)


def attention_sdpa(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float) -> torch.Tensor:
    """The reference forward's attention (Q/model.py:271-273) for one query token."""
    nq, hd = q.shape
    a = F.scaled_dot_product_attention(q.view(1, nq, 1, hd), K[None], V[None], is_causal=False,
                                       scale=scale, enable_gqa=True)
    return a[0].transpose(0, 1).reshape(nq * hd)


class LayerW:
    """Row-major weights of one layer for the oracle (fp8 matrices + fp32 scales + bf16 norms)."""

    def __init__(self, ln1, ln2, q_norm, k_norm, w_qkv, s_qkv, w_o, s_o, w_gu, s_gu, w_d, s_d):
        self.ln1, self.ln2, self.q_norm, self.k_norm = ln1, ln2, q_norm, k_norm
        self.w_qkv, self.s_qkv, self.w_o, self.s_o = w_qkv, s_qkv, w_o, s_o
        self.w_gu, self.s_gu, self.w_d, self.s_d = w_gu, s_gu, w_d, s_d


def decode_layer(h: torch.Tensor, L: LayerW, k_cache: torch.Tensor, v_cache: torch.Tensor, pos: int,
                 cos: torch.Tensor, sin: torch.Tensor, eps: float, n_heads: int = 32, n_kv: int = 8,
                 head_dim: int = 128, attn_impl: str = "f32", trace: dict | None = None) -> torch.Tensor:
    """One token through one layer. h bf16 [H]; k_cache/v_cache bf16 [n_kv, max_seq, 128] are written
    at `pos` in place. Returns the layer output (residual stream) bf16 [H]."""
    hd = head_dim
    x = rms_norm(h[None], L.ln1, eps)
    qkv = fp8_linear(x, L.w_qkv, L.s_qkv)[0]
    q, k, v = qkv.split([n_heads * hd, n_kv * hd, n_kv * hd])
    c, s = cos[pos], sin[pos]
    q = norm_rope(q.view(n_heads, hd), L.q_norm, c, s, eps)
    k = norm_rope(k.view(n_kv, hd), L.k_norm, c, s, eps)
    k_cache[:, pos] = k
    v_cache[:, pos] = v.view(n_kv, hd)
    K, V = k_cache[:, : pos + 1], v_cache[:, : pos + 1]
    scale = hd ** -0.5
    attn = attention_f32(q, K, V, scale) if attn_impl == "f32" else attention_sdpa(q, K, V, scale)
    h = h + fp8_linear(attn[None].contiguous(), L.w_o, L.s_o)[0]
    x = rms_norm(h[None], L.ln2, eps)
    gu = fp8_linear(x, L.w_gu, L.s_gu)[0]
    I = gu.shape[0] // 2
    g, u = gu.split([I, I])
    a = F.silu(g) * u
    if trace is not None:
        trace.update(qkv=qkv, attn=attn, h_mid=h.clone(), act=a)
    h = h + fp8_linear(a[None].contiguous(), L.w_d, L.s_d)[0]
    return h


def prefill_layer(h: torch.Tensor, L: LayerW, k_cache: torch.Tensor, v_cache: torch.Tensor, start: int,
                  cos: torch.Tensor, sin: torch.Tensor, eps: float, n_heads: int = 32, n_kv: int = 8,
                  head_dim: int = 128, attn_impl: str = "f32") -> torch.Tensor:
    """M positions through one layer (the reference's batched forward). h bf16 [M, H]; k_cache/v_cache bf16
    [n_kv, max_seq, 128] are written at start..start+M-1 in place. Returns the residual stream bf16 [M, H].
    attn_impl "f32": causal attention in fp32; "sdpa": torch SDPA exactly as Q/model.py:271-273 calls it
    (bf16, is_causal for M > 1), which the golden prefill fixture pins."""
    M, hd = h.shape[0], head_dim
    x = rms_norm(h, L.ln1, eps)
    qkv = fp8_linear(x, L.w_qkv, L.s_qkv)
    q, k, v = qkv.split([n_heads * hd, n_kv * hd, n_kv * hd], dim=-1)
    c, s = cos[start:start + M][:, None, :], sin[start:start + M][:, None, :]
    q = norm_rope(q.reshape(M, n_heads, hd), L.q_norm, c, s, eps)
    k = norm_rope(k.reshape(M, n_kv, hd), L.k_norm, c, s, eps)
    k_cache[:, start:start + M] = k.transpose(0, 1)
    v_cache[:, start:start + M] = v.reshape(M, n_kv, hd).transpose(0, 1)
    ctx = start + M
    if attn_impl == "sdpa":
        a = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k_cache[:, :ctx][None], v_cache[:, :ctx][None],
                                           is_causal=(M > 1), scale=hd ** -0.5, enable_gqa=True)
        attn = a[0].transpose(0, 1).reshape(M, n_heads * hd)
    else:
        K = k_cache[:, :ctx].float().repeat_interleave(n_heads // n_kv, 0)     # [n_heads, ctx, 128]
        V = v_cache[:, :ctx].float().repeat_interleave(n_heads // n_kv, 0)
        sc = torch.einsum("mhd,hjd->hmj", q.float(), K) * hd ** -0.5
        pos = start + torch.arange(M, device=h.device)
        sc = sc.masked_fill((torch.arange(ctx, device=h.device)[None, :] > pos[:, None])[None], float("-inf"))
        attn = torch.einsum("hmj,hjd->mhd", torch.softmax(sc, dim=-1), V).reshape(M, n_heads * hd).to(torch.bfloat16)
    h = h + fp8_linear(attn, L.w_o, L.s_o)
    x = rms_norm(h, L.ln2, eps)
    gu = fp8_linear(x, L.w_gu, L.s_gu)
    I = gu.shape[-1] // 2
    g, u = gu.split([I, I], dim=-1)
    a = F.silu(g) * u
    return h + fp8_linear(a.contiguous(), L.w_d, L.s_d)


def lm_head_logits(h: torch.Tensor, norm_w: torch.Tensor, head_w: torch.Tensor, head_scale, eps: float):
    """Final RMSNorm + lm_head. bf16 head (reference format): F.linear like Q/model.py:281.
    FP8 head: the same W8A8 recipe as the other linears."""
    x = rms_norm(h[None], norm_w, eps)
    if head_w.dtype == torch.bfloat16:
        return F.linear(x, head_w)[0]
    return fp8_linear(x, head_w, head_scale)[0]


def argmax_lowest(logits: torch.Tensor) -> int:
    """Greedy argmax over bf16 logits, ties to the lowest index (torch.argmax semantics)."""
    return int(logits.float().argmax())


def decode_step(tok: int, pos: int, embed: torch.Tensor, layers: list, k_cache: torch.Tensor,
                v_cache: torch.Tensor, cos, sin, norm_w, head_w, head_scale, eps: float,
                attn_impl: str = "f32"):
    """Full decode step: embed -> layers -> final norm -> lm_head -> argmax. Caches [L, n_kv, S, 128].
    Returns (next_token, logits bf16 [V])."""
    h = embed[tok].clone()
    for li, L in enumerate(layers):
        h = decode_layer(h, L, k_cache[li], v_cache[li], pos, cos, sin, eps, attn_impl=attn_impl)
    logits = lm_head_logits(h, norm_w, head_w, head_scale, eps)
    return argmax_lowest(logits), logits
