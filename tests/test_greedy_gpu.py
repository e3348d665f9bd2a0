"""256 greedy tokens of the benchmarked configuration against a torch restatement run on the GPU.

The configuration `bench.py` measures: all 36 layers, per-output-channel FP8 scales, the FP8 lm_head, the
fused persistent step (decode_step_kernel) replayed from one CUDA graph, a KV cache pre-filled with N(0,1)
to position 3840 and 256 greedy steps (contexts 3840..4095). The check (the parity contract's greedy row
for this mode) runs the reference's decode math restated in torch ops on the GPU (oracle/qwen3_ref.py's
arithmetic: per-128 activation quant, fp32 block dots times the activation and weight scales summed over
K blocks, bf16 rounding of every linear, fp32 attention with fp32 probabilities), teacher-forced on the
engine's own tokens so one near-tie cannot derail the rest of the sequence. Every step whose restated
top-2 logit gap is clearly above the measured logit difference must pick the same token, and at least
250 of the 256 steps must agree overall.
"""
import pytest
import torch

import model as M
from oracle import qwen3_ref as O

pytestmark = pytest.mark.gpu

START, STEPS = 3840, 256


class TorchDecode:
    """The decode step in torch ops on the GPU, from the row-major fp8 weights (fp32 copies cached per layer,
    [K/128, 128, N], so a linear is one batched matmul for the block dots)."""

    def __init__(self, m: M.Qwen3FP8Decode):
        self.m = m
        self.cfg = m.cfg
        self.layers = []
        for L in m.layers:
            d = {}
            for name, scale in (("qkv", L.qkv.scale), ("o_proj", L.o.scale), ("gate_up", L.gu.scale),
                                ("down_proj", L.down.scale)):
                w = L.rowmajor[name]
                N, K = w.shape
                d[name] = (w.float().view(N, K // 128, 128).permute(1, 2, 0).contiguous(), scale.float())
            d["norms"] = (L.ln1, L.ln2, L.q_norm, L.k_norm)
            self.layers.append(d)
        w = m.lm_head_rowmajor
        self.head = (w.float().view(w.shape[0], 32, 128).permute(1, 2, 0).contiguous(), m.lm_head.scale.float())
        self.k_cache = m.k_cache[:, 0].clone()
        self.v_cache = m.v_cache[:, 0].clone()

    @staticmethod
    def linear(x, wf_scale):
        wf, sw = wf_scale
        q, sx = O.act_quant(x[None])                          # [1, K] fp8, [1, K/128]
        KB = wf.shape[0]
        d = torch.bmm(q.float().view(KB, 1, 128), wf)[:, 0]   # [KB, N] fp32 block dots
        return ((d * sx[0][:, None]) * sw[None]).sum(0).to(torch.bfloat16)

    def step(self, tok: int, pos: int):
        cfg, eps = self.cfg, self.cfg.eps
        hd, nq, nkv = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
        cos, sin = self.m.cos[pos], self.m.sin[pos]
        h = self.m.embed[tok].clone()
        for li, L in enumerate(self.layers):
            ln1, ln2, qn, kn = L["norms"]
            qkv = self.linear(O.rms_norm(h[None], ln1, eps)[0], L["qkv"])
            q, k, v = qkv.split([nq * hd, nkv * hd, nkv * hd])
            q = O.norm_rope(q.view(nq, hd), qn, cos, sin, eps)
            k = O.norm_rope(k.view(nkv, hd), kn, cos, sin, eps)
            self.k_cache[li, :, pos] = k
            self.v_cache[li, :, pos] = v.view(nkv, hd)
            attn = O.attention_f32(q, self.k_cache[li, :, : pos + 1], self.v_cache[li, :, : pos + 1], hd ** -0.5)
            h = h + self.linear(attn, L["o_proj"])
            gu = self.linear(O.rms_norm(h[None], ln2, eps)[0], L["gate_up"])
            g, u = gu.split([cfg.inter, cfg.inter])
            h = h + self.linear(torch.nn.functional.silu(g) * u, L["down_proj"])
        return self.linear(O.rms_norm(h[None], self.m.norm, eps)[0], self.head)


def test_fused_step_256_greedy_tokens_vs_torch_restatement():
    from generate import Engine
    cfg = M.Config()
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=4096, device="cuda", seed=0, scale_mode="channel", head_dtype="fp8",
                                   norm_init="ones", keep_rowmajor=True)
    m.fill_cache_random(START, seed=1234)
    ref = TorchDecode(m)                      # copies the pre-filled caches before the engine writes them
    eng = Engine(m, fused=True)
    first = 1
    eng.token.fill_(first)
    eng.state.copy_(torch.tensor([START, 0], dtype=torch.int32))
    eng.capture()
    logits = []
    for _ in range(STEPS):
        eng.graph.replay()
        logits.append(eng.logits.clone())
    torch.cuda.synchronize()
    eng.check()
    toks = eng.out_tokens[:STEPS].tolist()
    got_logits = torch.stack(logits).float()

    agree, clear_mismatch, first_div = 0, [], None
    gaps, errs = [], []
    with torch.no_grad():
        cur = first
        for i in range(STEPS):
            lg = ref.step(cur, START + i).float()
            top2 = torch.topk(lg, 2).values
            gap = float(top2[0] - top2[1])
            err = float((got_logits[i] - lg).abs().max())
            ref_tok = int(lg.argmax())
            gaps.append(gap)
            errs.append(err)
            if ref_tok == toks[i]:
                agree += 1
            else:
                first_div = i if first_div is None else first_div
                if gap > 2 * err:
                    clear_mismatch.append((i, toks[i], ref_tok, gap, err))
            cur = toks[i]                    # teacher-forced on the engine's own tokens
    msg = (f"{agree}/{STEPS} tokens agree; first divergence at step {first_div}; max logit difference "
           f"{max(errs):.4f}; median top-2 gap {sorted(gaps)[STEPS // 2]:.4f}; clear mismatches {clear_mismatch[:5]}")
    print(msg)
    assert not clear_mismatch, msg
    assert agree >= 250, msg
