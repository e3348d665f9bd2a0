"""Decode attention over an FP8 KV cache (qk_attention_fp8kv; no reference counterpart) on the GPU.

The contract (include/qwen3_b200.h, oracle.quant_kv_rows / attention_fp8kv_f32):
* the appended K and V rows are the bf16 rows the bf16 cache would hold (the same K row, bit for bit, as the
  bf16 attention op writes), quantized to e4m3 with one fp32 scale per row: the scale equals amax/448 to within
  the division's 2 ulp, each byte equals the IEEE restatement's or lies one e4m3 step from it (a quotient on a
  rounding tie), and no other cache byte or scale changes;
* the output matches the fp32 restatement over the kernel's own cache within 5e-3 rel-L2 (the bf16 attention
  op's bar against fp32), at contexts across the 64-key split and 128-key block boundaries, ragged batches
  included, for both split sizes (128 keys, and 512 keys streamed as 4 double-buffered blocks);
* against the bf16 cache the quantization costs a few percent of the output (measured and bounded at 5e-2);
* a 2-layer model with an FP8 cache decodes through the op path; its first token's logits stay within 0.2
  rel-L2 of the bf16-cache model's (0.127 measured: every attention output moves by a few percent and the W8A8
  layers after it amplify that, as any one-ulp change does), and the token agrees unless the top-2 gap is a
  near-tie. The fused step and the chunked prefill refuse an FP8 cache.
"""
import pytest
import torch

import model as M
from oracle import qwen3_ref as O

pytestmark = pytest.mark.gpu
EPS = 1e-6
SCALE = 128 ** -0.5
FP8 = torch.float8_e4m3fn


def rel(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    return ((a - b).norm() / b.norm()).item()


def setup(lengths, max_seq, seed):
    batch = len(lengths)
    g = torch.Generator(device="cuda").manual_seed(seed)
    kb = torch.randn(batch, 8, max_seq, 128, generator=g, device="cuda").to(torch.bfloat16)
    vb = torch.randn(batch, 8, max_seq, 128, generator=g, device="cuda").to(torch.bfloat16)
    k8, ks = O.quant_kv_rows(kb)
    v8, vs = O.quant_kv_rows(vb)
    qkv = (torch.randn(batch, 6144, generator=g, device="cuda") * 2).to(torch.bfloat16)
    qn = M.synth_norm(seed, "kv8.qn", 128, "random", device="cuda")
    kn = M.synth_norm(seed, "kv8.kn", 128, "random", device="cuda")
    cos, sin = M.rope_tables(max_seq, 128, 1e6, "cuda")
    state = torch.tensor([[p, 0] for p in lengths], dtype=torch.int32, device="cuda").view(-1)
    return dict(kb=kb, vb=vb, k8=k8.view(torch.uint8), ks=ks, v8=v8.view(torch.uint8), vs=vs, qkv=qkv, qn=qn,
                kn=kn, cos=cos, sin=sin, state=state, batch=batch, max_seq=max_seq)


def parts(d):
    splits = (d["max_seq"] + 63) // 64
    return (torch.zeros(d["batch"], 32, splits, 128, device="cuda"),
            torch.zeros(d["batch"], 32, splits, 2, device="cuda"))


def run_fp8(d):
    from kernels import ops
    k8, ks, v8, vs = d["k8"].clone(), d["ks"].clone(), d["v8"].clone(), d["vs"].clone()
    o_part, ml = parts(d)
    out = torch.empty(d["batch"], 4096, dtype=torch.bfloat16, device="cuda")
    ops().attention_fp8kv(d["qkv"], d["qn"], d["kn"], d["cos"], d["sin"], d["state"], k8, ks, v8, vs, o_part, ml,
                          out, SCALE, EPS, batch=d["batch"])
    torch.cuda.synchronize()
    assert ops().device_error() == 0
    return out, k8, ks, v8, vs


def run_bf16(d):
    from kernels import ops
    kb, vb = d["kb"].clone(), d["vb"].clone()
    o_part, ml = parts(d)
    cnt = torch.zeros(d["batch"], 8, dtype=torch.int32, device="cuda")
    out = torch.empty(d["batch"], 4096, dtype=torch.bfloat16, device="cuda")
    ops().attention(d["qkv"], d["qn"], d["kn"], d["cos"], d["sin"], d["state"], kb, vb, o_part, ml, cnt, out, SCALE,
                    EPS, 0, 64, batch=d["batch"])
    torch.cuda.synchronize()
    return out, kb, vb


def e4m3_close(a8, b8):
    """Bytes equal, or their values one e4m3 step apart."""
    a, b = a8.view(FP8).float(), b8.view(FP8).float()
    return ((a - b).abs() <= 0.125 * torch.maximum(a.abs(), b.abs()) + 2.0 ** -9).all().item()


@pytest.mark.parametrize("lengths,max_seq", [([0], 4096), ([63], 4096), ([64, 127], 4096), ([128, 1000], 4096),
                                             ([4095, 2049], 4096), ([16383, 700, 5000], 16384)])
def test_fp8kv_append_and_attention(lengths, max_seq):
    """max_seq 4096: one 128-key block per split; 16384: 512-key splits of 4 double-buffered blocks."""
    d = setup(lengths, max_seq, seed=sum(lengths) + len(lengths))
    out8, k8, ks, v8, vs = run_fp8(d)
    out16, kb, vb = run_bf16(d)
    for b, pos in enumerate(lengths):
        # the appended rows: the bf16 op's rows, quantized per the contract
        for new8, news, bfrow, old8, olds in ((k8, ks, kb, d["k8"], d["ks"]), (v8, vs, vb, d["v8"], d["vs"])):
            want8, wants = O.quant_kv_rows(bfrow[b, :, pos])
            got_s = news[b, :, pos]
            assert ((got_s - wants).abs() <= 2.0 ** -21 * wants.abs()).all(), (got_s, wants)
            same = (new8[b, :, pos] == want8.view(torch.uint8)).float().mean().item()
            assert same > 0.99 and e4m3_close(new8[b, :, pos], want8.view(torch.uint8)), same
            # every other row and scale unchanged
            keep = torch.ones(max_seq, dtype=torch.bool, device="cuda")
            keep[pos] = False
            assert torch.equal(new8[b][:, keep], old8[b][:, keep]) and torch.equal(news[b][:, keep], olds[b][:, keep])
        # the output against the fp32 restatement over the kernel's own cache
        q = O.norm_rope(d["qkv"][b, :4096].view(32, 128), d["qn"], d["cos"][pos], d["sin"][pos], EPS)
        ref = O.attention_fp8kv_f32(q, k8[b, :, :pos + 1].view(FP8), ks[b, :, :pos + 1], v8[b, :, :pos + 1].view(FP8),
                                    vs[b, :, :pos + 1], SCALE)
        e = rel(out8[b], ref)
        assert e < 5e-3, (pos, e)
        # against the bf16 cache: the quantization's cost
        e16 = rel(out8[b], out16[b])
        assert e16 < 5e-2, (pos, e16)


def test_fp8kv_engine_decodes_and_refuses_the_bf16_only_paths():
    from generate import Engine
    cfg = M.Config(layers=2, vocab=4096)
    ids = [(i * 131 + 7) % cfg.vocab for i in range(20)]
    logits = {}
    toks = {}
    for kv in ("bf16", "fp8"):
        m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=256, seed=9, norm_init="random")
        if kv == "fp8":
            m.set_kv_dtype("fp8")
            with pytest.raises(ValueError, match="FP8 KV"):
                Engine(m, fused=True)
        eng = Engine(m)
        first = int(eng.prefill(ids))
        torch.cuda.synchronize()
        logits[kv] = eng.logits.float().clone()
        eng.step(8)
        toks[kv] = [first] + eng.out_tokens[:8].tolist()
        eng.check()
        if kv == "fp8":
            assert m.k_cache.dtype == torch.uint8 and bool((m.k_scale[:, 0, :, :len(ids) + 8] > 0).all())
            assert not bool(m.k_scale[:, 0, :, len(ids) + 8:].any())
            with pytest.raises(ValueError, match="bf16 KV"):
                eng.prefill_chunked(ids)
    e = rel(logits["fp8"], logits["bf16"])
    assert e < 0.2, e
    la = logits["bf16"]
    top2 = la.topk(2).values
    if toks["fp8"][0] != toks["bf16"][0]:
        assert float(top2[0] - top2[1]) <= 2 * float((logits["fp8"] - la).abs().max())
