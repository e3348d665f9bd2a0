"""Bit-exactness against the reference's own decode kernels, built for sm_100a and run on the same B200
(oracle/_ref/ref_decode.so from qwen3-8b-fp8_rtx-5090/kernels/decode.cu). Reference-format weights: block-128
scales and a bf16 lm_head. Skipped when the checker library was not built (no reference checkout)."""
import pytest
import torch

import model as M
from oracle import ref_gpu as R

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not R.available(), reason="oracle/_ref not built")]
EPS = 1e-6


def ops():
    from kernels import ops as _ops
    return _ops()


def lin(kind, seed=0):
    N, K = {0: (6144, 4096), 1: (4096, 4096), 2: (24576, 4096), 3: (4096, 12288)}[kind]
    w, s = M.synth_linear(seed, f"ref{kind}", N, K, "block", device="cuda")
    return w, s


@pytest.mark.parametrize("kind", [0, 1, 2, 3])
@pytest.mark.parametrize("inp", ["rnd", "big"])
def test_gemv_bitwise_vs_reference_kernel(kind, inp):
    w, s = lin(kind)
    N, K = w.shape
    g = torch.Generator(device="cuda").manual_seed(kind)
    std = 0.5 if inp == "rnd" else 8.0
    x = (torch.randn(K, generator=g, device="cuda") * std).to(torch.bfloat16)
    norm_w = (1 + 0.1 * torch.randn(K, generator=g, device="cuda")).to(torch.bfloat16) if kind in (0, 2) else None
    resid = torch.randn(N, generator=g, device="cuda").to(torch.bfloat16)
    if kind in (1, 3):
        ref_out, out = resid.clone(), resid.clone()
    else:
        ref_out = torch.empty(N // 2 if kind == 2 else N, dtype=torch.bfloat16, device="cuda")
        out = torch.empty_like(ref_out)
    rk = R.ref_ops()
    rk.set_pdl(False)
    rk.fp8_gemv(kind, R.ref_tile_fp8(w, True), s, x, norm_w, ref_out, N, EPS, R.RefEngine.DEPTH[kind],
                R.RefEngine.WARPS[kind], R.RefEngine.PRE[kind], R.RefEngine.TRIG[kind], 1)
    ops().fp8_gemv(kind, M.pack_fp8(w, pairs=(kind == 2)), s, x, norm_w, out, N, EPS)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16)), \
        f"{(out.view(torch.int16) != ref_out.view(torch.int16)).sum().item()} of {out.numel()} differ"


@pytest.mark.parametrize("pos,chunk", [(0, 64), (63, 64), (64, 64), (777, 64), (1500, 64), (31, 32), (1500, 32),
                                       (127, 128), (1500, 128)])
def test_attention_bitwise_vs_reference_kernel(pos, chunk):
    max_seq = 2048
    g = torch.Generator(device="cuda").manual_seed(pos + chunk)
    kc = torch.randn(8, max_seq, 128, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(8, max_seq, 128, generator=g, device="cuda").to(torch.bfloat16)
    qkv = (torch.randn(6144, generator=g, device="cuda") * 2).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(128, generator=g, device="cuda")).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(128, generator=g, device="cuda")).to(torch.bfloat16)
    cos, sin = M.rope_tables(max_seq, 128, 1e6, "cuda")
    state = torch.tensor([pos, 0], dtype=torch.int32, device="cuda")
    ms = (max_seq + 31) // 32

    def scratch():
        return (torch.zeros(32, ms, 128, device="cuda"), torch.zeros(32, ms, 2, device="cuda"),
                torch.zeros(8, dtype=torch.int32, device="cuda"), torch.empty(4096, dtype=torch.bfloat16, device="cuda"))
    rk = R.ref_ops()
    rk.set_pdl(False)
    kr, vr = kc.clone(), vc.clone()
    op, ml, cnt, ref_out = scratch()
    rk.attention(qkv, qn, kn, cos, sin, state, kr, vr, op, ml, cnt, ref_out, 128 ** -0.5, EPS, 0, chunk)
    km, vm = kc.clone(), vc.clone()
    op2, ml2, cnt2, out = scratch()
    ops().attention(qkv, qn, kn, cos, sin, state, km, vm, op2, ml2, cnt2, out, 128 ** -0.5, EPS, 0, chunk)
    torch.cuda.synchronize()
    assert torch.equal(km, kr) and torch.equal(vm, vr)          # KV append: same slot, same bits
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))
    assert int(cnt2.abs().sum()) == 0


def test_lm_head_bf16_bitwise_vs_reference_kernel():
    V = 151936
    g = torch.Generator(device="cuda").manual_seed(9)
    w = (torch.randn(V, 4096, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    x = (torch.randn(4096, generator=g, device="cuda") * 3).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(4096, generator=g, device="cuda")).to(torch.bfloat16)
    rk = R.ref_ops()
    rk.set_pdl(False)
    lr = torch.empty(V, dtype=torch.bfloat16, device="cuda")
    br = torch.zeros(1, dtype=torch.int64, device="cuda")
    rk.lm_head_argmax(w, x, nw, lr, br, EPS, torch.cuda.get_device_properties(0).multi_processor_count)
    lm = torch.empty_like(lr)
    bm = torch.zeros_like(br)
    ops().lm_head_argmax(w, x, nw, lm, bm, EPS, 0)
    torch.cuda.synchronize()
    assert torch.equal(lm.view(torch.int16), lr.view(torch.int16))
    assert int(bm.item()) == int(br.item())


@pytest.mark.parametrize("fused", [False, True], ids=["ops", "fused"])
def test_greedy_256_identical_to_reference_engine(fused):
    """Full 36-layer model, block-128 scales + bf16 lm_head (the reference's format): 256 greedy tokens from
    the B200 engine (CUDA graph; the op path or the fused one-launch step) == the reference engine's decode
    step run on its own kernels, and the KV caches equal."""
    from generate import Engine
    cfg = M.Config()
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=512, device="cuda", seed=0, scale_mode="block", head_dtype="bf16",
                                   norm_init="random", keep_rowmajor=True)
    layers = []
    for L in m.layers:
        layers.append(dict(ln1=L.ln1, ln2=L.ln2, q_norm=L.q_norm, k_norm=L.k_norm,
                           qkv=(L.rowmajor["qkv"], L.qkv.scale), o_proj=(L.rowmajor["o_proj"], L.o.scale),
                           gate_up=(L.rowmajor["gate_up"], L.gu.scale), down_proj=(L.rowmajor["down_proj"], L.down.scale)))
        L.rowmajor = {}
    ref = R.RefEngine(layers, m.embed, m.norm, m.lm_head, m.cos, m.sin, m.max_seq)
    del layers
    torch.cuda.empty_cache()
    prompt = [int(t) for t in torch.randint(0, cfg.vocab, (16,), generator=torch.Generator().manual_seed(5))]
    ref_tokens = ref.generate(prompt, 256)
    ref_k = ref.k_cache.clone()
    del ref
    torch.cuda.empty_cache()
    eng = Engine(m, fused=fused)
    tokens = eng.generate(prompt, 256)
    assert tokens == ref_tokens, next(i for i, (a, b) in enumerate(zip(tokens, ref_tokens)) if a != b)
    assert torch.equal(m.k_cache[:, 0, :, : len(prompt) + 255], ref_k[:, :, : len(prompt) + 255])
