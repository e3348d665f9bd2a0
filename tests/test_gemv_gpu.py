"""FP8 GEMV parity on the B200: every kind and both scale layouts against the CPU oracle, and bit-identity
across launch shapes (the split-K fold must not change a bit). Pattern of the reference's per-op checks
(qwen3-8b-fp8_rtx-5090/test_kernels.py:96-133)."""
import pytest
import torch
import torch.nn.functional as F

import model as M
from oracle import qwen3_ref as O

pytestmark = pytest.mark.gpu
EPS = 1e-6

SHAPES = {  # kind: (N, K)
    0: (6144, 4096),
    1: (4096, 4096),
    2: (24576, 4096),
    3: (4096, 12288),
}


def ops():
    from kernels import ops as _ops
    return _ops()


def rel_l2(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def same_frac(a, b):
    return (a.view(torch.int16) == b.view(torch.int16)).float().mean().item()


_cache = {}


def weights(kind, scale_mode, seed=0):
    key = (kind, scale_mode, seed)
    if key not in _cache:
        N, K = SHAPES[kind]
        w, s = M.synth_linear(seed, f"gemv{kind}", N, K, scale_mode)
        _cache[key] = (w, s, M.pack_fp8(w, pairs=(kind == 2)))
    return _cache[key]


def oracle(kind, w, s, x, norm_w, resid):
    if kind == 0:
        return O.fp8_linear(O.rms_norm(x[None], norm_w, EPS), w, s)[0]
    if kind in (1, 3):
        return resid + O.fp8_linear(x[None], w, s)[0]
    gu = O.fp8_linear(O.rms_norm(x[None], norm_w, EPS), w, s)[0]
    g, u = gu.split(gu.shape[0] // 2)
    return F.silu(g) * u


def run(kind, packed, s, x, norm_w, resid, N, **shape):
    k = ops()
    dev = "cuda"
    if kind in (1, 3):
        out = resid.to(dev).clone()
    else:
        out = torch.empty(N // 2 if kind == 2 else N, dtype=torch.bfloat16, device=dev)
    k.fp8_gemv(kind, packed.to(dev), s.to(dev), x.to(dev), None if norm_w is None else norm_w.to(dev), out, N,
               EPS, shape.get("depth", 0), shape.get("warps", 0), shape.get("pre", -1), -1, 1,
               stage_tiles=shape.get("stage_tiles", 0), ctas_per_sm=shape.get("ctas", 0))
    torch.cuda.synchronize()
    return out.cpu()


def inputs(kind, seed=1):
    N, K = SHAPES[kind]
    x = M.randn((K,), seed, f"x{kind}").to(torch.bfloat16)
    norm_w = M.synth_norm(seed, f"n{kind}", K, "random") if kind in (0, 2) else None
    resid = M.randn((N,), seed, f"r{kind}").to(torch.bfloat16) if kind in (1, 3) else None
    return x, norm_w, resid


@pytest.mark.parametrize("scale_mode", ["channel", "block"])
@pytest.mark.parametrize("kind", [0, 1, 2, 3])
def test_gemv_matches_oracle(kind, scale_mode):
    N, K = SHAPES[kind]
    w, s, packed = weights(kind, scale_mode)
    x, norm_w, resid = inputs(kind)
    ref = oracle(kind, w, s, x, norm_w, resid)
    got = run(kind, packed, s, x, norm_w, resid, N)
    # The oracle quantizes activations with IEEE division, the kernels (like the reference) with
    # div.full.f32, so x/s ties can round to the neighbouring e4m3 value; tensor-core block dots also
    # round differently from the oracle's fp32 sums. 1e-2 rel-L2 is the bar; bit-exactness is checked
    # against the reference's own kernel in test_ref_gpu.py.
    assert rel_l2(got, ref) < 1e-2, (rel_l2(got, ref), same_frac(got, ref))


@pytest.mark.parametrize("kind", [0, 1, 2, 3])
def test_gemv_bit_identical_across_launch_shapes(kind):
    """Different warp counts / ring shapes split K at different places; the fold replays the in-order
    accumulation, so every output bit is the same."""
    N, K = SHAPES[kind]
    w, s, packed = weights(kind, "channel")
    x, norm_w, resid = inputs(kind)
    base = run(kind, packed, s, x, norm_w, resid, N)
    for shape in (dict(warps=4, depth=2, stage_tiles=1, pre=0), dict(warps=16, depth=3, stage_tiles=1, pre=1),
                  dict(warps=8, depth=4, stage_tiles=1, pre=4, ctas=2), dict(warps=5, depth=1, stage_tiles=7)):
        got = run(kind, packed, s, x, norm_w, resid, N, **shape)
        assert torch.equal(got.view(torch.int16), base.view(torch.int16)), shape


def test_gemv_zero_group_and_repeat():
    """An all-zero 128-group quantizes with scale 0 (output 0 contribution), and repeated launches give the
    same bits (counters are left at zero by every launch)."""
    N, K = SHAPES[1]
    w, s, packed = weights(1, "channel")
    x, _, resid = inputs(1)
    x = x.clone()
    x[256:512] = 0
    ref = oracle(1, w, s, x, None, resid)
    a = run(1, packed, s, x, None, resid, N)
    b = run(1, packed, s, x, None, resid, N)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert rel_l2(a, ref) < 1e-2


@pytest.mark.parametrize("head", ["fp8", "bf16"])
def test_lm_head_argmax(head):
    V, H = 151936, 4096
    k = ops()
    x = (M.randn((H,), 5, "hx") * 3).to(torch.bfloat16)
    norm_w = M.synth_norm(5, "hn", H, "random")
    if head == "fp8":
        w, s = M.quantize_fp8(M.randn((V, H), 5, "head", std=0.02), "channel")
        ref = O.lm_head_logits(x, norm_w, w, s, EPS)
        wdev, sdev = M.pack_fp8(w).cuda(), s.cuda()
    else:
        w = M.randn((V, H), 5, "head", std=0.02).to(torch.bfloat16)
        ref = O.lm_head_logits(x, norm_w, w, None, EPS)
        wdev, sdev = w.cuda(), None
    logits = torch.empty(V, dtype=torch.bfloat16, device="cuda")
    best = torch.zeros(1, dtype=torch.int64, device="cuda")
    k.lm_head_argmax(wdev, x.cuda(), norm_w.cuda(), logits, best, EPS, 0, w_scale=sdev)
    torch.cuda.synchronize()
    got = logits.cpu()
    assert rel_l2(got, ref) < 1e-2
    if head == "bf16":                                    # no activation quantization: plain fp32 dots
        assert same_frac(got, ref) > 0.97
    tok = 0xFFFFFFFF - (int(best.item()) & 0xFFFFFFFF)
    assert tok == int(got.float().argmax())              # fused argmax == argmax of its own logits
    top2 = ref.float().topk(2).values
    err = (got.float() - ref.float()).abs().max().item()
    if (top2[0] - top2[1]).item() > 2 * err:              # a winner clearer than the logit error must match
        assert tok == O.argmax_lowest(ref)


def test_lm_head_argmax_ties_pick_lowest_index():
    """Identical rows give identical logits: the argmax must pick the lowest index (torch.argmax rule)."""
    V, H = 4096, 4096
    k = ops()
    w = torch.zeros(V, H, dtype=torch.bfloat16)
    w[3000] = 0.01
    w[1234] = 0.01
    w[777] = 0.009
    x = torch.ones(H, dtype=torch.bfloat16)
    logits = torch.empty(V, dtype=torch.bfloat16, device="cuda")
    best = torch.zeros(1, dtype=torch.int64, device="cuda")
    k.lm_head_argmax(w.cuda(), x.cuda(), torch.ones(H, dtype=torch.bfloat16, device="cuda"), logits, best, EPS, 0)
    torch.cuda.synchronize()
    assert 0xFFFFFFFF - (int(best.item()) & 0xFFFFFFFF) == 1234
