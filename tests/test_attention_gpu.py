"""Fused q/k norm + RoPE + KV append + split-KV attention on the B200 vs the CPU oracle. Same cases as the
reference's kernel check (qwen3-8b-fp8_rtx-5090/test_kernels.py:135-173): K/V rows written at `pos`, no other
cache byte touched, attention within 5e-3 rel-L2 of fp32, split counters back at zero."""
import pytest
import torch

import model as M
from oracle import qwen3_ref as O

pytestmark = pytest.mark.gpu
EPS = 1e-6


def ulp_dist(a, b):
    def line(x):
        i = x.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -(i + 32768), i)
    return (line(a) - line(b)).abs()


def setup(max_seq, batch, seed):
    g = torch.Generator().manual_seed(seed)
    kc = torch.randn(batch, 8, max_seq, 128, generator=g).to(torch.bfloat16)
    vc = torch.randn(batch, 8, max_seq, 128, generator=g).to(torch.bfloat16)
    qkv = (torch.randn(batch, 6144, generator=g) * 2).to(torch.bfloat16)
    qn = M.synth_norm(seed, "qn", 128, "random")
    kn = M.synth_norm(seed, "kn", 128, "random")
    return kc, vc, qkv, qn, kn


def run_attention(kc, vc, qkv, qn, kn, positions, chunk, max_splits=None):
    from kernels import ops
    k = ops()
    batch, _, max_seq, _ = kc.shape
    dev = "cuda"
    cos, sin = M.rope_tables(max_seq, 128, 1e6, dev)
    max_splits = max_splits or (max_seq + 31) // 32
    o_part = torch.zeros(batch, 32, max_splits, 128, device=dev)
    ml_part = torch.zeros(batch, 32, max_splits, 2, device=dev)
    counters = torch.zeros(batch, 8, dtype=torch.int32, device=dev)
    state = torch.tensor([[p, 0] for p in positions], dtype=torch.int32, device=dev).view(-1)
    kd, vd = kc.to(dev), vc.to(dev)
    out = torch.empty(batch, 4096, dtype=torch.bfloat16, device=dev)
    k.attention(qkv.to(dev), qn.to(dev), kn.to(dev), cos, sin, state, kd, vd, o_part, ml_part, counters, out,
                128 ** -0.5, EPS, 0, chunk, batch=batch)
    torch.cuda.synchronize()
    return kd.cpu(), vd.cpu(), out.cpu(), counters.cpu(), cos.cpu(), sin.cpu()


CASES = [(0, 64), (63, 64), (64, 64), (777, 64), (1500, 64), (31, 32), (1500, 32), (127, 128), (1500, 128),
         (2047, 64)]


@pytest.mark.parametrize("pos,chunk", CASES)
def test_attention_and_kv_append(pos, chunk):
    kc, vc, qkv, qn, kn = setup(2048, 1, seed=pos * 7 + chunk)
    kd, vd, out, counters, cos, sin = run_attention(kc, vc, qkv, qn, kn, [pos], chunk)
    q, kk, v = qkv[0].split([4096, 1024, 1024])
    qr = O.norm_rope(q.view(32, 128), qn, cos[pos], sin[pos], EPS)
    kr = O.norm_rope(kk.view(8, 128), kn, cos[pos], sin[pos], EPS)
    # the V row is a copy; the K row follows the same per-step bf16 rounding (rsqrt may differ by an ulp)
    assert torch.equal(vd[0, :, pos], v.view(8, 128))
    assert int(ulp_dist(kd[0, :, pos], kr).max()) <= 1
    # nothing else in the cache changed
    kref, vref = kc.clone(), vc.clone()
    kref[0, :, pos] = kd[0, :, pos]
    vref[0, :, pos] = vd[0, :, pos]
    assert torch.equal(kd, kref) and torch.equal(vd, vref)
    # attention vs fp32 over the cache as written
    ref = O.attention_f32(qr, kd[0, :, : pos + 1], vd[0, :, : pos + 1], 128 ** -0.5)
    e = ((out[0].float() - ref.float()).norm() / ref.float().norm()).item()
    assert e < 5e-3, e
    assert int(counters.abs().sum()) == 0


def test_attention_batch_ragged():
    """Batch of 8 sequences with different lengths in one launch (each writes only its own slot)."""
    positions = [5, 1023, 64, 700, 1, 999, 512, 130]
    kc, vc, qkv, qn, kn = setup(1024, 8, seed=11)
    kd, vd, out, counters, cos, sin = run_attention(kc, vc, qkv, qn, kn, positions, 64)
    for b, pos in enumerate(positions):
        q, kk, v = qkv[b].split([4096, 1024, 1024])
        qr = O.norm_rope(q.view(32, 128), qn, cos[pos], sin[pos], EPS)
        assert torch.equal(vd[b, :, pos], v.view(8, 128))
        kref = kc[b].clone()
        kref[:, pos] = kd[b, :, pos]
        assert torch.equal(kd[b], kref)
        ref = O.attention_f32(qr, kd[b, :, : pos + 1], vd[b, :, : pos + 1], 128 ** -0.5)
        e = ((out[b].float() - ref.float()).norm() / ref.float().norm()).item()
        assert e < 5e-3, (b, e)
    assert int(counters.abs().sum()) == 0


def test_attention_long_context_32k():
    """32k context (beyond the reference's 16k limit): compared with an fp32 torch computation on the GPU."""
    max_seq, pos = 32768, 32767
    g = torch.Generator(device="cuda").manual_seed(3)
    kc = torch.randn(1, 8, max_seq, 128, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(1, 8, max_seq, 128, generator=g, device="cuda").to(torch.bfloat16)
    qkv = (torch.randn(1, 6144, generator=g, device="cuda") * 2).to(torch.bfloat16)
    qn = torch.ones(128, dtype=torch.bfloat16, device="cuda")
    from kernels import ops
    k = ops()
    cos, sin = M.rope_tables(max_seq, 128, 1e6, "cuda")
    max_splits = max_seq // 64
    o_part = torch.zeros(1, 32, max_splits, 128, device="cuda")
    ml_part = torch.zeros(1, 32, max_splits, 2, device="cuda")
    counters = torch.zeros(1, 8, dtype=torch.int32, device="cuda")
    state = torch.tensor([pos, 0], dtype=torch.int32, device="cuda")
    out = torch.empty(1, 4096, dtype=torch.bfloat16, device="cuda")
    k.attention(qkv, qn, qn, cos, sin, state, kc, vc, o_part, ml_part, counters, out, 128 ** -0.5, EPS, 0, 64, batch=1)
    torch.cuda.synchronize()
    q = qkv[0, :4096].view(32, 128).cpu()
    qr = O.norm_rope(q, qn.cpu(), cos[pos].cpu(), sin[pos].cpu(), EPS).cuda().float().view(8, 4, 128)
    s = torch.einsum("ghd,gjd->ghj", qr, kc[0, :, : pos + 1].float()) * 128 ** -0.5
    ref = torch.einsum("ghj,gjd->ghd", torch.softmax(s, -1), vc[0, :, : pos + 1].float()).reshape(-1)
    e = ((out[0].float() - ref).norm() / ref.norm()).item()
    assert e < 5e-3, e
    assert int(counters.abs().sum()) == 0


def sweep_lengths(L: int, batch: int, seed: int = 0):
    """Benchmark configuration 4's sequence lengths: batch 1 holds L keys; batch 8 holds lengths ~ U[L/2, L], seeded.
    The new token goes at position len (so the attention covers len + 1 keys)."""
    if batch == 1:
        return [L]
    g = torch.Generator().manual_seed(seed + L)
    return [int(x) for x in torch.randint(L // 2, L + 1, (batch,), generator=g)]


@pytest.mark.parametrize("L", [1024, 4096, 8192, 16384, 32768])
@pytest.mark.parametrize("batch", [1, 8])
def test_attention_sweep_point(L, batch):
    """Every point of the attention sweep (bench.py --sweep attention): the drop-in op on the GPU against fp32
    attention in torch on the GPU from the same normalised, rotated q (the oracle's norm_rope), with the new
    K/V rows appended at each sequence's position: within 5e-3 rel-L2 (the reference's bar), V rows exact."""
    from kernels import ops
    lengths = sweep_lengths(L, batch)
    max_seq = L + 1
    g = torch.Generator(device="cuda").manual_seed(L * 10 + batch)
    kc = torch.randn(batch, 8, max_seq, 128, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(batch, 8, max_seq, 128, generator=g, device="cuda").to(torch.bfloat16)
    qkv = (torch.randn(batch, 6144, generator=g, device="cuda") * 2).to(torch.bfloat16)
    qn = torch.ones(128, dtype=torch.bfloat16, device="cuda")
    k = ops()
    cos, sin = M.rope_tables(max_seq, 128, 1e6, "cuda")
    max_splits = (max_seq + 63) // 64
    o_part = torch.zeros(batch, 32, max_splits, 128, device="cuda")
    ml_part = torch.zeros(batch, 32, max_splits, 2, device="cuda")
    counters = torch.zeros(batch, 8, dtype=torch.int32, device="cuda")
    state = torch.tensor([[p, 0] for p in lengths], dtype=torch.int32, device="cuda").view(-1)
    out = torch.empty(batch, 4096, dtype=torch.bfloat16, device="cuda")
    k.attention(qkv, qn, qn, cos, sin, state, kc, vc, o_part, ml_part, counters, out, 128 ** -0.5, EPS, 0, 64,
                batch=batch)
    torch.cuda.synchronize()
    assert k.device_error() == 0
    for b, pos in enumerate(lengths):
        q, _, v = qkv[b].split([4096, 1024, 1024])
        assert torch.equal(vc[b, :, pos], v.view(8, 128))
        qr = O.norm_rope(q.view(32, 128), qn, cos[pos], sin[pos], EPS).float().view(8, 4, 128)
        s = torch.einsum("ghd,gjd->ghj", qr, kc[b, :, : pos + 1].float()) * 128 ** -0.5
        ref = torch.einsum("ghj,gjd->ghd", torch.softmax(s, -1), vc[b, :, : pos + 1].float()).reshape(-1)
        e = ((out[b].float() - ref).norm() / ref.norm()).item()
        assert e < 5e-3, (b, pos, e)
