"""FP8 KV cache host side, on the CPU: the row quantizer the model uses to set up caches equals the contract's
restatement in the oracle, zero rows quantize to zeros with a zero scale, the largest value of a row maps to
±448, and `set_kv_dtype("fp8")` allocates e4m3 rows plus one fp32 scale per (layer, sequence, head, position)
that `fill_cache_random` fills."""
import torch

import model as M
from oracle import qwen3_ref as O


def test_quantize_kv_rows_matches_the_contract():
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(4, 8, 33, 128, generator=g) * 3).to(torch.bfloat16)
    x[0, 0, 5] = 0                                    # a zero row
    q, s = M.quantize_kv_rows(x)
    qo, so = O.quant_kv_rows(x)
    assert q.dtype == torch.float8_e4m3fn and s.dtype == torch.float32
    assert torch.equal(q.view(torch.uint8), qo.view(torch.uint8)) and torch.equal(s, so)
    assert s[0, 0, 5] == 0 and not q[0, 0, 5].view(torch.uint8).any()
    # the row's largest magnitude lands on the e4m3 maximum, and dequantized rows are within one e4m3 step
    amax_q = q.float().abs().amax(-1)
    nz = s > 0
    assert torch.all(amax_q[nz] == 448.0)
    deq = q.float() * s[..., None]
    assert torch.all((deq - x.float()).abs() <= 0.0625 * x.float().abs() + s[..., None] * 2.0 ** -9)


def test_set_kv_dtype_allocates_and_fills_fp8_rows():
    cfg = M.Config(layers=2, vocab=256)
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=64, device="cpu", seed=0, batch=2)
    assert m.kv_dtype == "bf16" and m.k_cache.dtype == torch.bfloat16 and m.k_scale is None
    m.set_kv_dtype("fp8")
    assert m.k_cache.dtype == torch.uint8 and tuple(m.k_cache.shape) == (2, 2, 8, 64, 128)
    assert m.k_scale.dtype == torch.float32 and tuple(m.k_scale.shape) == (2, 2, 8, 64)
    m.fill_cache_random(40, seed=5)
    assert bool((m.k_scale[:, :, :, :40] > 0).all()) and bool((m.v_scale[:, :, :, :40] > 0).all())
    assert not bool(m.k_scale[:, :, :, 40:].any()) and not bool(m.k_cache[:, :, :, 40:].any())
    try:
        m.set_kv_dtype("int4")
    except ValueError:
        pass
    else:
        raise AssertionError("an unknown KV dtype must be refused")
