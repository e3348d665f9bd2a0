"""The batched FP8 linear on the tcgen05 tensor cores (qk_fp8_gemm_rows) against the W8A8 recipe restated in
torch on the GPU (oracle/qwen3_ref.py: per-128 activation quant, fp32 block dots times the scales summed over K
blocks in order, bf16): the five decode shapes x rows 1, 4, 16, 64, 128 (and 2, 33, 100 for padding), both scale
layouts, with and without the RMSNorm prologue; 1e-2 rel-L2, the parity bar of the GEMV rows."""
import pytest
import torch

import model as M
from oracle import qwen3_ref as O

pytestmark = pytest.mark.gpu

SHAPES = [(6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288), (151936, 4096)]


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def run(N, K, rows, scale_mode, norm=False, seed=0):
    from kernels import ops
    w, s = M.synth_linear(seed, f"tc.{N}.{K}", N, K, scale_mode, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(seed + rows)
    x = (torch.randn(rows, K, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    nw = M.synth_norm(seed, "tc.norm", K, "random", device="cuda") if norm else None
    out = torch.empty(rows, N, dtype=torch.bfloat16, device="cuda")
    ops().fp8_gemm_rows(x, w, s, out, norm_w=nw)
    torch.cuda.synchronize()
    assert ops().device_error() == 0
    xin = O.rms_norm(x, nw, 1e-6) if norm else x
    ref = O.fp8_linear(xin, w, s)
    return out, ref


@pytest.mark.parametrize("rows", [1, 4, 16, 64, 128])
@pytest.mark.parametrize("N,K", SHAPES)
def test_gemm_rows_per_channel(N, K, rows):
    out, ref = run(N, K, rows, "channel")
    e = rel(out, ref)
    assert e < 1e-2, e


@pytest.mark.parametrize("rows", [2, 33, 100])
def test_gemm_rows_block_scales_and_norm(rows):
    out, ref = run(4096, 4096, rows, "block", norm=True, seed=1)
    e = rel(out, ref)
    assert e < 1e-2, e


def test_gemm_rows_repeat_and_rejects_packed_weights():
    """Two calls in a row give the same result (the tile counters are left zero); the packed GEMV layout
    and more than 64 rows are refused."""
    from kernels import ops
    out1, ref = run(6144, 4096, 16, "channel", seed=2)
    out2, _ = run(6144, 4096, 16, "channel", seed=2)
    assert torch.equal(out1, out2)
    w, s = M.synth_linear(0, "tc.rej", 256, 256, "channel", device="cuda")
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(4, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="row-major"):
        ops().fp8_gemm_rows(x, M.pack_fp8(w), s, out)
    with pytest.raises(RuntimeError):
        ops().fp8_gemm_rows(torch.zeros(129, 256, dtype=torch.bfloat16, device="cuda"), w, s,
                            torch.empty(129, 256, dtype=torch.bfloat16, device="cuda"))
    # above 64 rows the activation scales of at most K = 12288 fit in shared memory
    w2, s2 = M.synth_linear(0, "tc.rej2", 128, 16384, "channel", device="cuda")
    with pytest.raises(RuntimeError, match="12288"):
        ops().fp8_gemm_rows(torch.zeros(65, 16384, dtype=torch.bfloat16, device="cuda"), w2, s2,
                            torch.empty(65, 128, dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("rows", [1, 37, 64, 128])
@pytest.mark.parametrize("N,K", [(6144, 4096), (4096, 12288), (24576, 4096)])
def test_gemm_tiles_equal_row_major(N, K, rows):
    """The tile-packed weights (bulk copies) give the row-major path's (TMA boxes) results bit for bit: the
    same shared-memory images, the same arithmetic. Both scale layouts, RMSNorm prologue on the block one."""
    from kernels import ops
    for scale_mode, norm in (("channel", False), ("block", True)):
        w, s = M.synth_linear(3, f"tt.{N}.{K}", N, K, scale_mode, device="cuda")
        g = torch.Generator(device="cuda").manual_seed(rows)
        x = torch.randn(rows, K, generator=g, device="cuda").to(torch.bfloat16)
        nw = M.synth_norm(3, "tt.norm", K, "random", device="cuda") if norm else None
        a = torch.empty(rows, N, dtype=torch.bfloat16, device="cuda")
        b = torch.empty_like(a)
        ops().fp8_gemm_rows(x, w, s, a, norm_w=nw)
        ops().fp8_gemm_rows(x, M.pack_fp8_tiles(w), s, b, norm_w=nw)
        torch.cuda.synchronize()
        assert ops().device_error() == 0
        assert torch.equal(a, b), (scale_mode, (a.float() - b.float()).abs().max().item())

