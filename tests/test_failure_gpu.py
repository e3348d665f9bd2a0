"""Failure handling without a GPU fault: every wait in the kernels is bounded, and a wait that runs out sets the
device error word and returns instead of hanging. `qk_wait_probe` makes the two kinds of wait run out on
purpose — a ring stage that never lands (mbarrier) and a peer rank that never adds to a counter — with a short
limit. The test checks the status the host reads, and that the context stays usable: a GEMV launched right after
is exact again and leaves the error word clear."""
import ctypes

import pytest
import torch

import kernels

pytestmark = pytest.mark.gpu

LIMIT_NS = 20_000_000   # 20 ms


def _probe(mode):
    ops = kernels.ops()
    ops.device_error()                                   # start from a clear error word
    gave_up = torch.zeros(1, dtype=torch.int32, device="cuda")
    counter = torch.zeros(1, dtype=torch.int64, device="cuda")
    rc = ops.lib.qk_wait_probe(mode, ctypes.c_void_p(counter.data_ptr()), LIMIT_NS,
                               ctypes.c_void_p(gave_up.data_ptr()), None)
    assert rc == 0, ops.lib.qk_last_error()
    torch.cuda.synchronize()
    return int(gave_up.item()), ops.device_error()


@pytest.mark.parametrize("mode,bit", [(0, 1), (1, 4)], ids=["mbarrier", "counter"])
def test_bounded_wait_gives_up_and_reports(mode, bit):
    gave_up, err = _probe(mode)
    assert gave_up == 1
    assert err & bit, err
    assert kernels.ops().device_error() == 0             # reading cleared it


def test_context_usable_after_a_timeout():
    import model as M
    _probe(0)
    w, s = M.synth_linear(5, "after_timeout", 256, 4096, "channel", "cuda")
    x = (torch.randn(4096, device="cuda") * 0.5).to(torch.bfloat16)
    out = torch.zeros(256, dtype=torch.bfloat16, device="cuda")
    out2 = torch.zeros_like(out)
    packed = M.pack_fp8(w)
    ops = kernels.ops()
    for o in (out, out2):
        ops.fp8_gemv(3, packed, s, x, None, o, 256, 1e-6)   # kind 3: o_proj-style, residual in place (zero)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all() and out.float().abs().sum() > 0
    assert torch.equal(out, out2)
    assert ops.device_error() == 0


def test_probe_rejects_bad_arguments():
    ops = kernels.ops()
    g = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert ops.lib.qk_wait_probe(2, None, LIMIT_NS, ctypes.c_void_p(g.data_ptr()), None) != 0
    assert ops.lib.qk_wait_probe(0, None, 0, ctypes.c_void_p(g.data_ptr()), None) != 0
    assert ops.lib.qk_wait_probe(1, None, LIMIT_NS, ctypes.c_void_p(g.data_ptr()), None) != 0
