"""The C-ABI library (CPU-only checks): it loads, exports every entry point include/qwen3_b200.h declares, and
rejects bad arguments with QK_EINVAL and a message before touching the GPU."""
import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "qwen3_b200.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(qk_\w+)\s*\(", src, re.M)))


@pytest.fixture(scope="module")
def lib():
    from kernels import load_library, LIB_PATH
    if not os.path.exists(LIB_PATH):
        pytest.skip("library not built (run __graft_entry__.build())")
    return load_library()


def test_header_declares_the_reference_ops():
    names = declared()
    for n in ("qk_fp8_gemv", "qk_attention", "qk_lm_head_argmax", "qk_embed", "qk_finalize", "qk_set_pdl",
              "qk_set_timeline"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_version_and_pdl_switch(lib):
    assert lib.qk_version() >= 100
    assert lib.qk_set_pdl(1) == 0 and lib.qk_set_pdl(0) == 0


def test_bad_arguments_are_rejected_without_a_gpu(lib):
    # null weights
    st = lib.qk_fp8_gemv(0, None, None, 1, None, None, None, None, None, 6144, 4096, 1e-6, None, None,
                         0, 0, 0, -1, 0, None)
    assert st == 1 and b"null" in lib.qk_last_error()
    # bad attention chunk
    p = ctypes.c_void_p(16)
    st = lib.qk_attention(p, p, p, p, p, p, p, p, p, p, p, p, 1, 8, 4096, 128, 6144, 2, 0.088, 1e-6, 48, None)
    assert st == 1 and b"chunk" in lib.qk_last_error()
    # o_part too small for the context
    st = lib.qk_attention(p, p, p, p, p, p, p, p, p, p, p, p, 1, 8, 4096, 16, 6144, 2, 0.088, 1e-6, 64, None)
    assert st == 1 and b"max_splits" in lib.qk_last_error()
    # K not a multiple of 128
    st = lib.qk_fp8_gemv(1, p, p, 1, p, None, None, None, p, 4096, 100, 1e-6, p, p, 0, 0, 0, -1, 0, None)
    assert st == 1 and b"K=100" in lib.qk_last_error()
    # timeline: a buffer needs a positive slot count; disabling a never-enabled timeline needs no GPU
    assert lib.qk_set_timeline(p, 0) == 1 and lib.qk_set_timeline(None, 0) == 0


def test_ops_refuses_to_run_without_cuda():
    import torch
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    import kernels
    with pytest.raises(RuntimeError):
        kernels.ops()


def test_fused_step_scratch_sizes(lib):
    """The fused step's boundary-unit scratch covers the largest GEMV of a layer even for a small vocabulary."""
    assert lib.qk_decode_step_part_floats(4096) == 24576 * 4096 // 128
    assert lib.qk_decode_step_counters(4096) == 768
    assert lib.qk_decode_step_part_floats(151936) == 151936 * 32
    assert lib.qk_decode_step_counters(151936) == 151936 // 16


def test_tp_entry_points_check_arguments_without_a_gpu(lib):
    assert lib.qk_tp_area_bytes() >= 2 * 8 * 4096 * 4
    p = ctypes.c_void_p(16)

    class Comm(ctypes.Structure):
        _fields_ = [("tp", ctypes.c_int), ("rank", ctypes.c_int), ("areas", ctypes.c_void_p)]

    args = [p, 1, p, p, ctypes.c_longlong(8 * 4096 * 256), p, p, p, p, 151936, p, p, p, p, p, 4096, p, p, p, p, p,
            p, p, ctypes.c_longlong(151936 * 32), p, 151936 // 16, p, p, p, p, 4096, 128, ctypes.c_float(1e-6),
            None, p]
    for tp, rank, off, msg in ((3, 0, 0, b"tp must be"), (2, 2, 0, b"bad rank"), (2, 0, 8, b"vocab_offset")):
        comm = Comm(tp, rank, 16)
        st = lib.qk_decode_step_tp(*args, off, ctypes.byref(comm), None)
        assert st == 1 and msg in lib.qk_last_error(), lib.qk_last_error()
    st = lib.qk_decode_step_tp(*args, 0, None, None)
    assert st == 1 and b"null" in lib.qk_last_error()
