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
    assert lib.qk_decode_step_part_floats(4096) == 2 * 24576 * 4096 // 128   # u64 tagged words
    assert lib.qk_decode_step_counters(4096) == 768
    assert lib.qk_decode_step_part_floats(151936) == 2 * 151936 * 32
    assert lib.qk_decode_step_counters(151936) == 151936 // 16


def test_tp_entry_points_check_arguments_without_a_gpu(lib):
    assert lib.qk_tp_area_bytes() >= 2 * 8 * 4096 * 4
    p = ctypes.c_void_p(16)

    class Comm(ctypes.Structure):
        _fields_ = [("tp", ctypes.c_int), ("rank", ctypes.c_int), ("areas", ctypes.c_void_p)]

    args = [p, 1, p, p, ctypes.c_longlong(8 * 4096 * 256), p, p, p, p, 151936, p, p, p, p, p, 4096, p, p, p, p, p,
            p, p, ctypes.c_longlong(2 * 151936 * 32), p, 151936 // 16, p, p, p, p, 4096, 128, ctypes.c_float(1e-6),
            None, p]
    for tp, rank, off, msg in ((3, 0, 0, b"tp must be"), (2, 2, 0, b"bad rank"), (2, 0, 8, b"vocab_offset")):
        comm = Comm(tp, rank, 16)
        st = lib.qk_decode_step_tp(*args, off, ctypes.byref(comm), None)
        assert st == 1 and msg in lib.qk_last_error(), lib.qk_last_error()
    st = lib.qk_decode_step_tp(*args, 0, None, None)
    assert st == 1 and b"null" in lib.qk_last_error()


def _ref_tile_fp8(w, kmajor):
    """The reference's weight layout (qwen3-8b-fp8_rtx-5090/model.py:92-104), restated for the boundary test:
    8-row groups of 64-wide K chunks, group-major or K-major."""
    import torch
    N, K = w.shape
    v = w.view(torch.uint8).view(N // 8, 8, K // 64, 4, 4, 4)
    order = (2, 0, 1, 4, 3, 5) if kmajor else (0, 2, 1, 4, 3, 5)
    return v.permute(*order).contiguous().view(torch.float8_e4m3fn).view(N, K)


def test_boundary_rejects_weights_not_in_pack_fp8_layout(lib):
    """A reference caller handing its tile_fp8 weights (or any untagged fp8 tensor) to fp8_gemv gets the
    reference's RuntimeError instead of wrong numbers; pack_reference_tiled converts them."""
    import torch
    import kernels
    import model as M
    ops = kernels.DecodeOps(lib)    # no GPU needed: the layout check comes before any launch
    w = (torch.randn(256, 4096) * 4).to(torch.float8_e4m3fn)
    s = torch.ones(256)
    x = torch.zeros(4096, dtype=torch.bfloat16)
    out = torch.zeros(256, dtype=torch.bfloat16)
    for bad in (_ref_tile_fp8(w, True), w, M.pack_fp8(w).as_subclass(torch.Tensor)):
        with pytest.raises(RuntimeError, match="pack_fp8"):
            ops.fp8_gemv(0, bad, s, x, x, out, 256, 1e-6, 4, 4, 2, 24, 1)
    # gate|up needs the pairs packing, every other kind the plain one
    with pytest.raises(RuntimeError, match="pairs=True"):
        ops.fp8_gemv(2, M.pack_fp8(w), s, x, x, out, 256, 1e-6)
    with pytest.raises(RuntimeError, match="PackedFP8Pairs"):
        ops.fp8_gemv(0, M.pack_fp8(w, pairs=True), s, x, x, out, 256, 1e-6)
    with pytest.raises(RuntimeError, match="pack_fp8"):
        ops.lm_head_argmax(w, x, x, out, torch.zeros(1, dtype=torch.int64), 1e-6, 0, w_scale=s)
    with pytest.raises(RuntimeError, match="bf16"):
        ops.lm_head_argmax(M.pack_fp8(w), x, x, out, torch.zeros(1, dtype=torch.int64), 1e-6, 0)
    # the converter gives exactly pack_fp8 of the row-major matrix, for both reference orders
    for km in (False, True):
        got = M.pack_reference_tiled(_ref_tile_fp8(w, km), km)
        assert isinstance(got, kernels.PackedFP8)
        assert torch.equal(got.view(torch.uint8), M.pack_fp8(w).view(torch.uint8))
    # the tag survives moves and views
    assert isinstance(M.pack_fp8(w).to("cpu").view(-1), kernels.PackedFP8)


def test_boundary_validates_the_reference_tuning_knobs(lib):
    import torch
    import kernels
    import model as M
    ops = kernels.DecodeOps(lib)
    w = M.pack_fp8(torch.zeros(256, 4096).to(torch.float8_e4m3fn))
    s = torch.ones(256)
    x = torch.zeros(4096, dtype=torch.bfloat16)
    out = torch.zeros(256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="kmajor"):
        ops.fp8_gemv(0, w, s, x, x, out, 256, 1e-6, 4, 4, 2, 24, 2)
    with pytest.raises(RuntimeError, match="trig"):
        ops.fp8_gemv(0, w, s, x, x, out, 256, 1e-6, 4, 4, 2, 32, 1)
    with pytest.raises(RuntimeError, match="trig"):
        ops.fp8_gemv(0, w, s, x, x, out, 256, 1e-6, 4, 4, 2, -2, 1)


def test_noalloc_rejects_bad_arguments_before_enqueuing_anything(lib):
    """Every check of qk_fp8_gemv runs before the no-alloc entry point touches the device: these calls need
    no GPU, so nothing (not even its counter reset) was enqueued."""
    p = ctypes.c_void_p(16)
    # null weights
    st = lib.qk_fp8_gemv_noalloc(0, None, p, 1, p, p, None, None, p, 6144, 4096, 1e-6, None)
    assert st == 1 and b"null" in lib.qk_last_error()
    # gate|up with N not a multiple of 32
    st = lib.qk_fp8_gemv_noalloc(2, p, p, 1, p, p, None, None, p, 4112, 4096, 1e-6, None)
    assert st == 1 and b"multiple of 32" in lib.qk_last_error()
    # block-128 scales with N % 128 != 0
    st = lib.qk_fp8_gemv_noalloc(0, p, p, 0, p, p, None, None, p, 6160, 4096, 1e-6, None)
    assert st == 1 and b"block-128" in lib.qk_last_error()
    # misaligned output
    st = lib.qk_fp8_gemv_noalloc(1, p, p, 1, p, None, None, None, ctypes.c_void_p(18), 4096, 4096, 1e-6, None)
    assert st == 1 and b"aligned" in lib.qk_last_error()
    # the unknown kind is refused too
    st = lib.qk_fp8_gemv_noalloc(4, p, p, 1, p, p, None, None, p, 4096, 4096, 1e-6, None)
    assert st == 1 and b"kind" in lib.qk_last_error()


def test_pack_fp8_tiles_round_trip_and_swizzle():
    """The tcgen05 linear's tile-packed weight layout: a permutation of the bytes (round trip), with chunk c
    of row r of tile (t, kb) at chunk position c ^ (r % 8)."""
    import torch
    import model as M
    g = torch.Generator().manual_seed(0)
    w = torch.randint(0, 0x7F, (384, 256), generator=g, dtype=torch.uint8).view(torch.float8_e4m3fn)
    p = M.pack_fp8_tiles(w)
    assert p.shape == w.shape and p.dtype == w.dtype
    assert torch.equal(M.unpack_fp8_tiles(p).view(torch.uint8), w.view(torch.uint8))
    flat = p.as_subclass(torch.Tensor).view(torch.uint8).reshape(-1)
    wb = w.view(torch.uint8)
    for t, kb, r, c in ((0, 0, 0, 0), (2, 1, 13, 6), (1, 0, 127, 7)):
        off = ((t * 2 + kb) * 128 + r) * 128 + (c ^ (r % 8)) * 16
        assert torch.equal(flat[off:off + 16], wb[t * 128 + r, kb * 128 + c * 16: kb * 128 + c * 16 + 16])
