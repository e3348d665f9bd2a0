"""qk_fp8_gemv_noalloc: the GEMV for callers that cannot allocate device memory.

Such callers (an allocator-free host runtime, a plugin that only sees one op's tensors, a process whose
device memory is reserved up front) cannot provide the split-K scratch qk_fp8_gemv asks for; this entry point
keeps it in a fixed array inside the library. The test calls both entry points through the C ABI on the same
inputs and requires the same output bits, on two calls in a row (the second call finds the array holding the
first call's contents). It sits in its own file, collected last, and needs nothing from other tests.
"""
import ctypes

import pytest
import torch

import model as M

pytestmark = pytest.mark.gpu
EPS = 1e-6
_VP, _I, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def lib():
    from kernels import load_library
    L = load_library()
    L.qk_fp8_gemv_noalloc.argtypes = [_I, _VP, _VP, _I, _VP, _VP, _VP, _VP, _VP, _I, _I, _F, _VP]
    L.qk_fp8_gemv_noalloc.restype = _I
    return L


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("kind,N,K", [(2, 24576, 4096), (3, 4096, 12288), (0, 6144, 4096)])
def test_noalloc_matches_fp8_gemv_twice(kind, N, K):
    L = lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    w, s = M.synth_linear(kind, f"noalloc{kind}", N, K, "channel", device="cuda")
    packed = M.pack_fp8(w, pairs=(kind == 2))
    g = torch.Generator(device="cuda").manual_seed(kind)
    out_len = N // 2 if kind == 2 else N
    norm_w = (1 + 0.1 * torch.randn(K, generator=g, device="cuda")).to(torch.bfloat16) if kind != 3 else None
    part = torch.empty(N * K // 128, dtype=torch.float32, device="cuda")
    counters = torch.zeros(N // 16, dtype=torch.int32, device="cuda")
    for call in range(2):
        x = (torch.randn(K, generator=g, device="cuda") * (0.5 + call)).to(torch.bfloat16)
        resid = torch.randn(out_len, generator=g, device="cuda").to(torch.bfloat16)
        ref = resid.clone() if kind == 3 else torch.empty(out_len, dtype=torch.bfloat16, device="cuda")
        got = resid.clone() if kind == 3 else torch.full((out_len,), 7.0, dtype=torch.bfloat16, device="cuda")
        st = L.qk_fp8_gemv(kind, ptr(packed), ptr(s), 1, ptr(x), ptr(norm_w), None, None, ptr(ref), N, K, EPS,
                           ptr(part), ptr(counters), 0, 0, 0, -1, 0, stream)
        assert st == 0, L.qk_last_error()
        st = L.qk_fp8_gemv_noalloc(kind, ptr(packed), ptr(s), 1, ptr(x), ptr(norm_w), None, None, ptr(got), N, K,
                                   EPS, stream)
        assert st == 0, L.qk_last_error()
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), f"call {call}: outputs differ"


def test_noalloc_rejects_sizes_beyond_its_array():
    L = lib()
    p = ctypes.c_void_p(16)
    # the 151936-row FP8 lm_head needs more scratch than the fixed array holds
    st = L.qk_fp8_gemv_noalloc(0, p, p, 1, p, p, None, None, p, 151936, 4096, EPS, None)
    assert st == 1 and b"exceeds the no-alloc scratch" in L.qk_last_error()
