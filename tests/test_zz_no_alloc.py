"""The W4A16 GEMM entry point that allocates nothing (b2_w4_gemm_noalloc).

Some callers cannot allocate device memory where they call the GEMM: a host that reaches the
library through a C binding but does not own the process's device allocator, code running where
a cudaMalloc could stall every stream on the device or fail, and code with nowhere to keep a
workspace alive between calls. For them the library keeps the split-K scratch in a fixed array of
device memory and this entry point takes only operands. These tests call it through the C ABI and
check that it gives the same results as b2_w4_gemm (which takes a workspace), within the tolerance
of the other tests, on two calls in a row. This file is collected last on purpose.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import dev, stream_ptr, workspace

pytestmark = pytest.mark.gpu

SHAPES = [  # M, K, N, G
    (8, 4096, 4096, 128),
    (1, 2048, 1056, 32),
    (5, 2176, 5120, 128),
    (7, 1024, 384, 64),
]


def _call_noalloc(lib, x, qw, qz, sc, y, M, K, N, G):
    return lib.b2_w4_gemm_noalloc(x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(),
                                  y.data_ptr(), M, K, N, G, stream_ptr())


@pytest.mark.parametrize("M,K,N,G", SHAPES)
def test_noalloc_matches_workspace_entry_point(capi, oracle, M, K, N, G):
    lib = capi.lib()
    x, qw, qz, sc = oracle.gen_w4(M, K, N, G, seed=M * 7 + N)
    xd, qwd, qzd, scd = dev(x), dev(qw), dev(qz), dev(sc)
    ws = workspace(capi)
    y_ws = torch.empty(M, N, dtype=torch.float16, device="cuda")
    capi.check(lib.b2_w4_gemm(xd.data_ptr(), qwd.data_ptr(), qzd.data_ptr(), scd.data_ptr(),
                              y_ws.data_ptr(), M, K, N, G, ws.data_ptr(), ws.numel(), stream_ptr()),
               "b2_w4_gemm")
    y_ref = y_ws.double().cpu().numpy()
    ref64 = oracle.w4_ref(x, qw, qz, sc)
    for call in range(2):  # the scratch keeps the previous call's contents
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        capi.check(_call_noalloc(lib, xd, qwd, qzd, scd, y, M, K, N, G), "b2_w4_gemm_noalloc")
        torch.cuda.synchronize()
        yn = y.double().cpu().numpy()
        assert np.isfinite(yn).all(), f"call {call}: unwritten or non-finite outputs"
        st = oracle.error_stats(yn, y_ref)
        assert oracle.within_tolerance(st), f"call {call} vs b2_w4_gemm: {st}"
        st64 = oracle.error_stats(yn, ref64)
        assert oracle.within_tolerance(st64), f"call {call} vs float64 oracle: {st64}"


def test_noalloc_rejects_n_beyond_scratch(capi):
    lib = capi.lib()
    fake = 1 << 20  # validation fails before any pointer is used
    rc = lib.b2_w4_gemm_noalloc(fake, fake, fake, fake, fake, 4, 128, 524288 + 128, 128,
                                stream_ptr())
    assert rc == capi.B2_ERR_INVALID_ARG
    assert b"scratch" in lib.b2_last_error()


class _DeviceArray:
    """A raw device allocation seen through __cuda_array_interface__, so torch can write to it."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes // 4,), "typestr": "<i4",
                                         "data": (ptr, False), "version": 3}


def _scratch(capi):
    import ctypes as C

    p, n = C.c_void_p(), C.c_size_t()
    capi.check(capi.lib().b2_w4_noalloc_scratch(C.byref(p), C.byref(n)), "b2_w4_noalloc_scratch")
    return p.value, n.value


@pytest.mark.parametrize("path", [1, 2], ids=["stream-K", "cluster"])
@pytest.mark.parametrize("M,K,N,G", [(8, 4096, 4096, 128), (3, 2176, 5120, 128), (8, 4096, 1056, 32)])
def test_noalloc_each_split_k_path(capi, oracle, path, M, K, N, G):
    """Both split-K kernels, forced with B2_TUNE_W4_PATH: stream-K runs on the fixed array with its
    256-CTA cap, the cluster kernel uses none of it. Each call, made twice in a row, matches
    b2_w4_gemm with the same tuning and the float64 oracle."""
    lib = capi.lib()
    saved = lib.b2_get_tuning(4)
    lib.b2_set_tuning(4, path)
    try:
        x, qw, qz, sc = oracle.gen_w4(M, K, N, G, seed=path * 100 + M + N)
        xd, qwd, qzd, scd = dev(x), dev(qw), dev(qz), dev(sc)
        ws = workspace(capi)
        y_ws = torch.empty(M, N, dtype=torch.float16, device="cuda")
        capi.check(lib.b2_w4_gemm(xd.data_ptr(), qwd.data_ptr(), qzd.data_ptr(), scd.data_ptr(),
                                  y_ws.data_ptr(), M, K, N, G, ws.data_ptr(), ws.numel(),
                                  stream_ptr()), "b2_w4_gemm")
        ref64 = oracle.w4_ref(x, qw, qz, sc)
        for call in range(2):
            y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
            capi.check(_call_noalloc(lib, xd, qwd, qzd, scd, y, M, K, N, G), "b2_w4_gemm_noalloc")
            torch.cuda.synchronize()
            yn = y.double().cpu().numpy()
            assert np.isfinite(yn).all(), f"path {path} call {call}: unwritten outputs"
            assert oracle.within_tolerance(oracle.error_stats(yn, y_ws.double().cpu().numpy()))
            assert oracle.within_tolerance(oracle.error_stats(yn, ref64))
    finally:
        lib.b2_set_tuning(4, saved)


def test_noalloc_clears_what_an_earlier_call_left(capi, oracle):
    """The array keeps whatever the last call left; a call that gave up on a wait can leave tile
    counters and the status word non-zero. Fill the whole array with a non-zero pattern and check
    that the next stream-K call still gives the right result (it clears what it uses first)."""
    lib = capi.lib()
    M, K, N, G = 8, 4096, 4096, 128
    x, qw, qz, sc = oracle.gen_w4(M, K, N, G, seed=77)
    xd, qwd, qzd, scd = dev(x), dev(qw), dev(qz), dev(sc)
    y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    capi.check(_call_noalloc(lib, xd, qwd, qzd, scd, y, M, K, N, G), "b2_w4_gemm_noalloc")
    ptr, nbytes = _scratch(capi)
    assert ptr and nbytes == 2113792
    arr = torch.as_tensor(_DeviceArray(ptr, nbytes), device="cuda")
    saved = lib.b2_get_tuning(4)
    lib.b2_set_tuning(4, 1)  # stream-K: the kernel that uses the counters and partial slots
    try:
        for call in range(2):
            arr.fill_(0x01010101 + call)  # counters, status and partial slots all non-zero
            y.fill_(float("nan"))
            capi.check(_call_noalloc(lib, xd, qwd, qzd, scd, y, M, K, N, G), "b2_w4_gemm_noalloc")
            torch.cuda.synchronize()
            yn = y.double().cpu().numpy()
            assert np.isfinite(yn).all(), f"call {call}: unwritten outputs"
            st = oracle.error_stats(yn, oracle.w4_ref(x, qw, qz, sc))
            assert oracle.within_tolerance(st), f"call {call}: {st}"
    finally:
        lib.b2_set_tuning(4, saved)


def test_noalloc_scratch_address_is_stable(capi):
    """The array is looked up once per CUDA context: repeated queries give the same address and
    the documented size."""
    p1, n1 = _scratch(capi)
    p2, n2 = _scratch(capi)
    assert p1 == p2 and n1 == n2
