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
