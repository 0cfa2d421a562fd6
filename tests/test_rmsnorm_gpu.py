"""The row-parallel W4 layer with the all-reduce, residual add and RMSNorm in one launch
(b2_w4_gemm_allreduce_rmsnorm / gfx906_skinny.w4gemm_ar_rmsnorm) on one GPU.

A one-rank all-reduce handle runs the whole fused epilogue: the exchange (to itself), the
grid-wide barrier and the row norm. The norm is checked against the oracle's restatement of
vLLM's fused_add_rms_norm applied to the plain fused GEMM + all-reduce output of the same inputs
(which itself is checked against the float64 GEMM oracle): the new residual bit for bit, the
output within two fp16 ulps (the kernel's row sums are added in another order and rsqrtf is
not correctly rounded; the oracle pins vLLM's own code to within one ulp)."""

from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest
import torch

from gpu_util import check, dev, mismatch, stream_ptr, workspace

pytestmark = pytest.mark.gpu

EPS = 1e-6


@pytest.fixture(scope="module")
def handle(capi):
    """One-rank NVLink all-reduce handle on device 0 (room for M=8, N=8192 fp32 payloads)."""
    lib = capi.lib()
    h = C.c_void_p()
    capi.check(lib.b2_nvar_create(0, 0, 1, 8 * 8192 * 4, C.byref(h)), "nvar_create")
    assert lib.b2_nvar_is_connected(h) == 1
    yield h
    torch.cuda.synchronize()
    capi.check(lib.b2_nvar_destroy(h), "nvar_destroy")


@pytest.fixture(scope="module")
def ws(capi):
    return workspace(capi)


def layer_inputs(oracle, M, K, N, G, seed):
    x, qw, qz, sc = oracle.gen_w4(M, K, N, G, seed=seed)
    rng = np.random.default_rng(seed + 1)
    res = (rng.standard_normal((M, N)) * 4).astype(np.float16)
    w = (1.0 + rng.uniform(-0.3, 0.3, size=N)).astype(np.float16)
    return x, qw, qz, sc, res, w


def fused_ar(capi, h, ws, x, qw, qz, sc, M, K, N, G):
    y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    capi.check(capi.lib().b2_w4_gemm_allreduce(
        h, x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), y.data_ptr(), M, K, N, G,
        ws.data_ptr(), ws.numel(), stream_ptr()), "w4_gemm_allreduce")
    return y


def fused_norm(capi, h, ws, x, qw, qz, sc, res, w, M, K, N, G, eps=EPS):
    y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    capi.check(capi.lib().b2_w4_gemm_allreduce_rmsnorm(
        h, x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), res.data_ptr(),
        w.data_ptr(), eps, y.data_ptr(), M, K, N, G, ws.data_ptr(), ws.numel(), stream_ptr()),
        "w4_gemm_allreduce_rmsnorm")
    return y


def assert_norm_parity(oracle, y_ar, res0, w, out, new_res, eps=EPS, what=""):
    ref_out, ref_res = oracle.add_rmsnorm_ref(y_ar.cpu().numpy(), res0, w, eps)
    got_res = new_res.cpu().numpy()
    assert np.array_equal(got_res.view(np.int16), ref_res.view(np.int16)), \
        f"{what}: residual differs in {(got_res != ref_res).sum()} elements"
    o = out.cpu().numpy()
    assert np.isfinite(o).all(), f"{what}: non-finite output"
    ulp = oracle.fp16_ulp_distance(o, ref_out)
    exact = float((ulp == 0).mean())
    assert ulp.max() <= 2 and exact >= 0.99, f"{what}: max ulp {ulp.max()}, exact {exact:.5f}"
    return exact


SHAPES = [(8, 2176, 5120, 128), (1, 1024, 5120, 128), (5, 2048, 4128, 64), (3, 1024, 1024, 32),
          (8, 6144, 640, 128)]


@pytest.mark.parametrize("path", [0, 1, 2], ids=["auto", "stream-K", "cluster"])
@pytest.mark.parametrize("M,K,N,G", SHAPES)
def test_fused_rmsnorm_matches_oracle(capi, handle, ws, oracle, path, M, K, N, G):
    lib = capi.lib()
    saved = lib.b2_get_tuning(4)
    lib.b2_set_tuning(4, path)
    try:
        x, qw, qz, sc, res0, w = layer_inputs(oracle, M, K, N, G, seed=M * 13 + K + N + G)
        dx, dqw, dqz, dsc, dw = dev(x), dev(qw), dev(qz), dev(sc), dev(w)
        y_ar = fused_ar(capi, handle, ws, dx, dqw, dqz, dsc, M, K, N, G)
        check(y_ar, oracle.w4_ref(x, qw, qz, sc), f"all-reduced GEMM {M}x{K}x{N}")
        r = dev(res0)
        out = fused_norm(capi, handle, ws, dx, dqw, dqz, dsc, r, dw, M, K, N, G)
        torch.cuda.synchronize()
        assert_norm_parity(oracle, y_ar, res0, w, out, r, what=f"path {path} {M}x{K}x{N} G={G}")
        # deterministic: the same inputs again give the same bits
        r2 = dev(res0)
        out2 = fused_norm(capi, handle, ws, dx, dqw, dqz, dsc, r2, dw, M, K, N, G)
        assert torch.equal(out2, out), mismatch(out2, out)
        assert torch.equal(r2, r), mismatch(r2, r)
        st = C.c_int(-1)
        capi.check(lib.b2_nvar_status(handle, 1, C.byref(st)), "nvar_status")
        assert st.value == 0
    finally:
        lib.b2_set_tuning(4, saved)


def test_back_to_back_launches(capi, handle, ws, oracle):
    """Eight launches in a row on one stream (40 clusters of 12 CTAs each, near the 42 that fit
    the GPU), with a 500 ms bound on the grid-wide barrier: none may give up (status 0), and each
    normalises the residual the previous one left, as the oracle does."""
    lib = capi.lib()
    M, K, N, G = 8, 4352, 5120, 128
    x, qw, qz, sc, res0, w = layer_inputs(oracle, M, K, N, G, seed=21)
    dx, dqw, dqz, dsc, dw = dev(x), dev(qw), dev(qz), dev(sc), dev(w)
    y_ar = fused_ar(capi, handle, ws, dx, dqw, dqz, dsc, M, K, N, G).cpu().numpy()
    capi.check(lib.b2_nvar_set_timeout_ns(handle, 500_000_000), "set_timeout")
    try:
        r = dev(res0)
        outs = [fused_norm(capi, handle, ws, dx, dqw, dqz, dsc, r, dw, M, K, N, G)
                for _ in range(8)]
        torch.cuda.synchronize()
        st = C.c_int(-1)
        capi.check(lib.b2_nvar_status(handle, 1, C.byref(st)), "nvar_status")
        assert st.value == 0, f"a grid-wide barrier gave up (status {st.value})"
    finally:
        capi.check(lib.b2_nvar_set_timeout_ns(handle, 10_000_000_000), "set_timeout")
    res = res0
    for i, out in enumerate(outs):
        ref_out, res = oracle.add_rmsnorm_ref(y_ar, res, w, EPS)
        ulp = oracle.fp16_ulp_distance(out.cpu().numpy(), ref_out)
        assert ulp.max() <= 2 and (ulp == 0).mean() >= 0.99, (i, ulp.max(), (ulp == 0).mean())
    assert np.array_equal(r.cpu().numpy().view(np.int16), res.view(np.int16))


def test_fused_rmsnorm_edge_rows(capi, handle, ws, oracle):
    """A zero row (the residual cancels the layer output: x = 0, eps alone sets the scale) and
    large values (sum of squares far beyond fp16 range) in one call."""
    M, K, N, G = 4, 1024, 2048, 128
    x, qw, qz, sc, _, w = layer_inputs(oracle, M, K, N, G, seed=77)
    x[2] *= np.float16(8)
    dx, dqw, dqz, dsc, dw = dev(x), dev(qw), dev(qz), dev(sc), dev(w)
    y_ar = fused_ar(capi, handle, ws, dx, dqw, dqz, dsc, M, K, N, G)
    res0 = np.zeros((M, N), np.float16)
    res0[1] = -y_ar[1].cpu().numpy()          # row 1: x = 0 exactly
    res0[3] = np.float16(3000)                # row 3: |x| in the thousands
    r = dev(res0)
    out = fused_norm(capi, handle, ws, dx, dqw, dqz, dsc, r, dw, M, K, N, G)
    torch.cuda.synchronize()
    assert_norm_parity(oracle, y_ar, res0, w, out, r, what="edge rows")
    assert not out[1].any()


def test_fused_rmsnorm_chain_in_graph(capi, handle, ws, oracle):
    """Two layers chained through the residual (o_proj then down_proj of one decoder layer, as
    the decode step runs them), captured in a CUDA graph: replays equal the eager calls."""
    M, K1, K2, N, G = 8, 2048, 4352, 5120, 128
    a = layer_inputs(oracle, M, K1, N, G, seed=5)
    b = layer_inputs(oracle, M, K2, N, G, seed=6)
    A = [dev(v) for v in a]
    B = [dev(v) for v in b]
    res_init = A[4].clone()

    def step(res):
        o1 = fused_norm(capi, handle, ws, A[0], A[1], A[2], A[3], res, A[5], M, K1, N, G)
        o2 = fused_norm(capi, handle, ws, B[0], B[1], B[2], B[3], res, B[5], M, K2, N, G)
        return o1, o2

    res_e = res_init.clone()
    e1, e2 = step(res_e)
    torch.cuda.synchronize()
    res_g = res_init.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            g1, g2 = step(res_g)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        res_g.copy_(res_init)
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(g1, e1), mismatch(g1, e1)
    assert torch.equal(g2, e2), mismatch(g2, e2)
    assert torch.equal(res_g, res_e), mismatch(res_g, res_e)
    del g


def test_torch_op_one_rank(ops, oracle):
    """gfx906_skinny.w4gemm_ar_rmsnorm on a one-rank handle made by nvar_create: the residual is
    updated in place and the result equals the C-ABI path's."""
    M, K, N, G = 6, 2048, 3072, 128
    x, qw, qz, sc, res0, w = layer_inputs(oracle, M, K, N, G, seed=9)
    name = f"/b2_test_norm_{os.getpid()}"
    h = ops.nvar_create(name, M * N * 4, 0, 1)
    ops.hostar_unlink(name)
    dx, dqw, dqz, dsc, dw = dev(x), dev(qw), dev(qz), dev(sc), dev(w)
    y_ar = ops.w4gemm_ar(dx, dqw, dqz, dsc, h)
    r = dev(res0)
    out = ops.w4gemm_ar_rmsnorm(dx, dqw, dqz, dsc, h, r, dw, EPS)
    torch.cuda.synchronize()
    assert out.shape == (M, N) and out.dtype == torch.float16
    assert_norm_parity(oracle, y_ar, res0, w, out, r, what="torch op")
    assert ops.nvar_status(h, True) == 0
    with pytest.raises(RuntimeError, match="residual"):
        ops.w4gemm_ar_rmsnorm(dx, dqw, dqz, dsc, h, r[:, :-32].contiguous(), dw, EPS)
    with pytest.raises(RuntimeError, match="weight"):
        ops.w4gemm_ar_rmsnorm(dx, dqw, dqz, dsc, h, r, dw[:-8].contiguous(), EPS)


def test_rejects_bad_arguments(capi, handle, ws, oracle):
    """Host-side checks: nothing is launched for a missing, misaligned or overlapping residual
    or weight, or a bad eps."""
    lib = capi.lib()
    M, K, N, G = 2, 256, 256, 128
    x, qw, qz, sc, res0, w = layer_inputs(oracle, M, K, N, G, seed=3)
    dx, dqw, dqz, dsc, dw, r = dev(x), dev(qw), dev(qz), dev(sc), dev(w), dev(res0)
    y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    big = torch.empty(M * N * 2 + 8, dtype=torch.float16, device="cuda")

    def call(res_ptr, w_ptr, y_ptr, eps=EPS):
        return lib.b2_w4_gemm_allreduce_rmsnorm(
            handle, dx.data_ptr(), dqw.data_ptr(), dqz.data_ptr(), dsc.data_ptr(), res_ptr, w_ptr,
            eps, y_ptr, M, K, N, G, ws.data_ptr(), ws.numel(), stream_ptr())

    assert call(None, dw.data_ptr(), y.data_ptr()) == capi.B2_ERR_INVALID_ARG
    assert call(r.data_ptr(), None, y.data_ptr()) == capi.B2_ERR_INVALID_ARG
    assert call(r.data_ptr() + 2, dw.data_ptr(), y.data_ptr()) == capi.B2_ERR_INVALID_ARG
    assert call(big.data_ptr(), dw.data_ptr(), big.data_ptr() + 64) == capi.B2_ERR_INVALID_ARG
    assert call(r.data_ptr(), dw.data_ptr(), y.data_ptr(), eps=-1.0) == capi.B2_ERR_INVALID_ARG
    assert call(r.data_ptr(), dw.data_ptr(), y.data_ptr(), eps=float("nan")) == \
        capi.B2_ERR_INVALID_ARG
    torch.cuda.synchronize()
    assert torch.equal(r, dev(res0))  # untouched
