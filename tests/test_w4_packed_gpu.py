"""W4A16 on weights repacked at load time (b2_w4_repack / b2_w4_gemm_packed), through the C ABI.

The repack is a byte permutation, so its output is compared byte for byte with the oracle's
restatement, and the packed GEMM must equal the GEMM on the original tensors bit for bit (same
plan, same bytes in shared memory); both are also checked against the float64 reference
(kernels/check_w4.py:11-21)."""

from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch

from gpu_util import (check, dev, mismatch, sample_columns, stream_ptr, w4_device_inputs,
                      w4_ref_sampled, workspace)

pytestmark = pytest.mark.gpu


def repack(capi, qw, qz, sc, K, N, G) -> torch.Tensor:
    lib = capi.lib()
    nbytes = lib.b2_w4_packed_bytes(K, N, G)
    assert nbytes > 0
    out = torch.full((nbytes,), 0xAB, dtype=torch.uint8, device="cuda")  # every byte is written
    capi.check(lib.b2_w4_repack(qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), K, N, G,
                                out.data_ptr(), nbytes, stream_ptr()), "b2_w4_repack")
    return out


def gemm(capi, ws, x, qw, qz, sc, K, N, G) -> torch.Tensor:
    y = torch.full((x.shape[0], N), float("nan"), dtype=torch.float16, device="cuda")
    capi.check(capi.lib().b2_w4_gemm(x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(),
                                     y.data_ptr(), x.shape[0], K, N, G, ws.data_ptr(), ws.numel(),
                                     stream_ptr()), "b2_w4_gemm")
    return y


def gemm_packed(capi, ws, x, pk, K, N, G) -> torch.Tensor:
    y = torch.full((x.shape[0], N), float("nan"), dtype=torch.float16, device="cuda")
    capi.check(capi.lib().b2_w4_gemm_packed(x.data_ptr(), pk.data_ptr(), y.data_ptr(), x.shape[0],
                                            K, N, G, ws.data_ptr(), ws.numel(), stream_ptr()),
               "b2_w4_gemm_packed")
    return y


SMALL = [(1, 128, 32, 128), (3, 256, 96, 32), (5, 512, 352, 64), (8, 1024, 384, 128),
         (7, 1024, 160, 256), (8, 2176, 5120, 128), (2, 4096, 1056, 32)]


@pytest.mark.parametrize("M,K,N,G", SMALL)
def test_repack_bytes_match_oracle(capi, oracle, M, K, N, G):
    _, qw, qz, sc = oracle.gen_w4(M, K, N, G, seed=K + N + G)
    pk = repack(capi, dev(qw), dev(qz), dev(sc), K, N, G)
    torch.cuda.synchronize()
    ref = oracle.w4_repack(qw, qz, sc, G).reshape(-1)
    got = pk.cpu().numpy()
    assert got.shape == ref.shape
    bad = np.flatnonzero(got != ref)
    assert bad.size == 0, f"{bad.size} bytes differ, first at {bad[:8]}"


@pytest.mark.parametrize("path", [0, 1, 2], ids=["auto", "stream-K", "cluster"])
@pytest.mark.parametrize("M,K,N,G", SMALL)
def test_packed_equals_unpacked(capi, oracle, path, M, K, N, G):
    """Each split-K kernel on packed weights gives the bits of the same kernel on the original
    tensors (forced with B2_TUNE_W4_PATH), and both are within tolerance of the oracle."""
    lib = capi.lib()
    saved = lib.b2_get_tuning(4)
    lib.b2_set_tuning(4, path)
    try:
        ws = workspace(capi)
        x, qw, qz, sc = oracle.gen_w4(M, K, N, G, seed=M + K + N + G)
        xd, qwd, qzd, scd = dev(x), dev(qw), dev(qz), dev(sc)
        pk = repack(capi, qwd, qzd, scd, K, N, G)
        y0 = gemm(capi, ws, xd, qwd, qzd, scd, K, N, G)
        y1 = gemm_packed(capi, ws, xd, pk, K, N, G)
        assert torch.equal(y0, y1), mismatch(y0, y1)
        check(y1, oracle.w4_ref(x, qw, qz, sc), f"packed path {path} M={M} K={K} N={N} G={G}")
        torch.cuda.synchronize()
        assert int(ws[:4].view(torch.int32).item()) == 0
    finally:
        lib.b2_set_tuning(4, saved)


@pytest.mark.parametrize("name,M,K,N", [("cfg0", 7, 4096, 4096), ("gate_up", 8, 5120, 34816),
                                        ("down", 8, 17408, 5120), ("qkv", 8, 5120, 8192)])
def test_packed_full_size(capi, name, M, K, N):
    """BASELINE shapes: bit-equal to the unpacked GEMM over the whole output (a size-independent
    property), sampled columns against the float64 reference, and the original tensors may be
    freed once the repack has completed."""
    G = 128
    ws = workspace(capi)
    x, qw, qz, sc = w4_device_inputs(M, K, N, G, seed=N)
    y0 = gemm(capi, ws, x, qw, qz, sc, K, N, G)
    pk = repack(capi, qw, qz, sc, K, N, G)
    torch.cuda.synchronize()
    cols = sample_columns(N, 300, seed=1)
    ref = w4_ref_sampled(x, qw, qz, sc, cols)
    del qw, qz, sc
    torch.cuda.empty_cache()
    y1 = gemm_packed(capi, ws, x, pk, K, N, G)
    assert torch.equal(y0, y1), f"{name}: {mismatch(y0, y1)}"
    check(y1[:, torch.from_numpy(cols).cuda()], ref, name)


def test_packed_graph_replay(capi, oracle):
    ws = workspace(capi)
    K, N, G = 2048, 1024, 128
    x, qw, qz, sc = oracle.gen_w4(4, K, N, G, seed=3)
    xd = dev(x)
    pk = repack(capi, dev(qw), dev(qz), dev(sc), K, N, G)
    y = torch.empty(4, N, dtype=torch.float16, device="cuda")
    lib = capi.lib()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            capi.check(lib.b2_w4_gemm_packed(xd.data_ptr(), pk.data_ptr(), y.data_ptr(), 4, K, N,
                                             G, ws.data_ptr(), ws.numel(), s.cuda_stream), "packed")
    torch.cuda.current_stream().wait_stream(s)
    x2, _, _, _ = oracle.gen_w4(4, K, N, G, seed=4)
    xd.copy_(dev(x2))
    g.replay()
    torch.cuda.synchronize()
    check(y, oracle.w4_ref(x2, qw, qz, sc), "graph replay")


def test_packed_rejects(capi):
    lib = capi.lib()
    assert lib.b2_w4_packed_bytes(100, 64, 128) == 0      # K % 128
    assert lib.b2_w4_packed_bytes(128, 48, 128) == 0      # N % 32
    assert lib.b2_w4_packed_bytes(384, 64, 96) == 0       # group size outside the contract
    K, N, G = 256, 64, 128
    t = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    p = t.data_ptr()
    need = lib.b2_w4_packed_bytes(K, N, G)
    assert lib.b2_w4_repack(p, p, p, K, N, G, p, need - 16, stream_ptr()) != 0   # too small
    assert lib.b2_w4_repack(p, p, p, K, N, G, p + 8, need, stream_ptr()) != 0    # misaligned
    assert lib.b2_w4_gemm_packed(p, 0, p, 1, K, N, G, p, t.numel(), stream_ptr()) != 0  # null


@pytest.mark.parametrize("M,K,N,G", [(8, 1024, 384, 128), (3, 256, 96, 32), (7, 4096, 4096, 128)])
def test_torch_ops_packed(ops, capi, oracle, M, K, N, G):
    """torch.ops.gfx906_skinny.w4_repack / w4gemm_packed: the same bytes as the C ABI and the same
    product as w4gemm, bit for bit."""
    x, qw, qz, sc = (dev(a) for a in oracle.gen_w4(M, K, N, G, seed=M * K + N))
    pk = ops.w4_repack(qw, qz, sc)
    assert pk.dtype == torch.uint8 and pk.numel() == capi.lib().b2_w4_packed_bytes(K, N, G)
    assert torch.equal(pk, repack(capi, qw, qz, sc, K, N, G))
    y = ops.w4gemm(x, qw, qz, sc, 0, 0)
    yp = ops.w4gemm_packed(x, pk, N, G)
    torch.cuda.synchronize()
    assert torch.equal(y, yp), mismatch(yp, y)


def test_torch_ops_packed_rejects(ops, oracle):
    x, qw, qz, sc = (dev(a) for a in oracle.gen_w4(2, 256, 64, 128, seed=5))
    pk = ops.w4_repack(qw, qz, sc)
    with pytest.raises(RuntimeError, match="needs"):
        ops.w4gemm_packed(x, pk[:-16], 64, 128)          # image shorter than K, N, G need
    with pytest.raises(RuntimeError, match="G=96 needs 0"):
        ops.w4gemm_packed(x, pk, 64, 96)                 # group size outside the contract
    with pytest.raises(RuntimeError, match="uint8"):
        ops.w4gemm_packed(x, pk.view(torch.int32), 64, 128)
    with pytest.raises(RuntimeError, match="qz must be"):
        ops.w4_repack(qw, qz[:, :4], sc)


FUSED = [(8, 1024, 384, 128), (5, 512, 256, 64), (3, 4096, 1024, 32), (8, 2176, 5120, 128)]


@pytest.fixture(scope="module")
def solo(capi):
    """One-rank all-reduce handle on device 0: the fused kernels run their whole epilogue."""
    lib = capi.lib()
    h = ctypes.c_void_p()
    capi.check(lib.b2_nvar_create(0, 0, 1, 8 * 8192 * 4, ctypes.byref(h)), "nvar_create")
    yield h
    torch.cuda.synchronize()
    capi.check(lib.b2_nvar_destroy(h), "nvar_destroy")


@pytest.mark.parametrize("path", [1, 2], ids=["stream-K", "cluster"])
@pytest.mark.parametrize("M,K,N,G", FUSED)
def test_fused_packed_equals_unpacked(capi, oracle, solo, path, M, K, N, G):
    """b2_w4_gemm_allreduce(_rmsnorm)_packed give the bits of the same calls on the original
    tensors: the output, and for the norm the normalised rows and the updated residual."""
    lib = capi.lib()
    saved = lib.b2_get_tuning(4)
    lib.b2_set_tuning(4, path)
    try:
        ws = workspace(capi)
        x, qw, qz, sc = oracle.gen_w4(M, K, N, G, seed=3 * M + K + N)
        xd, qwd, qzd, scd = dev(x), dev(qw), dev(qz), dev(sc)
        pk = repack(capi, qwd, qzd, scd, K, N, G)
        sp = stream_ptr()
        y0, y1 = (torch.empty(M, N, dtype=torch.float16, device="cuda") for _ in range(2))
        capi.check(lib.b2_w4_gemm_allreduce(solo, xd.data_ptr(), qwd.data_ptr(), qzd.data_ptr(),
                                            scd.data_ptr(), y0.data_ptr(), M, K, N, G,
                                            ws.data_ptr(), ws.numel(), sp), "w4_gemm_allreduce")
        capi.check(lib.b2_w4_gemm_allreduce_packed(solo, xd.data_ptr(), pk.data_ptr(),
                                                   y1.data_ptr(), M, K, N, G, ws.data_ptr(),
                                                   ws.numel(), sp), "w4_gemm_allreduce_packed")
        rng = np.random.default_rng(M + N)
        res = dev((rng.standard_normal((M, N)) * 4).astype(np.float16))
        w = dev((1.0 + rng.uniform(-0.3, 0.3, size=N)).astype(np.float16))
        r0, r1 = res.clone(), res.clone()
        o0, o1 = (torch.empty(M, N, dtype=torch.float16, device="cuda") for _ in range(2))
        capi.check(lib.b2_w4_gemm_allreduce_rmsnorm(
            solo, xd.data_ptr(), qwd.data_ptr(), qzd.data_ptr(), scd.data_ptr(), r0.data_ptr(),
            w.data_ptr(), 1e-6, o0.data_ptr(), M, K, N, G, ws.data_ptr(), ws.numel(), sp),
            "w4_gemm_allreduce_rmsnorm")
        capi.check(lib.b2_w4_gemm_allreduce_rmsnorm_packed(
            solo, xd.data_ptr(), pk.data_ptr(), r1.data_ptr(), w.data_ptr(), 1e-6, o1.data_ptr(),
            M, K, N, G, ws.data_ptr(), ws.numel(), sp), "w4_gemm_allreduce_rmsnorm_packed")
        torch.cuda.synchronize()
        assert torch.equal(y0, y1), mismatch(y1, y0)
        assert torch.equal(o0, o1), mismatch(o1, o0)
        assert torch.equal(r0, r1), mismatch(r1, r0)
        check(y1, oracle.w4_ref(x, qw, qz, sc), f"fused packed path {path} M={M} K={K} N={N}")
        st = ctypes.c_int()
        capi.check(lib.b2_nvar_status(solo, 1, ctypes.byref(st)), "nvar_status")
        assert st.value == 0
    finally:
        lib.b2_set_tuning(4, saved)


def test_torch_ops_fused_packed(ops, oracle):
    """w4gemm_ar_packed / w4gemm_ar_rmsnorm_packed on a one-rank handle from nvar_create equal
    w4gemm_ar / w4gemm_ar_rmsnorm on the original tensors."""
    M, K, N, G = 6, 2048, 3072, 128
    x, qw, qz, sc = (dev(a) for a in oracle.gen_w4(M, K, N, G, seed=21))
    name = f"/b2_test_packed_{os.getpid()}"
    h = ops.nvar_create(name, M * N * 4, 0, 1)
    ops.hostar_unlink(name)
    pk = ops.w4_repack(qw, qz, sc)
    assert torch.equal(ops.w4gemm_ar(x, qw, qz, sc, h), ops.w4gemm_ar_packed(x, pk, N, G, h))
    rng = np.random.default_rng(3)
    res = dev((rng.standard_normal((M, N)) * 4).astype(np.float16))
    w = dev((1.0 + rng.uniform(-0.3, 0.3, size=N)).astype(np.float16))
    r0, r1 = res.clone(), res.clone()
    o0 = ops.w4gemm_ar_rmsnorm(x, qw, qz, sc, h, r0, w, 1e-6)
    o1 = ops.w4gemm_ar_rmsnorm_packed(x, pk, N, G, h, r1, w, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(o0, o1), mismatch(o1, o0)
    assert torch.equal(r0, r1), mismatch(r1, r0)
    assert ops.nvar_status(h, True) == 0
    with pytest.raises(RuntimeError, match="needs"):
        ops.w4gemm_ar_packed(x, pk[:-16], N, G, h)
    with pytest.raises(RuntimeError, match="residual"):
        ops.w4gemm_ar_rmsnorm_packed(x, pk, N, G, h, r1[:, :-32].contiguous(), w, 1e-6)
