"""W4A16 skinny GEMM on the GPU against the float64 dequantize-then-matmul oracle
(kernels/check_w4.py:11-21), on the golden fixtures, the benchmark configurations and edge cases."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from gpu_util import (check, dev, mismatch, sample_columns, stream_ptr, w4_device_inputs,
                      w4_ref_sampled, workspace)

pytestmark = pytest.mark.gpu


def run(ops, x, qw, qz, sc):
    return ops.w4gemm(x, qw, qz, sc, 128, 14)


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("w4_*.npz")), ids=lambda p: p.stem)
def test_golden(ops, oracle, path):
    d = np.load(path)
    y = run(ops, dev(d["x"]), dev(d["qw"]), dev(d["qz"]), dev(d["sc"]))
    check(y, d["ref"], path.stem)


@pytest.mark.parametrize("G", [32, 64, 128, 256])
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 6, 7, 8])
def test_groups_and_rows(ops, oracle, G, M):
    K, N = 1024, 384
    x, qw, qz, sc = oracle.gen_w4(M, K, N, G, seed=G * 10 + M)
    y = run(ops, dev(x), dev(qw), dev(qz), dev(sc))
    assert y.shape == (M, N) and y.dtype == torch.float16
    check(y, oracle.w4_ref(x, qw, qz, sc), f"G={G} M={M}")


@pytest.mark.parametrize("K,N", [(128, 32), (256, 96), (640, 160), (2176, 5120), (384, 4128)])
def test_ragged_shapes(ops, oracle, K, N):
    x, qw, qz, sc = oracle.gen_w4(5, K, N, 128 if K % 128 == 0 else 32, seed=K + N)
    check(run(ops, dev(x), dev(qw), dev(qz), dev(sc)), oracle.w4_ref(x, qw, qz, sc), f"{K}x{N}")


@pytest.mark.parametrize("path,cs", [(1, 0), (2, 0), (2, 1), (2, 3), (2, 8), (2, 16)],
                         ids=["stream-K", "cluster-auto", "cluster-1", "cluster-3", "cluster-8",
                              "cluster-16"])
@pytest.mark.parametrize("M,K,N,G", [(8, 2176, 5120, 128), (3, 5120, 992, 128), (8, 4096, 1056, 32),
                                     (1, 2048, 4128, 64)])
def test_split_k_paths(capi, ops, oracle, path, cs, M, K, N, G):
    """Both split-K kernels (stream-K with a global fix-up; thread-block clusters reducing
    through distributed shared memory) and several cluster sizes, forced with B2_TUNE_W4_PATH /
    B2_TUNE_W4_CLUSTER, against the oracle; ragged N (partial last tile) included. A cluster
    size the shape cannot use (more CTAs than k-units) falls back to stream-K."""
    lib = capi.lib()
    saved = (lib.b2_get_tuning(4), lib.b2_get_tuning(5))
    lib.b2_set_tuning(4, path)
    lib.b2_set_tuning(5, cs)
    try:
        x, qw, qz, sc = oracle.gen_w4(M, K, N, G, seed=M * 7 + K + N + cs)
        y = run(ops, dev(x), dev(qw), dev(qz), dev(sc))
        check(y, oracle.w4_ref(x, qw, qz, sc), f"path {path} cs {cs} M={M} K={K} N={N} G={G}")
        y2 = run(ops, dev(x), dev(qw), dev(qz), dev(sc))
        assert torch.equal(y, y2), f"not deterministic: {mismatch(y, y2)}"
        assert ops.workspace_status(False) == 0
    finally:
        lib.b2_set_tuning(4, saved[0])
        lib.b2_set_tuning(5, saved[1])


def test_config0(ops, oracle):
    """M=7, K=N=4096, G=128, raw max abs error <= 1e-2 as well."""
    x, qw, qz, sc = oracle.gen_w4(7, 4096, 4096, 128, seed=0)
    y = run(ops, dev(x), dev(qw), dev(qz), dev(sc))
    st = check(y, oracle.w4_ref(x, qw, qz, sc), "config 0")
    assert st["max_abs"] <= 1e-2, st


@pytest.mark.parametrize("M", [1, 4, 8])
def test_check_w4_fixture_shape(ops, oracle, M):
    """The reference's own check (kernels/check_w4.py:7-26): K=5120, N=1024, G=32,
    scales rand*0.02+0.001, x = randn*0.5 - reported there as max error / max |ref|."""
    g = torch.Generator(device="cuda").manual_seed(1)
    K, N, G = 5120, 1024, 32
    qw = torch.randint(-2**31, 2**31 - 1, (K // 8, N), device="cuda", dtype=torch.int32, generator=g)
    qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), device="cuda", dtype=torch.int32, generator=g)
    sc = (torch.rand(K // G, N, device="cuda", generator=g) * 0.02 + 0.001).half()
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.5).half()
    y = run(ops, x, qw, qz, sc)
    ref = oracle.w4_ref(x.cpu().numpy(), qw.cpu().numpy(), qz.cpu().numpy(), sc.cpu().numpy())
    check(y, ref, f"check_w4 M={M}")
    rel = float(np.abs(y.double().cpu().numpy() - ref).max() / np.abs(ref).max())
    assert rel < 2e-3, rel


LAYERS = {"qkv_proj": (5120, 8192, 31), "o_proj": (6144, 5120, 32), "gate_up": (5120, 34816, 33),
          "down_proj": (17408, 5120, 34)}


@pytest.mark.parametrize("M", [1, 8])
@pytest.mark.parametrize("layer", list(LAYERS))
def test_config2_layers_sampled(ops, layer, M):
    """BASELINE config 2 (decoder-layer sweep, G=128), checked on sampled columns."""
    K, N, seed = LAYERS[layer]
    x, qw, qz, sc = w4_device_inputs(M, K, N, 128, seed=seed * 10 + M)
    y = run(ops, x, qw, qz, sc)
    assert torch.isfinite(y).all()
    cols = sample_columns(N, 300, seed=M)
    check(y[:, torch.from_numpy(cols).cuda()], w4_ref_sampled(x, qw, qz, sc, cols), layer)
    assert torch.equal(y, run(ops, x, qw, qz, sc)), "not deterministic"


def test_weights_written_by_the_previous_kernel(ops):
    """Packed weights produced by the kernel launched just before the GEMM (no host sync in
    between) are read in full; every call is compared with a repeat made after a sync."""
    M, K, N = 8, 5120, 8192
    x, qw, qz, sc = w4_device_inputs(M, K, N, 128, seed=11)
    outs = []
    for i in range(8):
        qwi = qw ^ (0x11111111 * i)  # the kernel right before the GEMM writes the weights
        outs.append((run(ops, x, qwi, qz, sc), qwi))
    torch.cuda.synchronize()
    for i, (y, qwi) in enumerate(outs):
        y_again = run(ops, x, qwi, qz, sc)
        assert torch.equal(y, y_again), f"call {i}: {mismatch(y, y_again)}"


@pytest.mark.parametrize("P", [2, 4, 8])
def test_config3_shard_sum(ops, oracle, P):
    """BASELINE config 3 on one GPU: the K-shards' GEMMs summed in rank order match the full
    down_proj GEMM (linearity of the split), and each shard matches the oracle."""
    K, N, M = 17408, 5120, 8
    x, qw, qz, sc = w4_device_inputs(M, K, N, 128, seed=P)
    full = run(ops, x, qw, qz, sc).float()
    ks = K // P
    acc = torch.zeros(M, N, device="cuda")
    cols = sample_columns(N, 128, seed=P)
    parts = []
    for r in range(P):
        xs = x[:, r * ks:(r + 1) * ks].contiguous()
        qws = qw[r * ks // 8:(r + 1) * ks // 8].contiguous()
        qzs = qz[r * ks // 128:(r + 1) * ks // 128].contiguous()
        scs = sc[r * ks // 128:(r + 1) * ks // 128].contiguous()
        ys = run(ops, xs, qws, qzs, scs)
        if r == 0:
            check(ys[:, torch.from_numpy(cols).cuda()], w4_ref_sampled(xs, qws, qzs, scs, cols), "shard")
        acc += ys.float()
        parts.append(ys.float().cpu().numpy())
    # each shard's and the full output's fp16 rounding bound the difference
    bound = sum(oracle.fp16_half_ulp(p) for p in parts) + oracle.fp16_half_ulp(full.cpu().numpy())
    assert ((acc - full).abs().cpu().numpy() <= bound + 1e-3).all()


def test_capi_nan_prefilled_and_graph(capi, ops, oracle):
    lib = capi.lib()
    ws = workspace(capi)
    M, K, N, G = 8, 2048, 1056, 64
    x, qw, qz, sc = oracle.gen_w4(M, K, N, G, seed=5)
    xd, qwd, qzd, scd = dev(x), dev(qw), dev(qz), dev(sc)
    y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    rc = lib.b2_w4_gemm(xd.data_ptr(), qwd.data_ptr(), qzd.data_ptr(), scd.data_ptr(), y.data_ptr(),
                        M, K, N, G, ws.data_ptr(), ws.numel(), stream_ptr())
    capi.check(rc, "b2_w4_gemm")
    ref = oracle.w4_ref(x, qw, qz, sc)
    check(y, ref, "capi")
    # graph capture through the torch op, replayed with new activations
    y0 = run(ops, xd, qwd, qzd, scd)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            yg = run(ops, xd, qwd, qzd, scd)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(yg, y0)
    x2 = oracle.gen_w4(M, K, 8, G, seed=6)[0]
    xd.copy_(dev(x2))
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    check(yg, oracle.w4_ref(x2, qw, qz, sc), "graph replay")
    assert ops.workspace_status(False) == 0


def test_vllm_shim_routes(pkg, oracle):
    from mi50_vllm_lab_b200 import vllm_shim

    x, qw, qz, sc = oracle.gen_w4(4, 512, 256, 128, seed=8)
    y = vllm_shim.w4_skinny(dev(x), dev(qw), dev(qz), dev(sc))
    check(y, oracle.w4_ref(x, qw, qz, sc), "shim")
    assert vllm_shim.w4_skinny(dev(x[:, :500].copy()), dev(qw), dev(qz), dev(sc)) is None
    xf, w = oracle.gen_f16(3, 256, 1200, seed=9)
    y = vllm_shim.skinny8(dev(xf).reshape(1, 3, 256), dev(w))
    assert y.shape == (1, 3, 1200)
    check(y.reshape(3, 1200), oracle.gemm_ref(xf, w), "skinny8")
    assert vllm_shim.skinny8(torch.zeros(9, 256, dtype=torch.float16, device="cuda"), dev(w)) is None


def test_rejects_bad_inputs(ops):
    a = torch.zeros(4, 512, dtype=torch.float16, device="cuda")
    qw = torch.zeros(64, 256, dtype=torch.int32, device="cuda")
    qz = torch.zeros(4, 32, dtype=torch.int32, device="cuda")
    sc = torch.zeros(4, 256, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        ops.w4gemm(a, qw[:32], qz, sc, 128, 14)     # qw rows != K/8
    with pytest.raises(RuntimeError):
        ops.w4gemm(a, qw, qz[:, :16], sc, 128, 14)  # qz cols != N/8
    with pytest.raises(RuntimeError):
        ops.w4gemm(a, qw, qz[:3], sc[:3], 128, 14)  # K % G
    with pytest.raises(RuntimeError):
        ops.w4gemm(torch.zeros(9, 512, dtype=torch.float16, device="cuda"), qw, qz, sc, 128, 14)


@pytest.mark.parametrize("M,K,N", [(8, 5120, 34816), (8, 17408, 5120), (7, 4096, 4096), (3, 2176, 5120),
                                   (1, 5120, 1024)])
def test_cluster_aliased_buffers_same_bits(capi, ops, M, K, N):
    """With one tile per cluster and long k-ranges the cluster kernel keeps its reduction buffers
    on the drained stage ring and runs five stages; B2_TUNE_W4_NO_ALIAS keeps them apart (four
    stages); forced to one cluster size so that both layouts run on every shape here. Same
    sums in the same order, so the outputs must be identical, and sampled columns match the
    float64 reference."""
    lib = capi.lib()
    saved = lib.b2_get_tuning(8)
    x, qw, qz, sc = w4_device_inputs(M, K, N, 128, seed=K + N)
    saved_cs = lib.b2_get_tuning(5)
    try:
        lib.b2_set_tuning(5, 1)  # clusters of one CTA: every CTA has the whole k-range
        lib.b2_set_tuning(8, 0)
        y_alias = run(ops, x, qw, qz, sc)
        y_alias2 = run(ops, x, qw, qz, sc)
        lib.b2_set_tuning(8, 1)
        y_apart = run(ops, x, qw, qz, sc)
    finally:
        lib.b2_set_tuning(8, saved)
        lib.b2_set_tuning(5, saved_cs)
    assert torch.equal(y_alias, y_alias2), mismatch(y_alias, y_alias2)
    assert torch.equal(y_alias, y_apart), mismatch(y_alias, y_apart)
    cols = sample_columns(N, 200, seed=2)
    check(y_alias[:, torch.from_numpy(cols).cuda()], w4_ref_sampled(x, qw, qz, sc, cols), f"{M}x{K}x{N}")
    assert ops.workspace_status(False) == 0
