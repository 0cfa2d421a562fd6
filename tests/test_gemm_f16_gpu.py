"""fp16 skinny GEMM on the GPU against the oracle (kernels/bench_skinny.py:44 in float64)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from gpu_util import check, dev, f16_ref_sampled, mismatch, sample_columns, stream_ptr, workspace

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("f16_*.npz")), ids=lambda p: p.stem)
def test_golden(ops, oracle, path):
    d = np.load(path)
    y = ops.gemm(dev(d["x"]), dev(d["w"]), 20)
    check(y, d["ref"].astype(np.float64), path.stem)
    check(y, oracle.gemm_ref(d["x"], d["w"]), path.stem)


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("K,N", [(512, 1000), (5120, 1387), (1032, 128), (64, 129), (8, 7),
                                 (4096, 256), (2056, 300)])
def test_shapes(ops, oracle, M, K, N):
    x, w = oracle.gen_f16(M, K, N, seed=M * 1000 + K + N)
    y = ops.gemm(dev(x), dev(w), 0)
    assert y.shape == (M, N) and y.dtype == torch.float16
    check(y, oracle.gemm_ref(x, w), f"M={M} K={K} N={N}")


def test_config1_lm_head_sampled_columns(ops):
    """M=7, K=5120, N=151936 (1.56 GB of weights)."""
    g = torch.Generator(device="cuda").manual_seed(101)
    M, K, N = 7, 5120, 151936
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    y = ops.gemm(x, w, 20)
    assert torch.isfinite(y).all()
    cols = sample_columns(N, 1500, seed=5)
    check(y[:, torch.from_numpy(cols).cuda()], f16_ref_sampled(x, w, cols), "config 1")
    y2 = ops.gemm(x, w, 20)
    assert torch.equal(y, y2), f"not deterministic: {mismatch(y, y2)}"
    del w


# The drafter layers the reference times (kernels/bench_skinny.py:34-37), as (N, K), at its row
# counts (kernels/bench_skinny.py:12: 1, 3, 4, 7, 8).
DRAFTER = {"dr_qkv": (3072, 5120), "dr_o": (5120, 2048), "dr_gate_up": (17408, 5120),
           "dr_down": (5120, 8704), "dr_fc": (5120, 25600), "dr_ctx_kv": (5120, 5120),
           "dr_kproj": (1280, 5120)}


@pytest.mark.parametrize("M", [1, 3, 4, 7, 8])
@pytest.mark.parametrize("layer", list(DRAFTER))
def test_drafter_shapes(ops, layer, M):
    """Every drafter shape of the reference's fp16 benchmark, with its weights N(0, 0.02) and
    activations N(0, 1) (kernels/bench_skinny.py:41-43), checked on sampled columns against the
    float64 oracle, and deterministic."""
    N, K = DRAFTER[layer]
    g = torch.Generator(device="cuda").manual_seed(N + K + M)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    y = ops.gemm(x, w, 20)
    assert y.shape == (M, N) and torch.isfinite(y).all()
    cols = sample_columns(N, 400, seed=M)
    check(y[:, torch.from_numpy(cols).cuda()], f16_ref_sampled(x, w, cols), f"{layer} M={M}")
    assert torch.equal(y, ops.gemm(x, w, 20)), "not deterministic"


def test_weights_written_by_the_previous_kernel(ops):
    """Weights produced by the kernel launched just before the GEMM (no host sync in between)
    are read in full: the early start of the GEMM's CTAs must not read them before that
    kernel's stores have landed. Every call is compared with a repeat made after a sync."""
    g = torch.Generator(device="cuda").manual_seed(7)
    M, K, N = 8, 5120, 16384
    x = torch.randn(M, K, device="cuda", generator=g).half()
    base = torch.randn(N, K, device="cuda", generator=g)
    outs = []
    for i in range(8):
        w = (base * (0.02 + 0.001 * i)).half()  # the kernel right before the GEMM writes w
        outs.append((ops.gemm(x, w, 0), w))
    torch.cuda.synchronize()
    for i, (y, w) in enumerate(outs):
        y_again = ops.gemm(x, w, 0)
        assert torch.equal(y, y_again), f"call {i}: {mismatch(y, y_again)}"


def test_capi_nan_prefilled_output(capi, oracle):
    """Through the C ABI with a NaN-filled output: every element must be written."""
    lib = capi.lib()
    ws = workspace(capi)
    for M, K, N in [(8, 1024, 777), (3, 5120, 4096)]:
        x, w = oracle.gen_f16(M, K, N, seed=N)
        xd, wd = dev(x), dev(w)
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        rc = lib.b2_gemm_f16(xd.data_ptr(), wd.data_ptr(), y.data_ptr(), M, K, N, ws.data_ptr(),
                             ws.numel(), stream_ptr())
        capi.check(rc, "b2_gemm_f16")
        check(y, oracle.gemm_ref(x, w), "capi")
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 0


def test_deterministic_and_graph_replay(ops, oracle):
    x, w = oracle.gen_f16(8, 4096, 6000, seed=77)
    xd, wd = dev(x), dev(w)
    y0 = ops.gemm(xd, wd, 20)
    assert torch.equal(y0, ops.gemm(xd, wd, 20))
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            yg = ops.gemm(xd, wd, 20)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(yg, y0)
    # new activations through the same graph
    x2, _ = oracle.gen_f16(8, 4096, 1, seed=78)
    xd.copy_(dev(x2))
    g.replay()
    torch.cuda.synchronize()
    check(yg, oracle.gemm_ref(x2, w), "graph replay")
    assert ops.workspace_status(False) == 0


def test_rejects_bad_inputs(ops):
    x = torch.zeros(9, 64, dtype=torch.float16, device="cuda")
    w = torch.zeros(128, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        ops.gemm(x, w, 0)  # M = 9
    with pytest.raises(RuntimeError):
        ops.gemm(x[:4].float(), w, 0)  # dtype
    with pytest.raises(RuntimeError):
        ops.gemm(torch.zeros(4, 60, dtype=torch.float16, device="cuda"),
                 torch.zeros(128, 60, dtype=torch.float16, device="cuda"), 0)  # K % 8
    with pytest.raises(RuntimeError):
        ops.gemm(x[:4], w[:, :32], 0)  # K mismatch
