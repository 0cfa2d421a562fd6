"""Multi-rank all-reduce and fused GEMM epilogues on ONE GPU.

The reference proves its all-reduce with two processes on two GPUs (kernels/test_hostar.py):
random calls bit-identical to the collective, and a chain of calls captured in a CUDA graph. This
file runs the same protocol code with 2 and 3 ranks on one GPU: the ranks' handles live in one
process and are connected to one another's buffers (b2_nvar_connect_local), and one cooperative
launch runs every rank's CTAs (grid.y = rank). Each rank has its own operands, workspace and
all-reduce buffer, so the kernels take exactly the multi-rank code paths: the pushes into every
rank's slots, the fp32 flag protocol, the 64-bit (generation, value) exchange of both split-K
kernels, and the grid-wide barrier of the residual add + RMSNorm epilogue. Checks: the fixed
rank-order fp32 sum of the oracle (kernels/hostar.cu:107) bit for bit, bit-identity across ranks,
the float64 GEMM oracle within the tolerance of the other tests, and CUDA-graph replay.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from gpu_util import check, dev, mismatch, stream_ptr, workspace

pytestmark = pytest.mark.gpu

EPS = 1e-6
TIMEOUT_NS = 2_000_000_000  # a protocol mistake ends in B2_ERR_TIMEOUT after 2 s, never a hang


class Group:
    """`ranks` all-reduce handles on device 0, connected to one another."""

    def __init__(self, capi, ranks: int, slot_bytes: int):
        self.capi, self.lib, self.ranks = capi, capi.lib(), ranks
        self.h = []
        for r in range(ranks):
            h = C.c_void_p()
            capi.check(self.lib.b2_nvar_create(0, r, ranks, slot_bytes, C.byref(h)), "nvar_create")
            capi.check(self.lib.b2_nvar_set_timeout_ns(h, TIMEOUT_NS), "nvar_set_timeout_ns")
            self.h.append(h)
        self.arr = (C.c_void_p * ranks)(*[h.value for h in self.h])
        capi.check(self.lib.b2_nvar_connect_local(self.arr, ranks), "nvar_connect_local")
        for h in self.h:
            assert self.lib.b2_nvar_is_connected(h) == 1

    def status(self):
        out = []
        for h in self.h:
            st = C.c_int()
            self.capi.check(self.lib.b2_nvar_status(h, 0, C.byref(st)), "nvar_status")
            out.append(st.value)
        return out

    def close(self):
        torch.cuda.synchronize()
        for h in self.h:
            self.capi.check(self.lib.b2_nvar_destroy(h), "nvar_destroy")


def allreduce(g: Group, ins, outs, dtype_code):
    p = g.capi.ptr_array
    g.capi.check(g.lib.b2_nvar_allreduce_emulated(
        g.arr, g.ranks, p([t.data_ptr() for t in ins]), p([t.data_ptr() for t in outs]),
        ins[0].numel(), dtype_code, stream_ptr()), "nvar_allreduce_emulated")


def fused(g: Group, xs, ws_, ys, M, K, N, G, wss, residuals=None, nws=None):
    p = g.capi.ptr_array
    g.capi.check(g.lib.b2_w4_gemm_allreduce_emulated(
        g.arr, g.ranks, p([x.data_ptr() for x in xs]), p([w[0].data_ptr() for w in ws_]),
        p([w[1].data_ptr() for w in ws_]), p([w[2].data_ptr() for w in ws_]),
        p([r.data_ptr() for r in residuals]) if residuals else None,
        p([w.data_ptr() for w in nws]) if nws else None, EPS,
        p([y.data_ptr() for y in ys]), M, K, N, G, p([w.data_ptr() for w in wss]),
        wss[0].numel(), stream_ptr()), "w4_gemm_allreduce_emulated")


def test_world1_allreduce_is_identity(capi, ops):
    """A one-rank handle: the sum over one rank is the input itself, fp16 and fp32, through the
    C ABI and through the torch operator (nvar_create with world 1)."""
    lib = capi.lib()
    h = C.c_void_p()
    capi.check(lib.b2_nvar_create(0, 0, 1, 1 << 18, C.byref(h)), "nvar_create")
    try:
        g = torch.Generator(device="cuda").manual_seed(3)
        for n, dt, code in ((40960, torch.float16, 0), (64, torch.float16, 0),
                            (65536, torch.float32, 1), (5120, torch.float32, 1)):
            x = torch.randn(n, device="cuda", generator=g, dtype=dt) * 30
            y = torch.full_like(x, float("nan"))
            capi.check(lib.b2_nvar_allreduce(h, x.data_ptr(), y.data_ptr(), n, code, stream_ptr()),
                       "nvar_allreduce")
            torch.cuda.synchronize()
            assert torch.equal(x, y), f"n={n} {dt}"
        st = C.c_int()
        capi.check(lib.b2_nvar_status(h, 0, C.byref(st)), "nvar_status")
        assert st.value == 0
    finally:
        torch.cuda.synchronize()
        lib.b2_nvar_destroy(h)
    name = "/b2_test_world1"
    th = ops.nvar_create(name, 1 << 17, 0, 1)
    ops.hostar_unlink(name)
    x = torch.randn(8 * 5120, device="cuda", dtype=torch.float16)
    assert torch.equal(ops.nvar_allreduce(x, th), x)
    assert ops.nvar_status(th, False) == 0


@pytest.mark.parametrize("ranks", [2, 3])
def test_emulated_allreduce_random_calls(capi, oracle, ranks):
    """Random calls cycling the reference's sizes and dtypes (kernels/test_hostar.py:11-22): every
    rank's output equals the rank-order fp32 sum of the oracle bit for bit, on every rank."""
    g = Group(capi, ranks, 65536 * 4)
    try:
        rng = np.random.default_rng(100 + ranks)
        for it in range(60):
            n = [8 * 5120, 5120, 2 * 5120, 64, 65536][it % 5]
            f16 = it % 7 != 0
            dt = np.float16 if f16 else np.float32
            ins_np = [(rng.standard_normal(n) * 10.0 ** (it % 4 - 1)).astype(dt) for _ in range(ranks)]
            ins = [dev(a) for a in ins_np]
            outs = [torch.full_like(t, float("nan")) for t in ins]
            allreduce(g, ins, outs, 0 if f16 else 1)
            torch.cuda.synchronize()
            ref = oracle.allreduce_ref(ins_np)
            for r in range(ranks):
                got = outs[r].cpu().numpy()
                assert np.array_equal(got.view(np.uint8), ref.view(np.uint8)), \
                    f"call {it}, rank {r}, n={n}, {dt.__name__}: {(got != ref).sum()} elements differ"
        assert g.status() == [0] * ranks
    finally:
        g.close()


def test_emulated_allreduce_graph_chain(capi, oracle):
    """A chain of all-reduces, each output halved and fed to the next, captured in one CUDA graph
    and replayed (the reference's graph test, kernels/test_hostar.py:31-48): the device generation
    counter keeps the parity slots straight across replays."""
    ranks, n, steps = 2, 8 * 5120, 12
    g = Group(capi, ranks, n * 4)
    try:
        rng = np.random.default_rng(9)
        x0 = [rng.standard_normal(n).astype(np.float16) for _ in range(ranks)]
        bufs = [dev(a) for a in x0]
        outs = [torch.empty_like(b) for b in bufs]

        def chain():
            for _ in range(steps):
                allreduce(g, bufs, outs, 0)
                for r in range(ranks):
                    bufs[r].copy_(outs[r] * 0.5)

        ref = [a.copy() for a in x0]
        for _ in range(steps):
            s = oracle.allreduce_ref(ref)
            ref = [(s.astype(np.float32) * np.float32(0.5)).astype(np.float16) for _ in range(ranks)]
        chain()
        torch.cuda.synchronize()
        eager = [b.clone() for b in bufs]
        for r in range(ranks):
            assert np.array_equal(eager[r].cpu().numpy(), ref[r])
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for r in range(ranks):
                bufs[r].copy_(dev(x0[r]))
            with torch.cuda.graph(graph, stream=s):
                chain()
        torch.cuda.current_stream().wait_stream(s)
        for rep in range(3):
            for r in range(ranks):
                bufs[r].copy_(dev(x0[r]))
            graph.replay()
            torch.cuda.synchronize()
            for r in range(ranks):
                assert torch.equal(bufs[r], eager[r]), f"replay {rep}, rank {r}"
        del graph
        assert g.status() == [0] * ranks
    finally:
        g.close()


def shard_inputs(oracle, ranks, M, K, N, G, seed):
    """Full-K inputs and their K-shards (row-parallel layer: rank r owns k in [r K/P, (r+1) K/P))."""
    x, qw, qz, sc = oracle.gen_w4(M, K, N, G, seed=seed)
    ks = K // ranks
    shards = []
    for r in range(ranks):
        shards.append((dev(x[:, r * ks:(r + 1) * ks]),
                       (dev(qw[r * ks // 8:(r + 1) * ks // 8]), dev(qz[r * ks // G:(r + 1) * ks // G]),
                        dev(sc[r * ks // G:(r + 1) * ks // G]))))
    return (x, qw, qz, sc), shards


# (path, low-latency exchange): path 0 = the planner's choice, 1 = stream-K, 2 = clusters. The
# fp32 partials travel as 64-bit (generation, value) words, or (B2_TUNE_AR_FLAGS) as fp32 values
# published by per-tile flags.
VARIANTS = [(0, True), (1, True), (2, True), (1, False), (2, False)]


@pytest.mark.parametrize("ranks", [2, 3, 4])
@pytest.mark.parametrize("two_shot", [1, 2], ids=["two-shot", "one-shot"])
def test_emulated_fused_exchange_forms(capi, oracle, ranks, two_shot):
    """The cluster kernel's two exchange forms (B2_TUNE_AR_TWO_SHOT): one-shot, where every rank
    adds every rank's partials, and two-shot, where each tile's owner rank adds them and sends the
    rounded result back. Same bits on every rank, within tolerance of the float64 oracle, and the
    two forms give the same bits (the owner adds in the same rank order)."""
    lib = capi.lib()
    M, N, G = 8, 5120, 128
    K = 2176 * ranks
    saved = lib.b2_get_tuning(7)
    g = Group(capi, ranks, M * N * 8)
    try:
        full, shards = shard_inputs(oracle, ranks, M, K, N, G, seed=ranks * 7)
        wss = [workspace(capi) for _ in range(ranks)]
        outs = {}
        for form in (two_shot, 3 - two_shot):
            lib.b2_set_tuning(7, form)
            ys = [torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
                  for _ in range(ranks)]
            for _ in range(2):
                fused(g, [s[0] for s in shards], [s[1] for s in shards], ys, M, K // ranks, N, G, wss)
            torch.cuda.synchronize()
            for r in range(1, ranks):
                assert torch.equal(ys[0], ys[r]), f"form {form} rank {r}: {mismatch(ys[0], ys[r])}"
            check(ys[0], oracle.w4_ref(*full), f"form {form}, {ranks} ranks")
            outs[form] = ys[0]
        assert torch.equal(outs[1], outs[2]), mismatch(outs[1], outs[2])
        assert g.status() == [0] * ranks
    finally:
        lib.b2_set_tuning(7, saved)
        g.close()


@pytest.mark.parametrize("path,ll", VARIANTS, ids=[f"path{p}-{'ll' if l else 'flags'}" for p, l in VARIANTS])
@pytest.mark.parametrize("M,K,N,G", [(8, 4352, 5120, 128), (3, 2048, 1024, 64), (5, 1024, 352, 32)])
def test_emulated_fused_gemm_allreduce(capi, oracle, path, ll, M, K, N, G):
    """The row-parallel layer at 2 ranks: every rank gets the same fp16 result bit for bit, within
    the tolerance of the float64 oracle of the whole K; the same call again gives the same bits."""
    ranks = 2
    lib = capi.lib()
    if path == 2 and N % 128:
        pytest.skip("the fused cluster kernel needs whole 128-column tiles")
    saved = (lib.b2_get_tuning(4), lib.b2_get_tuning(6))
    lib.b2_set_tuning(4, path)
    lib.b2_set_tuning(6, 0 if ll else 1)
    g = Group(capi, ranks, M * N * 8)
    try:
        full, shards = shard_inputs(oracle, ranks, M, K, N, G, seed=M * 31 + K + N)
        wss = [workspace(capi) for _ in range(ranks)]
        ref = oracle.w4_ref(*full)
        prev = None
        for call in range(2):
            ys = [torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
                  for _ in range(ranks)]
            fused(g, [s[0] for s in shards], [s[1] for s in shards], ys, M, K // ranks, N, G, wss)
            torch.cuda.synchronize()
            for r in range(1, ranks):
                assert torch.equal(ys[0], ys[r]), f"rank {r} differs: {mismatch(ys[0], ys[r])}"
            check(ys[0], ref, f"fused {ranks} ranks path {path} ll {ll}")
            if prev is not None:
                assert torch.equal(prev, ys[0]), f"not deterministic: {mismatch(prev, ys[0])}"
            prev = ys[0]
        assert g.status() == [0] * ranks
        for w in wss:
            st = C.c_int()
            capi.check(lib.b2_workspace_status(w.data_ptr(), 0, C.byref(st)), "workspace_status")
            assert st.value == 0
    finally:
        lib.b2_set_tuning(4, saved[0])
        lib.b2_set_tuning(6, saved[1])
        g.close()


@pytest.mark.parametrize("path", [1, 2], ids=["stream-K", "cluster"])
@pytest.mark.parametrize("ranks", [2, 3])
def test_emulated_fused_rmsnorm(capi, oracle, path, ranks):
    """The layer followed by the residual add + RMSNorm at several ranks: the grid-wide barrier and
    the row sums run on every rank; the new residual is fp16(y + residual) of the plain fused
    output bit for bit, the normalised rows within two fp16 ulps of the oracle, and every rank
    holds the same bits."""
    lib = capi.lib()
    M, N, G = 8, 5120, 128
    K = 768 * ranks
    saved = lib.b2_get_tuning(4)
    lib.b2_set_tuning(4, path)
    g = Group(capi, ranks, M * N * 8)
    try:
        full, shards = shard_inputs(oracle, ranks, M, K, N, G, seed=ranks * 13 + path)
        wss = [workspace(capi) for _ in range(ranks)]
        xs, wts = [s[0] for s in shards], [s[1] for s in shards]
        y_plain = [torch.empty(M, N, dtype=torch.float16, device="cuda") for _ in range(ranks)]
        fused(g, xs, wts, y_plain, M, K // ranks, N, G, wss)
        rng = np.random.default_rng(5)
        res0 = (rng.standard_normal((M, N)) * 4).astype(np.float16)
        w = (1.0 + rng.uniform(-0.3, 0.3, size=N)).astype(np.float16)
        res = [dev(res0) for _ in range(ranks)]
        nw = [dev(w) for _ in range(ranks)]
        out = [torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda") for _ in range(ranks)]
        fused(g, xs, wts, out, M, K // ranks, N, G, wss, residuals=res, nws=nw)
        torch.cuda.synchronize()
        assert g.status() == [0] * ranks
        yp = y_plain[0].cpu().numpy()
        ref_out, ref_res = oracle.add_rmsnorm_ref(yp, res0, w, EPS)
        for r in range(ranks):
            assert torch.equal(y_plain[0], y_plain[r])
            assert torch.equal(out[0], out[r]), f"rank {r}: {mismatch(out[0], out[r])}"
            assert torch.equal(res[0], res[r])
        got_res = res[0].cpu().numpy()
        assert np.array_equal(got_res.view(np.int16), ref_res.view(np.int16))
        ulp = oracle.fp16_ulp_distance(out[0].cpu().numpy(), ref_out)
        assert ulp.max() <= 2 and float((ulp == 0).mean()) >= 0.99, ulp.max()
    finally:
        lib.b2_set_tuning(4, saved)
        g.close()


def test_emulated_fused_graph_replay(capi, oracle):
    """Two fused layers at 2 ranks captured in one CUDA graph and replayed: the results equal the
    eager ones on every replay (generation and parity of the exchange carried on the device)."""
    ranks, M, K, N, G = 2, 8, 2 * 2176, 5120, 128
    g = Group(capi, ranks, M * N * 8)
    try:
        full, shards = shard_inputs(oracle, ranks, M, K, N, G, seed=21)
        wss = [workspace(capi) for _ in range(ranks)]
        xs, wts = [s[0] for s in shards], [s[1] for s in shards]
        ys = [torch.empty(M, N, dtype=torch.float16, device="cuda") for _ in range(ranks)]
        ys2 = [torch.empty(M, N, dtype=torch.float16, device="cuda") for _ in range(ranks)]

        def two_layers():
            fused(g, xs, wts, ys, M, K // ranks, N, G, wss)
            fused(g, xs, wts, ys2, M, K // ranks, N, G, wss)

        two_layers()
        torch.cuda.synchronize()
        eager = ys[0].clone()
        check(eager, oracle.w4_ref(*full), "eager")
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                two_layers()
        torch.cuda.current_stream().wait_stream(s)
        for rep in range(3):
            for y in ys + ys2:
                y.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            for r in range(ranks):
                assert torch.equal(ys[r], eager) and torch.equal(ys2[r], eager), f"replay {rep} rank {r}"
        del graph
        assert g.status() == [0] * ranks
    finally:
        g.close()


def test_emulated_rejects_unconnected_and_mismatched(capi):
    """Host-side checks: handles of another world size, or not connected, are refused before any
    launch."""
    lib = capi.lib()
    h = [C.c_void_p(), C.c_void_p()]
    capi.check(lib.b2_nvar_create(0, 0, 2, 4096, C.byref(h[0])), "nvar_create")
    capi.check(lib.b2_nvar_create(0, 1, 3, 4096, C.byref(h[1])), "nvar_create")
    try:
        arr = (C.c_void_p * 2)(h[0].value, h[1].value)
        assert lib.b2_nvar_connect_local(arr, 2) == capi.B2_ERR_INVALID_ARG
        x = torch.zeros(1024, dtype=torch.float16, device="cuda")
        p = capi.ptr_array([x.data_ptr(), x.data_ptr()])
        rc = lib.b2_nvar_allreduce_emulated(arr, 2, p, p, 1024, 0, stream_ptr())
        assert rc == capi.B2_ERR_STATE  # not connected
    finally:
        for hh in h:
            lib.b2_nvar_destroy(hh)
