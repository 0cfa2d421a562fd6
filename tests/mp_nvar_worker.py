"""Multi-GPU checks of the NVLink all-reduce and of the W4 GEMM with the all-reduce fused into its
epilogue. Run one process per GPU:

    python -m torch.distributed.run --nnodes=1 --nproc-per-node P --master-addr 127.0.0.1 \
        --master-port 29531 tests/mp_nvar_worker.py [--quick]

Follows the reference's own multi-GPU test (kernels/test_hostar.py): random calls cycling sizes
and dtypes compared with NCCL, a chain of all-reduces captured in one CUDA graph; then the fused
row-parallel layer against the float64 oracle, bit-identity across ranks,
graph replay, a wait that is made to time out, and timings (max over ranks). Exits non-zero on the
first failed check. Prints one JSON line of timings on rank 0.
"""

from __future__ import annotations

import datetime
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import __graft_entry__ as entry  # noqa: E402

B2_ERR_TIMEOUT = 5


def fail(msg):
    print(f"rank {dist.get_rank()}: FAIL {msg}", flush=True)
    sys.exit(1)


def gather_equal(t: torch.Tensor) -> bool:
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t.contiguous())
    return all(torch.equal(parts[0], p) for p in parts[1:])


def max_over_ranks(v: float) -> float:
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def graph_time_us(fn, reps=20, iters=10):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(reps):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    align = torch.zeros(1, device="cuda")
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # align the GPUs on the device (no host sync between this collective and the replay), so
        # host-side skew between the ranks' launches does not land inside the timed region
        dist.all_reduce(align)
        e0.record()
        g.replay()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3 / reps)
    del g
    return max_over_ranks(sorted(ts)[len(ts) // 2])


def main():
    quick = "--quick" in sys.argv
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=90),
                            device_id=torch.device("cuda", local))
    cpu = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=90))
    r, P = dist.get_rank(), dist.get_world_size()
    entry.load_package()
    from mi50_vllm_lab_b200 import vllm_shim
    from oracle import skinny_oracle as so

    import gpu_util

    ops = entry.load_package().ops()
    M, N, G, K = 8, 5120, 128, 17408
    ar = vllm_shim.NvlinkAllReduce(cpu, r, list(range(P)), slot_bytes=M * 8192 * 8)
    if not ar.should_use(torch.empty(8 * 5120, dtype=torch.float16, device="cuda")):
        fail("should_use rejects an 80 KB fp16 tensor")

    # 1. random calls against NCCL (kernels/test_hostar.py:11-22)
    g = torch.Generator(device="cuda").manual_seed(100 + r)
    bad, calls = 0, (300 if quick else 1500)
    for it in range(calls):
        n = [8 * 5120, 5120, 2 * 5120, 64, 8 * 8192][it % 5]
        dt = torch.float16 if it % 7 else torch.float32
        if n * (2 if dt == torch.float16 else 4) > ar.max_bytes:
            dt = torch.float16
        x = torch.randn(n, device="cuda", dtype=dt, generator=g) * (10 ** (it % 4 - 1))
        y = ar.all_reduce(x)
        if P == 2:
            ref = x.clone()
            dist.all_reduce(ref)
            ok = torch.equal(y, ref)
        else:  # fixed rank-order fp32 sum (the oracle), NCCL only to within rounding
            parts = [torch.empty_like(x) for _ in range(P)]
            dist.all_gather(parts, x)
            acc = torch.zeros(n, dtype=torch.float32, device="cuda")
            for p in parts:
                acc = acc + p.float()
            ok = torch.equal(y, acc.to(dt))
        bad += 0 if ok else 1
    torch.cuda.synchronize()
    if bad:
        fail(f"{bad} of {calls} all-reduce calls differ from the reference sum")
    if not gather_equal(y):
        fail("all-reduce results differ across ranks")
    if ar.status() != 0:
        fail(f"all-reduce status {ar.status()}")

    # 2. 200 chained all-reduces captured in one CUDA graph (kernels/test_hostar.py:31-48)
    base = torch.randn(8 * 5120, device="cuda", dtype=torch.float16, generator=g) * 0.01
    buf = base.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(gr, stream=s):
            yg = buf
            for _ in range(200):
                yg = ar.all_reduce(yg) * 0.5
    torch.cuda.current_stream().wait_stream(s)
    dist.barrier()
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    ref = base.clone()
    for _ in range(200):
        if P == 2:
            dist.all_reduce(ref)
        else:
            parts = [torch.empty_like(ref) for _ in range(P)]
            dist.all_gather(parts, ref)
            acc = torch.zeros_like(ref, dtype=torch.float32)
            for p in parts:
                acc = acc + p.float()
            ref = acc.half()
        ref = ref * 0.5
    if not torch.equal(yg, ref):
        fail("graph chain of 200 all-reduces differs from the reference chain")
    del gr

    # 3. fused row-parallel W4 layer (config 3): this rank's K-shard, all-reduce in the epilogue
    ks = K // P
    x, qw, qz, sc = gpu_util.w4_device_inputs(M, K, N, G, seed=7)  # same full weights on all ranks
    xs = x[:, r * ks:(r + 1) * ks].contiguous()
    qws = qw[r * ks // 8:(r + 1) * ks // 8].contiguous()
    qzs = qz[r * ks // G:(r + 1) * ks // G].contiguous()
    scs = sc[r * ks // G:(r + 1) * ks // G].contiguous()
    yf = ar.w4_gemm_all_reduce(xs, qws, qzs, scs)
    torch.cuda.synchronize()
    if not gather_equal(yf):
        fail("fused GEMM+all-reduce results differ across ranks")
    cols = gpu_util.sample_columns(N, 200 if quick else 600, seed=3)
    if r == 0:
        st = so.error_stats(yf[:, torch.from_numpy(cols).cuda()].double().cpu().numpy(),
                            gpu_util.w4_ref_sampled(x, qw, qz, sc, cols))
        if not so.within_tolerance(st):
            fail(f"fused GEMM+all-reduce outside tolerance: {st}")
        print(f"fused config-3 TP{P} error vs float64 oracle: {st}", flush=True)
    for _ in range(3):  # repeated calls: deterministic
        y2 = ar.w4_gemm_all_reduce(xs, qws, qzs, scs)
    if not torch.equal(y2, yf):
        fail("fused GEMM+all-reduce not deterministic")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(gr, stream=s):
            yfg = ar.w4_gemm_all_reduce(xs, qws, qzs, scs)
    torch.cuda.current_stream().wait_stream(s)
    dist.barrier()
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    if not torch.equal(yfg, yf):
        fail("fused GEMM+all-reduce under graph replay differs from eager")
    del gr
    if ar.status() != 0:
        fail(f"fused status {ar.status()}")

    # 3c. the same layer with the decoder layer's residual add + RMSNorm in the epilogue:
    # bit-identical on every rank, the residual updated in place, and equal to the oracle's norm
    # of the plain fused output (new residual bit for bit, output within two fp16 ulps)
    gn = torch.Generator(device="cuda").manual_seed(55)  # the same residual on every rank
    res0 = (torch.randn(M, N, device="cuda", generator=gn) * 4).half()
    wn = (1.0 + (torch.rand(N, device="cuda", generator=gn) - 0.5) * 0.4).half()
    rn = res0.clone()
    yn = ar.w4_gemm_all_reduce_rmsnorm(xs, qws, qzs, scs, rn, wn, 1e-6)
    torch.cuda.synchronize()
    same_y, same_res = gather_equal(yn), gather_equal(rn)  # both collectives on every rank
    if not (same_y and same_res):
        fail("fused GEMM+all-reduce+RMSNorm results differ across ranks")
    if r == 0:
        ref_out, ref_res = so.add_rmsnorm_ref(yf.cpu().numpy(), res0.cpu().numpy(),
                                              wn.cpu().numpy(), 1e-6)
        if not np.array_equal(rn.cpu().numpy().view(np.int16), ref_res.view(np.int16)):
            fail("fused RMSNorm: residual differs from the oracle")
        ulp = so.fp16_ulp_distance(yn.cpu().numpy(), ref_out)
        if ulp.max() > 2 or (ulp == 0).mean() < 0.99:
            fail(f"fused RMSNorm: max ulp {ulp.max()}, exact {(ulp == 0).mean():.5f}")
    if ar.status() != 0:
        fail(f"fused RMSNorm status {ar.status()}")

    # 3d. both fused layers on this rank's shard repacked at load time (w4_repack): the same bits
    pks = ar.ops.w4_repack(qws, qzs, scs)
    yp = ar.w4_gemm_all_reduce_packed(xs, pks, N, G)
    rp = res0.clone()
    ynp = ar.w4_gemm_all_reduce_rmsnorm_packed(xs, pks, N, G, rp, wn, 1e-6)
    torch.cuda.synchronize()
    if not (torch.equal(yp, yf) and torch.equal(ynp, yn) and torch.equal(rp, rn)):
        fail("fused layers on repacked weights differ from the same layers on GPTQ tensors")
    if ar.status() != 0:
        fail(f"fused packed status {ar.status()}")
    del pks

    # 3b. the same layer through the other split-K kernel's fused epilogue (the default is the
    # cluster kernel; B2_TUNE_W4_PATH = 1 selects stream-K with its global fix-up)
    from mi50_vllm_lab_b200 import capi

    lib = capi.lib()
    lib.b2_set_tuning(4, 1)
    yc = ar.w4_gemm_all_reduce(xs, qws, qzs, scs)
    torch.cuda.synchronize()
    if not gather_equal(yc):
        fail("stream-K fused GEMM+all-reduce results differ across ranks")
    if r == 0:
        st = so.error_stats(yc[:, torch.from_numpy(cols).cuda()].double().cpu().numpy(),
                            gpu_util.w4_ref_sampled(x, qw, qz, sc, cols))
        if not so.within_tolerance(st):
            fail(f"stream-K fused GEMM+all-reduce outside tolerance: {st}")
    for _ in range(2):
        yc2 = ar.w4_gemm_all_reduce(xs, qws, qzs, scs)
    if not torch.equal(yc2, yc):
        fail("stream-K fused GEMM+all-reduce not deterministic")
    t_fused_streamk = graph_time_us(lambda: ar.w4_gemm_all_reduce(xs, qws, qzs, scs))
    lib.b2_set_tuning(4, 0)
    if ar.status() != 0:
        fail(f"stream-K fused status {ar.status()}")

    # 4. timings (max over ranks): fused vs GEMM + NCCL, and the bare all-reduce vs NCCL at 80 KB
    a80 = torch.randn(8 * 5120, device="cuda", dtype=torch.float16, generator=g)
    t_fused = graph_time_us(lambda: ar.w4_gemm_all_reduce(xs, qws, qzs, scs))
    t_fused_norm = graph_time_us(
        lambda: ar.w4_gemm_all_reduce_rmsnorm(xs, qws, qzs, scs, rn, wn, 1e-6))

    def unfused():
        yy = ops.w4gemm(xs, qws, qzs, scs, 0, 0)
        dist.all_reduce(yy)

    t_unfused = graph_time_us(unfused)
    t_gemm = graph_time_us(lambda: ops.w4gemm(xs, qws, qzs, scs, 0, 0))
    t_ar = graph_time_us(lambda: ar.all_reduce(a80))
    t_nccl = graph_time_us(lambda: dist.all_reduce(a80))
    if ar.status() != 0:
        fail(f"status after timing {ar.status()}")

    # 5. a wait that runs out (on 2-4 ranks): rank 0 all-reduces on a fresh handle that no other
    # rank calls; its kernel gives up after 300 ms and reports B2_ERR_TIMEOUT
    arf = vllm_shim.NvlinkAllReduce(cpu, r, list(range(P)), slot_bytes=1 << 16)
    ops.nvar_set_timeout_ms(arf.handle, 300)
    dist.barrier()
    if r == 0 and P <= 4:
        arf.all_reduce(torch.ones(4096, device="cuda", dtype=torch.float16))
        torch.cuda.synchronize()
        stt = arf.status(clear=True)
        if stt != B2_ERR_TIMEOUT:
            fail(f"expected a timeout status ({B2_ERR_TIMEOUT}), got {stt}")
    dist.barrier()
    if ar.status() != 0:
        fail("the timeout leaked into the main handle")

    if r == 0:
        bytes_rank = ks * N // 2 + (ks // G) * N * 2 + (ks // G) * N // 2 + 2 * M * ks + 2 * M * N
        print(json.dumps({"world": P, "config": f"3: down_proj K={K} sharded {P} ways, M={M}, N={N}",
                          "fused_us": round(t_fused, 2),
                          "fused_streamk_us": round(t_fused_streamk, 2),
                          "fused_with_rmsnorm_us": round(t_fused_norm, 2),
                          "gemm_plus_nccl_us": round(t_unfused, 2),
                          "gemm_only_us": round(t_gemm, 2), "nvlink_ar_80KB_us": round(t_ar, 2),
                          "nccl_ar_80KB_us": round(t_nccl, 2),
                          "gemm_bytes_per_rank": bytes_rank,
                          "nvlink_bytes_per_rank": (P - 1) * M * N * 4}), flush=True)
        print("mp_nvar_worker: all checks passed", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
