"""Phase timeline of the W4 GEMM with the all-reduce fused into its epilogue, on P GPUs, from the
trace build (builder.py --trace). One process per GPU:

    python -m torch.distributed.run --nnodes=1 --nproc-per-node P --master-addr 127.0.0.1 \\
        --master-port 29541 bench.py --trace-fused K,N[,norm] [--tune KEY=VALUE ...]

Each rank builds an all-reduce handle through the C ABI (IPC handles exchanged over gloo), runs a
chain of `chain` fused launches back to back (the exchange keeps the ranks in step, as inside a
decode step) and reads the per-CTA stamps of the last one. Rank 0 prints one JSON line: per rank,
the median over CTAs of each phase - dep_wait (an early-launched CTA waiting for the previous
grid), units (its k-units), reduce (cluster reduction and the sends to every rank), wait (phase 2:
gathering every rank's words), tail (norm, finish, exit) - and the kernel span (first CTA start to
last CTA end on that GPU). Durations only: each GPU's global timer is read on that GPU.
"""

from __future__ import annotations

import ctypes as C
import datetime
import json
import os
import statistics

CTA_WORDS = 12


def main(argv) -> dict | None:
    import torch
    import torch.distributed as dist

    from . import builder, capi

    K, N = (int(v) for v in argv[0].split(","))
    norm = "--norm" in argv[1:]
    tune = [a for a in argv[1:] if a != "--norm"]
    M, G, chain = 8, 128, 40
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    capi.CAPI_LIB = builder.TRACE_LIB
    lib = capi.lib()
    lib.b2_trace_read.argtypes = [C.c_void_p, C.c_void_p]
    lib.b2_trace_clear.restype = C.c_int
    for kv in tune:
        k, v = (int(t) for t in kv.split("="))
        capi.check(lib.b2_set_tuning(k, v), "b2_set_tuning")

    h = C.c_void_p()
    capi.check(lib.b2_nvar_create(local, rank, world, M * N * 8, C.byref(h)), "b2_nvar_create")
    mine = (C.c_ubyte * 64)()
    capi.check(lib.b2_nvar_export(h, mine), "b2_nvar_export")
    allh = [None] * world
    dist.all_gather_object(allh, bytes(mine))
    joined = (C.c_ubyte * (64 * world)).from_buffer_copy(b"".join(allh))
    capi.check(lib.b2_nvar_connect(h, joined), "b2_nvar_connect")

    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    qw = torch.randint(-2**31, 2**31 - 1, (K // 8, N), device="cuda", dtype=torch.int32, generator=g)
    qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), device="cuda", dtype=torch.int32, generator=g)
    sc = (torch.rand(K // G, N, device="cuda", generator=g) * 0.015 + 0.005).half()
    y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    res = torch.randn(M, N, device="cuda", generator=g).half()
    nw = torch.ones(N, device="cuda", dtype=torch.float16)
    ws = torch.zeros(lib.b2_workspace_bytes(local), dtype=torch.uint8, device="cuda")
    sp = torch.cuda.current_stream().cuda_stream

    def launch():
        if norm:
            capi.check(lib.b2_w4_gemm_allreduce_rmsnorm(
                h, x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), res.data_ptr(),
                nw.data_ptr(), 1e-6, y.data_ptr(), M, K, N, G, ws.data_ptr(), ws.numel(), sp),
                "b2_w4_gemm_allreduce_rmsnorm")
            return
        capi.check(lib.b2_w4_gemm_allreduce(h, x.data_ptr(), qw.data_ptr(), qz.data_ptr(),
                                            sc.data_ptr(), y.data_ptr(), M, K, N, G,
                                            ws.data_ptr(), ws.numel(), sp), "b2_w4_gemm_allreduce")

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    dist.barrier()
    capi.check(lib.b2_trace_clear(), "b2_trace_clear")
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(chain):
        launch()
    e1.record()
    torch.cuda.synchronize()
    per_launch_us = e0.elapsed_time(e1) * 1e3 / chain
    st = C.c_int(0)
    capi.check(lib.b2_nvar_status(h, 1, C.byref(st)), "b2_nvar_status")
    units = (C.c_ulonglong * (5 * 4096))()
    ctas = (C.c_ulonglong * (4096 * CTA_WORDS))()
    capi.check(lib.b2_trace_read(units, ctas), "b2_trace_read")
    plan = capi.w4_plan(M, K, N, G, True)
    n = plan["ctas"]
    rows = [[ctas[CTA_WORDS * i + k] for k in range(CTA_WORDS)] for i in range(n)]

    def med(xs):
        return round(statistics.median(xs)) if xs else None

    t0 = min(r[0] for r in rows)
    mine = {
        "rank": rank, "status": st.value, "us_per_launch_in_chain": round(per_launch_us, 2),
        "span_ns": max(r[1] for r in rows) - t0,
        "dep_wait_ns": med([r[7] - r[0] for r in rows]),
        "units_ns": med([r[3] - r[7] for r in rows]),
        "reduce_and_send_ns": med([r[4] - r[3] for r in rows]),
        "to_phase2_ns": med([r[5] - r[4] for r in rows]),
        "wait_gather_ns": med([r[6] - r[5] for r in rows]),
        "wait_gather_ns_max": max(r[6] - r[5] for r in rows),
        "tail_ns": med([r[1] - r[6] for r in rows]),
        "start_spread_ns": max(r[0] for r in rows) - t0,
    }
    if norm:
        lead = [rows[i] for i in range(0, n, plan["cluster"])]
        mine.update({
            "norm_sums_sent_ns": med([r[8] - r[6] for r in rows]),
            "norm_leader_gathered_ns": med([r[9] - r[8] for r in lead]),
            "norm_leader_grid_barrier_ns": med([r[10] - r[9] for r in lead]),
            "norm_rstd_received_ns": med([r[11] - r[8] for r in rows]),
            "norm_finish_and_exit_ns": med([r[1] - r[11] for r in rows]),
        })
        # the last cluster (its leader counted last) finishes every row
        cs = plan["cluster"]
        li = max(range(0, n, cs), key=lambda i: rows[i][10])
        last = rows[li:li + cs]
        mine.update({
            "last_cluster_units_end_to_count_ns": rows[li][10] - max(r[3] for r in last),
            "last_cluster_count_to_rstd_ns": med([r[11] for r in last]) - rows[li][10],
            "last_cluster_finish_and_exit_ns": med([r[1] - r[11] for r in last]),
            "last_cluster_end_minus_kernel_others_end_ns":
                max(r[1] for r in last) - max(r[1] for i, r in enumerate(rows) if not li <= i < li + cs),
        })
    every = [None] * world
    dist.all_gather_object(every, mine)
    capi.check(lib.b2_nvar_destroy(h), "b2_nvar_destroy")
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        return {"world": world, "shape": {"M": M, "K": K, "N": N, "G": G}, "norm": norm,
                "plan": plan, "tune": tune, "ranks": every}
    return None
