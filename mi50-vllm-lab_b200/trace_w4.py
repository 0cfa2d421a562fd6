"""Per-unit timeline of the W4 cluster kernel, from the trace build (builder.py --trace).

    python bench.py --trace M,K,N[,G] [--trace-units] [--tune KEY=VALUE ...]

runs one launch of b2_w4_gemm on random weights after the GPU has gone idle, and prints a JSON
summary: how the CTAs sat on the SMs and how long they ran, and for CTA 0, per unit, how long a
stage's copies took from the producer's issue until the consumers saw them land ("copy"), how
long the consumers spent on the unit ("consume"), and how long they then waited for the next
unit ("starve"). The first `stages` units are issued into an empty ring (unloaded latency); the
rest are issued as stages free up (latency under load). --units adds the raw stamps.
"""

from __future__ import annotations

import argparse
import collections
import ctypes as C
import json
import statistics

CTA_WORDS = 12  # per CTA: start, end, SM, units done, reduction done, exchange phase 2, ...


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser()
    ap.add_argument("shape", type=int, nargs="+", help="M K N [G]")
    ap.add_argument("--units", action="store_true")
    ap.add_argument("--tune", action="append", default=[], metavar="KEY=VALUE")
    a = ap.parse_args(argv)
    M, K, N = a.shape[:3]
    G = a.shape[3] if len(a.shape) > 3 else 128

    import torch

    from . import builder, capi

    capi.CAPI_LIB = builder.TRACE_LIB  # before the first capi.lib() of this process
    if not capi.CAPI_LIB.exists():
        raise RuntimeError(f"{capi.CAPI_LIB} is not built (python builder.py --trace)")
    lib = capi.lib()
    lib.b2_trace_read.argtypes = [C.c_void_p, C.c_void_p]
    lib.b2_trace_read.restype = C.c_int
    lib.b2_trace_clear.restype = C.c_int
    for kv in a.tune:
        k, v = (int(t) for t in kv.split("="))
        capi.check(lib.b2_set_tuning(k, v), "b2_set_tuning")

    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    qw = torch.randint(-2**31, 2**31 - 1, (K // 8, N), device="cuda", dtype=torch.int32, generator=g)
    qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), device="cuda", dtype=torch.int32, generator=g)
    sc = (torch.rand(K // G, N, device="cuda", generator=g) * 0.015 + 0.005).half()
    y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    ws = torch.zeros(lib.b2_workspace_bytes(0), dtype=torch.uint8, device="cuda")
    sp = torch.cuda.current_stream().cuda_stream

    def launch():
        capi.check(lib.b2_w4_gemm(x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(),
                                  y.data_ptr(), M, K, N, G, ws.data_ptr(), ws.numel(), sp), "w4")

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    capi.check(lib.b2_trace_clear(), "b2_trace_clear")
    torch.cuda.synchronize()
    launch()
    torch.cuda.synchronize()
    units = (C.c_ulonglong * (5 * 4096))()
    ctas = (C.c_ulonglong * (4096 * CTA_WORDS))()
    capi.check(lib.b2_trace_read(units, ctas), "b2_trace_read")
    plan = capi.w4_plan(M, K, N, G)
    if plan["kernel"] != "w4c_kernel":
        return {"plan": plan, "note": "this shape does not take the cluster kernel: no trace"}

    n = plan["ctas"]
    c = [(ctas[CTA_WORDS * i], ctas[CTA_WORDS * i + 1], ctas[CTA_WORDS * i + 2]) for i in range(n)]
    t0 = min(s for s, _, _ in c)
    dur = [e - s for s, e, _ in c]
    per_sm = collections.Counter(sm for _, _, sm in c)
    sm_end = collections.defaultdict(int)
    for s, e, sm in c:
        sm_end[sm] = max(sm_end[sm], e - t0)
    ends = sorted(sm_end.values())
    u = [[units[e * 4096 + j] for j in range(4096)] for e in range(5)]
    nu = sum(1 for v in u[3] if v)
    base = u[0][0]
    # the planner's rule for the five-stage layout (one tile per cluster, >= 16 k-units per CTA)
    cs = plan["cluster"]
    tiles, upt = (N + 127) // 128, K // 128
    stages = 5 if (G >= 128 and plan["ctas"] // cs >= tiles and (upt + cs - 1) // cs >= 16
                   and not lib.b2_get_tuning(8)) else 4

    def med(xs):
        return round(statistics.median(xs)) if xs else None

    copy = [u[2][j] - u[0][j] for j in range(nu)]
    consume = [u[3][j] - u[2][j] for j in range(nu)]
    starve = [u[2][j + 1] - u[3][j] for j in range(nu - 1)]
    out = {
        "shape": {"M": M, "K": K, "N": N, "G": G}, "plan": plan,
        "ctas": {"count": n, "span_ns": max(e for _, e, _ in c) - t0,
                 "start_spread_ns": max(s for s, _, _ in c) - t0,
                 "duration_ns_min_med_max": [min(dur), med(dur), max(dur)],
                 "ctas_per_sm": dict(sorted(collections.Counter(per_sm.values()).items())),
                 "sms": len(per_sm), "sm_last_end_ns_min_med_max": [ends[0], med(ends), ends[-1]]},
        "cta0": {"units": nu, "stages_assumed": stages,
                 "copy_ns_unloaded": med(copy[:stages]), "copy_ns_loaded": med(copy[stages:]),
                 "consume_ns": med(consume), "starve_ns": med(starve),
                 "ns_per_unit": round((u[3][nu - 1] - u[2][0]) / max(1, nu - 1)) if nu > 1 else None},
    }
    # per CTA (medians): start -> units done (3), units done -> reduction done (4), -> end (1)
    full = [[ctas[CTA_WORDS * i + k] for k in range(CTA_WORDS)] for i in range(n)]
    ok_rows = [r for r in full if r[3] and r[4]]
    if ok_rows:
        out["ctas"]["start_to_units_done_ns"] = med([r[3] - r[0] for r in ok_rows])
        out["ctas"]["units_done_to_reduced_ns"] = med([r[4] - r[3] for r in ok_rows])
        out["ctas"]["reduced_to_end_ns"] = med([r[1] - r[4] for r in ok_rows])
    if nu:
        out["cta0"]["start_to_first_issue_ns"] = u[0][0] - c[0][0]
    if a.units:
        out["cta0"]["stamps_ns"] = [[(u[e][j] - base) if u[e][j] else None for e in range(4)]
                                    for j in range(nu)]
    return out


if __name__ == "__main__":
    print(json.dumps(main()))
