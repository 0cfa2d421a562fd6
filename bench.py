"""Benchmark of the skinny-GEMM hot path on B200.

Default (the driver's line): BASELINE config 1, the fp16 skinny GEMM at lm_head shape
M=7, K=5120, N=151936 (1.56 GB of weights, larger than the 126 MB L2, so no flush is needed).
One step = one GEMM through the C ABI on device-resident operands. With N GPUs (torchrun, one
rank per GPU) every rank runs its own config-1 GEMM (weak scaling; column-parallel shards need no
collective); `value` is the aggregate HBM throughput of all ranks, timed as the max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W]
    python bench.py --impl reference      # the reference's CPU path (torch dequant+matmul)
    python bench.py --sweep               # every BASELINE config, one JSON line each (not timed by the driver)
    python bench.py --norm-epilogue       # row-parallel layer + residual add + RMSNorm, fused vs separate

Metric: HBM TB/s of algorithmic bytes (2*N*K + 2*M*K + 2*M*N for fp16; the W4 formula for W4),
and us per GEMM.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "W4A16/fp16 skinny-GEMM HBM throughput at M<=8 (config 1: fp16 lm_head GEMM)"
UNIT = "TB/s"
CFG1 = dict(M=7, K=5120, N=151936)
FALLBACK_HBM_GBS = 6650.0


def f16_bytes(M, K, N):
    return 2 * N * K + 2 * M * K + 2 * M * N


def w4_bytes(M, K, N, G):
    return K * N // 2 + (K // G) * N * 2 + (K // G) * N // 2 + 2 * M * K + 2 * M * N


def hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def recorded_traffic(kernel: str, workload: str):
    """DRAM bytes per launch of `kernel` on `workload` from a committed ncu summary, or None."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(kernel, {}).get(workload)
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int, period_s: float = 0.01):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
        self.period = period_s

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------------
# distributed plumbing
# ------------------------------------------------------------------------------------------------


def dist_setup(n_gpus: int):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    if world != n_gpus and not (world == 1 and n_gpus == 1):
        print(f"warning: --gpus {n_gpus} but WORLD_SIZE={world}", file=sys.stderr)
    return rank, world, local


def barrier_sync(world):
    import torch

    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------------------------
# CPU baseline: the reference's own torch path (kernels/bench_skinny.py:44; kernels/check_w4.py)
# ------------------------------------------------------------------------------------------------


def cpu_baseline_f16(x_cpu, w_rows_cpu, budget_s: float = 10.0):
    """Time `x.float() @ w.float().T` (the reference's fp16 GEMM reference) on the host cores
    over a row sample of the weights; returns (TB/s, seconds per call, cores, description)."""
    import torch

    from oracle import cpu_baseline

    return cpu_baseline.time_f16(x_cpu, w_rows_cpu, budget_s=budget_s)


# ------------------------------------------------------------------------------------------------
# GPU legs
# ------------------------------------------------------------------------------------------------


def time_steps(fn, steps: int, world: int, stream):
    """Time exactly `steps` calls of fn between barriers with one pair of CUDA events on `stream`
    around all of them (events between the steps would put gaps between the launches)."""
    import torch

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier_sync(world)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    barrier_sync(world)
    return start.elapsed_time(end)


def run_gpu(args):
    import torch

    import __graft_entry__ as entry

    rank, world, local = dist_setup(args.gpus)
    pkg = entry.load_package()
    from mi50_vllm_lab_b200 import capi

    ops = pkg.ops()
    lib = capi.lib()
    M, K, N = CFG1["M"], CFG1["K"], CFG1["N"]
    nbytes = f16_bytes(M, K, N)

    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    ws = torch.zeros(lib.b2_workspace_bytes(local), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def step():
        rc = lib.b2_gemm_f16(x.data_ptr(), w.data_ptr(), y.data_ptr(), M, K, N, ws.data_ptr(),
                             ws.numel(), sp)
        if rc:
            capi.check(rc, "b2_gemm_f16")

    for _ in range(args.warmup):
        step()
    with ClockSampler(local) as clk:
        total_ms = time_steps(step, args.steps, world, stream)
    ms_step = max_over_ranks(total_ms / args.steps, world)
    # the timed region holds exactly one launch of the kernel per step: its per-launch period
    kern_ms = total_ms / args.steps
    value = world * nbytes / (ms_step * 1e-3) / 1e12

    # end to end through the plugin API with host buffers: H2D of the activations, the GEMM,
    # D2H of the logits, every step
    x_host = torch.randn(M, K, generator=torch.Generator().manual_seed(7)).half().pin_memory()
    y_host = torch.empty(M, N, dtype=torch.float16).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        out = ops.gemm(x_dev, w, 20)
        y_host.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    e2e_ms = time_steps(e2e_step, args.steps, world, stream)
    e2e_step_ms = max_over_ranks(e2e_ms / args.steps, world)
    e2e_value = world * nbytes / (e2e_step_ms * 1e-3) / 1e12

    peak, peak_kind = hbm_peak()
    achieved = nbytes / (kern_ms * 1e-3) / 1e9
    clocks = clk.summary()
    status = ops.workspace_status(False)
    assert status == 0, f"device status {status}"

    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "us_per_gemm": round(ms_step * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 (fp32 accumulate)", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
            "config": {"workload": "config 1: fp16 skinny GEMM, lm_head shape", "M": M, "K": K,
                       "N": N, "per_gpu_bytes_per_step": nbytes,
                       "l2": "weights 1.56 GB > 126 MB L2 (no flush needed)",
                       "parallelism": f"{world} independent column shards (no collective)"},
            "e2e": {"value": round(e2e_value, 4), "unit": UNIT, "ms_per_step": round(e2e_step_ms, 5),
                    "api": "torch.ops.gfx906_skinny.gemm, pinned host x -> device, y -> pinned host",
                    "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": "gemm_f16_kernel", "kernel_us": round(kern_ms * 1e3, 2),
                         "traffic": recorded_traffic("gemm_f16_kernel", "config1")},
            "gpu_launches": args.steps,
            "clocks": clocks,
        }
    if rank == 0 and world == 1 and not args.no_cpu:
        rows = 8192
        cpu = cpu_baseline_f16(x.cpu(), w[:rows].cpu(), budget_s=args.cpu_seconds)
        line["cpu_baseline"] = cpu
    if line:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_reference(args):
    """The reference's CPU implementation of the path (oracle port of kernels/bench_skinny.py:44:
    `x.float() @ w.float().T`), on the same config and metric, all host threads."""
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import cpu_baseline

    M, K, N = CFG1["M"], CFG1["K"], CFG1["N"]
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(1234)
    x = torch.randn(M, K, generator=g).half()
    w = (torch.randn(8192, K, generator=g) * 0.02).half()
    # size the per-step sample so that warm-up + steps stay within about two minutes
    t0 = time.perf_counter()
    cpu_baseline.f16_reference(x, w)
    t_full = time.perf_counter() - t0
    per_step = 120.0 / (args.steps + args.warmup)
    rows = int(max(256, min(8192, 8192 * per_step / max(t_full, 1e-6))) // 256 * 256)
    w = w[:rows].contiguous()
    step = lambda: cpu_baseline.f16_reference(x, w)  # noqa: E731
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    sample_bytes = f16_bytes(M, K, rows)
    value = sample_bytes / sec / 1e12
    desc = (f"{rows} of {N} weight rows per step ({sample_bytes / f16_bytes(M, K, N):.3f} of a "
            f"config-1 GEMM); torch {torch.__version__} float32 matmul")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": UNIT,
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
        "ms_per_full_gemm": round(sec * 1e3 * N / rows, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (reference computes x.float() @ w.float().T)", "data": "synthetic",
        "config": {"workload": "config 1: fp16 skinny GEMM, lm_head shape", "M": M, "K": K,
                   "N": N, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 6), "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 6), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


SWEEP = (
    [("cfg1_lm_head", "f16", 7, 5120, 151936, 0), ("cfg0", "w4", 7, 4096, 4096, 128)]
    + [(f"cfg2_{nm}_M{M}", "w4", M, K, N, 128) for M in (1, 2, 4, 8)
       for nm, (K, N) in {"qkv": (5120, 8192), "o_proj": (6144, 5120), "gate_up": (5120, 34816),
                          "down": (17408, 5120)}.items()]
    + [(f"cfg3_down_TP{P}", "w4", 8, 17408 // P, 5120, 128) for P in (2, 4, 8)]
    + [(f"drafter_fc_M{M}", "f16", M, 25600, 5120, 0) for M in (1, 8)]
    + [("check_w4_G32", "w4", 8, 5120, 1024, 32)]
)
# Extra cases for --profile only: the lm_head kernel on a 335 MB slice (above L2, small enough
# for a multi-pass ncu capture); traffic scales with N for this kernel.
PROFILE_ONLY = [("cfg1_lm_head_N32768", "f16", 7, 5120, 32768, 0)]


def run_sweep(args):
    """Every BASELINE config on one GPU. Launches are captured in a CUDA graph that rotates over
    enough weight copies to exceed 3x L2 (so every launch reads HBM), and timed by replaying the
    graph: the time per launch excludes host launch overhead, as in a captured decode step."""
    import torch

    import __graft_entry__ as entry

    entry.load_package()
    from mi50_vllm_lab_b200 import capi

    lib = capi.lib()
    torch.cuda.set_device(0)
    ws = torch.zeros(lib.b2_workspace_bytes(0), dtype=torch.uint8, device="cuda")
    if args.no_pdl:
        capi.check(lib.b2_set_tuning(3, 1), "b2_set_tuning")  # B2_TUNE_NO_PDL
    for kv in args.tune:
        k, v = (int(t) for t in kv.split("="))
        capi.check(lib.b2_set_tuning(k, v), "b2_set_tuning")
    peak, _ = hbm_peak()
    l2 = torch.cuda.get_device_properties(0).L2_cache_size

    def measure(name, kind, M, K, N, G):
        wbytes = K * N // 2 if kind == "w4" else 2 * N * K
        nb = w4_bytes(M, K, N, G) if kind == "w4" else f16_bytes(M, K, N)
        copies = max(1, int(3 * l2 // wbytes) + 1)
        g = torch.Generator(device="cuda").manual_seed(M * K + N)
        x = torch.randn(M, K, device="cuda", generator=g).half()
        y = torch.empty(M, N, dtype=torch.float16, device="cuda")
        calls = []
        for _ in range(copies):
            if kind == "w4":
                qw = torch.randint(-2**31, 2**31 - 1, (K // 8, N), device="cuda", dtype=torch.int32, generator=g)
                qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), device="cuda", dtype=torch.int32, generator=g)
                sc = (torch.rand(K // G, N, device="cuda", generator=g) * 0.015 + 0.005).half()
                calls.append((qw, qz, sc))
            else:
                calls.append((torch.randn(N, K, device="cuda", generator=g) * 0.02).half(),)

        def launch(t, sp):
            if kind == "w4":
                qw, qz, sc = t
                rc = lib.b2_w4_gemm(x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(),
                                    y.data_ptr(), M, K, N, G, ws.data_ptr(), ws.numel(), sp)
            else:
                rc = lib.b2_gemm_f16(x.data_ptr(), t[0].data_ptr(), y.data_ptr(), M, K, N,
                                     ws.data_ptr(), ws.numel(), sp)
            capi.check(rc, name)

        reps = max(copies, min(64, 20 * copies))
        reps = (reps // copies) * copies
        sp0 = torch.cuda.current_stream().cuda_stream
        for t in calls:
            launch(t, sp0)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                for i in range(reps):
                    launch(calls[i % copies], s.cuda_stream)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        times = []
        for _ in range(max(3, args.steps // reps)):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            graph.replay()
            e1.record(st)
            e1.synchronize()
            times.append(e0.elapsed_time(e1) * 1e3 / reps)
        us = statistics.median(times)
        del graph
        return {"workload": name, "kind": kind, "M": M, "K": K, "N": N, "G": G, "us": round(us, 2),
                "TBps": round(nb / us / 1e6, 3), "frac": round(nb / us / 1e3 / peak, 3),
                "bytes": nb, "l2_rotation_copies": copies, "launches_per_graph": reps}

    for w in SWEEP:
        if args.only and not any(o in w[0] for o in args.only.split(",")):
            continue
        print(json.dumps(measure(*w)), flush=True)
        torch.cuda.empty_cache()


def run_profile(args):
    """A few eager launches of one sweep workload, for ncu: warm-up launches, then `steps`."""
    import torch

    import __graft_entry__ as entry

    entry.load_package()
    from mi50_vllm_lab_b200 import capi

    lib = capi.lib()
    torch.cuda.set_device(0)
    ws = torch.zeros(lib.b2_workspace_bytes(0), dtype=torch.uint8, device="cuda")
    name, kind, M, K, N, G = next(w for w in PROFILE_ONLY + list(SWEEP) if args.only in w[0])
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    sp = torch.cuda.current_stream().cuda_stream
    if kind == "w4":
        qw = torch.randint(-2**31, 2**31 - 1, (K // 8, N), device="cuda", dtype=torch.int32, generator=g)
        qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), device="cuda", dtype=torch.int32, generator=g)
        sc = (torch.rand(K // G, N, device="cuda", generator=g) * 0.015 + 0.005).half()
        step = lambda: capi.check(lib.b2_w4_gemm(x.data_ptr(), qw.data_ptr(), qz.data_ptr(),  # noqa: E731
                                                 sc.data_ptr(), y.data_ptr(), M, K, N, G,
                                                 ws.data_ptr(), ws.numel(), sp))
    else:
        w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
        step = lambda: capi.check(lib.b2_gemm_f16(x.data_ptr(), w.data_ptr(), y.data_ptr(), M, K,  # noqa: E731
                                                  N, ws.data_ptr(), ws.numel(), sp))
    for _ in range(args.warmup + args.steps):
        step()
    torch.cuda.synchronize()
    print(json.dumps({"profiled": name, "launches": args.warmup + args.steps}))


# the decode-verify step of a 64-layer W4A16 model at M = 8 (speculative k = 7),
# tensor parallel over the ranks: qkv and gate_up column-parallel, o_proj and down_proj
# row-parallel with the NVLink all-reduce fused into their epilogues, then the fp16 lm_head
# (column-parallel, 151936 / P rows per rank), all captured in one CUDA graph.
CFG4 = dict(layers=64, M=8, hidden=5120, qkv=8192, o_in=6144, inter=17408, vocab=151936, G=128)


def decode_step_bytes(P: int) -> int:
    c = CFG4
    per_layer = (w4_bytes(c["M"], c["hidden"], c["qkv"] // P, c["G"])
                 + w4_bytes(c["M"], c["o_in"] // P, c["hidden"], c["G"])
                 + w4_bytes(c["M"], c["hidden"], 2 * c["inter"] // P, c["G"])
                 + w4_bytes(c["M"], c["inter"] // P, c["hidden"], c["G"]))
    return c["layers"] * per_layer + f16_bytes(c["M"], c["hidden"], c["vocab"] // P)


def run_decode_step(args):
    """Config 4 on N GPUs (TP = N): one graph replay per step, timed as the max over ranks."""
    import torch

    import __graft_entry__ as entry

    rank, world, local = dist_setup(args.gpus)
    pkg = entry.load_package()
    from mi50_vllm_lab_b200 import vllm_shim

    ops = pkg.ops()
    c = CFG4
    M, H, G, P = c["M"], c["hidden"], c["G"], world
    ar = None
    if P > 1:
        import datetime

        import torch.distributed as dist

        cpu = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=120))
        # 8 bytes per output element: room for the low-latency (value + generation) exchange
        ar = vllm_shim.NvlinkAllReduce(cpu, rank, list(range(P)), slot_bytes=M * H * 8)
    g = torch.Generator(device="cuda").manual_seed(4000 + rank)

    def w4(K, N):
        return (torch.randint(-2**31, 2**31 - 1, (K // 8, N), device="cuda", dtype=torch.int32,
                              generator=g),
                torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), device="cuda",
                              dtype=torch.int32, generator=g),
                (torch.rand(K // G, N, device="cuda", generator=g) * 0.015 + 0.005).half())

    layers = [dict(qkv=w4(H, c["qkv"] // P), o=w4(c["o_in"] // P, H),
                   gu=w4(H, 2 * c["inter"] // P), down=w4(c["inter"] // P, H))
              for _ in range(c["layers"])]
    lm = (torch.randn(c["vocab"] // P, H, device="cuda", generator=g) * 0.02).half()
    x0 = torch.randn(M, H, device="cuda", generator=g).half()
    # attention output and activated MLP input of this rank's shard (synthetic, fixed)
    a_o = (torch.randn(M, c["o_in"] // P, device="cuda", generator=g) * 0.05).half()
    a_d = (torch.randn(M, c["inter"] // P, device="cuda", generator=g) * 0.05).half()

    def row_parallel(a, w):
        return ar.w4_gemm_all_reduce(a, *w) if ar else ops.w4gemm(a, *w, 0, 0)

    def step():
        h = x0
        for L in layers:
            ops.w4gemm(h, *L["qkv"], 0, 0)
            h = row_parallel(a_o, L["o"])
            ops.w4gemm(h, *L["gu"], 0, 0)
            h = row_parallel(a_d, L["down"])
        return ops.gemm(h, lm, 0)

    eager = step()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            out = step()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    same = bool(torch.equal(out, eager))
    st = torch.cuda.current_stream()
    align = torch.zeros(1, device="cuda")
    times = []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            if P > 1:
                import torch.distributed as dist

                dist.all_reduce(align)  # line the ranks up on the device, not on the host
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            graph.replay()
            e1.record(st)
            e1.synchronize()
            times.append(e0.elapsed_time(e1) * 1e3)
    us = max_over_ranks(statistics.median(times), world)
    status = ar.status() if ar else ops.workspace_status(False)
    nbytes = decode_step_bytes(P)
    peak, peak_kind = hbm_peak()
    if rank == 0:
        kernels = c["layers"] * 4 + 1
        print(json.dumps({
            "metric": "config 4: decode-verify step (64 W4A16 layers + fp16 lm_head, M=8), us per step",
            "value": round(us, 1), "unit": "us", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": False, "scaling": "strong",
            "dtype": "W4A16 / f16 (fp32 accumulate)", "data": "synthetic (seeded random weights)",
            "config": {"workload": "config 4", "tp": P, "layers": c["layers"], "M": M,
                       "kernels_per_step": kernels, "fused_allreduces_per_step": 2 * c["layers"] if P > 1 else 0,
                       "graph": "one CUDA graph per step (programmatic dependent launch between GEMMs)",
                       "per_rank_bytes_per_step": nbytes},
            "per_rank_TBps": round(nbytes / us / 1e6, 3),
            "roofline": {"bound": "hbm", "achieved": round(nbytes / us / 1e3, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(nbytes / us / 1e3 / peak, 4),
                         "peak_source": peak_kind},
            "graph_equals_eager": same, "device_status": status, "clocks": clk.summary()}),
            flush=True)
    del graph
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_norm_epilogue(args):
    """Row-parallel W4 layer + residual add + RMSNorm on one GPU (one-rank all-reduce handle):
    the fused launch (w4gemm_ar_rmsnorm) against the fused GEMM + all-reduce followed by a
    separate norm - vLLM's own CUDA kernel (torch.ops._C.fused_add_rms_norm) when vLLM loads, and
    the torch restatement of its reference code (vllm/ir/ops/layernorm.py:48-58). Per-rank
    shards of o_proj and down_proj at TP 1..8, M=8; graph replay over weight copies that exceed
    3x L2, as in --sweep. One JSON line per shape."""
    import torch

    import __graft_entry__ as entry

    ops = entry.load_package().ops()
    from mi50_vllm_lab_b200 import capi

    lib = capi.lib()
    torch.cuda.set_device(0)
    M, N, G, eps = 8, CFG4["hidden"], CFG4["G"], 1e-6
    name = f"/b2_bench_norm_{os.getpid()}"
    h = ops.nvar_create(name, M * N * 8, 0, 1)
    ops.hostar_unlink(name)
    try:
        import vllm._C  # noqa: F401

        vllm_norm = torch.ops._C.fused_add_rms_norm
    except Exception as e:  # vLLM's compiled ops are optional here
        vllm_norm = None
        print(json.dumps({"note": f"vLLM CUDA ops unavailable: {type(e).__name__}: {e}"[:200]}),
              flush=True)
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    g = torch.Generator(device="cuda").manual_seed(11)
    w = (1.0 + (torch.rand(N, device="cuda", generator=g) - 0.5) * 0.4).half()
    res0 = (torch.randn(M, N, device="cuda", generator=g) * 4).half()

    def torch_norm(x, r):
        xf = x.float() + r.float()
        r.copy_(xf.half())
        var = xf.pow(2).mean(dim=-1, keepdim=True)
        return (xf * torch.rsqrt(var + eps)).half() * w

    for layer, K_full in (("down", CFG4["inter"]), ("o_proj", CFG4["o_in"])):
        for P in (1, 2, 4, 8):
            K = K_full // P
            copies = max(1, int(3 * l2 // (K * N // 2)) + 1)
            # small activations: the residual grows by y at every replayed call
            x = (torch.randn(M, K, device="cuda", generator=g) * 0.01).half()
            ws = [(torch.randint(-2**31, 2**31 - 1, (K // 8, N), device="cuda", dtype=torch.int32,
                                 generator=g),
                   torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), device="cuda",
                                 dtype=torch.int32, generator=g),
                   (torch.rand(K // G, N, device="cuda", generator=g) * 0.015 + 0.005).half())
                  for _ in range(copies)]
            r = res0.clone()
            variants = {
                "gemm_ar": lambda t: ops.w4gemm_ar(x, *t, h),
                # the same launch without early start, as the norm epilogue is launched
                "gemm_ar_no_early_launch": lambda t: ops.w4gemm_ar(x, *t, h),
                "gemm_ar_norm_fused": lambda t: ops.w4gemm_ar_rmsnorm(x, *t, h, r, w, eps),
                "gemm_ar_then_torch_norm": lambda t: torch_norm(ops.w4gemm_ar(x, *t, h), r),
            }
            if vllm_norm is not None:
                def vl(t):
                    y = ops.w4gemm_ar(x, *t, h)
                    vllm_norm(y, r, w, eps)
                    return y
                variants["gemm_ar_then_vllm_norm"] = vl
            row = {"workload": f"{layer} shard TP{P}", "M": M, "K": K, "N": N, "G": G,
                   "l2_rotation_copies": copies}
            for vname, fn in variants.items():
                reps = max(copies, min(64, 20 * copies)) // copies * copies
                capi.check(lib.b2_set_tuning(3, 1 if vname == "gemm_ar_no_early_launch" else 0),
                           "b2_set_tuning")  # B2_TUNE_NO_PDL, read at launch (and capture) time
                try:
                    for t in ws:
                        fn(t)
                    torch.cuda.synchronize()
                except RuntimeError as e:  # e.g. a library kernel built for other GPUs
                    row[vname + "_error"] = str(e)[:160]
                    continue
                graph = torch.cuda.CUDAGraph()
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s):
                    with torch.cuda.graph(graph, stream=s):
                        for i in range(reps):
                            fn(ws[i % copies])
                torch.cuda.current_stream().wait_stream(s)
                for _ in range(args.warmup):
                    graph.replay()
                torch.cuda.synchronize()
                st = torch.cuda.current_stream()
                times = []
                for _ in range(max(3, args.steps // reps)):
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(st)
                    graph.replay()
                    e1.record(st)
                    e1.synchronize()
                    times.append(e0.elapsed_time(e1) * 1e3 / reps)
                row[vname + "_us"] = round(statistics.median(times), 2)
                del graph
            capi.check(lib.b2_set_tuning(3, 0), "b2_set_tuning")
            row["status"] = int(ops.nvar_status(h, False))
            print(json.dumps(row), flush=True)
            del ws
            torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--sweep", action="store_true")
    ap.add_argument("--decode-step", action="store_true",
                    help="config 4: the 64-layer decode-verify step in one CUDA graph, TP = --gpus")
    ap.add_argument("--only", default="", help="with --sweep: workloads whose name contains one of these comma-separated "
                         "strings; with --profile: the first workload whose name contains it")
    ap.add_argument("--profile", action="store_true", help="eager launches of one --only workload (for ncu)")
    ap.add_argument("--norm-epilogue", action="store_true",
                    help="row-parallel W4 layer + residual add + RMSNorm: fused vs separate, 1 GPU")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--tune", action="append", default=[], metavar="KEY=VALUE",
                    help="with --sweep: b2_set_tuning(KEY, VALUE) first (B2_TUNE_* in b2_skinny.h)")
    ap.add_argument("--no-pdl", action="store_true",
                    help="with --sweep: launch each GEMM only after the previous one has finished")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.profile:
        run_profile(args)
    elif args.sweep:
        run_sweep(args)
    elif args.decode_step:
        run_decode_step(args)
    elif args.norm_epilogue:
        run_norm_epilogue(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
