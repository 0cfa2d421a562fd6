"""Benchmark of the skinny-GEMM hot path on B200.

Default (the driver's line): BASELINE config 4, the synthetic decode-verify step of a 64-layer
W4A16 model at M = 8 (speculative k = 7), tensor parallel over the N ranks (TP = N, one process
per GPU under torchrun): per layer qkv_proj and gate_up (column-parallel, N-sharded) and o_proj
and down_proj (row-parallel, K-sharded, with the NVLink all-reduce fused into the GEMM epilogue
when N > 1), then the fp16 lm_head (column-parallel). All 257 launches of a step are captured in
one CUDA graph; one step = one replay. `value` is microseconds per step, timed on the device with
CUDA events and taken as the max over ranks. The line also carries:
  * `roofline`: the kernel that takes most of the step, timed alone (a graph of its 64 launches
    of the step, CUDA events), against its algorithmic bytes and the measured HBM peak;
  * `kernels`: the same per-launch figures for every kind of launch of the step;
  * `e2e`: the step through the operator library with the step's input activations copied from
    pinned host memory and the logits copied back, every step;
  * `cpu_baseline` (N = 1): the reference's CPU path (torch dequantize-then-matmul,
    kernels/check_w4.py:11-21; `x.float() @ w.float().T`, kernels/bench_skinny.py:44) timed on
    the host cores over a column sample of every GEMM of one layer and a row sample of the
    lm_head, scaled to a full step;
  * `config4_with_norms`: the step with the decoder layer's residual add + RMSNorm after each
    row-parallel layer, fused into its epilogue and as separate steps;
  * `config4_packed_weights`: the step with every W4 weight repacked at load time (w4_repack,
    then the *_packed operators), and whether its logits equal the plain step's bit for bit;
  * `extra` (N = 1): config 1 (fp16 lm_head GEMM) and config 0 (W4 4096 x 4096) on their own, as
    in the earlier default line.

    python bench.py [--gpus N] [--steps K] [--warmup W]
    python bench.py --impl reference      # the reference's CPU path on the same step and metric
    python bench.py --sweep               # every single-GEMM BASELINE config, one JSON line each
    python bench.py --config1             # config 1 alone (fp16 lm_head GEMM, TB/s)
    python bench.py --norm-epilogue       # row-parallel layer + residual add + RMSNorm, fused vs separate
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

METRIC = ("W4A16/fp16 skinny-GEMM decode-verify step, config 4 (64 W4A16 layers + fp16 lm_head, "
          "M=8, TP=N with the all-reduce fused into the row-parallel GEMMs): us per step")
UNIT = "us"
CFG1 = dict(M=7, K=5120, N=151936)
CFG0 = dict(M=7, K=4096, N=4096, G=128)
CFG4 = dict(layers=64, M=8, hidden=5120, qkv=8192, o_in=6144, inter=17408, vocab=151936, G=128)
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


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while the timed region runs
    (every millisecond by default)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int, period_s: float = 0.001):
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
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples),
                "period_ms": self.period * 1e3}


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


def capture(fn):
    """Capture fn() in a CUDA graph on a side stream; returns (graph, fn's return value)."""
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            out = fn()
    torch.cuda.current_stream().wait_stream(s)
    return graph, out


# ------------------------------------------------------------------------------------------------
# the decode-verify step
# ------------------------------------------------------------------------------------------------


def decode_step_bytes(P: int) -> int:
    """Algorithmic HBM bytes one rank moves per step at TP = P."""
    c = CFG4
    return c["layers"] * sum(w4_bytes(c["M"], K, N, c["G"]) for K, N in layer_shapes(P).values()) \
        + f16_bytes(c["M"], c["hidden"], c["vocab"] // P)


def layer_shapes(P: int) -> dict:
    """(K, N) of this rank's four W4 GEMMs per layer at TP = P."""
    c = CFG4
    return {"qkv": (c["hidden"], c["qkv"] // P), "o": (c["o_in"] // P, c["hidden"]),
            "gate_up": (c["hidden"], 2 * c["inter"] // P), "down": (c["inter"] // P, c["hidden"])}


class DecodeModel:
    """Random-initialised weights of one rank's shard of config 4 and the step that runs them
    through torch.ops.gfx906_skinny (the operators vLLM calls).

    `norm` adds the decoder layer's two residual-add + RMSNorm steps, which vLLM runs on the
    all-reduced outputs of o_proj and down_proj (fused_add_rms_norm): "fused" in the GEMM's
    epilogue (w4gemm_ar_rmsnorm; at TP=1 through a one-rank handle `h1`), "unfused" as a separate
    step after it (the torch restatement of vLLM's reference code, vllm/ir/ops/layernorm.py:48-58).
    The residual stream restarts from the step's input every step."""

    def __init__(self, ops, P: int, rank: int, ar, seed: int = 4000, norm=None, h1=None):
        import torch

        c = CFG4
        self.ops, self.ar, self.P = ops, ar, P
        M, H, G = c["M"], c["hidden"], c["G"]
        g = torch.Generator(device="cuda").manual_seed(seed + rank)
        sh = layer_shapes(P)

        def w4(K, N):
            return (torch.randint(-2**31, 2**31 - 1, (K // 8, N), device="cuda", dtype=torch.int32,
                                  generator=g),
                    torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), device="cuda",
                                  dtype=torch.int32, generator=g),
                    (torch.rand(K // G, N, device="cuda", generator=g) * 0.015 + 0.005).half())

        self.layers = [{k: w4(*sh[k]) for k in ("qkv", "o", "gate_up", "down")}
                       for _ in range(c["layers"])]
        self.lm = (torch.randn(c["vocab"] // P, H, device="cuda", generator=g) * 0.02).half()
        self.x0 = torch.randn(M, H, device="cuda", generator=g).half()
        # attention output and activated MLP input of this rank's shard (synthetic, fixed: the
        # attention and the activation are not part of this path)
        self.a_o = (torch.randn(M, c["o_in"] // P, device="cuda", generator=g) * 0.05).half()
        self.a_d = (torch.randn(M, c["inter"] // P, device="cuda", generator=g) * 0.05).half()
        self.norm, self.h1, self.packed = norm, h1, False
        self.res = torch.empty(M, H, device="cuda", dtype=torch.float16)
        self.nw = [(1.0 + (torch.rand(2, H, device="cuda", generator=g) - 0.5) * 0.2).half()
                   for _ in range(c["layers"])]

    def pack(self):
        """Repack every layer's weights at load time (w4_repack); `packed` then switches the
        launches to the operators on the packed image (w4gemm_packed, w4gemm_ar_packed,
        w4gemm_ar_rmsnorm_packed)."""
        for L in self.layers:
            for k in ("qkv", "o", "gate_up", "down"):
                L["packed_" + k] = self.ops.w4_repack(*L[k])
        self.packed = True

    def w4(self, a, L, kind):
        if self.packed:
            return self.ops.w4gemm_packed(a, L["packed_" + kind], L[kind][0].shape[1], CFG4["G"])
        return self.ops.w4gemm(a, *L[kind], 0, 0)

    def row_parallel(self, a, L, kind):
        if not self.ar:
            return self.w4(a, L, kind)
        if self.packed:
            return self.ar.w4_gemm_all_reduce_packed(a, L["packed_" + kind], L[kind][0].shape[1],
                                                     CFG4["G"])
        return self.ar.w4_gemm_all_reduce(a, *L[kind])

    def row_parallel_norm(self, a, L, kind, nw):
        """Row-parallel GEMM, all-reduce, then residual add + RMSNorm (fused or not)."""
        eps = 1e-6
        w = L[kind]
        if self.norm == "fused":
            if self.packed:
                n, pk = w[0].shape[1], L["packed_" + kind]
                if self.ar:
                    return self.ar.w4_gemm_all_reduce_rmsnorm_packed(a, pk, n, CFG4["G"], self.res,
                                                                     nw, eps)
                return self.ops.w4gemm_ar_rmsnorm_packed(a, pk, n, CFG4["G"], self.h1, self.res,
                                                         nw, eps)
            if self.ar:
                return self.ar.w4_gemm_all_reduce_rmsnorm(a, *w, self.res, nw, eps)
            return self.ops.w4gemm_ar_rmsnorm(a, *w, self.h1, self.res, nw, eps)
        y = self.row_parallel(a, L, kind)
        xf = y.float() + self.res.float()
        self.res.copy_(xf.half())
        return ((xf * (xf.pow(2).mean(dim=-1, keepdim=True) + eps).rsqrt()).half() * nw)

    def launch(self, kind: str, L: dict, h):
        if kind in ("o", "down"):
            return self.row_parallel(self.a_o if kind == "o" else self.a_d, L, kind)
        return self.w4(h, L, kind)

    def step(self):
        h = self.x0
        if self.norm:
            self.res.copy_(self.x0)
            for L, nw in zip(self.layers, self.nw):
                self.launch("qkv", L, h)
                h = self.row_parallel_norm(self.a_o, L, "o", nw[0])
                self.launch("gate_up", L, h)
                h = self.row_parallel_norm(self.a_d, L, "down", nw[1])
            return self.ops.gemm(h, self.lm, 0)
        for L in self.layers:
            self.launch("qkv", L, h)
            h = self.launch("o", L, h)
            self.launch("gate_up", L, h)
            h = self.launch("down", L, h)
        return self.ops.gemm(h, self.lm, 0)

    def kind_step(self, kind: str):
        """The step's launches of one kind only (64 of a layer kind, or 8 lm_head launches)."""
        if kind == "lm_head":
            for _ in range(8):
                self.ops.gemm(self.x0, self.lm, 0)
            return
        for L in self.layers:
            self.launch(kind, L, self.x0)


def kernel_breakdown(model: DecodeModel, world: int, capi, reps: int = 5) -> dict:
    """Per-launch device time of every kind of launch of the step: a graph of that kind's launches
    (the step's own weights, so every launch reads HBM), replayed `reps` times between CUDA
    events, max over ranks."""
    import torch

    c, P = CFG4, model.P
    st = torch.cuda.current_stream()
    out = {}
    for kind in ("qkv", "o", "gate_up", "down", "lm_head"):
        if kind == "lm_head":
            K, N, launches = c["hidden"], c["vocab"] // P, 8
            nb, name = f16_bytes(c["M"], K, N), "gemm_f16_kernel"
            plan = None
        else:
            K, N = layer_shapes(P)[kind]
            launches = c["layers"]
            nb = w4_bytes(c["M"], K, N, c["G"])
            fused = P > 1 and kind in ("o", "down")
            plan = capi.w4_plan(c["M"], K, N, c["G"], fused)
            name = plan["kernel"] + ("<fused all-reduce>" if fused else "")
        graph, _ = capture(lambda: model.kind_step(kind))
        graph.replay()
        ms = time_steps(graph.replay, reps, world, st)
        us = max_over_ranks(ms * 1e3 / (reps * launches), world)
        del graph
        out[kind] = {"kernel": name, "K": K, "N": N, "us_per_launch": round(us, 2),
                     "launches_per_step": 1 if kind == "lm_head" else c["layers"],
                     "bytes_per_launch": nb}
        if plan:
            out[kind]["plan"] = {k: plan[k] for k in ("cluster", "ctas")}
    return out


# ------------------------------------------------------------------------------------------------
# single-GEMM measurements (--sweep, and the `extra` keys of the default line)
# ------------------------------------------------------------------------------------------------


def measure_gemm(lib, capi, ws, name, kind, M, K, N, G, steps, warmup, peak, l2):
    """One GEMM shape: launches captured in a CUDA graph that rotates over enough weight copies
    to exceed 3x L2 (so every launch reads HBM), timed by replaying the graph."""
    import torch

    w4 = kind in ("w4", "w4p", "w4n")
    wbytes = K * N // 2 if w4 else 2 * N * K
    nb = w4_bytes(M, K, N, G) if w4 else f16_bytes(M, K, N)
    copies = max(1, int(3 * l2 // wbytes) + 1)
    g = torch.Generator(device="cuda").manual_seed(M * K + N)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    calls = []
    for _ in range(copies):
        if w4:
            qw = torch.randint(-2**31, 2**31 - 1, (K // 8, N), device="cuda", dtype=torch.int32, generator=g)
            qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), device="cuda", dtype=torch.int32, generator=g)
            sc = (torch.rand(K // G, N, device="cuda", generator=g) * 0.015 + 0.005).half()
            if kind == "w4p":  # repacked once, as at weight-load time; the originals are freed
                pk = torch.empty(lib.b2_w4_packed_bytes(K, N, G), dtype=torch.uint8, device="cuda")
                capi.check(lib.b2_w4_repack(qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), K, N, G,
                                            pk.data_ptr(), pk.numel(), 0), "b2_w4_repack")
                torch.cuda.synchronize()
                calls.append((pk,))
                del qw, qz, sc
            else:
                calls.append((qw, qz, sc))
        else:
            calls.append((torch.randn(N, K, device="cuda", generator=g) * 0.02).half(),)

    def launch(t, sp):
        if kind == "w4n":  # the entry point that allocates nothing (fixed scratch in the library)
            qw, qz, sc = t
            rc = lib.b2_w4_gemm_noalloc(x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(),
                                        y.data_ptr(), M, K, N, G, sp)
        elif kind == "w4p":
            rc = lib.b2_w4_gemm_packed(x.data_ptr(), t[0].data_ptr(), y.data_ptr(), M, K, N, G,
                                       ws.data_ptr(), ws.numel(), sp)
        elif kind == "w4":
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
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    times = []
    for _ in range(max(3, steps // reps)):
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


# ------------------------------------------------------------------------------------------------
# the default line
# ------------------------------------------------------------------------------------------------


def run_gpu(args):
    import torch

    import __graft_entry__ as entry

    rank, world, local = dist_setup(args.gpus)
    pkg = entry.load_package()
    from mi50_vllm_lab_b200 import capi, vllm_shim

    ops = pkg.ops()
    lib = capi.lib()
    c = CFG4
    M, H, P = c["M"], c["hidden"], world
    ar = None
    if P > 1:
        import datetime

        import torch.distributed as dist

        cpu = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=120))
        # 8 bytes per output element: room for the low-latency (value + generation) exchange
        ar = vllm_shim.NvlinkAllReduce(cpu, rank, list(range(P)), slot_bytes=M * H * 8)
    model = DecodeModel(ops, P, rank, ar)
    eager = model.step()
    torch.cuda.synchronize()
    graph, out = capture(model.step)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    same = bool(torch.equal(out, eager))
    stream = torch.cuda.current_stream()

    with ClockSampler(local) as clk:
        total_ms = time_steps(graph.replay, args.steps, world, stream)
    us_step = max_over_ranks(total_ms * 1e3 / args.steps, world)

    # end to end: the step's input activations from pinned host memory, the graph of operator
    # calls, the logits back to pinned host memory, every step
    x_host = torch.randn(M, H, generator=torch.Generator().manual_seed(7)).half().pin_memory()
    logits_host = torch.empty(out.shape, dtype=torch.float16).pin_memory()

    def e2e_step():
        model.x0.copy_(x_host, non_blocking=True)
        graph.replay()
        logits_host.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    e2e_ms = time_steps(e2e_step, args.steps, world, stream)
    e2e_us = max_over_ranks(e2e_ms * 1e3 / args.steps, world)

    # the same step with the decoder layer's two residual-add + RMSNorm steps per layer: fused
    # into the row-parallel GEMMs' epilogue, and as separate steps after them (one graph each)
    norms = {}
    if P == 1:
        name = f"/b2_bench_h1_{os.getpid()}"
        model.h1 = ops.nvar_create(name, M * H * 8, 0, 1)
        ops.hostar_unlink(name)
    for mode in ("fused", "unfused"):
        model.norm = mode
        model.step()
        torch.cuda.synchronize()
        g_n, _ = capture(model.step)
        for _ in range(args.warmup):
            g_n.replay()
        torch.cuda.synchronize()
        ms = time_steps(g_n.replay, args.steps, world, stream)
        norms[f"{mode}_us_per_step"] = round(max_over_ranks(ms * 1e3 / args.steps, world), 1)
        del g_n
    model.norm = None
    norms["norms_per_step"] = 2 * c["layers"]

    kernels = kernel_breakdown(model, world, capi)

    # the same step with the weights repacked at load time (w4_repack, then w4gemm_packed for the
    # launches without a fused all-reduce); the logits must be bit-identical
    ref = model.step()
    model.pack()
    eager_p = model.step()
    torch.cuda.synchronize()
    g_p, out_p = capture(model.step)
    for _ in range(args.warmup):
        g_p.replay()
    torch.cuda.synchronize()
    ms = time_steps(g_p.replay, args.steps, world, stream)
    packed = {"us_per_step": round(max_over_ranks(ms * 1e3 / args.steps, world), 1),
              "operators": "w4_repack once per weight; w4gemm_packed"
                           + (", w4gemm_ar_packed" if P > 1 else "") + ", gemm",
              "logits_equal_plain": bool(torch.equal(ref, eager_p) and torch.equal(out_p, eager_p))}
    del g_p
    status = ar.status() if ar else ops.workspace_status(False)
    peak, peak_kind = hbm_peak()
    nbytes = decode_step_bytes(P)
    for k in kernels.values():
        k["GBps"] = round(k["bytes_per_launch"] / k["us_per_launch"] / 1e3, 1)
        k["frac"] = round(k["GBps"] / peak, 4)
        k["us_per_step"] = round(k["us_per_launch"] * k["launches_per_step"], 1)
    dom_kind = max(kernels, key=lambda k: kernels[k]["us_per_step"])
    dom = kernels[dom_kind]
    del graph

    line = None
    if rank == 0:
        workload = f"config 4 TP={P} {dom_kind}"
        line = {
            "metric": METRIC, "value": round(us_step, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us_step / 1e3, 4),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "W4A16 / f16 (fp32 accumulate)",
            "data": "synthetic (seeded random int4 weights, U[0.005,0.02] scales, N(0,1) activations)",
            "config": {"workload": "config 4: decode-verify step, 64 W4A16 layers + fp16 lm_head",
                       "M": M, "tp": P, "layers": c["layers"], "hidden": H, "qkv": c["qkv"],
                       "o_in": c["o_in"], "intermediate": c["inter"], "vocab": c["vocab"],
                       "group_size": c["G"], "kernels_per_step": 4 * c["layers"] + 1,
                       "fused_allreduces_per_step": 2 * c["layers"] if P > 1 else 0,
                       "parallelism": f"tp{P}", "per_rank_bytes_per_step": nbytes,
                       "graph": "one CUDA graph per step; programmatic dependent launch between GEMMs",
                       "l2": f"each step streams {nbytes / 1e9:.2f} GB of weights per rank "
                             f"(> 126 MB L2; no flush needed)"},
            "step_hbm": {"GBps_per_rank": round(nbytes / us_step / 1e3, 1),
                         "frac": round(nbytes / us_step / 1e3 / peak, 4)},
            "e2e": {"value": round(e2e_us, 1), "unit": UNIT, "ms_per_step": round(e2e_us / 1e3, 4),
                    "api": "torch.ops.gfx906_skinny (w4gemm, w4gemm_ar, gemm) captured in one CUDA "
                           "graph; pinned host x -> device, logits -> pinned host every step",
                    "h2d_bytes_per_step": M * H * 2, "d2h_bytes_per_step": int(out.numel()) * 2},
            "roofline": {"bound": "hbm", "achieved": dom["GBps"], "peak": peak, "unit": "GB/s",
                         "frac": dom["frac"],
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, copy bandwidth)",
                         "kernel": dom["kernel"], "launch": dom_kind, "kernel_us": dom["us_per_launch"],
                         "bytes_per_launch": dom["bytes_per_launch"],
                         "traffic": recorded_traffic(dom["kernel"].split("<")[0], workload)},
            "kernels": kernels,
            "config4_with_norms": norms,
            "config4_packed_weights": packed,
            "gpu_launches": args.steps * (4 * c["layers"] + 1),
            "graph_equals_eager": same, "device_status": int(status),
            "clocks": clk.summary(),
        }
    if world == 1:
        del model
        torch.cuda.empty_cache()
        ws = torch.zeros(lib.b2_workspace_bytes(local), dtype=torch.uint8, device="cuda")
        l2 = torch.cuda.get_device_properties(local).L2_cache_size
        extra = {}
        for key, kind, cfg in (("config1_fp16_lm_head", "f16", dict(CFG1, G=0)),
                               ("config0_w4", "w4", CFG0)):
            r = measure_gemm(lib, capi, ws, key, kind, cfg["M"], cfg["K"], cfg["N"], cfg["G"],
                             200, args.warmup, peak, l2)
            extra[key] = {k: r[k] for k in ("M", "K", "N", "G", "us", "TBps", "frac", "bytes",
                                            "l2_rotation_copies")}
            torch.cuda.empty_cache()
        line["extra"] = extra
        if not args.no_cpu:
            from oracle import cpu_baseline

            cb = cpu_baseline.time_decode_step(CFG4, budget_s=args.cpu_seconds)
            cb["cpu_model"] = cpu_model()
            line["cpu_baseline"] = cb
    if line:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_reference(args):
    """The reference's CPU implementation of the path (oracle port of kernels/check_w4.py:11-21
    and kernels/bench_skinny.py:44) on the default line's step and metric, all host threads.
    Each step is a sample (a column sample of every GEMM of one layer and a row sample of the
    lm_head) scaled to a full config-4 step; the CPU computes the whole step, all ranks' shards.
    Under torchrun only rank 0 runs."""
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import cpu_baseline

    torch.set_num_threads(os.cpu_count() or 1)
    sample = cpu_baseline.DecodeStepSample(CFG4)
    for _ in range(args.warmup):
        sample.estimate_step_seconds()
    est = [sample.estimate_step_seconds() for _ in range(args.steps)]
    sec = sum(est) / len(est)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    line = {
        "impl": "reference", "metric": METRIC, "value": round(sec * 1e6, 1), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32 (the reference's torch check computes (q - z) * s and x @ deq; float32 here)",
        "data": "synthetic",
        "config": {"workload": "config 4: decode-verify step, 64 W4A16 layers + fp16 lm_head",
                   "M": CFG4["M"], "tp": world, "layers": CFG4["layers"],
                   "parallelism": "host cores (the whole step, every rank's shard)"},
        "cpu_baseline": {"value": round(sec * 1e6, 1), "unit": UNIT,
                         "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample.describe(), "cpu_model": cpu_model()},
        "e2e": {"value": round(sec * 1e6, 1), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_config1(args):
    """BASELINE config 1 alone (the earlier default line): the fp16 lm_head GEMM through the C
    ABI on device-resident operands, back to back; TB/s of algorithmic bytes."""
    import torch

    import __graft_entry__ as entry

    rank, world, local = dist_setup(args.gpus)
    entry.load_package()
    from mi50_vllm_lab_b200 import capi

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
        capi.check(lib.b2_gemm_f16(x.data_ptr(), w.data_ptr(), y.data_ptr(), M, K, N,
                                   ws.data_ptr(), ws.numel(), sp), "b2_gemm_f16")

    for _ in range(args.warmup):
        step()
    with ClockSampler(local) as clk:
        total_ms = time_steps(step, args.steps, world, stream)
    ms_step = max_over_ranks(total_ms / args.steps, world)
    peak, peak_kind = hbm_peak()
    if rank == 0:
        print(json.dumps({
            "metric": "config 1: fp16 skinny GEMM (lm_head shape) HBM throughput", "unit": "TB/s",
            "value": round(world * nbytes / (ms_step * 1e-3) / 1e12, 4), "n_gpus": world,
            "us_per_gemm": round(ms_step * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "roofline": {"bound": "hbm", "achieved": round(nbytes / (ms_step * 1e-3) / 1e9, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(nbytes / (ms_step * 1e6) / peak, 4),
                         "peak_source": peak_kind, "kernel": "gemm_f16_kernel",
                         "traffic": recorded_traffic("gemm_f16_kernel", "config1")},
            "clocks": clk.summary()}), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


# fp16 drafter layers of kernels/bench_skinny.py:34-37, as (N, K) - the reference's own table
DRAFTER = {"qkv": (3072, 5120), "o": (5120, 2048), "gate_up": (17408, 5120), "down": (5120, 8704),
           "fc": (5120, 25600), "ctx_kv": (5120, 5120), "kproj": (1280, 5120)}

SWEEP = (
    [("cfg1_lm_head", "f16", 7, 5120, 151936, 0), ("cfg0", "w4", 7, 4096, 4096, 128)]
    + [(f"cfg2_{nm}_M{M}", "w4", M, K, N, 128) for M in (1, 2, 4, 8)
       for nm, (K, N) in {"qkv": (5120, 8192), "o_proj": (6144, 5120), "gate_up": (5120, 34816),
                          "down": (17408, 5120)}.items()]
    + [(f"cfg3_down_TP{P}", "w4", 8, 17408 // P, 5120, 128) for P in (2, 4, 8)]
    + [(f"cfg4_TP8_{nm}", "w4", 8, K, N, 128) for nm, (K, N) in layer_shapes(8).items()]
    + [(f"drafter_{nm}_M{M}", "f16", M, K, N, 0) for M in (1, 7, 8)
       for nm, (N, K) in DRAFTER.items()]
    + [("check_w4_G32", "w4", 8, 5120, 1024, 32)]
    # the same shapes through b2_w4_gemm_noalloc (no workspace argument)
    + [("cfg0_noalloc", "w4n", 7, 4096, 4096, 128)]
    + [(f"cfg2_{nm}_M8_noalloc", "w4n", 8, K, N, 128)
       for nm, (K, N) in {"qkv": (5120, 8192), "o_proj": (6144, 5120), "gate_up": (5120, 34816),
                          "down": (17408, 5120)}.items()]
    # weights repacked at load time (b2_w4_repack): the same shapes through b2_w4_gemm_packed
    + [("cfg0_packed", "w4p", 7, 4096, 4096, 128)]
    + [(f"cfg2_{nm}_M8_packed", "w4p", 8, K, N, 128)
       for nm, (K, N) in {"qkv": (5120, 8192), "o_proj": (6144, 5120), "gate_up": (5120, 34816),
                          "down": (17408, 5120)}.items()]
    + [(f"cfg3_down_TP{P}_packed", "w4p", 8, 17408 // P, 5120, 128) for P in (2, 4, 8)]
    + [(f"cfg4_TP8_{nm}_packed", "w4p", 8, K, N, 128) for nm, (K, N) in layer_shapes(8).items()]
)
# Extra cases for --profile only: the lm_head kernel on a 335 MB slice (above L2, small enough
# for a multi-pass ncu capture); traffic scales with N for this kernel.
PROFILE_ONLY = [("cfg1_lm_head_N32768", "f16", 7, 5120, 32768, 0)]


def run_sweep(args):
    """Every single-GEMM BASELINE config (and the drafter shapes of kernels/bench_skinny.py:34-38)
    on one GPU, timed by graph replay over > 3x L2 of weight copies (see measure_gemm)."""
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
    for w in SWEEP:
        if args.only and not any(o in w[0] for o in args.only.split(",")):
            continue
        r = measure_gemm(lib, capi, ws, *w, args.steps, args.warmup, peak, l2)
        if w[1] in ("w4", "w4p", "w4n"):
            r["plan"] = capi.w4_plan(w[2], w[3], w[4], w[5])
        print(json.dumps(r), flush=True)
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
    for kv in args.tune:
        k, v = (int(t) for t in kv.split("="))
        capi.check(lib.b2_set_tuning(k, v), "b2_set_tuning")
    cases = PROFILE_ONLY + list(SWEEP)  # an exact workload name, else the first that contains it
    name, kind, M, K, N, G = next((w for w in cases if args.only == w[0]), None) or \
        next(w for w in cases if args.only in w[0])
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    y = torch.empty(M, N, dtype=torch.float16, device="cuda")
    sp = torch.cuda.current_stream().cuda_stream
    if kind in ("w4", "w4p"):
        qw = torch.randint(-2**31, 2**31 - 1, (K // 8, N), device="cuda", dtype=torch.int32, generator=g)
        qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), device="cuda", dtype=torch.int32, generator=g)
        sc = (torch.rand(K // G, N, device="cuda", generator=g) * 0.015 + 0.005).half()
        step = lambda: capi.check(lib.b2_w4_gemm(x.data_ptr(), qw.data_ptr(), qz.data_ptr(),  # noqa: E731
                                                 sc.data_ptr(), y.data_ptr(), M, K, N, G,
                                                 ws.data_ptr(), ws.numel(), sp))
        if kind == "w4p":
            pk = torch.empty(lib.b2_w4_packed_bytes(K, N, G), dtype=torch.uint8, device="cuda")
            capi.check(lib.b2_w4_repack(qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), K, N, G,
                                        pk.data_ptr(), pk.numel(), sp), "b2_w4_repack")
            step = lambda: capi.check(lib.b2_w4_gemm_packed(  # noqa: E731
                x.data_ptr(), pk.data_ptr(), y.data_ptr(), M, K, N, G, ws.data_ptr(), ws.numel(), sp))
    else:
        w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
        step = lambda: capi.check(lib.b2_gemm_f16(x.data_ptr(), w.data_ptr(), y.data_ptr(), M, K,  # noqa: E731
                                                  N, ws.data_ptr(), ws.numel(), sp))
    for _ in range(args.warmup + args.steps):
        step()
    torch.cuda.synchronize()
    print(json.dumps({"profiled": name, "launches": args.warmup + args.steps}))



def run_norm_epilogue(args):
    """Row-parallel W4 layer + residual add + RMSNorm on one GPU (one-rank all-reduce handle):
    the fused call (w4gemm_ar_rmsnorm: the GEMM + all-reduce launch, then its finishing launch;
    and with the norm inside the GEMM's launch) against the fused GEMM + all-reduce followed by a
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
                # the norm inside the GEMM's launch instead of a finishing launch
                # (B2_TUNE_NORM_IN_LAUNCH)
                "gemm_ar_norm_in_launch": lambda t: ops.w4gemm_ar_rmsnorm(x, *t, h, r, w, eps),
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
                capi.check(lib.b2_set_tuning(10, 1 if vname == "gemm_ar_norm_in_launch" else 0),
                           "b2_set_tuning")
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
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--sweep", action="store_true")
    ap.add_argument("--config1", action="store_true",
                    help="config 1 alone: the fp16 lm_head GEMM back to back (TB/s)")
    ap.add_argument("--only", default="", help="with --sweep: workloads whose name contains one of these comma-separated "
                         "strings; with --profile: the first workload whose name contains it")
    ap.add_argument("--profile", action="store_true", help="eager launches of one --only workload (for ncu)")
    ap.add_argument("--trace", default="", metavar="M,K,N[,G]",
                    help="per-unit timeline of one W4 cluster-kernel launch (trace build: "
                         "python mi50-vllm-lab_b200/builder.py --trace)")
    ap.add_argument("--trace-units", action="store_true", help="with --trace: the raw stamps too")
    ap.add_argument("--trace-fused", default="", metavar="K,N",
                    help="under torchrun: phase timeline of the fused GEMM + all-reduce (trace build)")
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
    if args.trace_fused:
        import __graft_entry__ as entry

        entry.load_package()
        from mi50_vllm_lab_b200 import trace_fused

        kn = args.trace_fused.split(",")
        out = trace_fused.main([",".join(kn[:2])] + (["--norm"] if "norm" in kn[2:] else [])
                               + list(args.tune))
        if out is not None:
            print(json.dumps(out))
        return
    if args.impl == "reference":
        run_reference(args)
    elif args.trace:
        import __graft_entry__ as entry

        entry.load_package()
        from mi50_vllm_lab_b200 import trace_w4

        argv = args.trace.split(",") + (["--units"] if args.trace_units else [])
        for kv in args.tune:
            argv += ["--tune", kv]
        print(json.dumps(trace_w4.main(argv)))
    elif args.profile:
        run_profile(args)
    elif args.sweep:
        run_sweep(args)
    elif args.config1:
        run_config1(args)
    elif args.norm_epilogue:
        run_norm_epilogue(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
