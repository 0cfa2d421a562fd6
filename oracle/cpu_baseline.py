"""The reference's CPU path for the skinny GEMMs, timed on the host cores (test / bench only).

The reference computes its correctness references with torch on the host side of the same
expressions the GPU kernels implement:
  * fp16 GEMM: ``x.float() @ w.float().T``           (kernels/bench_skinny.py:44)
  * W4A16:     unpack, ``(w - z) * s``, ``x @ deq``    (kernels/check_w4.py:11-21)
These functions run those expressions in float32 with all host threads; ``bench.py`` reports
their throughput as the CPU baseline beside the B200 number.
"""

from __future__ import annotations

import os
import time

import torch


def f16_reference(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """kernels/bench_skinny.py:44."""
    return x.float() @ w.float().T


def w4_reference(x: torch.Tensor, qw: torch.Tensor, qz: torch.Tensor, sc: torch.Tensor) -> torch.Tensor:
    """kernels/check_w4.py:11-18,21 in float32 (the reference runs it in float64 for checking)."""
    K, N = x.shape[1], qw.shape[1]
    G = K // sc.shape[0]
    u = qw.to(torch.int64) & 0xFFFFFFFF
    w = torch.empty(K, N, dtype=torch.float32)
    for i in range(4):
        w[2 * i::8] = ((u >> (4 * i)) & 0xF).float()
        w[2 * i + 1::8] = ((u >> (16 + 4 * i)) & 0xF).float()
    zu = qz.to(torch.int64) & 0xFFFFFFFF
    z = torch.stack([(zu >> (4 * c)) & 0xF for c in range(8)], dim=-1).reshape(K // G, N).float()
    deq = (w - z.repeat_interleave(G, 0)) * sc.float().repeat_interleave(G, 0)
    return x.float() @ deq


def _bytes_f16(M, K, N):
    return 2 * N * K + 2 * M * K + 2 * M * N


def time_f16(x: torch.Tensor, w_rows: torch.Tensor, budget_s: float = 10.0) -> dict:
    """Median time of f16_reference on a row sample of the weights, with all host threads,
    repeated for about `budget_s` seconds. Returns the cpu_baseline record of bench.py."""
    torch.set_num_threads(os.cpu_count() or 1)
    x = x.cpu()
    w_rows = w_rows.cpu()
    M, K = x.shape
    rows = w_rows.shape[0]
    f16_reference(x, w_rows)  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 5:
        t0 = time.perf_counter()
        f16_reference(x, w_rows)
        times.append(time.perf_counter() - t0)
    times.sort()
    sec = times[len(times) // 2]
    return {
        "value": round(_bytes_f16(M, K, rows) / sec / 1e12, 6),
        "unit": "TB/s",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": (f"x.float() @ w.float().T (kernels/bench_skinny.py:44) on {rows} weight rows "
                   f"x K={K}, M={M}; median of {len(times)} calls over {budget_s:.0f} s; "
                   f"{sec * 1e3:.2f} ms per call"),
    }


def _bytes_w4(M, K, N, G):
    return K * N // 2 + (K // G) * N * 2 + (K // G) * N // 2 + 2 * M * K + 2 * M * N


class DecodeStepSample:
    """A bounded CPU sample of the decode-verify step of BASELINE config 4 (64 W4A16 layers of
    qkv_proj, o_proj, gate_up, down_proj and an fp16 lm_head, M rows), run with the reference's
    torch expressions: every W4 GEMM of one layer at its full K on `cols` of its output columns
    (w4_reference, kernels/check_w4.py:11-21), and the lm_head on `lm_rows` of its rows
    (f16_reference, kernels/bench_skinny.py:44). The work of these expressions is linear in the
    number of output columns, so each part's time scales by N / sample to the full GEMM, and the
    layer by the number of layers, to estimate one full step (all ranks' shards)."""

    def __init__(self, cfg: dict, cols: int = 2048, lm_rows: int = 8192, seed: int = 7):
        torch.set_num_threads(os.cpu_count() or 1)
        g = torch.Generator().manual_seed(seed)
        M, H, G = cfg["M"], cfg["hidden"], cfg["G"]
        self.cfg, self.cols, self.lm_rows = cfg, cols, lm_rows
        shapes = {"qkv": (H, cfg["qkv"]), "o_proj": (cfg["o_in"], H),
                  "gate_up": (H, 2 * cfg["inter"]), "down": (cfg["inter"], H)}
        self.parts = []
        for name, (K, N) in shapes.items():
            n = min(cols, N)
            x = torch.randn(M, K, generator=g).half()
            qw = torch.randint(-2**31, 2**31 - 1, (K // 8, n), dtype=torch.int32, generator=g)
            qz = torch.randint(-2**31, 2**31 - 1, (K // G, n // 8), dtype=torch.int32, generator=g)
            sc = (torch.rand(K // G, n, generator=g) * 0.015 + 0.005).half()
            self.parts.append((name, (x, qw, qz, sc), cfg["layers"] * N / n, (K, N)))
        self.lm_x = torch.randn(M, H, generator=g).half()
        self.lm_w = (torch.randn(lm_rows, H, generator=g) * 0.02).half()
        self.lm_scale = cfg["vocab"] / lm_rows

    def estimate_step_seconds(self) -> float:
        total = 0.0
        for _, args, scale, _ in self.parts:
            t0 = time.perf_counter()
            w4_reference(*args)
            total += (time.perf_counter() - t0) * scale
        t0 = time.perf_counter()
        f16_reference(self.lm_x, self.lm_w)
        return total + (time.perf_counter() - t0) * self.lm_scale

    def describe(self) -> str:
        c = self.cfg
        return (f"one layer's 4 W4A16 GEMMs (full K, {self.cols} output columns each; torch "
                f"dequantize-then-matmul of kernels/check_w4.py:11-21 in float32) x {c['layers']} "
                f"layers, plus the fp16 lm_head on {self.lm_rows} of {c['vocab']} rows "
                f"(x.float() @ w.float().T, kernels/bench_skinny.py:44), each part scaled by its "
                f"full N / sampled N; M={c['M']}, torch {torch.__version__}")


def time_decode_step(cfg: dict, budget_s: float = 10.0) -> dict:
    """Median estimated seconds per full config-4 step over ~budget_s of samples (at least 3),
    with all host threads. Returns the cpu_baseline record of bench.py (value in us per step)."""
    sample = DecodeStepSample(cfg)
    sample.estimate_step_seconds()  # warm-up
    est = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(est) < 3:
        est.append(sample.estimate_step_seconds())
    est.sort()
    sec = est[len(est) // 2]
    return {"value": round(sec * 1e6, 1), "unit": "us", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": sample.describe() + f"; median of {len(est)} samples over {budget_s:.0f} s"}
