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
