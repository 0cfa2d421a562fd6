"""Helpers for the GPU tests: device inputs in the reference's layouts, oracle checks on full
outputs or on sampled columns, and C-ABI calls with torch-owned device buffers."""

from __future__ import annotations

import numpy as np
import torch

from oracle import skinny_oracle as so


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check(y: torch.Tensor, ref: np.ndarray, what: str = "") -> dict:
    yn = y.float().cpu().numpy()
    assert np.isfinite(yn).all(), f"{what}: non-finite output"
    st = so.error_stats(yn, ref)
    assert so.within_tolerance(st), f"{what}: outside tolerance {st}"
    return st


def mismatch(a: torch.Tensor, b: torch.Tensor, tile: int = 128) -> str:
    """Where two results of the same call differ: element count, rows, 128-column tiles, the
    columns inside a tile, and the largest difference (for the message of a failed assert)."""
    d = a != b
    if not bool(d.any()):
        return "equal"
    idx = d.nonzero()
    cols = idx[:, 1].unique()
    big = float((a.float() - b.float()).abs().nan_to_num(float("inf")).max())
    return (f"{int(d.sum())} elements differ; rows {idx[:, 0].unique().tolist()}; "
            f"tiles {sorted(set((cols // tile).tolist()))[:16]}; "
            f"columns in tile {sorted(set((cols % tile).tolist()))[:16]}; max |diff| {big}; "
            f"nan {int(torch.isnan(a).sum())}/{int(torch.isnan(b).sum())}")


def sample_columns(N: int, n: int, seed: int, tile: int = 128) -> np.ndarray:
    """Sorted columns: `n` random ones plus both edges of every 16th tile and the last column."""
    rng = np.random.default_rng(seed)
    cols = set(rng.choice(N, size=min(n, N), replace=False).tolist())
    for t in range(0, (N + tile - 1) // tile, 16):
        cols.update({t * tile, min(N - 1, t * tile + tile - 1)})
    cols.add(N - 1)
    return np.array(sorted(cols))


def w4_device_inputs(M: int, K: int, N: int, G: int, seed: int, x_scale: float = 1.0):
    """Large W4 inputs made on the GPU: every nibble uniform 0..15 (full-range int32 words as in
    kernels/check_w4.py:8-9), scales U[0.005, 0.02], x ~ N(0,1) * x_scale."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    qw = torch.randint(-2**31, 2**31 - 1, (K // 8, N), device="cuda", dtype=torch.int32, generator=g)
    qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), device="cuda", dtype=torch.int32,
                       generator=g)
    sc = (torch.rand(K // G, N, device="cuda", generator=g) * 0.015 + 0.005).half()
    x = (torch.randn(M, K, device="cuda", generator=g) * x_scale).half()
    return x, qw, qz, sc


def w4_ref_sampled(x, qw, qz, sc, cols: np.ndarray) -> np.ndarray:
    blocks = np.unique(cols // 8)
    full = np.concatenate([np.arange(b * 8, b * 8 + 8) for b in blocks])
    fi = torch.from_numpy(full).cuda()
    bi = torch.from_numpy(blocks).cuda()
    sub = so.w4_ref(x.cpu().numpy(), qw.index_select(1, fi).cpu().numpy(),
                    qz.index_select(1, bi).cpu().numpy(), sc.index_select(1, fi).cpu().numpy())
    pos = {c: i for i, c in enumerate(full)}
    return sub[:, [pos[c] for c in cols]]


def f16_ref_sampled(x, w, cols: np.ndarray) -> np.ndarray:
    wi = w.index_select(0, torch.from_numpy(cols).cuda()).cpu().numpy()
    return so.gemm_ref(x.cpu().numpy(), wi)


def workspace(capi) -> torch.Tensor:
    """A zero-filled workspace owned by torch (what a non-torch host would cudaMalloc)."""
    nbytes = capi.lib().b2_workspace_bytes(0)
    return torch.zeros(nbytes, dtype=torch.uint8, device="cuda")


def stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream
