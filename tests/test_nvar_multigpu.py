"""NVLink all-reduce and the fused W4 GEMM + all-reduce on 2 (and 4, 8 when present) GPUs, one
process per GPU (tests/mp_nvar_worker.py under torch.distributed.run)."""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(nproc: int, quick: bool) -> subprocess.CompletedProcess:
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", B2_NVAR_TIMEOUT_MS="5000")
    cmd = ["timeout", "-k", "30", "420", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), str(ROOT / "tests" / "mp_nvar_worker.py")]
    if quick:
        cmd.append("--quick")
    return subprocess.run(cmd, env=env, capture_output=True, text=True, cwd=ROOT)


@pytest.mark.parametrize("nproc", [2, 4, 8])
def test_nvlink_allreduce_and_fused_gemm(nproc):
    import torch

    if torch.cuda.device_count() < nproc:
        pytest.skip(f"needs {nproc} GPUs")
    r = _run(nproc, quick=nproc > 2)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert "all checks passed" in out, out[-4000:]
