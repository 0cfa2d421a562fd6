"""B200-native (sm_100a) skinny-GEMM path of 0c33/mi50-vllm-lab.

Speculative-decode verify steps run their projections at M <= 8 rows. This package provides the
kernels for them behind the reference's operator library ``gfx906_skinny``:

* ``gfx906_skinny.so`` (``torch.ops.gfx906_skinny``): ``gemm``, ``w4gemm``, ``hostar_*`` with the
  reference's schemas, plus ``nvar_*`` (N-rank NVLink all-reduce) and ``w4gemm_ar`` (row-parallel
  W4 GEMM with the all-reduce fused into its epilogue);
* ``libb2skinny.so``: the CUDA kernels and their C ABI (``include/b2_skinny.h``);
* :mod:`.vllm_shim`: the vLLM call sites of the reference (predicates and set-up), ported;
* :mod:`.capi`: a ctypes binding of the C ABI.

There is no CPU fallback: on a machine without the built libraries or without an sm_100 GPU the
operators raise.
"""

from __future__ import annotations

import threading
from pathlib import Path

HERE = Path(__file__).resolve().parent
OPS_LIB = HERE / "gfx906_skinny.so"
CAPI_LIB = HERE / "libb2skinny.so"

_lock = threading.Lock()
_ops_loaded = False


def lib_path() -> str:
    """Path of the operator library (the value for VLLM_GFX906_SKINNY8_LIB / _HOSTAR_LIB)."""
    return str(OPS_LIB)


def build(verbose: bool = False):
    """Compile both libraries in place (nvcc for sm_100a, g++ for the torch bindings)."""
    from . import builder

    return builder.build(verbose=verbose)


def ops():
    """Load ``gfx906_skinny.so`` once and return ``torch.ops.gfx906_skinny``."""
    global _ops_loaded
    import torch

    with _lock:
        if not _ops_loaded:
            if not OPS_LIB.exists():
                raise RuntimeError(
                    f"{OPS_LIB} is not built; call build() (nvcc for sm_100a) first")
            torch.ops.load_library(str(OPS_LIB))
            _ops_loaded = True
    return torch.ops.gfx906_skinny


def load_capi():
    """The C ABI through ctypes (see :mod:`.capi`)."""
    from . import capi

    return capi.lib()
