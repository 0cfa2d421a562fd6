"""ctypes binding of the C ABI in ``include/b2_skinny.h`` (libb2skinny.so).

This is the binding a non-torch host (or a test) uses: plain pointers, sizes and a stream
handle. Every function returns a status code; :func:`check` turns a non-zero code into an
exception carrying ``b2_last_error()``.
"""

from __future__ import annotations

import ctypes as C
import re
import threading
from pathlib import Path

from . import CAPI_LIB

HEADER = Path(__file__).resolve().parents[1] / "include" / "b2_skinny.h"

B2_OK = 0
B2_ERR_INVALID_ARG = 1
B2_ERR_UNSUPPORTED = 2
B2_ERR_CUDA = 3
B2_ERR_WORKSPACE = 4
B2_ERR_TIMEOUT = 5
B2_ERR_STATE = 6
B2_DTYPE_F16 = 0
B2_DTYPE_F32 = 1
B2_BLOB_BYTES = 64
B2_TUNE_CTAS_PER_SM = 1
B2_TUNE_MIN_UNITS = 2
B2_TUNE_NO_PDL = 3
B2_TUNE_W4_PATH = 4
B2_TUNE_W4_CLUSTER = 5
B2_TUNE_AR_FLAGS = 6
B2_TUNE_AR_TWO_SHOT = 7
B2_TUNE_W4_NO_ALIAS = 8
B2_TUNE_NORM_NO_COOP = 9
B2_TUNE_NORM_IN_LAUNCH = 10

_vp, _i, _sz, _u64 = C.c_void_p, C.c_int, C.c_size_t, C.c_uint64
_SIGS = {
    "b2_status_string": (C.c_char_p, [_i]),
    "b2_last_error": (C.c_char_p, []),
    "b2_abi_version": (_i, []),
    "b2_workspace_bytes": (_sz, [_i]),
    "b2_workspace_init": (_i, [_vp, _sz, _vp]),
    "b2_workspace_status": (_i, [_vp, _i, C.POINTER(_i)]),
    "b2_gemm_f16": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    "b2_w4_gemm": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    "b2_w4_packed_bytes": (_sz, [_i, _i, _i]),
    "b2_w4_repack": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    "b2_w4_gemm_packed": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    "b2_w4_gemm_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "b2_w4_noalloc_scratch": (_i, [C.POINTER(_vp), C.POINTER(_sz)]),
    "b2_registry_open": (_i, [C.c_char_p, _i, _i, C.POINTER(_vp)]),
    "b2_registry_put": (_i, [_vp, _i, _vp]),
    "b2_registry_get": (_i, [_vp, _i, _vp]),
    "b2_registry_close": (_i, [_vp]),
    "b2_registry_unlink": (_i, [C.c_char_p]),
    "b2_nvar_create": (_i, [_i, _i, _i, _sz, C.POINTER(_vp)]),
    "b2_nvar_export": (_i, [_vp, _vp]),
    "b2_nvar_connect": (_i, [_vp, _vp]),
    "b2_nvar_is_connected": (_i, [_vp]),
    "b2_nvar_max_bytes": (_sz, [_vp]),
    "b2_nvar_set_timeout_ns": (_i, [_vp, _u64]),
    "b2_nvar_allreduce": (_i, [_vp, _vp, _vp, _sz, _i, _vp]),
    "b2_w4_gemm_allreduce": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    "b2_w4_gemm_allreduce_rmsnorm": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, C.c_float, _vp, _i, _i,
                                          _i, _i, _vp, _sz, _vp]),
    "b2_w4_gemm_allreduce_packed": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    "b2_w4_gemm_allreduce_rmsnorm_packed": (_i, [_vp, _vp, _vp, _vp, _vp, C.c_float, _vp, _i, _i,
                                                 _i, _i, _vp, _sz, _vp]),
    "b2_nvar_status": (_i, [_vp, _i, C.POINTER(_i)]),
    "b2_nvar_rank": (_i, [_vp]),
    "b2_nvar_world": (_i, [_vp]),
    "b2_nvar_destroy": (_i, [_vp]),
    "b2_nvar_connect_local": (_i, [C.POINTER(_vp), _i]),
    "b2_nvar_allreduce_emulated": (_i, [C.POINTER(_vp), _i, C.POINTER(_vp), C.POINTER(_vp), _sz,
                                        _i, _vp]),
    "b2_w4_gemm_allreduce_emulated": (_i, [C.POINTER(_vp), _i, C.POINTER(_vp), C.POINTER(_vp),
                                           C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp),
                                           C.POINTER(_vp), C.c_float, C.POINTER(_vp), _i, _i, _i,
                                           _i, C.POINTER(_vp), _sz, _vp]),
    "b2_set_tuning": (_i, [_i, _i]),
    "b2_get_tuning": (_i, [_i]),
    "b2_w4_plan": (_i, [_i, _i, _i, _i, _i, C.POINTER(_i), C.POINTER(_i), C.POINTER(_i)]),
}

_lib = None
_lock = threading.Lock()


def declared_functions() -> list[str]:
    """Names of the functions ``include/b2_skinny.h`` declares."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", text)))


def lib() -> C.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not CAPI_LIB.exists():
                raise RuntimeError(f"{CAPI_LIB} is not built")
            L = C.CDLL(str(CAPI_LIB))
            for name, (res, args) in _SIGS.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _lib = L
    return _lib


class B2Error(RuntimeError):
    def __init__(self, status: int, where: str):
        L = lib()
        super().__init__(f"{where}: {L.b2_status_string(status).decode()} "
                         f"({status}): {L.b2_last_error().decode()}")
        self.status = status


def check(status: int, where: str = "b2") -> None:
    if status != B2_OK:
        raise B2Error(status, where)


def w4_plan(M: int, K: int, N: int, G: int, fused: bool = False) -> dict:
    """The split-K plan the W4 entry points would launch (b2_w4_plan): the kernel's name, the
    path (1 stream-K, 2 clusters), CTAs per cluster and the grid size."""
    path, cs, ctas = C.c_int(), C.c_int(), C.c_int()
    check(lib().b2_w4_plan(M, K, N, G, 1 if fused else 0, C.byref(path), C.byref(cs),
                           C.byref(ctas)), "b2_w4_plan")
    kernel = "w4c_kernel" if path.value == 2 else "w4_kernel"
    return {"kernel": kernel, "path": path.value, "cluster": cs.value, "ctas": ctas.value}


def ptr_array(ptrs) -> "C.Array":
    """A C array of void* (for the entry points that take one pointer per rank); None -> NULL."""
    return (_vp * len(ptrs))(*[p if p is None else int(p) for p in ptrs])
