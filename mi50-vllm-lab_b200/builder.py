"""Build the two in-tree shared libraries of the package.

* ``libb2skinny.so``  - the CUDA kernels and their C ABI (``include/b2_skinny.h``), compiled by
  nvcc for sm_100a only, with the CUDA runtime linked statically. No torch dependency.
* ``gfx906_skinny.so`` - the PyTorch operator library: registers ``torch.ops.gfx906_skinny.*``
  with the reference's schemas (kernels/skinny.cu:330-333, kernels/w4.cu:506-509,
  kernels/hostar.cu:155-166) and forwards to the C ABI. Load it with
  ``torch.ops.load_library`` exactly like the reference's ``gfx906_skinny.so``
  (kernels/build.py:12-14, patches/vllm/utils.patch:17).

Both land next to this file so that they travel with the source tree. Objects go to ``_build/``.
Rebuilds only what changed (by modification time).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
BUILD = HERE / "_build"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU_SOURCES = ["b2_runtime.cu", "b2_gemm_f16.cu", "b2_w4.cu", "b2_nvar.cu"]
HEADERS = ["b2_device.cuh", "b2_internal.h", "b2_nvar.cuh"]

CAPI_LIB = HERE / "libb2skinny.so"
TORCH_LIB = HERE / "gfx906_skinny.so"


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... ({r.returncode})")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)


def build_capi(verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    common_deps = [CSRC / h for h in HEADERS] + [INCLUDE / "b2_skinny.h"]
    objs = []
    for src in CU_SOURCES:
        obj = BUILD / (src + ".o")
        objs.append(obj)
        if _newer(obj, [CSRC / src] + common_deps) or ptxas_verbose:
            cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                   "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(CSRC / src),
                   "-o", str(obj)]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            _run(cmd, verbose or ptxas_verbose)
    if _newer(CAPI_LIB, objs):
        tmp = BUILD / CAPI_LIB.name
        _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lrt"], verbose)
        shutil.move(str(tmp), CAPI_LIB)
    return CAPI_LIB


def build_torch_ops(verbose: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "torch_ops.cpp"
    if not _newer(TORCH_LIB, [src, INCLUDE / "b2_skinny.h", CAPI_LIB]):
        return TORCH_LIB
    inc = [f"-I{p}" for p in cpp_extension.include_paths()]
    libdirs = cpp_extension.library_paths()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    py_inc = sysconfig.get_paths()["include"]
    tmp = BUILD / TORCH_LIB.name
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=gfx906_skinny", *inc, f"-I{py_inc}", f"-I{CUDA_HOME / 'include'}",
           f"-I{INCLUDE}", str(src), "-o", str(tmp), f"-L{HERE}", "-lb2skinny",
           "-Wl,-rpath,$ORIGIN"]
    for d in libdirs:
        cmd += [f"-L{d}", f"-Wl,-rpath,{d}"]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu"]
    _run(cmd, verbose)
    shutil.move(str(tmp), TORCH_LIB)
    return TORCH_LIB


TRACE_LIB = HERE / "libb2skinny_trace.so"


def build_trace(verbose: bool = False) -> Path:
    """The C ABI again with -DB2_TRACE: the cluster kernel stamps a per-unit timeline (see
    trace_w4.py). Built only on request; the product library compiles none of the stamps."""
    tdir = BUILD / "trace"
    tdir.mkdir(parents=True, exist_ok=True)
    deps = [CSRC / h for h in HEADERS] + [INCLUDE / "b2_skinny.h"]
    objs = []
    for src in CU_SOURCES:
        obj = tdir / (src + ".o")
        objs.append(obj)
        if _newer(obj, [CSRC / src] + deps):
            _run([NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                  "--expt-relaxed-constexpr", "-DB2_TRACE", f"-I{INCLUDE}", f"-I{CSRC}", "-c",
                  str(CSRC / src), "-o", str(obj)], verbose)
    if _newer(TRACE_LIB, objs):
        tmp = tdir / TRACE_LIB.name
        _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lrt"], verbose)
        shutil.move(str(tmp), TRACE_LIB)
    return TRACE_LIB


def build(verbose: bool = False) -> tuple[Path, Path]:
    BUILD.mkdir(exist_ok=True)
    capi = build_capi(verbose)
    ops = build_torch_ops(verbose)
    return capi, ops


if __name__ == "__main__":
    v = "-v" in sys.argv
    if "--ptxas" in sys.argv:
        build_capi(verbose=True, ptxas_verbose=True)
    elif "--trace" in sys.argv:
        print(build_trace(verbose=v))
    else:
        print(build(verbose=v))
