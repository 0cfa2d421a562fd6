"""The C ABI and the operator library without a GPU: both load, every declared symbol is
exported, argument validation rejects what the contract excludes (before touching a device),
and the host-side rendezvous registry works."""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import pytest


def test_every_declared_symbol_is_exported(capi):
    names = capi.declared_functions()
    assert len(names) >= 25
    lib = capi.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(capi._SIGS), set(names) ^ set(capi._SIGS)


def test_abi_version_and_strings(capi):
    lib = capi.lib()
    assert lib.b2_abi_version() == 1
    assert lib.b2_status_string(0) == b"ok"
    assert b"timed out" in lib.b2_status_string(capi.B2_ERR_TIMEOUT)
    assert lib.b2_workspace_bytes(0) > 4 << 20


def test_operator_schemas_match_reference(ops):
    # kernels/skinny.cu:331, kernels/w4.cu:507, kernels/hostar.cu:156-159
    expect = {
        "gemm": "gfx906_skinny::gemm(Tensor x, Tensor w, int variant=0) -> Tensor",
        "w4gemm": "gfx906_skinny::w4gemm(Tensor a, Tensor qw, Tensor qz, Tensor sc, int kw, "
                  "int waves) -> Tensor",
        "hostar_create": "gfx906_skinny::hostar_create(str name, int slot_bytes, bool create) -> int",
        "hostar_unlink": "gfx906_skinny::hostar_unlink(str name) -> ()",
        "hostar_max_bytes": "gfx906_skinny::hostar_max_bytes() -> int",
        "hostar_allreduce": "gfx906_skinny::hostar_allreduce(Tensor inp, int handle, int rank) -> Tensor",
    }
    for name, schema in expect.items():
        assert str(getattr(ops, name).default._schema) == schema
    assert ops.hostar_max_bytes() == 128 * 1024


def test_meta_shapes(ops):
    import torch

    x = torch.empty(7, 512, dtype=torch.float16, device="meta")
    w = torch.empty(1000, 512, dtype=torch.float16, device="meta")
    assert ops.gemm(x, w, 0).shape == (7, 1000)
    qw = torch.empty(64, 256, dtype=torch.int32, device="meta")
    qz = torch.empty(4, 32, dtype=torch.int32, device="meta")
    sc = torch.empty(4, 256, dtype=torch.float16, device="meta")
    assert ops.w4gemm(x, qw, qz, sc, 128, 14).shape == (7, 256)
    pk = ops.w4_repack(qw, qz, sc)
    assert pk.dtype == torch.uint8 and pk.numel() >= 512 * 256 // 2
    assert ops.w4gemm_packed(x, pk, 256, 128).shape == (7, 256)


def test_repack_operator_schemas(ops):
    assert str(ops.w4_repack.default._schema) == \
        "gfx906_skinny::w4_repack(Tensor qw, Tensor qz, Tensor sc) -> Tensor"
    assert str(ops.w4gemm_packed.default._schema) == \
        "gfx906_skinny::w4gemm_packed(Tensor a, Tensor packed, int N, int group_size) -> Tensor"
    assert str(ops.w4gemm_ar_packed.default._schema) == \
        "gfx906_skinny::w4gemm_ar_packed(Tensor a, Tensor packed, int N, int group_size, " \
        "int handle) -> Tensor"
    assert str(ops.w4gemm_ar_rmsnorm_packed.default._schema) == \
        "gfx906_skinny::w4gemm_ar_rmsnorm_packed(Tensor a, Tensor packed, int N, int group_size, " \
        "int handle, Tensor(a!) residual, Tensor weight, float eps) -> Tensor"


_ALIGNED = 1 << 20  # a fake, 16-byte aligned address: validation fails before it is used


@pytest.mark.parametrize("M,K,N,expect", [
    (0, 512, 256, 1), (9, 512, 256, 1), (4, 100, 256, 1), (4, 0, 256, 1), (4, 512, 0, 1),
])
def test_gemm_f16_rejects_bad_shapes(capi, M, K, N, expect):
    lib = capi.lib()
    rc = lib.b2_gemm_f16(_ALIGNED, _ALIGNED, _ALIGNED, M, K, N, _ALIGNED, 1 << 30, None)
    assert rc == expect
    assert lib.b2_last_error()


def test_gemm_f16_rejects_misaligned_and_missing_workspace(capi):
    lib = capi.lib()
    assert lib.b2_gemm_f16(_ALIGNED + 2, _ALIGNED, _ALIGNED, 4, 512, 256, _ALIGNED, 1 << 30,
                           None) == capi.B2_ERR_INVALID_ARG
    assert lib.b2_gemm_f16(_ALIGNED, _ALIGNED, _ALIGNED, 4, 512, 256, None, 0,
                           None) == capi.B2_ERR_WORKSPACE
    assert lib.b2_gemm_f16(None, _ALIGNED, _ALIGNED, 4, 512, 256, _ALIGNED, 1 << 30,
                           None) == capi.B2_ERR_INVALID_ARG


@pytest.mark.parametrize("M,K,N,G", [
    (4, 500, 256, 100),   # K % 128
    (4, 512, 250, 128),   # N % 32
    (4, 512, 256, 96),    # G not 32/64/128k
    (4, 384, 256, 256),   # K % G
    (0, 512, 256, 128),   # M
    (9, 512, 256, 128),
])
def test_w4_rejects_bad_shapes(capi, M, K, N, G):
    lib = capi.lib()
    rc = lib.b2_w4_gemm(_ALIGNED, _ALIGNED, _ALIGNED, _ALIGNED, _ALIGNED, M, K, N, G, _ALIGNED,
                        1 << 30, None)
    assert rc == capi.B2_ERR_INVALID_ARG, capi.lib().b2_last_error()


def test_w4_rejects_small_workspace(capi):
    lib = capi.lib()
    rc = lib.b2_w4_gemm(_ALIGNED, _ALIGNED, _ALIGNED, _ALIGNED, _ALIGNED, 4, 512, 256, 128,
                        _ALIGNED, 1024, None)
    assert rc == capi.B2_ERR_WORKSPACE


def test_allreduce_rejects_bad_arguments(capi):
    lib = capi.lib()
    assert lib.b2_nvar_allreduce(None, _ALIGNED, _ALIGNED, 64, 0, None) == capi.B2_ERR_STATE
    assert lib.b2_nvar_allreduce(None, _ALIGNED, _ALIGNED, 64, 7, None) == capi.B2_ERR_INVALID_ARG
    assert lib.b2_nvar_allreduce(None, _ALIGNED, _ALIGNED, 3, 0, None) == capi.B2_ERR_INVALID_ARG
    out = C.c_void_p()
    assert lib.b2_nvar_create(0, 3, 2, 1024, C.byref(out)) == capi.B2_ERR_INVALID_ARG
    assert lib.b2_nvar_create(0, 0, 9, 1024, C.byref(out)) == capi.B2_ERR_INVALID_ARG
    assert lib.b2_w4_gemm_allreduce(None, _ALIGNED, _ALIGNED, _ALIGNED, _ALIGNED, _ALIGNED, 4, 512,
                                    256, 128, _ALIGNED, 1 << 30, None) == capi.B2_ERR_STATE
    assert lib.b2_w4_gemm_allreduce_rmsnorm(None, _ALIGNED, _ALIGNED, _ALIGNED, _ALIGNED, _ALIGNED,
                                            _ALIGNED, 1e-6, _ALIGNED, 4, 512, 256, 128, _ALIGNED,
                                            1 << 30, None) == capi.B2_ERR_STATE


def test_tuning_knobs(capi):
    lib = capi.lib()
    assert lib.b2_set_tuning(capi.B2_TUNE_CTAS_PER_SM, 2) == 0
    assert lib.b2_get_tuning(capi.B2_TUNE_CTAS_PER_SM) == 2
    assert lib.b2_set_tuning(capi.B2_TUNE_CTAS_PER_SM, 0) == 0
    assert lib.b2_set_tuning(99, 1) == capi.B2_ERR_INVALID_ARG


def test_tuning_keys_match_header(capi):
    """Every B2_TUNE_* key of include/b2_skinny.h has the same value in the Python bindings, and
    the library accepts it."""
    import re

    header = (Path(__file__).resolve().parent.parent / "include" / "b2_skinny.h").read_text()
    keys = dict(re.findall(r"#define (B2_TUNE_\w+) (\d+)", header))
    assert len(keys) >= 10
    lib = capi.lib()
    for name, value in keys.items():
        assert getattr(capi, name) == int(value), name
        saved = lib.b2_get_tuning(int(value))
        assert lib.b2_set_tuning(int(value), saved) == 0, name


def test_registry_put_get_unlink(capi):
    lib = capi.lib()
    name = f"/b2_test_reg_{os.getpid()}".encode()
    reg = C.c_void_p()
    assert lib.b2_registry_open(name, 3, 1, C.byref(reg)) == 0
    other = C.c_void_p()
    assert lib.b2_registry_open(name, 3, 0, C.byref(other)) == 0
    bad = C.c_void_p()
    assert lib.b2_registry_open(name, 4, 0, C.byref(bad)) == capi.B2_ERR_STATE  # world mismatch
    blob = (C.c_ubyte * 64)(*range(64))
    out = (C.c_ubyte * 64)()
    assert lib.b2_registry_get(other, 1, out) == capi.B2_ERR_STATE  # not published yet
    assert lib.b2_registry_put(reg, 1, blob) == 0
    assert lib.b2_registry_get(other, 1, out) == 0
    assert bytes(out) == bytes(blob)
    assert lib.b2_registry_put(reg, 3, blob) == capi.B2_ERR_INVALID_ARG
    assert lib.b2_registry_unlink(name) == 0
    assert lib.b2_registry_open(name, 3, 0, C.byref(bad)) == capi.B2_ERR_STATE  # gone
    # mappings stay valid after unlink (the reference unlinks right after attaching)
    assert lib.b2_registry_get(reg, 1, out) == 0
    assert lib.b2_registry_close(reg) == 0 and lib.b2_registry_close(other) == 0


def test_tuning_presets_from_environment(built):
    """B2_TUNE="key=value,..." presets the tuning keys before first use (no GPU needed)."""
    import subprocess
    import sys

    from conftest import ROOT

    code = ("import sys; sys.path.insert(0, %r); import __graft_entry__ as e; e.load_package(); "
            "from mi50_vllm_lab_b200 import capi; L = capi.lib(); "
            "print(L.b2_get_tuning(3), L.b2_get_tuning(4), L.b2_get_tuning(5))") % str(ROOT)
    env = dict(os.environ, B2_TUNE="4=1,5=7")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.split()[-3:] == ["0", "1", "7"]

