"""The CPU oracle against the golden fixtures made by the reference's own code, plus its own
invariants (packing round trips, bit layout, summation order, tolerance arithmetic)."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN

W4_GOLDEN = sorted(GOLDEN.glob("w4_*.npz"))
F16_GOLDEN = sorted(GOLDEN.glob("f16_*.npz"))
NORM_GOLDEN = sorted(GOLDEN.glob("rmsnorm_*.npz"))


def test_golden_files_present():
    assert len(W4_GOLDEN) >= 7 and len(F16_GOLDEN) >= 4 and len(NORM_GOLDEN) >= 4


@pytest.mark.parametrize("path", NORM_GOLDEN, ids=lambda p: p.stem)
def test_add_rmsnorm_oracle_matches_vllm(oracle, path):
    """The restated residual add + RMSNorm against vLLM 0.22.0's own fused_add_rms_norm: the new
    residual bit for bit; the output within one fp16 ulp (the oracle takes the mean and rsqrt
    in float64, torch in float32), equal almost everywhere."""
    d = np.load(path)
    out, res = oracle.add_rmsnorm_ref(d["y"], d["residual"], d["weight"], float(d["eps"]))
    assert np.array_equal(res.view(np.int16), d["new_residual"].view(np.int16))
    ulp = oracle.fp16_ulp_distance(out, d["out"])
    assert ulp.max() <= 1 and (ulp == 0).mean() >= 0.999, (ulp.max(), (ulp == 0).mean())
    assert np.isfinite(out).all()


def test_add_rmsnorm_oracle_invariants(oracle):
    rng = np.random.default_rng(5)
    y = (rng.standard_normal((3, 512)) * 3).astype(np.float16)
    r = rng.standard_normal((3, 512)).astype(np.float16)
    ones = np.ones(512, np.float16)
    out, res = oracle.add_rmsnorm_ref(y, r, ones, 1e-6)
    # unit weight: each output row has mean square 1 (up to fp16 rounding)
    ms = (out.astype(np.float64) ** 2).mean(axis=1)
    np.testing.assert_allclose(ms, 1.0, rtol=2e-3)
    # the norm is scale-invariant up to rounding: scaling y and the residual by 2 (exact in
    # fp16) leaves the output unchanged, and doubles the new residual exactly
    out2, res2 = oracle.add_rmsnorm_ref(y * np.float16(2), r * np.float16(2), ones, 0.0)
    out1, _ = oracle.add_rmsnorm_ref(y, r, ones, 0.0)
    assert np.array_equal(out1, out2)
    assert np.array_equal(res2, res * np.float16(2))
    # a zero row gives zeros (eps keeps the scale finite)
    z = np.zeros((1, 64), np.float16)
    o0, _ = oracle.add_rmsnorm_ref(z, z, ones[:64], 1e-6)
    assert not o0.any() and np.isfinite(o0).all()


def test_fp16_ulp_distance(oracle):
    one = np.float16(1)
    nxt = np.nextafter(one, np.float16(2))
    assert oracle.fp16_ulp_distance(np.array([one, -0.0], np.float16),
                                    np.array([nxt, 0.0], np.float16)).tolist() == [1, 0]
    assert oracle.fp16_ulp_distance(np.array([-nxt], np.float16),
                                    np.array([-one], np.float16)).tolist() == [1]


@pytest.mark.parametrize("path", W4_GOLDEN, ids=lambda p: p.stem)
def test_w4_oracle_matches_reference_code(oracle, path):
    d = np.load(path)
    ref = oracle.w4_ref(d["x"], d["qw"], d["qz"], d["sc"])
    # float64 both sides; only the matmul summation order may differ
    np.testing.assert_allclose(ref, d["ref"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("path", F16_GOLDEN, ids=lambda p: p.stem)
def test_f16_oracle_matches_reference_code(oracle, path):
    d = np.load(path)
    ref = oracle.gemm_ref(d["x"], d["w"])
    # the reference line computes in float32; the oracle in float64
    np.testing.assert_allclose(ref, d["ref"].astype(np.float64), rtol=1e-5, atol=2e-6)


def test_pack_unpack_round_trip(oracle):
    rng = np.random.default_rng(0)
    q = rng.integers(0, 16, size=(64, 24), dtype=np.uint8)
    assert np.array_equal(oracle.unpack_qw(oracle.pack_qw(q)), q)
    z = rng.integers(0, 16, size=(4, 24), dtype=np.uint8)
    assert np.array_equal(oracle.unpack_qz(oracle.pack_qz(z)), z)


def test_exllama_bit_layout(oracle):
    # nibble i (bits 4i) -> k = 2i, nibble 4+i (bits 16+4i) -> k = 2i+1  (check_w4.py:13)
    for k in range(8):
        q = np.zeros((8, 1), dtype=np.uint8)
        q[k, 0] = 0xA
        word = int(oracle.pack_qw(q).view(np.uint32)[0, 0])
        shift = 4 * (k // 2) + (16 if k % 2 else 0)
        assert word == 0xA << shift
    z = np.zeros((1, 8), dtype=np.uint8)
    z[0, 5] = 0x7
    assert int(oracle.pack_qz(z).view(np.uint32)[0, 0]) == 0x7 << 20


def test_dequant_is_exact(oracle):
    x, qw, qz, sc = oracle.gen_w4(1, 256, 64, 32, seed=3)
    deq = oracle.dequant_f64(qw, qz, sc)
    q = oracle.unpack_qw(qw).astype(np.int64)
    z = np.repeat(oracle.unpack_qz(qz).astype(np.int64), 32, axis=0)
    assert np.array_equal(deq, (q - z) * np.repeat(sc.astype(np.float64), 32, axis=0))


def test_column_subset_reference(oracle):
    x, qw, qz, sc = oracle.gen_w4(3, 256, 128, 64, seed=4)
    full = oracle.w4_ref(x, qw, qz, sc)
    cols = np.array([0, 5, 17, 64, 127])
    np.testing.assert_array_equal(oracle.w4_ref_columns(x, qw, qz, sc, cols), full[:, cols])


def test_allreduce_reference_order(oracle):
    # fp16 inputs: the sum is accumulated in fp32 and rounded once, in rank order
    parts = [np.array([60000, 1, -60000], dtype=np.float16),
             np.array([10000, 1, -10000], dtype=np.float16)]
    out = oracle.allreduce_ref(parts)
    assert out.dtype == np.float16
    assert np.isinf(out[0]) and out[1] == 2 and np.isinf(out[2])
    # two ranks: a + b rounded once == fp16 add (kernels/hostar.cu:107)
    rng = np.random.default_rng(1)
    a = rng.standard_normal(1000).astype(np.float16)
    b = rng.standard_normal(1000).astype(np.float16)
    assert np.array_equal(oracle.allreduce_ref([a, b]), (a + b).astype(np.float16))


def test_half_ulp(oracle):
    assert oracle.fp16_half_ulp(np.array([1.0]))[0] == 2.0**-11
    assert oracle.fp16_half_ulp(np.array([24.0]))[0] == 2.0**-7
    assert oracle.fp16_half_ulp(np.array([48.0]))[0] == 2.0**-6
    assert oracle.fp16_half_ulp(np.array([1e-6]))[0] == 2.0**-25


def test_tolerance_accepts_rounded_reference(oracle):
    ref = np.random.default_rng(2).standard_normal((8, 1000)) * 20
    y = ref.astype(np.float16)
    st = oracle.error_stats(y, ref)
    assert oracle.within_tolerance(st)
    assert st["max_abs_excess"] <= 1e-9


def test_tolerance_rejects_planted_error(oracle):
    # a mistake planted in the oracle side: one output off by 0.05 must fail the check
    ref = np.random.default_rng(3).standard_normal((4, 500))
    y = ref.astype(np.float16)
    bad = ref.copy()
    bad[2, 17] += 0.05
    assert not oracle.within_tolerance(oracle.error_stats(y, bad))


def test_generators_are_seeded(oracle):
    a = oracle.gen_w4(2, 256, 64, 128, seed=9)
    b = oracle.gen_w4(2, 256, 64, 128, seed=9)
    for u, v in zip(a, b):
        assert np.array_equal(u, v)
    x, qw, qz, sc = a
    assert x.dtype == np.float16 and qw.dtype == np.int32 and qz.dtype == np.int32
    assert sc.dtype == np.float16 and sc.min() >= 0.005 and sc.max() <= 0.02


@pytest.mark.parametrize("K,N,G", [(256, 96, 32), (512, 352, 64), (1024, 384, 128), (1024, 160, 256)])
def test_repack_image_inverts(oracle, K, N, G):
    """The repack image holds every qw word, scale and zero of its unit at the documented place
    (block w, word row r, chunk c at w * 2048 + r * 128 + ((c ^ (r & 7)) << 4); then the group
    rows of scales and zeros), and zeros past N."""
    _, qw, qz, sc = oracle.gen_w4(2, K, N, G, seed=K + N)
    img = oracle.w4_repack(qw, qz, sc, G)
    RG = 1 if G >= 128 else 128 // G
    tiles, kus, unit = img.shape
    assert (tiles, kus, unit) == ((N + 127) // 128, K // 128, 8192 + RG * 320)
    qwu, scu, qzu = qw.view(np.uint32), sc.view(np.uint16), qz.view(np.uint32)
    for t in range(tiles):
        cols = np.arange(t * 128, t * 128 + 128)
        inside = cols < N
        for ku in range(kus):
            words = img[t, ku, :8192].view(np.uint32).reshape(4, 16, 8, 4)
            for r in range(16):
                logical = words[:, r, [c ^ (r & 7) for c in range(8)], :].reshape(128)
                exp = np.where(inside, qwu[ku * 16 + r, np.minimum(cols, N - 1)], 0)
                assert (logical == exp).all(), (t, ku, r)
            s = img[t, ku, 8192:8192 + RG * 256].view(np.uint16).reshape(RG, 128)
            z = img[t, ku, 8192 + RG * 256:].view(np.uint32).reshape(RG, 16)
            for g in range(RG):
                row = (ku * 128) // G + g
                assert (s[g] == np.where(inside, scu[row, np.minimum(cols, N - 1)], 0)).all()
                wc = np.arange(t * 16, t * 16 + 16)
                assert (z[g] == np.where(wc < N // 8, qzu[row, np.minimum(wc, N // 8 - 1)], 0)).all()
