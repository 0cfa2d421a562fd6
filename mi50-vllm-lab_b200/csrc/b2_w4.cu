// W4A16 skinny GEMM for sm_100a over GPTQ/Exllama-shuffled 4-bit weights, 1 <= M <= 8.
//
// Replaces w4_gemm / w4_skinny_s_kernel / w4_reduce_kernel of kernels/w4.cu:154-346,479-504 with
// the same operand layouts (kernels/w4.cu:477-478): a [M,K] fp16, qw [K/8,N] int32, qz [K/G,N/8]
// int32 (v2 zeros), sc [K/G,N] fp16. Design:
//   - one thread of a producer warp streams 128-column x 128-k units (8 KB of qw, that unit's
//     scale and zero rows, and the unit's activations, 8 rows x 128 k = 2 KB) into a ring of
//     shared-memory stages with TMA (128-byte swizzle for qw and x, L2 evict-first for the
//     weights), so every activation is read from L2 once per CTA unit instead of once per warp;
//   - each of four consumer warps owns 32 columns of the unit. A lane reads one 16-byte chunk
//     (4 columns of one 8-k word row) per 32 k, unpacks the 8 nibbles of each word to (q - z)
//     in fp16 exactly (lop3 magic-number trick + add.f16x2) and feeds them to mma.sync
//     m16n8k16 as the A operand against the <= 8 activation rows (B operand). Each weight is
//     dequantized once and used for all M rows.
//   - (q - z) * x is accumulated per quantization group in fp32 and multiplied by the group's
//     scale in fp32 once per group, so no product is rounded to fp16 (the reference rounds
//     (q - z) * s to fp16 per weight, kernels/w4.cu:33-36).
//   - stream-K over a persistent grid; tiles shared by CTAs are summed by the last CTA to
//     finish, in CTA order, from fp32 slots (one launch; replaces the workspace + second
//     reduce kernel of kernels/w4.cu:154-166,330-346).
//   - programmatic dependent launch: the first weight stages are prefetched into L2 before the
//     kernel waits for the previous grid on the stream; every load into shared memory and every
//     access to activations, workspace and y comes after that wait.
//   - optionally the NVLink all-reduce of a row-parallel layer is fused into the epilogue: the
//     finished fp32 tile is pushed to every rank, and each rank adds the ranks' tiles in rank
//     order (bit-identical on every rank); and optionally, after it, the decoder layer's
//     residual add + RMSNorm (row sums through one grid-wide barrier, see norm_rstd).
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "b2_device.cuh"
#include "b2_internal.h"
#include "b2_nvar.cuh"

namespace b2 {

int nvar_view(b2_nvar* ar, ArView* out, size_t need_slot_bytes, int* tiles_cap);

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kUnitK = 128;                 // k per unit = 16 word rows
constexpr int kQwBox = 16 * 128;            // 16 word rows x 32 columns x 4 B (one TMA box)
constexpr int kQwStage = kWarps * kQwBox;   // 8 KB

constexpr int align128(int v) { return (v + 127) & ~127; }
// shared memory of the RMSNorm epilogue: per-warp row sums [kWarps][kMaxM], then rstd [kMaxM]
constexpr int kNormFloats = (kWarps + 1) * kMaxM;

// Shared memory of one CTA (offsets from a 1024-byte aligned base). Every TMA destination must
// start on a 128-byte boundary, and the swizzled qw boxes on a 1024-byte one.
template <int GP>  // GP: 32-k pairs per scale group inside a unit (1: G=32, 2: G=64, 4: G>=128)
struct Cfg {
  // 5 stages x 10.6 KB let four CTAs (16 consumer warps) share an SM's 228 KB when G >= 128
  // (the exact-dequant variants need more registers and run three CTAs per SM).
  static constexpr int kStages = 5;
  static constexpr int RG = 4 / GP;                        // group rows per unit
  static constexpr int kScBytes = RG * kTileN * 2;         // scales of one unit
  static constexpr int kQzBytes = RG * (kTileN / 8) * 4;   // zeros of one unit
  static constexpr int kScStride = align128(kScBytes);
  static constexpr int kQzStride = align128(kQzBytes);
  // activations of one unit, x[8 rows][128 k] fp16: two TMA boxes of 64 k x 8 rows, 128-byte
  // swizzle (chunk c of row m of box b at b * 1024 + m * 128 + ((c ^ m) << 4))
  static constexpr int kXBytes = kMaxM * kUnitK * 2;
  static constexpr int kTx = kQwStage + kXBytes + kScBytes + kQzBytes;
  static constexpr int kXOff = kStages * kQwStage;
  static constexpr int kScOff = kXOff + kStages * kXBytes;
  static constexpr int kQzOff = kScOff + kStages * kScStride;
  static constexpr int kBarOff = kQzOff + kStages * kQzStride;
  static constexpr int kNormOff = align128(kBarOff + 2 * kStages * 8 + 32);  // kNormFloats fp32
  static constexpr int kSmem = 1024 + kNormOff + kNormFloats * 4;
  static_assert(kQwBox % 1024 == 0 && kQwStage % 1024 == 0, "swizzled boxes need 1024 B");
  static_assert(kXOff % 1024 == 0 && kXBytes % 1024 == 0, "swizzled boxes need 1024 B");
  static_assert(kScOff % 128 == 0 && kScStride % 128 == 0, "TMA destination alignment");
  static_assert(kQzOff % 128 == 0 && kQzStride % 128 == 0, "TMA destination alignment");
  static_assert(kBarOff % 8 == 0, "mbarrier alignment");
};

struct W4Args {
  const __half* x;
  __half* y;
  int M, K, N, G;
  StreamK sk;
  float* partials;
  int* counters;
  int* status;
  int cl_size, cl_count;  // cluster kernel: CTAs per cluster, clusters
  int ll;                 // fused: exchange as 64-bit value+generation words
  int two_shot;           // fused cluster kernel with ll: reduce at the tile's owner rank, then
                          // send the result back (instead of every rank reducing every tile)
  // fused launches only: residual add + RMSNorm of the all-reduced rows (norm != 0)
  int norm;
  float eps;
  const __half* nw;  // [N] norm weight
  __half* res;       // [M, N] residual: read, then overwritten with the sum
  float* npart;      // [grid][kMaxM] per-CTA sums of squares (workspace)
  int norm_v16;      // y, res and nw all 16-byte aligned: the last cluster moves 16-byte vectors
  // weights repacked at load time (b2_w4_repack), or null: unit (tile, ku) is pk_unit contiguous
  // bytes at pk + (tile * K / 128 + ku) * pk_unit holding exactly the stage's shared-memory image:
  // its qw block (8 KB, already swizzled), then its scale rows, then its zero rows
  const uint8_t* pk;
  int pk_unit;
};

// The repacked bytes of unit (tile, ku).
__device__ __forceinline__ const uint8_t* packed_unit(const W4Args& p, int tile, int ku) {
  return p.pk + ((size_t)tile * (size_t)(p.K / kUnitK) + (size_t)ku) * (size_t)p.pk_unit;
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;  // (a & b) | c
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hadd2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// (q - z) for the 8 nibbles of one shuffled word, as four fp16 pairs in k order
// (k0,k1) (k2,k3) (k4,k5) (k6,k7). Nibble i sits at bits 4i (k = 2i) and nibble 4+i at bits
// 16+4i (k = 2i+1). OR-ing a low nibble (bits 0..3 of a half) into the mantissa of fp16 1024.0
// (0x6400, ulp 1) gives 1024 + q; OR-ing a high nibble (bits 4..7) into fp16 64.0 (0x5400,
// ulp 1/16) gives 64 + q. zlo = -(1024 + z) and zhi = -(64 + z) in both halves; every step is
// exact in fp16: four lop3, one shift, four add.f16x2.
__device__ __forceinline__ void dequant_word(uint32_t q, uint32_t zlo, uint32_t zhi,
                                             uint32_t (&d)[4]) {
  constexpr uint32_t kLo = 0x64006400u;  // 1024.0 | 1024.0
  constexpr uint32_t kHi = 0x54005400u;  // 64.0 | 64.0
  const uint32_t q8 = q >> 8;
  d[0] = hadd2_u(lop_and_or(q, 0x000F000Fu, kLo), zlo);
  d[1] = hadd2_u(lop_and_or(q, 0x00F000F0u, kHi), zhi);
  d[2] = hadd2_u(lop_and_or(q8, 0x000F000Fu, kLo), zlo);
  d[3] = hadd2_u(lop_and_or(q8, 0x00F000F0u, kHi), zhi);
}

// The same 8 nibbles without the zero point: (1024 + q) for the nibbles at bits 0..3 of a half
// (k = 0,1,4,5 of the word) and (64 + q) for those at bits 4..7 (k = 2,3,6,7). One shift and four
// lop3 per word; the offsets and the zero point are removed once per group (GroupFix).
__device__ __forceinline__ void dequant_word_off(uint32_t q, uint32_t (&d)[4]) {
  constexpr uint32_t kLo = 0x64006400u;  // 1024.0 | 1024.0
  constexpr uint32_t kHi = 0x54005400u;  // 64.0 | 64.0
  const uint32_t q8 = q >> 8;
  d[0] = lop_and_or(q, 0x000F000Fu, kLo);
  d[1] = lop_and_or(q, 0x00F000F0u, kHi);
  d[2] = lop_and_or(q8, 0x000F000Fu, kLo);
  d[3] = lop_and_or(q8, 0x00F000F0u, kHi);
}

// Per-lane shared-memory geometry of the consumer warps. Lane (g = lane/4, t = lane%4) of warp w
// owns columns colw .. colw+3 of a unit (colw = w*32 + 4*ch, ch = the lane's 16-byte chunk of a
// 128-byte word row, permuted so the swizzled loads are conflict-free). For 32-k step q it reads
// word row 4q+t of its chunk and the matching 16 bytes of activations of row g (chunk 4q+t of
// the stage's two 64-k boxes). Under the 128-byte swizzle, steps 2 and 3 sit exactly 1024 bytes
// after steps 0 and 1 in both blocks, so two base offsets per block cover the four steps.
struct LaneGeo {
  int g, t, ch, colw;
  uint32_t xa, xb;  // activations of steps 0 / 1 inside a stage's x block (+1024: steps 2 / 3)
  uint32_t wa, wb;  // weight chunks of steps 0 / 1 inside the warp's qw box (+1024: steps 2 / 3)
  uint32_t one, zero;  // 1.0|1.0 and 0 in registers (a constant A operand kept live)
  __device__ __forceinline__ LaneGeo(int warp, int lane, int M) {
    g = lane >> 2;
    t = lane & 3;
    ch = ((g & 1) << 2) | (g >> 1);
    colw = warp * 32 + ch * 4;
    xa = (uint32_t)(g * 128 + ((t ^ g) << 4));
    xb = (uint32_t)(g * 128 + ((t ^ g ^ 4) << 4));
    wa = (uint32_t)(t * 128 + ((ch ^ t) << 4));
    wb = (uint32_t)((4 + t) * 128 + ((ch ^ t ^ 4) << 4));
    // M <= 8, so M >> 8 is 0; taken from a kernel argument, the compiler keeps these values in
    // registers instead of rebuilding the constant operand at every use
    zero = (uint32_t)M >> 8;
    one = 0x3C003C00u | zero;
  }
};

// Consume one unit (128 columns x 128 k) from a stage: acc[T][i] += this unit's contribution,
// scaled per quantization group, for the lane's columns colw + 2T + (i >> 1) and rows 2t + (i & 1).
// x_base / qw_base: shared addresses of the stage's activations and of this warp's qw box;
// sc_row / qz_row: the stage's scale rows [RG][128] fp16 and zero rows [RG][16] int32.
//
// G >= 128 (one group per unit) uses the offset form: the tensor cores multiply the activations
// by (off_k + q) straight from dequant_word_off (off_k = 1024 for the nibbles at bits 0..3 of a
// half, 64 for bits 4..7), and two more mma per 32 k against a constant A (ones on the 1024
// slots in rows 0..7, ones on the 64 slots in rows 8..15) give every lane XL[m] and XH[m], the
// row sums of the activations on the two kinds of slot. Per group, for column n and row m:
//   sum_k (q - z) x  =  raw - 1024 XL - 64 XH - z (XL + XH),
// which is multiplied by the group's scale in fp32. Per 8-weight word that is one shift and four
// lop3 (the exact form below needs four add.f16x2 more), at the price of carrying the offsets
// through the fp32 accumulation (rounding error ~1e-3 of a group sum of ~1e4, far inside the
// fp16 output rounding).
// G = 32 / 64 use the exact form: A = (q - z) exactly in fp16 (dequant_word), scale per group.
template <int GP>
__device__ __forceinline__ void consume_unit(const LaneGeo& L, uint32_t x_base, uint32_t qw_base,
                                             const __half* sc_rows, const uint32_t* qz_rows,
                                             float (&acc)[2][4]) {
  constexpr int RG = 4 / GP;
  uint4 xv[4], wv[4];
  const uint32_t xa = x_base + L.xa, xb = x_base + L.xb;
  const uint32_t wa = qw_base + L.wa, wb = qw_base + L.wb;
  xv[0] = lds128(xa);
  xv[1] = lds128(xb);
  xv[2] = lds128_1k(xa);
  xv[3] = lds128_1k(xb);
  wv[0] = lds128(wa);
  wv[1] = lds128(wb);
  wv[2] = lds128_1k(wa);
  wv[3] = lds128_1k(wb);
  if constexpr (GP == 4) {
    float raw[2][4], xs[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = wv[q];
      uint32_t d0[4], d1[4], d2[4], d3[4];
      dequant_word_off(w.x, d0);
      dequant_word_off(w.y, d1);
      dequant_word_off(w.z, d2);
      dequant_word_off(w.w, d3);
      // n-tile 0: A rows g / g+8 = columns colw / colw+1; n-tile 1: colw+2 / colw+3. In every
      // mma the A registers a0/a1 hold the 1024-offset pairs and a2/a3 the 64-offset pairs.
      if (q == 0) {
        mma_16816_first(raw[0], d0[0], d1[0], d0[1], d1[1], xv[q].x, xv[q].y);
        mma_16816_first(raw[1], d2[0], d3[0], d2[1], d3[1], xv[q].x, xv[q].y);
        mma_16816_first(xs, L.one, L.zero, L.zero, L.one, xv[q].x, xv[q].y);
      } else {
        mma_16816(raw[0], d0[0], d1[0], d0[1], d1[1], xv[q].x, xv[q].y);
        mma_16816(raw[1], d2[0], d3[0], d2[1], d3[1], xv[q].x, xv[q].y);
        mma_16816(xs, L.one, L.zero, L.zero, L.one, xv[q].x, xv[q].y);
      }
      mma_16816(raw[0], d0[2], d1[2], d0[3], d1[3], xv[q].z, xv[q].w);
      mma_16816(raw[1], d2[2], d3[2], d2[3], d3[3], xv[q].z, xv[q].w);
      mma_16816(xs, L.one, L.zero, L.zero, L.one, xv[q].z, xv[q].w);
    }
    // xs: XL[2t], XL[2t+1] (rows 0..7 of D), XH[2t], XH[2t+1] (rows 8..15)
    const float x0[2] = {xs[0] + xs[2], xs[1] + xs[3]};
    const float c1[2] = {fmaf(1024.f, xs[0], 64.f * xs[2]), fmaf(1024.f, xs[1], 64.f * xs[3])};
    const uint32_t zw = qz_rows[L.colw >> 3] >> ((L.colw & 7) * 4);
    const uint2 sv = *reinterpret_cast<const uint2*>(sc_rows + L.colw);
    const __half2 s01 = *reinterpret_cast<const __half2*>(&sv.x);
    const __half2 s23 = *reinterpret_cast<const __half2*>(&sv.y);
    const float s[4] = {__low2float(s01), __high2float(s01), __low2float(s23), __high2float(s23)};
#pragma unroll
    for (int T = 0; T < 2; ++T)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = 2 * T + (i >> 1), j = i & 1;
        const float z = (float)((zw >> (4 * c)) & 0xFu);
        acc[T][i] = fmaf(s[c], raw[T][i] - fmaf(z, x0[j], c1[j]), acc[T][i]);
      }
  } else {
    // zero points and scales of the lane's 4 columns for each group row of the unit
    uint32_t zlo[RG][4], zhi[RG][4];
    float scl[RG][4];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      const uint32_t zw = qz_rows[r * (kTileN / 8) + (L.colw >> 3)] >> ((L.colw & 7) * 4);
      const uint2 sv = *reinterpret_cast<const uint2*>(sc_rows + r * kTileN + L.colw);
      const __half2 s01 = *reinterpret_cast<const __half2*>(&sv.x);
      const __half2 s23 = *reinterpret_cast<const __half2*>(&sv.y);
      scl[r][0] = __low2float(s01);
      scl[r][1] = __high2float(s01);
      scl[r][2] = __low2float(s23);
      scl[r][3] = __high2float(s23);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t z = (zw >> (4 * i)) & 0xFu;
        zlo[r][i] = (0xE400u + z) * 0x00010001u;         // -(1024 + z)
        zhi[r][i] = (0xD400u + (z << 4)) * 0x00010001u;  // -(64 + z)
      }
    }
    float accg[2][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) accg[0][i] = accg[1][i] = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // 32-k step q: word rows 4q..4q+3, lane t takes row 4q+t
      const uint4 w = wv[q];
      const int r = (RG == 1) ? 0 : (q / GP);
      uint32_t d0[4], d1[4], d2[4], d3[4];
      dequant_word(w.x, zlo[r][0], zhi[r][0], d0);
      dequant_word(w.y, zlo[r][1], zhi[r][1], d1);
      dequant_word(w.z, zlo[r][2], zhi[r][2], d2);
      dequant_word(w.w, zlo[r][3], zhi[r][3], d3);
      mma_16816(accg[0], d0[0], d1[0], d0[1], d1[1], xv[q].x, xv[q].y);
      mma_16816(accg[0], d0[2], d1[2], d0[3], d1[3], xv[q].z, xv[q].w);
      mma_16816(accg[1], d2[0], d3[0], d2[1], d3[1], xv[q].x, xv[q].y);
      mma_16816(accg[1], d2[2], d3[2], d2[3], d3[3], xv[q].z, xv[q].w);
      if ((q + 1) % GP == 0) {
#pragma unroll
        for (int T = 0; T < 2; ++T)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[T][i] = fmaf(scl[r][2 * T + (i >> 1)], accg[T][i], acc[T][i]);
            accg[T][i] = 0.f;
          }
      }
    }
  }
}

// Lane output layout of a 128-column tile: lane (g, t) of warp w owns columns
// w*32 + 4*ch(g) .. +3 for rows m = 2t (v[0]) and m = 2t+1 (v[1]).
__device__ __forceinline__ void store_y(const W4Args& p, int tile, int colw, int t,
                                        const float4 (&v)[2]) {
  const int n = tile * kTileN + colw;
  if (n >= p.N) return;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int m = 2 * t + j;
    if (m >= p.M) continue;
    __half2 h0 = __floats2half2_rn(v[j].x, v[j].y);
    __half2 h1 = __floats2half2_rn(v[j].z, v[j].w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&h0);
    u.y = *reinterpret_cast<uint32_t*>(&h1);
    *reinterpret_cast<uint2*>(p.y + (size_t)m * p.N + n) = u;
  }
}

// ------------------------------------------------------------------------------------------------
// Residual add + RMSNorm of the all-reduced rows (fused launches with p.norm). Follows vLLM's
// fused_add_rms_norm (vllm/ir/ops/layernorm.py:40-60 in vLLM 0.22), which the decoder layers of
// the reference's models run on the all-reduced output of o_proj and down_proj:
//   x        = float(y) + float(residual)      y: the fp16 all-reduce result; x stays fp32
//   residual <- fp16(x)
//   out      = fp16(fp16(x * rsqrt(sum_n(x^2) / N + eps)) * weight)
// A row's sum needs every CTA's columns. Phase a, while the all-reduced sums are stored: y gets
// fp16(sum) and each thread adds x^2 per row over its elements in a fixed order. norm_rstd:
// the CTA's row sums go to the workspace, one grid-wide barrier, then every CTA adds all CTAs'
// sums in CTA order, so every CTA (and every rank) computes the same rstd bit for bit. Phase c:
// each thread re-reads y and the still untouched residual of its own elements and writes the
// new residual and `out` (into y).
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float norm_x(__half yh, __half r) {
  return __half2float(yh) + __half2float(r);
}
__device__ __forceinline__ __half norm_out(float x, float rstd, __half w) {
  return __float2half_rn(__half2float(__float2half_rn(x * rstd)) * __half2float(w));
}
// ss[m] += q for a row index known only at run time (kept in registers)
__device__ __forceinline__ void row_add(float (&ss)[kMaxM], int m, float q) {
#pragma unroll
  for (int i = 0; i < kMaxM; ++i)
    if (i == m) ss[i] += q;
}

// Phase a for the lane layout of store_y: columns n..n+3 of rows 2t, 2t+1 with fp32 sums v.
__device__ __forceinline__ void norm_accum_lane(const W4Args& p, int t, int n,
                                                const float4 (&v)[2], float (&ss)[kMaxM]) {
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int m = 2 * t + j;
    if (m >= p.M) continue;
    const uint2 rv = *reinterpret_cast<const uint2*>(p.res + (size_t)m * p.N + n);
    const __half* r = reinterpret_cast<const __half*>(&rv);
    const float x0 = norm_x(__float2half_rn(v[j].x), r[0]);
    const float x1 = norm_x(__float2half_rn(v[j].y), r[1]);
    const float x2 = norm_x(__float2half_rn(v[j].z), r[2]);
    const float x3 = norm_x(__float2half_rn(v[j].w), r[3]);
    row_add(ss, m, fmaf(x3, x3, fmaf(x2, x2, fmaf(x1, x1, x0 * x0))));
  }
}

// Phase c for columns n..n+3 of row m.
__device__ __forceinline__ void norm_finish4(const W4Args& p, int m, int n, float rstd) {
  const size_t o = (size_t)m * p.N + n;
  uint2 yv = *reinterpret_cast<const uint2*>(p.y + o);
  uint2 rv = *reinterpret_cast<const uint2*>(p.res + o);
  const uint2 wv = *reinterpret_cast<const uint2*>(p.nw + n);
  __half* yh = reinterpret_cast<__half*>(&yv);
  __half* rh = reinterpret_cast<__half*>(&rv);
  const __half* wh = reinterpret_cast<const __half*>(&wv);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float x = norm_x(yh[i], rh[i]);
    rh[i] = __float2half_rn(x);
    yh[i] = norm_out(x, rstd, wh[i]);
  }
  *reinterpret_cast<uint2*>(p.res + o) = rv;
  *reinterpret_cast<uint2*>(p.y + o) = yv;
}
// Phase c for one element.
__device__ __forceinline__ void norm_finish1(const W4Args& p, int m, int n, float rstd) {
  const size_t o = (size_t)m * p.N + n;
  const float x = norm_x(p.y[o], p.res[o]);
  p.res[o] = __float2half_rn(x);
  p.y[o] = norm_out(x, rstd, p.nw[n]);
}

// Called by every consumer thread of every CTA with its per-row sums of squares. Leaves
// rstd[m] for m < M at s_norm[kWarps * kMaxM + m]. Returns false if the grid-wide barrier gave
// up (after the handle's timeout; the caller records B2_ERR_TIMEOUT).
__device__ __forceinline__ bool norm_rstd(const W4Args& p, const ArView& ar, uint32_t e,
                                          const float (&ss)[kMaxM], float* s_norm,
                                          volatile int* s_flag) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // the CTA's row sums: a fixed shuffle tree per warp, then the warps in order
#pragma unroll
  for (int m = 0; m < kMaxM; ++m) {
    float v = ss[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) s_norm[warp * kMaxM + m] = v;
  }
  named_bar_sync(1, kWarps * 32);
  if (tid < kMaxM) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += s_norm[w * kMaxM + tid];
    p.npart[(size_t)blockIdx.x * kMaxM + tid] = v;
  }
  named_bar_sync(1, kWarps * 32);
  // grid-wide barrier: the last CTA to arrive resets the count and releases generation e (the
  // release orders the reset before the store). The fence before each arrival makes the CTA's
  // row sums, ordered before it by the CTA barrier, visible to whoever observes the arrival;
  // a CTA's other threads see the released sums through the CTA barrier after thread 0's
  // acquire.
  if (tid == 0) {
    ArHeader* h = ar_header(ar);
    bool ok = true;
    __threadfence();
    if (atomicAdd(&h->norm_count, 1u) == gridDim.x - 1) {
      atomicExch(&h->norm_count, 0u);
      st_release_gpu(&h->norm_gen, e);  // the grid barrier is on this GPU: gpu scope
    } else {
      const unsigned long long t0 = globaltimer_ns();
      unsigned int it = 0;
      while ((int)(ld_acquire_gpu(&h->norm_gen) - e) < 0) {
        if (++it >= kMaxSpin || ((it & 15u) == 0 && globaltimer_ns() - t0 > ar.timeout_ns)) {
          ok = false;
          break;
        }
        __nanosleep(32);
      }
    }
    *s_flag = ok ? 1 : 0;
  }
  named_bar_sync(1, kWarps * 32);
  const bool ok = *s_flag != 0;
  // All CTAs' row sums: thread i takes CTAs i, i + 128, ... (both 16-byte halves of each CTA's
  // eight sums, four CTAs' loads in flight at a time), adds them in that order, then the same
  // fixed shuffle tree and warp order as above. Every CTA runs the same sequence on the same
  // data, so every CTA gets the same sums.
  float acc[kMaxM];
#pragma unroll
  for (int m = 0; m < kMaxM; ++m) acc[m] = 0.f;
  const int nb = (int)gridDim.x;
  for (int b0 = tid; b0 < nb; b0 += 4 * kWarps * 32) {
    float4 lo[4], hi[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = b0 + j * kWarps * 32;
      if (b < nb) {
        lo[j] = __ldcg(reinterpret_cast<const float4*>(p.npart + (size_t)b * kMaxM));
        hi[j] = __ldcg(reinterpret_cast<const float4*>(p.npart + (size_t)b * kMaxM + 4));
      } else {
        lo[j] = hi[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[0] += lo[j].x;
      acc[1] += lo[j].y;
      acc[2] += lo[j].z;
      acc[3] += lo[j].w;
      acc[4] += hi[j].x;
      acc[5] += hi[j].y;
      acc[6] += hi[j].z;
      acc[7] += hi[j].w;
    }
  }
#pragma unroll
  for (int m = 0; m < kMaxM; ++m) {
    float v = acc[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) s_norm[warp * kMaxM + m] = v;
  }
  named_bar_sync(1, kWarps * 32);
  if (tid < p.M) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += s_norm[w * kMaxM + tid];
    s_norm[kWarps * kMaxM + tid] = rsqrtf(v / (float)p.N + p.eps);
  }
  named_bar_sync(1, kWarps * 32);
  return ok;
}

// Timeline trace (builds with -DB2_TRACE only; the library proper compiles none of it): CTA 0 of
// a cluster-kernel launch stamps the global timer per unit at the producer's issue (event 0), its
// wait for a free stage (1), consumer warp 0's wait for the data (2) and its end of the unit (3),
// and per tile at the start of the reduction (4). Every CTA records [0] its start, [1] its end,
// [2] its SM, [3] the end of its last tile's units, [4] the end of that tile's cluster reduction
// (and, fused, of its sends to the ranks), [5] / [6] the start / end of the fused exchange's
// second phase (gathering the ranks' partials), [7] the end of the wait for the previous grid;
// RMSNorm launches: [8] its row sums sent to the cluster leader, [9] (leader) every CTA's sums in,
// [10] (leader) past the grid-wide barrier, [11] rstd received.
#ifdef B2_TRACE
constexpr int kTraceUnits = 4096, kTraceCtas = 4096, kTraceCtaWords = 12;
__device__ unsigned long long g_trace_units[5][kTraceUnits];
__device__ unsigned long long g_trace_ctas[kTraceCtas][kTraceCtaWords];
#define B2_TRC(k)                                                                    \
  do {                                                                               \
    if (threadIdx.x == 0 && blockIdx.x < kTraceCtas) g_trace_ctas[blockIdx.x][k] = globaltimer_ns(); \
  } while (0)
#define B2_TR(e, j)                                                                   \
  do {                                                                                \
    if (blockIdx.x == 0 && (j) < kTraceUnits) g_trace_units[e][j] = globaltimer_ns(); \
  } while (0)
#else
#define B2_TR(e, j) \
  do {              \
  } while (0)
#define B2_TRC(k) \
  do {            \
  } while (0)
#endif

// The last cluster's share of the final RMSNorm step over all M x N elements, in vectors V of
// fp16 (uint4: 8, uint2: 4; N is a multiple of 8, so a vector never crosses a row): each thread
// issues the loads of up to 4 vectors of y, residual and weight before it uses any, so its share
// costs about one round trip to L2 instead of one per vector.
template <typename V>
__device__ __forceinline__ void norm_finish_all(const W4Args& p, const float* s_rstd, int crank,
                                                int CS) {
  constexpr int kH = (int)(sizeof(V) / 2);
  const int per = p.M * p.N / kH, stride = CS * kWarps * 32;
  for (int i0 = crank * kWarps * 32 + (int)threadIdx.x; i0 < per; i0 += 4 * stride) {
    V yv[4], rv[4], wv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = i0 + j * stride;
      if (i < per) {
        const int m = (i * kH) / p.N, n = i * kH - m * p.N;
        const size_t o = (size_t)m * p.N + n;
        yv[j] = __ldcg(reinterpret_cast<const V*>(p.y + o));
        rv[j] = __ldcg(reinterpret_cast<const V*>(p.res + o));
        wv[j] = __ldg(reinterpret_cast<const V*>(p.nw + n));
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = i0 + j * stride;
      if (i >= per) continue;
      const int m = (i * kH) / p.N, n = i * kH - m * p.N;
      const size_t o = (size_t)m * p.N + n;
      const __half* yh = reinterpret_cast<const __half*>(&yv[j]);
      __half* rh = reinterpret_cast<__half*>(&rv[j]);
      const __half* wh = reinterpret_cast<const __half*>(&wv[j]);
      V ov;
      __half* oh = reinterpret_cast<__half*>(&ov);
      const float rstd = s_rstd[m];
#pragma unroll
      for (int k = 0; k < kH; ++k) {
        const float x = norm_x(yh[k], rh[k]);
        rh[k] = __float2half_rn(x);
        oh[k] = norm_out(x, rstd, wh[k]);
      }
      *reinterpret_cast<V*>(p.res + o) = rv[j];
      *reinterpret_cast<V*>(p.y + o) = ov;
    }
  }
}

// The cluster kernel's RMSNorm, without a grid-wide barrier. (1) Each CTA adds its threads' row
// sums (shuffle tree, warps in order) and writes them into its cluster leader's shared memory
// (distributed shared memory, slot crank), then arrives on the leader's norm_bar. (2) The leader
// adds the CS slots in rank order, writes the cluster's sums to the workspace and counts its
// cluster in the handle's header (a release: its cluster's y stores and sums are ordered before).
// Every leader but the last tells its CTAs that they are done. (3) The last leader (whose counter
// update acquires every other cluster's) adds the NC cluster sums in cluster order - the same
// order on every rank, so every rank computes the same rstd bit for bit - advances the handle's
// generation (every cluster has finished reading its slots; these launches skip ar_finish) and
// sends rstd to its CTAs, which then finish every element of y: x = y + residual, residual <-
// fp16(x), y <- fp16(fp16(x * rstd) * weight). No CTA waits for another cluster, so the launch
// needs no co-residency (it may start early). Every wait is bounded; the leader always tells its
// CTAs, so none of them waits in vain. Returns false if a wait gave up.
__device__ __forceinline__ bool norm_finish_cluster(const W4Args& p, const ArView& ar, uint32_t e,
                                                    const float (&ss)[kMaxM], float* s_norm,
                                                    uint64_t* norm_bar, uint64_t* rstd_bar,
                                                    volatile int* s_flag, volatile int* s_abort,
                                                    int crank, int CS, int cid, int NC) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* s_rstd = s_norm + kWarps * kMaxM;   // [kMaxM]
  float* s_fin = s_rstd + kMaxM;             // [0]: nonzero in the CTAs of the last cluster
  float* s_gather = s_fin + kMaxM;           // [16][kMaxM] (leader)
  float* s_part = s_gather + 16 * kMaxM;     // [16][kMaxM] (leader)
  volatile int* s_last = reinterpret_cast<volatile int*>(s_part + 16 * kMaxM);
#pragma unroll
  for (int m = 0; m < kMaxM; ++m) {
    float v = ss[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) s_norm[warp * kMaxM + m] = v;
  }
  named_bar_sync(1, kWarps * 32);
  if (tid < kMaxM) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += s_norm[w * kMaxM + tid];
    st_dsmem_f32(mapa_shared(smem_u32(s_gather + crank * kMaxM + tid), 0u), v);
  }
  named_bar_sync(1, kWarps * 32);  // (also orders every thread's y stores before the arrival)
  if (tid == 0) {
    fence_acq_rel_cluster();
    mbar_arrive_remote(mapa_shared(smem_u32(norm_bar), 0u));
  }
  B2_TRC(8);
  bool ok = true;
  if (crank == 0) {
    if (tid == 0) *s_flag = mbar_wait_cluster(norm_bar, 0u, s_abort) ? 1 : 0;
    B2_TRC(9);
    named_bar_sync(1, kWarps * 32);
    ok = *s_flag != 0;
    if (tid < kMaxM) {
      float v = 0.f;
      for (int q = 0; q < CS; ++q) v += s_gather[q * kMaxM + tid];
      p.npart[(size_t)cid * kMaxM + tid] = v;
    }
    named_bar_sync(1, kWarps * 32);
    if (tid == 0) {
      ArHeader* h = ar_header(ar);
      __threadfence();  // the cluster's y stores and sums before its count
      const bool last = atomicAdd(&h->norm_count, 1u) == (unsigned)NC - 1u;
      if (last) {
        __threadfence();  // every other cluster's stores after their counts
        atomicExch(&h->norm_count, 0u);
      }
      *s_last = last ? 1 : 0;
    }
    named_bar_sync(1, kWarps * 32);
    const bool last = *s_last != 0;
    B2_TRC(10);
    if (last) {
      {
        const int m = tid & (kMaxM - 1), j = tid / kMaxM;  // 16 threads per row
        float v = 0.f;
        for (int b = j; b < NC; b += 16) v += __ldcg(p.npart + (size_t)b * kMaxM + m);
        s_part[j * kMaxM + m] = v;
      }
      named_bar_sync(1, kWarps * 32);
      if (tid == 0) {  // in place of ar_finish (read by this GPU's next launch: gpu scope)
        __threadfence();
        atomicExch(&ar_header(ar)->gen, e);
      }
    }
    if (last && tid < kMaxM) {
      float v = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) v += s_part[j * kMaxM + tid];
      s_rstd[tid] = rsqrtf(v / (float)p.N + p.eps);  // (this CTA's own copy, read below)
    }
    named_bar_sync(1, kWarps * 32);
    // to every CTA of the cluster at once: thread q * kMaxM + m stores row m's rstd into CTA q,
    // thread q the "finish" word, then (after the CTA barrier) arrives on CTA q's rstd_bar
    {
      const int q = tid / kMaxM, m = tid - q * kMaxM;
      if (q < CS && q > 0 && last) st_dsmem_f32(mapa_shared(smem_u32(s_rstd + m), (uint32_t)q), s_rstd[m]);
      if (tid < CS) st_dsmem_f32(mapa_shared(smem_u32(s_fin), (uint32_t)tid), last ? 1.f : 0.f);
    }
    named_bar_sync(1, kWarps * 32);
    if (tid < CS) {
      fence_acq_rel_cluster();
      mbar_arrive_remote(mapa_shared(smem_u32(rstd_bar), (uint32_t)tid));
    }
  }
  if (tid == 0) *s_flag = mbar_wait_cluster(rstd_bar, 0u, s_abort) ? 1 : 0;
  B2_TRC(11);
  named_bar_sync(1, kWarps * 32);
  ok = ok && *s_flag != 0;
  if (s_fin[0] != 0.f) {  // the last cluster finishes every element
    if (p.norm_v16)
      norm_finish_all<uint4>(p, s_rstd, crank, CS);
    else
      norm_finish_all<uint2>(p, s_rstd, crank, CS);
  }
  return ok;
}

// p.norm == 2 (the default): the fused launch stops after phase a. Each CTA adds its threads' row
// sums (shuffle tree per warp, warps in order) into npart[blockIdx.x]; norm_finish_kernel, the
// next launch on the stream, adds the grid's sums and finishes every element.
__device__ __forceinline__ void norm_cta_sums(const W4Args& p, const float (&ss)[kMaxM],
                                              float* s_norm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int m = 0; m < kMaxM; ++m) {
    float v = ss[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) s_norm[warp * kMaxM + m] = v;
  }
  named_bar_sync(1, kWarps * 32);
  if (tid < kMaxM) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += s_norm[w * kMaxM + tid];
    p.npart[(size_t)blockIdx.x * kMaxM + tid] = v;
  }
}

// Phases b and c of the split RMSNorm, after a fused launch with p.norm == 2 (programmatic
// dependent launch: nothing of that launch is read before grid_dep_wait). Every CTA adds the
// `nparts` CTA sums of each row in the same fixed order (16 strided partial sums, then those in
// order), so every CTA and every rank computes the same rstd bit for bit, then finishes its share
// of the M x N elements in vectors V (uint4: 8 fp16, uint2: 4; N % 32 == 0, so a vector never
// crosses a row): x = y + residual, residual <- fp16(x), y <- fp16(fp16(x * rstd) * weight).
template <typename V>
__global__ void __launch_bounds__(256) norm_finish_kernel(const __grid_constant__ W4Args p,
                                                          int nparts) {
  __shared__ float s_part[16 * kMaxM];
  __shared__ float s_rstd[kMaxM];
  grid_dep_launch();
  grid_dep_wait();
  constexpr int kH = (int)(sizeof(V) / 2);
  const int tid = threadIdx.x;
  const int per = p.M * p.N / kH, i0 = blockIdx.x * blockDim.x + tid;
  // this thread's first vector is loaded before the row sums are added, to overlap the two
  V y0 = {}, r0 = {}, w0 = {};
  if (i0 < per) {
    const int m = (i0 * kH) / p.N, n = i0 * kH - m * p.N;
    const size_t o = (size_t)m * p.N + n;
    y0 = __ldcg(reinterpret_cast<const V*>(p.y + o));
    r0 = __ldcg(reinterpret_cast<const V*>(p.res + o));
    w0 = __ldg(reinterpret_cast<const V*>(p.nw + n));
  }
  if (tid < 16 * kMaxM) {  // partial sum j of row m: CTAs j, j + 16, ... in order
    const int m = tid & (kMaxM - 1), j = tid / kMaxM;
    float v = 0.f;
    for (int b0 = j; b0 < nparts; b0 += 16 * 16) {
      float t[16];  // 16 independent loads in flight, then added in CTA order
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int b = b0 + 16 * u;
        t[u] = b < nparts ? __ldcg(p.npart + (size_t)b * kMaxM + m) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) v += t[u];
    }
    s_part[j * kMaxM + m] = v;
  }
  __syncthreads();
  if (tid < kMaxM) {
    float v = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) v += s_part[j * kMaxM + tid];
    s_rstd[tid] = rsqrtf(v / (float)p.N + p.eps);
  }
  __syncthreads();
  for (int i = i0; i < per; i += gridDim.x * blockDim.x) {
    const int m = (i * kH) / p.N, n = i * kH - m * p.N;
    const size_t o = (size_t)m * p.N + n;
    V yv = y0, rv = r0, wv = w0;
    if (i != i0) {
      yv = __ldcg(reinterpret_cast<const V*>(p.y + o));
      rv = __ldcg(reinterpret_cast<const V*>(p.res + o));
      wv = __ldg(reinterpret_cast<const V*>(p.nw + n));
    }
    const __half* yh = reinterpret_cast<const __half*>(&yv);
    __half* rh = reinterpret_cast<__half*>(&rv);
    const __half* wh = reinterpret_cast<const __half*>(&wv);
    V ov;
    __half* oh = reinterpret_cast<__half*>(&ov);
    const float rstd = s_rstd[m];
#pragma unroll
    for (int k = 0; k < kH; ++k) {
      const float x = norm_x(yh[k], rh[k]);
      rh[k] = __float2half_rn(x);
      oh[k] = norm_out(x, rstd, wh[k]);
    }
    *reinterpret_cast<V*>(p.res + o) = rv;
    *reinterpret_cast<V*>(p.y + o) = ov;
  }
}

// A = (q - z) in fp16 (exact, see dequant_word) against B = x; the fp32 sum of each quantization
// group is scaled once: acc += s * sum. Every weight is dequantized once per CTA and used for all
// M rows.
template <int GP, bool FUSED>
__device__ __forceinline__ void w4_body(const CUtensorMap& tm_qw, const CUtensorMap& tm_sc,
                                        const CUtensorMap& tm_qz, const CUtensorMap& tm_x,
                                        const W4Args& p, const ArView& ar) {
  using C = Cfg<GP>;
  constexpr int kStages = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* s_qw = smem;
  uint8_t* s_x = smem + C::kXOff;    // stage st at s_x + st * kXBytes
  uint8_t* s_sc = smem + C::kScOff;  // stage st at s_sc + st * kScStride: [RG][128] fp16
  uint8_t* s_qz = smem + C::kQzOff;  // stage st at s_qz + st * kQzStride: [RG][16] int32
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);  // TMA bytes landed
  uint64_t* empty = full + kStages;                                 // consumers done
  volatile int* s_abort = reinterpret_cast<volatile int*>(empty + kStages);
  volatile int* s_flag = s_abort + 1;
  volatile uint32_t* s_gen = reinterpret_cast<volatile uint32_t*>(s_abort + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const StreamK& sk = p.sk;
  const long long u_lo = sk_begin(sk, blockIdx.x), u_hi = sk_begin(sk, blockIdx.x + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    *s_abort = 0;
    *s_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  grid_dep_launch();

  // ------------------------------------------------------------------ producer warp (1 thread)
  if (warp == kWarps) {
    if (lane == 0) {
      if (!p.pk) {
        tma_prefetch_desc(&tm_qw);
        tma_prefetch_desc(&tm_sc);
        tma_prefetch_desc(&tm_qz);
      }
      tma_prefetch_desc(&tm_x);
      const uint64_t pol_w = l2_evict_first_policy();   // weights: read once
      const uint64_t pol_x = l2_evict_normal_policy();  // activations: read by every CTA
      auto issue_w = [&](int st, const UnitCursor& c) {
        const int n0 = c.tile * kTileN;
        const int grow = (c.ku * kUnitK) / p.G;
        mbar_arrive_expect_tx(&full[st], C::kTx);
        if (p.pk) {
          const uint8_t* u = packed_unit(p, c.tile, c.ku);
          bulk_load(s_qw + st * kQwStage, u, kQwStage, &full[st], pol_w);
          bulk_load(s_sc + st * C::kScStride, u + kQwStage, C::kScBytes, &full[st], pol_w);
          bulk_load(s_qz + st * C::kQzStride, u + kQwStage + C::kScBytes, C::kQzBytes, &full[st],
                    pol_w);
          return;
        }
        tma_load_3d(s_qw + st * kQwStage, &tm_qw, &full[st], 0, c.ku * 16, n0 / 32, pol_w);
        tma_load_2d(s_sc + st * C::kScStride, &tm_sc, &full[st], n0, grow, pol_w);
        tma_load_2d(s_qz + st * C::kQzStride, &tm_qz, &full[st], n0 / 8, grow, pol_w);
      };
      auto issue_x = [&](int st, const UnitCursor& c) {
        tma_load_3d(s_x + st * C::kXBytes, &tm_x, &full[st], 0, 0, c.ku * 2, pol_x);
      };
      // Until the previous grid on the stream has completed, its stores may not be visible:
      // only warm L2 with the first stages' weights, then wait, then load.
      const UnitCursor c0(sk, u_lo, u_hi);
      {
        UnitCursor cp = c0;
        for (int j = 0; j < kStages && cp.left > 0; ++j, cp.next(sk)) {
          const int n0 = cp.tile * kTileN, grow = (cp.ku * kUnitK) / p.G;
          if (p.pk) {
            bulk_prefetch_l2(packed_unit(p, cp.tile, cp.ku), (uint32_t)p.pk_unit);
            continue;
          }
          tma_prefetch_l2_3d(&tm_qw, 0, cp.ku * 16, n0 / 32);
          tma_prefetch_l2_2d(&tm_sc, n0, grow);
          tma_prefetch_l2_2d(&tm_qz, n0 / 8, grow);
        }
      }
      grid_dep_wait();
      UnitCursor c = c0;
      int issued = 0;
      for (; issued < kStages && c.left > 0; ++issued, c.next(sk)) {
        issue_w(issued, c);
        issue_x(issued, c);
      }
      int st = 0;
      uint32_t ph = 0;  // parity of the consumers' release of the unit kStages back
      for (; c.left > 0; ++issued, c.next(sk)) {
        if (!mbar_wait_backoff(&empty[st], ph, s_abort)) break;
        issue_w(st, c);
        issue_x(st, c);
        if (++st == kStages) st = 0, ph ^= 1u;
      }
      // Do not retire while copies this thread issued may still be landing in shared memory:
      // units 0..issued-1 were requested; the last unit of stage s is the largest u < issued
      // with u % kStages == s.
      for (int s = 0; s < kStages && s < issued; ++s) {
        const int u = s + ((issued - 1 - s) / kStages) * kStages;
        const uint32_t par = (uint32_t)((u / kStages) & 1);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_test(&full[s], par) && globaltimer_ns() - t0 < kPipeWaitNs) {
        }
      }
      if (*s_abort) atomicCAS(p.status, 0, B2_ERR_TIMEOUT);
    }
    return;
  }

  // ------------------------------------------------------------------ consumer warps
  grid_dep_wait();
  if (FUSED && threadIdx.x == 0) *s_gen = ar_begin(ar);
  named_bar_sync(1, kWarps * 32);
  const LaneGeo L(warp, lane, p.M);
  const int t = L.t, colw = L.colw;
  const uint32_t e = FUSED ? *s_gen : 0u;
  const uint32_t x_base0 = smem_u32(s_x), qw_base0 = smem_u32(s_qw + warp * kQwBox);

  float acc[2][4];
#pragma unroll
  for (int T = 0; T < 2; ++T)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[T][i] = 0.f;

  int st = 0;
  uint32_t ph = 0;
  bool ok = true;
  for (UnitCursor cu(sk, u_lo, u_hi); cu.left > 0; cu.next(sk)) {
    const int tile = cu.tile;
    if (ok) ok = mbar_wait(&full[st], ph, s_abort);
    // The lanes poll the barrier one by one, so the warp may be diverged here;
    // mma.sync.aligned needs all 32 lanes converged.
    __syncwarp();
    consume_unit<GP>(L, x_base0 + st * C::kXBytes, qw_base0 + st * kQwStage,
                     reinterpret_cast<const __half*>(s_sc + st * C::kScStride),
                     reinterpret_cast<const uint32_t*>(s_qz + st * C::kQzStride), acc);
    fence_proxy_async_smem();  // this lane's reads of the stage precede its next TMA fill
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (++st == kStages) st = 0, ph ^= 1u;

    if (!cu.segment_end(sk)) continue;
    // ---------------------------------------------------------------- end of a tile segment
    float4 v[2];
    v[0] = make_float4(acc[0][0], acc[0][2], acc[1][0], acc[1][2]);  // m = 2t
    v[1] = make_float4(acc[0][1], acc[0][3], acc[1][1], acc[1][3]);  // m = 2t + 1
#pragma unroll
    for (int T = 0; T < 2; ++T)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[T][i] = 0.f;

    const long long ts = (long long)tile * sk.upt;
    const int first = sk_owner(sk, ts), last = sk_owner(sk, ts + sk.upt - 1);
    bool finisher = true;
    if (first != last) {
      float* slot =
          p.partials + ((size_t)blockIdx.x * 2 + sk_slot_from_begin(u_lo, ts)) * kSlotFloats;
#pragma unroll
      for (int j = 0; j < 2; ++j)
        if (2 * t + j < p.M)
          __stcg(reinterpret_cast<float4*>(slot + (2 * t + j) * kTileN + colw), v[j]);
      // every writer makes its partials visible device-wide before the barrier; then one
      // thread counts the CTA's arrival
      __threadfence();
      named_bar_sync(1, kWarps * 32);
      if (threadIdx.x == 0) {
        const int prev = atomicAdd(&p.counters[tile], 1);
        const int fin = (prev == last - first);
        if (fin) {
          p.counters[tile] = 0;  // next used by a later launch, which the kernel boundary orders
          __threadfence();       // acquire side: the contributors' partials are read after this
        }
        *s_flag = fin;
      }
      named_bar_sync(1, kWarps * 32);
      finisher = *s_flag != 0;
      if (finisher) {
        // add the contributors' slots in CTA order, eight loads in flight at a time
        v[0] = v[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        const int first_slot = sk_slot_from_begin(sk_begin(sk, first), ts);
        for (int c0 = first; c0 <= last; c0 += 8) {
          float4 a[8][2];
#pragma unroll
          for (int b = 0; b < 8; ++b) {
            const int c = c0 + b;
            const float* sl =
                p.partials + ((size_t)c * 2 + (c == first ? first_slot : 0)) * kSlotFloats;
#pragma unroll
            for (int j = 0; j < 2; ++j)
              a[b][j] = (c <= last && 2 * t + j < p.M)
                            ? __ldcg(reinterpret_cast<const float4*>(sl + (2 * t + j) * kTileN + colw))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int b = 0; b < 8; ++b)
            if (c0 + b <= last)
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                v[j].x += a[b][j].x;
                v[j].y += a[b][j].y;
                v[j].z += a[b][j].z;
                v[j].w += a[b][j].w;
              }
        }
      }
    }
    if (!finisher) continue;
    if (!FUSED) {
      store_y(p, tile, colw, t, v);
      continue;
    }
    // Fused all-reduce: push this rank's finished fp32 tile into slot[e&1][rank] of every rank
    // ([M][N] layout). Low-latency form: 64-bit value+generation words, nothing else to publish.
    // Otherwise fp32 values, then the tile's flag on every rank.
    const int n = tile * kTileN + colw;
    if (p.ll) {
      if (n < p.N)
        for (int r = 0; r < ar.world; ++r) {
          uint64_t* dst = reinterpret_cast<uint64_t*>(ar_slot(ar, r, e & 1u, ar.rank));
#pragma unroll
          for (int j = 0; j < 2; ++j)
            if (2 * t + j < p.M) {
              uint64_t* d = dst + (size_t)(2 * t + j) * p.N + n;
              ll_store(d + 0, v[j].x, e);
              ll_store(d + 1, v[j].y, e);
              ll_store(d + 2, v[j].z, e);
              ll_store(d + 3, v[j].w, e);
            }
        }
      continue;
    }
    if (n < p.N) {
      for (int r = 0; r < ar.world; ++r) {
        float* dst = reinterpret_cast<float*>(ar_slot(ar, r, e & 1u, ar.rank));
#pragma unroll
        for (int j = 0; j < 2; ++j)
          if (2 * t + j < p.M) *reinterpret_cast<float4*>(dst + (size_t)(2 * t + j) * p.N + n) = v[j];
      }
    }
    named_bar_sync(1, kWarps * 32);
    if (threadIdx.x == 0) ar_publish(ar, tile, e);  // one release fence covers the CTA's stores
  }
  if (!ok && lane == 0) atomicCAS(p.status, 0, B2_ERR_TIMEOUT);
  if constexpr (FUSED) {
    // -------------------------------------------------------------- fused all-reduce, phase 2
    // CTA b adds tiles b, b + grid, ... over all ranks in rank order and writes the fp16 result.
    const unsigned long long deadline = globaltimer_ns() + ar.timeout_ns;
    float ss[kMaxM];  // RMSNorm: this thread's sums of squares per row
#pragma unroll
    for (int i = 0; i < kMaxM; ++i) ss[i] = 0.f;
    for (int tile = blockIdx.x; tile < sk.tiles; tile += gridDim.x) {
      const int n = tile * kTileN + colw;
      if (p.ll) {
        if (n >= p.N) continue;
        float4 v[2];
        v[0] = v[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        bool got = true;
        for (int src = 0; src < ar.world; ++src) {
          const uint64_t* sl = reinterpret_cast<const uint64_t*>(ar_slot(ar, ar.rank, e & 1u, src));
#pragma unroll
          for (int j = 0; j < 2; ++j)
            if (2 * t + j < p.M) {
              const uint64_t* q = sl + (size_t)(2 * t + j) * p.N + n;
              const uint64_t* ptr[4] = {q, q + 1, q + 2, q + 3};
              float a[4];
              got &= ll_gather<4>(ptr, 4, e, deadline, a);
              v[j].x += a[0];
              v[j].y += a[1];
              v[j].z += a[2];
              v[j].w += a[3];
            }
        }
        if (!got) atomicCAS(&ar_header(ar)->status, 0, B2_ERR_TIMEOUT);
        store_y(p, tile, colw, t, v);
        if (p.norm) norm_accum_lane(p, t, n, v, ss);
        continue;
      }
      named_bar_sync(1, kWarps * 32);
      if (threadIdx.x == 0) *s_flag = ar_wait(ar, tile, e) ? 1 : 0;
      named_bar_sync(1, kWarps * 32);
      __threadfence();
      if (n >= p.N) continue;
      float4 v[2];
      v[0] = v[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int src = 0; src < ar.world; ++src) {
        const float* sl = reinterpret_cast<const float*>(ar_slot(ar, ar.rank, e & 1u, src));
#pragma unroll
        for (int j = 0; j < 2; ++j)
          if (2 * t + j < p.M) {
            const float4 a =
                __ldcg(reinterpret_cast<const float4*>(sl + (size_t)(2 * t + j) * p.N + n));
            v[j].x += a.x;
            v[j].y += a.y;
            v[j].z += a.z;
            v[j].w += a.w;
          }
      }
      store_y(p, tile, colw, t, v);
      if (p.norm) norm_accum_lane(p, t, n, v, ss);
    }
    if (p.norm == 2) norm_cta_sums(p, ss, reinterpret_cast<float*>(smem + C::kNormOff));
    if (p.norm == 1) {
      float* s_norm = reinterpret_cast<float*>(smem + C::kNormOff);
      if (!norm_rstd(p, ar, e, ss, s_norm, s_flag) && threadIdx.x == 0)
        atomicCAS(&ar_header(ar)->status, 0, B2_ERR_TIMEOUT);
      for (int tile = blockIdx.x; tile < sk.tiles; tile += gridDim.x) {
        const int n = tile * kTileN + colw;
        if (n >= p.N) continue;
#pragma unroll
        for (int j = 0; j < 2; ++j)
          if (2 * t + j < p.M) norm_finish4(p, 2 * t + j, n, s_norm[kWarps * kMaxM + 2 * t + j]);
      }
    }
    named_bar_sync(1, kWarps * 32);
    if (threadIdx.x == 0) ar_finish(ar, e);
  }
}

template <int GP, bool FUSED>
__global__ void __launch_bounds__(kThreads, GP == 4 ? 4 : 3)
    w4_kernel(const __grid_constant__ CUtensorMap tm_qw, const __grid_constant__ CUtensorMap tm_sc,
              const __grid_constant__ CUtensorMap tm_qz, const __grid_constant__ CUtensorMap tm_x,
              const __grid_constant__ W4Args p, const __grid_constant__ ArView ar) {
  w4_body<GP, FUSED>(tm_qw, tm_sc, tm_qz, tm_x, p, ar);
}

// =================================================================================================
// Cluster split-K variant. The CTAs of one thread-block cluster share output tiles: cluster c
// owns tiles c, c + NC, ... and CTA rank r of the cluster computes k-units
// [r * upt / CS, (r + 1) * upt / CS) of each. A tile's partial sums are reduced through
// distributed shared memory: every CTA leaves its fp32 partial tile in its own shared memory,
// and CTA r adds column slice r of all CS partials in rank order (deterministic) and writes it.
// No workspace, no global atomics, no second pass; the fused all-reduce pushes each slice.
// =================================================================================================
// A (aliased): every cluster of the launch reduces exactly one output tile, so its reduction
// buffers are needed only once the stage ring has drained; they then take the place of the first
// stages' weights, and the 8.6 KB they would hold apart buys a fifth stage instead.
template <int GP, bool A = false>
struct CfgC {
  // 4 stages + a 4 KB reduction buffer, or 5 stages with the buffers aliased: four CTAs per SM
  static constexpr int kStages = A ? 5 : 4;
  static constexpr int RG = 4 / GP;
  static constexpr int kScBytes = RG * kTileN * 2;
  static constexpr int kQzBytes = RG * (kTileN / 8) * 4;
  static constexpr int kScStride = align128(kScBytes);
  static constexpr int kQzStride = align128(kQzBytes);
  static constexpr int kXBytes = kMaxM * kUnitK * 2;
  static constexpr int kTx = kQwStage + kXBytes + kScBytes + kQzBytes;
  static constexpr int kXOff = kStages * kQwStage;
  static constexpr int kScOff = kXOff + kStages * kXBytes;
  static constexpr int kQzOff = kScOff + kStages * kScStride;
  // reduction buffers: my partial tile arranged by destination CTA ([8 rows][W_r] fp32 per CTA
  // r), and the CS slices the cluster sends me ([CS][8 rows][W] fp32, W <= 128 / CS + 1)
  static constexpr int kRingEnd = kQzOff + kStages * kQzStride;
  static constexpr int kSendOff = A ? 0 : kRingEnd;
  static constexpr int kRecvOff = kSendOff + kMaxM * kTileN * 4;
  static constexpr int kRecvBytes = kMaxM * (kTileN + 16) * 4;
  static constexpr int kBarOff = A ? kRingEnd : kRecvOff + kRecvBytes;
  // full[S], empty[S], red_full, red_empty, pub_bar, norm_bar, rstd_bar
  static constexpr int kNormOff = align128(kBarOff + (2 * kStages + 5) * 8 + 32);
  // RMSNorm epilogue (fused launches): warp row sums [kWarps][kMaxM], rstd [kMaxM], the "finish"
  // word [kMaxM], the cluster's CTA row sums gathered at its leader [16][kMaxM], the leader's
  // partial sums [16][kMaxM], the leader's "last cluster" word [kMaxM]
  static constexpr int kNormClusterFloats = (kWarps + 2) * kMaxM + 2 * 16 * kMaxM + kMaxM;
  static constexpr int kSmem = 1024 + kNormOff + (A ? 0 : kNormClusterFloats * 4);
  static_assert(kXOff % 1024 == 0 && kXBytes % 1024 == 0, "swizzled boxes need 1024 B");
  static_assert(kScOff % 128 == 0 && kQzOff % 128 == 0 && kSendOff % 128 == 0 &&
                    kRecvOff % 128 == 0, "alignment");
  static_assert(!A || kRecvOff + kRecvBytes <= kXOff, "aliased buffers lie inside the qw ring");
};


template <int GP, bool FUSED, bool A = false>
__device__ __forceinline__ void w4c_body(const CUtensorMap& tm_qw, const CUtensorMap& tm_sc,
                                        const CUtensorMap& tm_qz, const CUtensorMap& tm_x,
                                        const W4Args& p, const ArView& ar) {
  static_assert(!(A && FUSED), "the exchange epilogue keeps its buffers apart");
  using C = CfgC<GP, A>;
  constexpr int kStages = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* s_qw = smem;
  uint8_t* s_x = smem + C::kXOff;
  uint8_t* s_sc = smem + C::kScOff;
  uint8_t* s_qz = smem + C::kQzOff;
  float* s_send = reinterpret_cast<float*>(smem + C::kSendOff);
  const float* s_recv = reinterpret_cast<const float*>(smem + C::kRecvOff);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + kStages;
  uint64_t* red_full = empty + kStages;  // the CS slices of the tile have landed in s_recv
  uint64_t* red_empty = red_full + 1;    // every receiver has added up my previous tile
  uint64_t* pub_bar = red_empty + 1;     // (CTA 0, fp32 flag exchange) every CTA pushed its slice
  uint64_t* norm_bar = pub_bar + 1;      // (leader, RMSNorm) every CTA's row sums have landed
  uint64_t* rstd_bar = norm_bar + 1;     // (RMSNorm) the leader has sent this CTA the rstd
  volatile int* s_abort = reinterpret_cast<volatile int*>(rstd_bar + 1);
  volatile int* s_flag = s_abort + 1;
  volatile uint32_t* s_gen = reinterpret_cast<volatile uint32_t*>(s_abort + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int CS = p.cl_size, NC = p.cl_count;
  const int crank = (int)cluster_ctarank();
  const int cid = blockIdx.x / CS;
  const int upt = p.sk.upt, tiles = p.sk.tiles;
  const int k0 = upt * crank / CS, k1 = upt * (crank + 1) / CS, nk = k1 - k0;
  const int ntile = (tiles - 1 - cid) / NC + 1;
  const int n_units = ntile * nk;
  if (A && ntile != 1) {  // the host launches the aliased layout only with one tile per cluster
    if (threadIdx.x == 0) atomicCAS(p.status, 0, B2_ERR_STATE);
    return;  // the whole cluster returns (ntile is the same for all its CTAs)
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    mbar_init(red_full, 1);  // my own expect-tx; the senders' copies complete the bytes
    mbar_init(red_empty, CS);
    mbar_init(pub_bar, CS);
    mbar_init(norm_bar, CS);
    mbar_init(rstd_bar, 1);
    *s_abort = 0;
    *s_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  cluster_sync_all();  // no CTA arrives on a peer's barrier before the peer initialised it
  grid_dep_launch();
#ifdef B2_TRACE
  if (threadIdx.x == 0 && blockIdx.x < kTraceCtas) {
    unsigned int smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    g_trace_ctas[blockIdx.x][0] = globaltimer_ns();
    g_trace_ctas[blockIdx.x][2] = smid;
  }
#endif

  // ------------------------------------------------------------------ producer warp (1 thread)
  if (warp == kWarps) {
    if (lane == 0) {
      if (!p.pk) {
        tma_prefetch_desc(&tm_qw);
        tma_prefetch_desc(&tm_sc);
        tma_prefetch_desc(&tm_qz);
      }
      tma_prefetch_desc(&tm_x);
      const uint64_t pol_w = l2_evict_first_policy();
      const uint64_t pol_x = l2_evict_normal_policy();
      // unit j of this CTA: tile cid + (j / nk) * NC, k-unit k0 + j % nk
      auto where = [&](int j, int& tile, int& ku) {
        const int i = j / nk;
        tile = cid + i * NC;
        ku = k0 + (j - i * nk);
      };
      auto issue = [&](int st, int j, bool with_w, bool with_x) {
        int tile, ku;
        where(j, tile, ku);
        const int n0 = tile * kTileN;
        if (with_w) {
          const int grow = (ku * kUnitK) / p.G;
          B2_TR(0, j);
          mbar_arrive_expect_tx(&full[st], C::kTx);
          if (p.pk) {
            const uint8_t* u = packed_unit(p, tile, ku);
            bulk_load(s_qw + st * kQwStage, u, kQwStage, &full[st], pol_w);
            bulk_load(s_sc + st * C::kScStride, u + kQwStage, C::kScBytes, &full[st], pol_w);
            bulk_load(s_qz + st * C::kQzStride, u + kQwStage + C::kScBytes, C::kQzBytes,
                      &full[st], pol_w);
          } else {
            tma_load_3d(s_qw + st * kQwStage, &tm_qw, &full[st], 0, ku * 16, n0 / 32, pol_w);
            tma_load_2d(s_sc + st * C::kScStride, &tm_sc, &full[st], n0, grow, pol_w);
            tma_load_2d(s_qz + st * C::kQzStride, &tm_qz, &full[st], n0 / 8, grow, pol_w);
          }
        }
        if (with_x) {
          tma_load_3d(s_x + st * C::kXBytes, &tm_x, &full[st], 0, 0, ku * 2, pol_x);
        }
      };
      // until the previous grid has completed only warm L2 with the first stages' weights
      for (int j = 0; j < kStages && j < n_units; ++j) {
        int tile, ku;
        where(j, tile, ku);
        const int n0 = tile * kTileN, grow = (ku * kUnitK) / p.G;
        if (p.pk) {
          bulk_prefetch_l2(packed_unit(p, tile, ku), (uint32_t)p.pk_unit);
          continue;
        }
        tma_prefetch_l2_3d(&tm_qw, 0, ku * 16, n0 / 32);
        tma_prefetch_l2_2d(&tm_sc, n0, grow);
        tma_prefetch_l2_2d(&tm_qz, n0 / 8, grow);
      }
      grid_dep_wait();
      int issued = 0;
      for (; issued < kStages && issued < n_units; ++issued) issue(issued, issued, true, true);
      int st = 0;
      uint32_t ph = 0;
      for (; issued < n_units; ++issued) {
        if (!mbar_wait_backoff(&empty[st], ph, s_abort)) break;
        B2_TR(1, issued);
        issue(st, issued, true, true);
        if (++st == kStages) st = 0, ph ^= 1u;
      }
      for (int s = 0; s < kStages && s < issued; ++s) {
        const int u = s + ((issued - 1 - s) / kStages) * kStages;
        const uint32_t par = (uint32_t)((u / kStages) & 1);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_test(&full[s], par) && globaltimer_ns() - t0 < kPipeWaitNs) {
        }
      }
      if (*s_abort) atomicCAS(p.status, 0, B2_ERR_TIMEOUT);
    }
    return;
  }

  // ------------------------------------------------------------------ consumer warps
  grid_dep_wait();
  B2_TRC(7);
  if (FUSED && threadIdx.x == 0) *s_gen = ar_begin(ar);
  named_bar_sync(1, kWarps * 32);
  const LaneGeo L(warp, lane, p.M);
  const int t = L.t, colw = L.colw;
  const uint32_t e = FUSED ? *s_gen : 0u;
  const int tid = threadIdx.x;
  // column slice of every tile that this CTA reduces and writes
  const int c0 = kTileN * crank / CS, c1 = kTileN * (crank + 1) / CS, W = c1 - c0;
  const uint32_t send_addr = smem_u32(s_send), recv_addr = smem_u32(s_recv);
  const uint32_t x_base0 = smem_u32(s_x), qw_base0 = smem_u32(s_qw + warp * kQwBox);

  float acc[2][4];
#pragma unroll
  for (int T = 0; T < 2; ++T)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[T][i] = 0.f;

  int st = 0;
  uint32_t ph = 0;
  bool ok = true;
  // one rank (a one-rank handle): there is nothing to exchange, so the reduced tile is stored as
  // y at once, with the RMSNorm's sums of squares, and the exchange's second phase is skipped
  const bool solo = FUSED && ar.world == 1;
  float ss1[kMaxM];
#pragma unroll
  for (int i = 0; i < kMaxM; ++i) ss1[i] = 0.f;
  for (int it = 0; it < ntile; ++it) {
    const int tile = cid + it * NC;
    for (int ku = k0; ku < k1; ++ku) {
      if (ok) ok = mbar_wait(&full[st], ph, s_abort);
      if (warp == 0 && lane == 0) B2_TR(2, it * nk + ku - k0);
      __syncwarp();
      consume_unit<GP>(L, x_base0 + st * C::kXBytes, qw_base0 + st * kQwStage,
                       reinterpret_cast<const __half*>(s_sc + st * C::kScStride),
                       reinterpret_cast<const uint32_t*>(s_qz + st * C::kQzStride), acc);
      fence_proxy_async_smem();  // this lane's reads of the stage precede its next TMA fill
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (warp == 0 && lane == 0) B2_TR(3, it * nk + ku - k0);
      if (++st == kStages) st = 0, ph ^= 1u;
    }
    if (warp == 0 && lane == 0) B2_TR(4, it);
    B2_TRC(3);

    // ---------------------------------------------------------------- tile epilogue: reduce
    // Push, not pull: every CTA writes its partial tile into its send buffer arranged by the CTA
    // that owns each column slice, and sends slice r to CTA r with one bulk copy (shared::cta ->
    // shared::cluster) that completes its bytes on CTA r's red_full. A CTA then adds the CS
    // slices it received in cluster rank order from its own shared memory. With one tile per
    // CTA there is no round trip at all; with more, the next tile's copies wait until every
    // receiver has added up the previous one (red_empty).
    // (a) the send buffer: the copies that read it for the previous tile must be done reading.
    // Aliased layout: the buffers lie on the stage ring, so every consumer warp must be done with
    // the ring before they are written, and no peer may push into my receive buffer before I say
    // so: lane r arrives on CTA r's red_empty, and CTA r pushes only once all CS CTAs have.
    if (it > 0) {
      if (tid < CS) bulk_wait_read_all();
      named_bar_sync(1, kWarps * 32);
    }
    if (A) {
      named_bar_sync(1, kWarps * 32);
      if (tid < CS) mbar_arrive_remote(mapa_shared(smem_u32(red_empty), (uint32_t)tid));
    }
    {
      const float v[2][4] = {{acc[0][0], acc[0][2], acc[1][0], acc[1][2]},   // row 2t
                             {acc[0][1], acc[0][3], acc[1][1], acc[1][3]}};  // row 2t + 1
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = colw + j;
        const int r = ((col + 1) * CS - 1) / kTileN;  // the CTA whose slice holds col
        const int cr0 = kTileN * r / CS, wr = kTileN * (r + 1) / CS - cr0;
        float* dst = s_send + kMaxM * cr0 + (col - cr0);
        dst[(2 * t) * wr] = v[0][j];
        dst[(2 * t + 1) * wr] = v[1][j];
      }
    }
#pragma unroll
    for (int T = 0; T < 2; ++T)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[T][i] = 0.f;
    fence_proxy_async_smem();  // these generic writes precede the copies' (async proxy) reads
    named_bar_sync(1, kWarps * 32);
    // (b) lane r of warp 0 sends slice r into CTA r's receive buffer, at my rank's place
    if (tid < CS) {
      const bool go = (it == 0 && !A) ||
                      mbar_wait_cluster(red_empty, (uint32_t)((A ? it : it - 1) & 1), s_abort);
      if (go) {
        const int cr0 = kTileN * tid / CS, wr = kTileN * (tid + 1) / CS - cr0;
        const uint32_t bytes = (uint32_t)(kMaxM * wr * 4);
        bulk_copy_to_peer(mapa_shared(recv_addr + (uint32_t)crank * bytes, (uint32_t)tid),
                          send_addr + (uint32_t)(kMaxM * cr0 * 4), bytes,
                          mapa_shared(smem_u32(red_full), (uint32_t)tid));
        bulk_commit();
      }
    }
    // (c) my slice from every CTA of the cluster
    if (tid == 0) {
      mbar_arrive_expect_tx(red_full, (uint32_t)(CS * kMaxM * W * 4));
      *s_flag = mbar_wait_cluster(red_full, (uint32_t)(it & 1), s_abort);
    }
    named_bar_sync(1, kWarps * 32);
    ok = ok && *s_flag;
    // slice [c0, c1) of the tile: the CS partials added in rank order
    for (int idx = tid; idx < p.M * W; idx += kWarps * 32) {
      const int m = idx / W, col = c0 + (idx - m * W);
      const float* src = s_recv + idx;  // [q][8 rows][W]: element (m, col) of sender q
      float part[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) part[q] = (q < CS) ? src[q * kMaxM * W] : 0.f;
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < 16; ++q)
        if (q < CS) s += part[q];
      const int n = tile * kTileN + col;
      if (n < p.N) {
        if (!FUSED || solo) {
          const __half yh = __float2half_rn(s);
          p.y[(size_t)m * p.N + n] = yh;
          if (FUSED && p.norm) {
            const float x = norm_x(yh, p.res[(size_t)m * p.N + n]);
            row_add(ss1, m, x * x);
          }
        } else {
          // exchange layout: slice (tile, crank) is one block of M x W floats at
          // (tile * 128 + c0) * M, element idx in the order the threads produce them, so a
          // warp's pushes over NVLink are coalesced (needs N % 128 == 0, checked on the host)
          const size_t at = ((size_t)tile * kTileN + c0) * p.M + idx;
          if (p.ll && p.two_shot) {  // to the tile's owner only (possibly this rank)
            ll_store(reinterpret_cast<uint64_t*>(ar_slot(ar, tile % ar.world, e & 1u, ar.rank)) + at,
                     s, e);
          } else if (p.ll) {
            for (int r = 0; r < ar.world; ++r)
              ll_store(reinterpret_cast<uint64_t*>(ar_slot(ar, r, e & 1u, ar.rank)) + at, s, e);
          } else {
            for (int r = 0; r < ar.world; ++r)
              reinterpret_cast<float*>(ar_slot(ar, r, e & 1u, ar.rank))[at] = s;
          }
        }
      }
    }
    B2_TRC(4);
    // (d) tell every sender that my receive buffer is free again (only if it will be reused)
    if (it + 1 < ntile) {
      fence_proxy_async_smem();  // my reads precede the next copies into the buffer
      named_bar_sync(1, kWarps * 32);
      if (tid < CS) mbar_arrive_remote(mapa_shared(smem_u32(red_empty), (uint32_t)tid));
    }
    // fp32 flag exchange: every CTA of the cluster has pushed its slice once CTA 0's pub_bar
    // completes; CTA 0 then publishes the tile with one system-scope fence (the peers' pushes
    // happen before it through their CTA barrier and cluster-scope release, which the fence's
    // cumulativity covers).
    if (FUSED && !p.ll && !solo) {
      named_bar_sync(1, kWarps * 32);
      if (tid == 0) mbar_arrive_remote(mapa_shared(smem_u32(pub_bar), 0u));
      if (crank == 0 && tid == 0 && mbar_wait_cluster(pub_bar, (uint32_t)(it & 1), s_abort))
        ar_publish(ar, tile, e);
    }
  }
  if constexpr (FUSED) {
    // -------------------------------------------------------------- fused all-reduce, phase 2
    B2_TRC(5);
    const unsigned long long deadline = globaltimer_ns() + ar.timeout_ns;
    float ss[kMaxM];  // RMSNorm: this thread's sums of squares per row
#pragma unroll
    for (int i = 0; i < kMaxM; ++i) ss[i] = ss1[i];
    for (int it = 0; it < (solo ? 0 : ntile); ++it) {
      const int tile = cid + it * NC;
      const size_t blk = ((size_t)tile * kTileN + c0) * p.M;
      if (p.ll) {
        bool got = true;
        // Two-shot: the owner of the tile has every rank's partial of it in its slots; it adds
        // them and sends the fp16 result (as an exactly representable fp32 word) to the other
        // ranks' slot of the owner, at the same offsets: no rank sends partials of a tile it
        // owns, so those words are free. One-shot: every rank has every rank's partials.
        const int owner = tile % ar.world;
        const bool wait_result = p.two_shot && owner != ar.rank;
        for (int idx = tid; idx < p.M * W; idx += kWarps * 32) {
          const int m = idx / W, col = c0 + (idx - m * W);
          const int n = tile * kTileN + col;
          if (n >= p.N) continue;
          __half yh;
          if (wait_result) {
            const uint64_t* ptr[1] = {
                reinterpret_cast<const uint64_t*>(ar_slot(ar, ar.rank, e & 1u, owner)) + blk + idx};
            float a[1];
            got &= ll_gather<1>(ptr, 1, e, deadline, a);
            yh = __float2half_rn(a[0]);
          } else {
            const uint64_t* ptr[kArMaxWorld];
#pragma unroll
            for (int src = 0; src < kArMaxWorld; ++src)
              ptr[src] = reinterpret_cast<const uint64_t*>(
                             ar_slot(ar, ar.rank, e & 1u, src < ar.world ? src : 0)) + blk + idx;
            float a[kArMaxWorld];
            got &= ll_gather<kArMaxWorld>(ptr, ar.world, e, deadline, a);
            float s = 0.f;
#pragma unroll
            for (int src = 0; src < kArMaxWorld; ++src)
              if (src < ar.world) s += a[src];
            yh = __float2half_rn(s);
            if (p.two_shot) {
              const float v = __half2float(yh);
              for (int r = 0; r < ar.world; ++r)
                if (r != ar.rank)
                  ll_store(reinterpret_cast<uint64_t*>(ar_slot(ar, r, e & 1u, ar.rank)) + blk + idx,
                           v, e);
            }
          }
          p.y[(size_t)m * p.N + n] = yh;
          if (p.norm) {
            const float x = norm_x(yh, p.res[(size_t)m * p.N + n]);
            row_add(ss, m, x * x);
          }
        }
        if (!got) atomicCAS(&ar_header(ar)->status, 0, B2_ERR_TIMEOUT);
        continue;
      }
      named_bar_sync(1, kWarps * 32);
      if (tid == 0) *s_flag = ar_wait(ar, tile, e) ? 1 : 0;
      named_bar_sync(1, kWarps * 32);
      __threadfence();
      for (int idx = tid; idx < p.M * W; idx += kWarps * 32) {
        const int m = idx / W, col = c0 + (idx - m * W);
        const int n = tile * kTileN + col;
        if (n >= p.N) continue;
        float s = 0.f;
        for (int src = 0; src < ar.world; ++src)
          s += __ldcg(reinterpret_cast<const float*>(ar_slot(ar, ar.rank, e & 1u, src)) + blk + idx);
        const __half yh = __float2half_rn(s);
        p.y[(size_t)m * p.N + n] = yh;
        if (p.norm) {
          const float x = norm_x(yh, p.res[(size_t)m * p.N + n]);
          row_add(ss, m, x * x);
        }
      }
    }
    B2_TRC(6);
    if (p.norm == 2) norm_cta_sums(p, ss, reinterpret_cast<float*>(smem + C::kNormOff));
    if (p.norm == 1) {
      float* s_norm = reinterpret_cast<float*>(smem + C::kNormOff);
      if (!norm_finish_cluster(p, ar, e, ss, s_norm, norm_bar, rstd_bar, s_flag, s_abort, crank,
                               CS, cid, NC) &&
          tid == 0)
        atomicCAS(&ar_header(ar)->status, 0, B2_ERR_TIMEOUT);
    }
    named_bar_sync(1, kWarps * 32);
    // (in-launch norm launches advanced the generation above)
    if (tid == 0 && p.norm != 1) ar_finish(ar, e);
  }
  // Before this CTA exits, no peer may still write into its shared memory or arrive on its
  // barriers, and its own outgoing copies must be done reading its send buffer. On the normal
  // path every such access was waited for above; after a wait gave up, wait for the last ones
  // again with the full bound (exiting under a peer's copy is worse than waiting).
  {
    volatile int* no_abort = s_flag + 2;  // a zeroed word of its own
    named_bar_sync(1, kWarps * 32);
    if (tid == 0 && *s_abort) {
      *no_abort = 0;
      mbar_wait_cluster(red_full, (uint32_t)((ntile - 1) & 1), no_abort);
      *no_abort = 0;
      if (A) mbar_wait_cluster(red_empty, 0u, no_abort);  // every peer's "drained" arrival
      else if (ntile > 1) mbar_wait_cluster(red_empty, (uint32_t)((ntile - 2) & 1), no_abort);
      *no_abort = 0;
      if (FUSED && !p.ll && !solo && crank == 0)
        mbar_wait_cluster(pub_bar, (uint32_t)((ntile - 1) & 1), no_abort);
      if (FUSED && p.norm == 1) {  // the leader's rstd here, and (leader) every CTA's row sums
        *no_abort = 0;
        mbar_wait_cluster(rstd_bar, 0u, no_abort);
        *no_abort = 0;
        if (crank == 0) mbar_wait_cluster(norm_bar, 0u, no_abort);
      }
    }
    if (tid < CS) bulk_wait_read_all();
    named_bar_sync(1, kWarps * 32);
  }
  if (!ok && lane == 0) atomicCAS(p.status, 0, B2_ERR_TIMEOUT);
#ifdef B2_TRACE
  if (threadIdx.x == 0 && blockIdx.x < kTraceCtas) g_trace_ctas[blockIdx.x][1] = globaltimer_ns();
#endif
}

template <int GP, bool FUSED, bool A = false>
__global__ void __launch_bounds__(kThreads, GP == 4 ? 4 : 3)
    w4c_kernel(const __grid_constant__ CUtensorMap tm_qw, const __grid_constant__ CUtensorMap tm_sc,
               const __grid_constant__ CUtensorMap tm_qz, const __grid_constant__ CUtensorMap tm_x,
               const __grid_constant__ W4Args p, const __grid_constant__ ArView ar) {
  w4c_body<GP, FUSED, A>(tm_qw, tm_sc, tm_qz, tm_x, p, ar);
}

// =================================================================================================
// Several ranks of a tensor-parallel group emulated on one GPU, in one launch: grid.y = rank, and
// every rank's operands, tensor maps and all-reduce view are kernel arguments indexed by it. The
// ranks' CTAs wait for one another, so the launch is cooperative: either all of them are resident
// at once or the launch fails. For testing the multi-rank exchange without several GPUs.
// =================================================================================================
constexpr int kEmuMaxRanks = 4;
struct W4Emu {
  CUtensorMap qw[kEmuMaxRanks], sc[kEmuMaxRanks], qz[kEmuMaxRanks], x[kEmuMaxRanks];
  W4Args p[kEmuMaxRanks];
  ArView ar[kEmuMaxRanks];
};

template <int GP>
__global__ void __launch_bounds__(kThreads, GP == 4 ? 4 : 3) w4_kernel_emu(const __grid_constant__ W4Emu E) {
  const int r = blockIdx.y;
  w4_body<GP, true>(E.qw[r], E.sc[r], E.qz[r], E.x[r], E.p[r], E.ar[r]);
}

template <int GP>
__global__ void __launch_bounds__(kThreads, GP == 4 ? 4 : 3) w4c_kernel_emu(const __grid_constant__ W4Emu E) {
  const int r = blockIdx.y;
  w4c_body<GP, true>(E.qw[r], E.sc[r], E.qz[r], E.x[r], E.p[r], E.ar[r]);
}

struct KernelCache {
  bool configured = false;
  int occ = 0;
};
KernelCache g_cache[64][3][2];

// The four tensor maps of a launch (weights, scales, zeros, activations).
template <int RG>
int encode_maps(const W4Args& a, const void* qw, const void* qz, const void* sc, CUtensorMap* m_qw,
                CUtensorMap* m_sc, CUtensorMap* m_qz, CUtensorMap* m_x) {
  const int K = a.K, N = a.N, G = a.G;
  if (a.pk) {  // repacked weights come in by plain bulk copies: no weight maps (left zeroed)
    std::memset(m_qw, 0, sizeof(CUtensorMap));
    std::memset(m_sc, 0, sizeof(CUtensorMap));
    std::memset(m_qz, 0, sizeof(CUtensorMap));
  } else {
    // qw [K/8 word rows, N] int32 as (32 columns, word rows, 32-column blocks): one box is a
    // unit's 4 blocks x 16 rows, laid out [block][row][32 words] with each 128-byte row swizzled
    // by its row index, as 4 separate 32 x 16 boxes would be (N % 32 == 0: whole blocks)
    const uint64_t qd[3] = {32, (uint64_t)(K / 8), (uint64_t)(N / 32)};
    const uint64_t qs[2] = {(uint64_t)N * 4, 128};
    const uint32_t qb[3] = {32, 16, (uint32_t)kWarps};
    int rc = encode_3d(m_qw, CU_TENSOR_MAP_DATA_TYPE_INT32, qw, qd, qs, qb,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = encode_2d(m_sc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc, (uint64_t)N, (uint64_t)(K / G),
                   (uint64_t)N * 2, kTileN, RG, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = encode_2d(m_qz, CU_TENSOR_MAP_DATA_TYPE_INT32, qz, (uint64_t)(N / 8), (uint64_t)(K / G),
                   (uint64_t)N / 2, kTileN / 8, RG, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  // activations [M rows, K] fp16 as (64 k, rows, 64-k chunks): one box is a unit's two chunks of
  // 8 rows, [chunk][row][64] (K % 128 == 0); rows M..7 of a box read as zeros (out of bounds)
  const uint64_t xd[3] = {64, (uint64_t)a.M, (uint64_t)(K / 64)};
  const uint64_t xs[2] = {(uint64_t)K * 2, 128};
  const uint32_t xb[3] = {64, kMaxM, 2};
  return encode_3d(m_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x, xd, xs, xb,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

// B2_LOG_PLAN=1 in the environment prints the split-K plan of every W4 launch to stderr.
bool plan_log() {
  static const bool on = [] {
    const char* v = std::getenv("B2_LOG_PLAN");
    return v && v[0] && v[0] != '0';
  }();
  return on;
}

// How many clusters of 1..16 CTAs of the cluster kernel can be resident at once (per device).
struct ClusterCaps {
  bool configured = false;
  int max_clusters[17] = {0};
  int occ = 0;  // resident CTAs per SM
};
ClusterCaps g_ccaps[64][3][2][2];

template <int GP, bool FUSED, bool A = false>
int cluster_caps(int dev, const ClusterCaps** out) {
  using C = CfgC<GP, A>;
  ClusterCaps& cc = g_ccaps[dev][GP == 1 ? 0 : GP == 2 ? 1 : 2][FUSED ? 1 : 0][A ? 1 : 0];
  if (!cc.configured) {
    auto kern = w4c_kernel<GP, FUSED, A>;
    B2_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    // clusters of more than 8 CTAs are allowed on this part when asked for
    const bool big = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
                     cudaSuccess;
    (void)cudaGetLastError();
    for (int cs = 1; cs <= 16; ++cs) {
      cc.max_clusters[cs] = 0;
      if (cs > 8 && !big) continue;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(cs * 64));
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = C::kSmem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = (unsigned)cs;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess) cc.max_clusters[cs] = n;
      (void)cudaGetLastError();
    }
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&cc.occ, kern, kThreads, C::kSmem) !=
        cudaSuccess)
      cc.occ = 0;
    (void)cudaGetLastError();
    cc.configured = true;
  }
  *out = &cc;
  return B2_OK;
}

// Cluster plan for `tiles` output tiles of `upt` k-units: the cluster size with the smallest
// critical path. Returns the plain model's cost of the chosen size in unit-times (the scale of
// the stream-K comparison), or a negative value when no cluster size fits.
// Plain model (fused launches): tiles per cluster x (k-units per CTA + half a unit for the
// reduction when the tile is split). Placement model (`occ` > 0, CTAs of the kernel per SM, on
// `sms` SMs): clusters of cs CTAs fill at most max_clusters[cs] * cs / occ SMs (clusters of 11 to
// 14 leave ~20 of 148 SMs without work), a CTA on an SM holding more than three runs 10 % slower
// per extra CTA, and the reduction grows with the cluster (0.3 unit-times per CTA). Fitted on
// forced cluster sizes 1..16 of seven shapes (config 0, config 2 at M = 8, config 4 TP=8
// qkv/gate_up), where it picks the fastest size on every one: o_proj 9.4 -> 8.7 us and TP=8
// qkv 5.3 -> 4.4 us against the plain model.
double plan_clusters(const ClusterCaps& cc, int tiles, int upt, int want, int max_cs, int* cs_out,
                     int* nc_out, int share = 1, int occ = 0, int sms = 0) {
  double best = -1.0, best_plain = -1.0;
  for (int cs = 1; cs <= 16 && cs <= upt && cs <= max_cs; ++cs) {
    if (want > 0 && cs != want) continue;
    const int ncmax = cc.max_clusters[cs] / share;
    if (ncmax < 1) continue;
    const int nc = std::min(tiles, ncmax);
    const int per_cluster = (tiles + nc - 1) / nc;
    const int ku = (upt + cs - 1) / cs;
    const double plain = per_cluster * (ku + (cs > 1 ? 0.5 : 0.0));
    double cost = plain;
    if (occ > 0 && sms > 0) {
      const double usable = std::min((double)sms / share, (double)ncmax * cs / occ);
      const int per_sm = (int)std::ceil((double)nc * cs / usable - 1e-9);
      cost = per_cluster * (ku * (1.0 + 0.1 * std::max(0, per_sm - 3)) + (cs > 1 ? 0.3 * cs : 0.0));
    }
    if (best < 0.0 || cost < best - 1e-9) {
      best = cost;
      best_plain = plain;
      *cs_out = cs;
      *nc_out = nc;
    }
  }
  return best_plain;
}

// Split-K plan of one launch: stream-K over sk.ctas CTAs (cs == 0), or nc clusters of cs CTAs.
struct Plan {
  StreamK sk;
  int cs = 0, nc = 0;
  bool alias = false;  // cluster kernel with its reduction buffers on the drained ring
};

// `share`: the launch gets 1/share of the GPU (several emulated ranks in one launch).
template <int GP, bool FUSED>
int make_plan(const W4Args& a, int max_ctas, Plan* out, int share = 1) {
  // (every launch may take the cluster kernel: it needs no workspace partials or counters)
  using C = Cfg<GP>;
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  int dev = 0;
  B2_CUDA_TRY(cudaGetDevice(&dev));
  auto kern = w4_kernel<GP, FUSED>;
  KernelCache& kc = g_cache[dev][GP == 1 ? 0 : GP == 2 ? 1 : 2][FUSED ? 1 : 0];
  if (!kc.configured) {
    B2_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    B2_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&kc.occ, kern, kThreads, C::kSmem));
    if (kc.occ < 1) return fail(B2_ERR_UNSUPPORTED, "w4: kernel does not fit on an SM");
    kc.configured = true;
  }
  const int K = a.K, N = a.N;
  Plan pl;
  StreamK& sk = pl.sk;
  sk.upt = K / kUnitK;
  sk.tiles = (N + kTileN - 1) / kTileN;
  sk.total = (long long)sk.tiles * sk.upt;
  sk.ctas = std::min(streamk_ctas(sk.total, di.sm_count, kc.occ, 4), max_ctas);
  if (FUSED) {
    // Every CTA must be resident at once: a CTA waiting for peers must not hold back another
    // CTA of the same launch.
    sk.ctas = std::min(sk.ctas, std::max(1, di.sm_count * kc.occ / share));
  }

  // Split-K path. Stream-K needs the partial slots and tile counters of a workspace (at most
  // max_ctas CTAs); the cluster kernel reduces through distributed shared memory and needs none.
  // Fused launches take the cluster kernel when its exchange blocks fit the slot (N a whole
  // number of tiles) and the slot holds the 64-bit value+generation words (TP=2 down_proj shard:
  // 17.5 us, against 20.3 us for stream-K fused and 23.8 us for GEMM + NCCL). With fp32 slots
  // and flags stream-K fused was faster (24.8 against 29.9 us), so it is the choice there.
  const int path = tuning(B2_TUNE_W4_PATH);
  const bool cluster_ok = !FUSED || N % kTileN == 0;
  const bool cluster_default = !FUSED || a.ll;
  if (cluster_ok &&
      (path == 2 || (path == 0 && cluster_default))) {
    const ClusterCaps* cc = nullptr;
    rc = cluster_caps<GP, FUSED>(dev, &cc);
    if (rc) return rc;
    int cs = 0, nc = 0;
    const int max_cs = 16;
    // B2_TUNE_CTAS_PER_SM below the kernel's occupancy caps the resident clusters likewise
    const int cps = tuning(B2_TUNE_CTAS_PER_SM);
    const int occ_share = (cps > 0 && cps < kc.occ) ? share * kc.occ / cps : share;
    const int cocc = FUSED ? 0 : cc->occ;  // placement model for plain launches
    const double cost = plan_clusters(*cc, sk.tiles, sk.upt, tuning(B2_TUNE_W4_CLUSTER), max_cs,
                                      &cs, &nc, occ_share, cocc, di.sm_count);
    // stream-K: even units per CTA, plus the tail of the CTAs that finish a shared tile
    const long long per_cta = (sk.total + sk.ctas - 1) / sk.ctas;
    const double sk_cost = (double)per_cta + ((sk.total % sk.upt == 0 && sk.ctas <= sk.tiles &&
                                               sk.tiles % sk.ctas == 0) ? 0.0 : 4.0);
    if (plan_log()) {
      std::fprintf(stderr, "b2 w4 plan: M=%d K=%d N=%d tiles=%d upt=%d | stream-K ctas=%d cost=%.1f | "
                   "cluster cs=%d nc=%d cost=%.1f | max clusters:", a.M, K, N, sk.tiles, sk.upt,
                   sk.ctas, sk_cost, cs, nc, cost);
      for (int i = 1; i <= 16; ++i) std::fprintf(stderr, " %d", cc->max_clusters[i]);
      std::fprintf(stderr, "\n");
    }
    // (the RMSNorm epilogue keeps kMaxM row sums per CTA in the workspace: kWsMaxCtas CTAs)
    if (cost > 0.0 && (path == 2 || cost <= sk_cost) && (!a.norm || nc * cs <= kWsMaxCtas)) {
      pl.cs = cs;
      pl.nc = nc;
      // One tile per cluster and a long k-range per CTA: the variant with a fifth stage. Its
      // "drained" handshake costs a cluster round trip before the first push, which a long
      // k-range repays: gate_up (20 units per CTA, clusters of 2) 25.7 -> 24.5 us, while with
      // 3 to 11 units per CTA and clusters of 6 to 14 every shape lost 0.3 to 1 us.
      if constexpr (GP == 4 && !FUSED) {
        if (nc >= sk.tiles && (sk.upt + cs - 1) / cs >= 16 && !tuning(B2_TUNE_W4_NO_ALIAS)) {
          const ClusterCaps* ca = nullptr;
          rc = cluster_caps<GP, FUSED, true>(dev, &ca);
          if (rc) return rc;
          pl.alias = ca->max_clusters[cs] / occ_share >= nc;
        }
      }
    }
  }
  *out = pl;
  return B2_OK;
}

template <int GP, bool FUSED>
int launch(const W4Args& a0, const void* qw, const void* qz, const void* sc, const ArView* ar,
           const Plan& pl, bool early, cudaStream_t stream) {
  using C = Cfg<GP>;
  W4Args a = a0;
  a.sk = pl.sk;
  CUtensorMap m_qw, m_sc, m_qz, m_x;
  int rc = encode_maps<C::RG>(a, qw, qz, sc, &m_qw, &m_sc, &m_qz, &m_x);
  if (rc) return rc;
  const ArView view = ar ? *ar : ArView{};
  if (pl.cs > 0) {
    a.cl_size = pl.cs;
    a.cl_count = pl.nc;
    if constexpr (GP == 4 && !FUSED) {
      if (pl.alias)
        return launch_kernel_clusters(w4c_kernel<GP, FUSED, true>, pl.nc * pl.cs, pl.cs, kThreads,
                                      CfgC<GP, true>::kSmem, stream, early, m_qw, m_sc, m_qz, m_x,
                                      a, view);
    }
    return launch_kernel_clusters(w4c_kernel<GP, FUSED>, pl.nc * pl.cs, pl.cs, kThreads,
                                  CfgC<GP>::kSmem, stream, early, m_qw, m_sc, m_qz, m_x, a, view);
  }
  a.cl_size = a.cl_count = 0;
  // The stream-K kernel's RMSNorm epilogue has a grid-wide barrier: every CTA must be resident at
  // once. A cooperative launch gets that guarantee from the driver (or is refused), and it starts
  // only after the previous kernel: launched early, a grid's first CTAs take whatever slots the
  // previous grid leaves free and the rest may not fit beside them.
  const bool barrier = FUSED && a.norm == 1;
  return launch_kernel_ex(w4_kernel<GP, FUSED>, pl.sk.ctas, kThreads, C::kSmem, stream,
                          early && !barrier, barrier && !tuning(B2_TUNE_NORM_NO_COOP), m_qw, m_sc,
                          m_qz, m_x, a, view);
}

// The plan of a launch for the group size in args.G.
template <bool FUSED>
int plan_for(const W4Args& args, int max_ctas, Plan* pl, int share = 1) {
  switch (args.G) {
    case 32: return make_plan<1, FUSED>(args, max_ctas, pl, share);
    case 64: return make_plan<2, FUSED>(args, max_ctas, pl, share);
    default: return make_plan<4, FUSED>(args, max_ctas, pl, share);
  }
}

template <bool FUSED>
int launch_plan(const W4Args& args, const void* qw, const void* qz, const void* sc,
                const ArView* ar, const Plan& pl, bool early, cudaStream_t stream) {
  switch (args.G) {
    case 32: return launch<1, FUSED>(args, qw, qz, sc, ar, pl, early, stream);
    case 64: return launch<2, FUSED>(args, qw, qz, sc, ar, pl, early, stream);
    default: return launch<4, FUSED>(args, qw, qz, sc, ar, pl, early, stream);
  }
}

int validate(const void* a, const void* qw, const void* qz, const void* sc, const void* y, int M,
             int K, int N, int G);

int validate(const void* a, const void* qw, const void* qz, const void* sc, const void* y, int M,
             int K, int N, int G, const void* ws, size_t ws_bytes) {
  const int rc = validate(a, qw, qz, sc, y, M, K, N, G);
  if (rc) return rc;
  if (!ws || ws_bytes < ws_total_bytes())
    return fail(B2_ERR_WORKSPACE, "w4: workspace of %zu B, need %zu B", ws_bytes, ws_total_bytes());
  return B2_OK;
}

// Operand checks shared by every W4 entry point.
int validate(const void* a, const void* qw, const void* qz, const void* sc, const void* y, int M,
             int K, int N, int G) {
  if (!a || !qw || !qz || !sc || !y) return fail(B2_ERR_INVALID_ARG, "w4: null pointer");
  if (M < 1 || M > kMaxM) return fail(B2_ERR_INVALID_ARG, "w4: M=%d outside 1..8", M);
  if (K < kUnitK || K % kUnitK != 0)
    return fail(B2_ERR_INVALID_ARG, "w4: K=%d must be a positive multiple of 128", K);
  if (N < 32 || N % 32 != 0)
    return fail(B2_ERR_INVALID_ARG, "w4: N=%d must be a positive multiple of 32", N);
  if (!(G == 32 || G == 64 || (G >= 128 && G % 128 == 0)) || K % G != 0)
    return fail(B2_ERR_INVALID_ARG,
                "w4: group size %d unsupported (32, 64 or a multiple of 128 dividing K=%d)", G, K);
  if (!aligned16(a) || !aligned16(qw) || !aligned16(qz) || !aligned16(sc))
    return fail(B2_ERR_INVALID_ARG, "w4: a, qw, qz and sc must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(y) & 7u) != 0)
    return fail(B2_ERR_INVALID_ARG, "w4: y must be 8-byte aligned");
  if ((N + kTileN - 1) / kTileN > kWsMaxTiles) return fail(B2_ERR_INVALID_ARG, "w4: N=%d too large", N);
  return B2_OK;
}

W4Args make_args(const void* a, void* y, int M, int K, int N, int G, void* ws) {
  W4Args r;
  r.x = static_cast<const __half*>(a);
  r.y = static_cast<__half*>(y);
  r.M = M;
  r.K = K;
  r.N = N;
  r.G = G;
  char* wsb = static_cast<char*>(ws);
  r.status = reinterpret_cast<int*>(wsb);
  r.counters = reinterpret_cast<int*>(wsb + ws_counters_offset());
  r.partials = reinterpret_cast<float*>(wsb + ws_partials_offset());
  r.cl_size = r.cl_count = 0;
  r.ll = 0;
  r.two_shot = 0;
  r.norm = 0;
  r.eps = 0.f;
  r.nw = nullptr;
  r.res = nullptr;
  r.npart = nullptr;
  r.norm_v16 = 0;
  r.pk = nullptr;
  r.pk_unit = 0;
  return r;
}

// `early`: programmatic dependent launch.
template <bool FUSED>
int dispatch(const W4Args& args, const void* qw, const void* qz, const void* sc, const ArView* ar,
             cudaStream_t stream, bool early) {
  Plan pl;
  const int rc = plan_for<FUSED>(args, kWsMaxCtas, &pl);
  if (rc) return rc;
  return launch_plan<FUSED>(args, qw, qz, sc, ar, pl, early, stream);
}

// ------------------------------------------------------------------------------------------------
// Scratch for b2_w4_gemm_noalloc: a fixed array in device memory, created when the library is
// loaded on a device and kept until the process exits. Layout: [status 256 B][arrival counters of
// up to kNoAllocMaxTiles output tiles][two fp32 partial slots for each of up to kNoAllocMaxCtas
// CTAs]. 2,113,792 bytes per device.
// ------------------------------------------------------------------------------------------------
constexpr int kNoAllocMaxTiles = 4096;  // N <= 4096 * 128 = 524288 output columns
constexpr int kNoAllocMaxCtas = 256;
constexpr size_t kNoAllocCountersOff = 256;
constexpr size_t kNoAllocPartialsOff = kNoAllocCountersOff + (size_t)kNoAllocMaxTiles * 4;
constexpr size_t kNoAllocBytes =
    kNoAllocPartialsOff + (size_t)kNoAllocMaxCtas * 2 * kSlotFloats * sizeof(float);
static_assert(kNoAllocPartialsOff % 256 == 0, "partial slots stay 256-byte aligned");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// Device address of g_noalloc_scratch. In host code the name g_noalloc_scratch is only a
// host-side stand-in for the symbol; a kernel must be given the address cudaGetSymbolAddress
// returns in the calling thread's current context (the device's primary context for runtime-API
// callers). The address is looked up at the first call in a context and cached per device with
// that context's unique id, so a call from another context, or after cudaDeviceReset has replaced
// the primary context (which reloads the module and the array), looks it up again. One lock per
// device: threads that drive different GPUs do not wait for each other.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

template <typename Fn>
Fn driver_fn(const char* name, int version) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion(name, &p, version, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

struct NoAllocEntry {
  std::mutex mu;
  unsigned long long ctx_id = 0;
  unsigned char* ptr = nullptr;
};
NoAllocEntry g_noalloc[64];

int noalloc_scratch(cudaStream_t stream, unsigned char** out) {
  static const CtxGetCurrentFn get_ctx = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent", 12000);
  static const CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId", 12000);
  int dev = 0;
  B2_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(B2_ERR_UNSUPPORTED, "w4_noalloc: device ordinal %d", dev);
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_ctx || !get_id || get_ctx(&ctx) != CUDA_SUCCESS)
    return fail(B2_ERR_CUDA, "w4_noalloc: cannot query the current CUDA context");
  if (!ctx) {  // no context current on this thread yet: make the device's primary context current
    B2_CUDA_TRY(cudaSetDevice(dev));
    if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx)
      return fail(B2_ERR_CUDA, "w4_noalloc: no CUDA context on device %d", dev);
  }
  if (get_id(ctx, &id) != CUDA_SUCCESS)
    return fail(B2_ERR_CUDA, "w4_noalloc: cannot identify the current CUDA context");
  NoAllocEntry& e = g_noalloc[dev];
  std::lock_guard<std::mutex> lk(e.mu);
  if (!e.ptr || e.ctx_id != id) {
    // The set-up: not inside a stream capture, where looking up a symbol may load the module.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    B2_CUDA_TRY(cudaStreamIsCapturing(stream, &cs));
    if (cs != cudaStreamCaptureStatusNone)
      return fail(B2_ERR_STATE,
                  "w4_noalloc: the first call in a CUDA context looks up the scratch array and "
                  "must come before any stream capture (make one eager call first)");
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || !p)
      return fail(B2_ERR_CUDA, "w4_noalloc: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(err));
    e.ptr = static_cast<unsigned char*>(p);
    e.ctx_id = id;
  }
  *out = e.ptr;
  return B2_OK;
}

// ------------------------------------------------------------------------------------------------
// Weight repack (load time). Unit (tile, ku) becomes unit_bytes contiguous bytes at
// out + (tile * K / 128 + ku) * unit_bytes: the stage image the kernels' consumers read.
//   [0, 8192)            qw: block w (32 columns), word row r (k = 8 (16 ku + r) ..), 16-byte
//                        chunk c (columns 4c..4c+3 of the block) at w * 2048 + r * 128 +
//                        ((c ^ (r & 7)) << 4): the 128-byte swizzle the tensor copy applies
//   [8192, +RG * 256)    scales of the unit's RG group rows, 128 fp16 each
//   [.., +RG * 64)       zeros of those rows, 16 packed words each
// with RG = 128 / G group rows per unit (1 for G >= 128: the unit's own group row). Columns past
// N hold zeros (a zero scale: they add nothing). A pure permutation of the bytes the kernels read
// from the original layout, so the products are bit-identical.
// ------------------------------------------------------------------------------------------------
int packed_unit_bytes(int G) {
  const int RG = G >= kUnitK ? 1 : kUnitK / G;
  return kQwStage + RG * (kTileN * 2 + (kTileN / 8) * 4);
}

__global__ void __launch_bounds__(256) w4_repack_kernel(const uint32_t* __restrict__ qw,
                                                        const uint32_t* __restrict__ qz,
                                                        const __half* __restrict__ sc,
                                                        uint8_t* __restrict__ out, int K, int N,
                                                        int G, int unit_bytes) {
  const int ku = blockIdx.x, tile = blockIdx.y;
  const int RG = G >= kUnitK ? 1 : kUnitK / G;
  const int grow0 = (ku * kUnitK) / G;
  const int sc_chunks = RG * kTileN * 2 / 16;
  uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)tile * (size_t)(K / kUnitK) + ku) *
                                                  (size_t)unit_bytes);
  for (int q = threadIdx.x; q < unit_bytes / 16; q += blockDim.x) {
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (q < kQwStage / 16) {
      const int blk = q >> 7, r = (q >> 3) & 15, c = (q & 7) ^ (r & 7);
      const int col = tile * kTileN + blk * 32 + c * 4;
      const size_t row = (size_t)ku * 16 + r;
      if (col < N)  // N % 32 == 0: a chunk is wholly inside or wholly past N
        for (int i = 0; i < 4; ++i) w[i] = qw[row * N + col + i];
    } else if (q < kQwStage / 16 + sc_chunks) {
      const int i16 = q - kQwStage / 16, g = i16 >> 4, col = tile * kTileN + (i16 & 15) * 8;
      if (col < N) {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(sc + (size_t)(grow0 + g) * N + col);
        for (int i = 0; i < 4; ++i) w[i] = src[i];
      }
    } else {
      const int i16 = q - kQwStage / 16 - sc_chunks, g = i16 >> 2;
      const int wcol = tile * (kTileN / 8) + (i16 & 3) * 4;
      if (wcol < N / 8)
        for (int i = 0; i < 4; ++i) w[i] = qz[(size_t)(grow0 + g) * (N / 8) + wcol + i];
    }
    dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace

int launch_w4(const void* a, const void* qw, const void* qz, const void* sc, void* y, int M, int K,
              int N, int G, void* ws, size_t ws_bytes, cudaStream_t stream) {
  int rc = validate(a, qw, qz, sc, y, M, K, N, G, ws, ws_bytes);
  if (rc) return rc;
  return dispatch<false>(make_args(a, y, M, K, N, G, ws), qw, qz, sc, nullptr, stream,
                         /*early=*/true);
}

size_t w4_packed_bytes(int K, int N, int G) {
  if (K < kUnitK || K % kUnitK != 0 || N < 32 || N % 32 != 0 ||
      !(G == 32 || G == 64 || (G >= kUnitK && G % kUnitK == 0)) || K % G != 0)
    return 0;
  return (size_t)((N + kTileN - 1) / kTileN) * (size_t)(K / kUnitK) * (size_t)packed_unit_bytes(G);
}

int w4_repack(const void* qw, const void* qz, const void* sc, int K, int N, int G, void* out,
              size_t out_bytes, cudaStream_t stream) {
  int rc = validate(qw, qw, qz, sc, out, 1, K, N, G);
  if (rc) return rc;
  if (!aligned16(out)) return fail(B2_ERR_INVALID_ARG, "w4_repack: out must be 16-byte aligned");
  const size_t need = w4_packed_bytes(K, N, G);
  if (out_bytes < need)
    return fail(B2_ERR_INVALID_ARG, "w4_repack: out holds %zu bytes, needs %zu", out_bytes, need);
  const dim3 grid((unsigned)(K / kUnitK), (unsigned)((N + kTileN - 1) / kTileN));
  w4_repack_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint32_t*>(qw),
                                             static_cast<const uint32_t*>(qz),
                                             static_cast<const __half*>(sc),
                                             static_cast<uint8_t*>(out), K, N, G,
                                             packed_unit_bytes(G));
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

int launch_w4_packed(const void* a, const void* packed, void* y, int M, int K, int N, int G,
                     void* ws, size_t ws_bytes, cudaStream_t stream) {
  int rc = validate(a, packed, packed, packed, y, M, K, N, G, ws, ws_bytes);
  if (rc) return rc;
  W4Args args = make_args(a, y, M, K, N, G, ws);
  args.pk = static_cast<const uint8_t*>(packed);
  args.pk_unit = packed_unit_bytes(G);
  return dispatch<false>(args, nullptr, nullptr, nullptr, nullptr, stream, /*early=*/true);
}

int launch_w4_noalloc(const void* a, const void* qw, const void* qz, const void* sc, void* y, int M,
                      int K, int N, int G, cudaStream_t stream) {
  const int tiles = (N + kTileN - 1) / kTileN;
  if (N > 0 && tiles > kNoAllocMaxTiles)
    return fail(B2_ERR_INVALID_ARG,
                "w4_noalloc: N=%d needs %d output tiles; the fixed scratch holds at most %d "
                "(N <= %d)", N, tiles, kNoAllocMaxTiles, kNoAllocMaxTiles * kTileN);
  unsigned char* scratch = nullptr;
  int rc = validate(a, qw, qz, sc, y, M, K, N, G);
  if (rc) return rc;
  rc = noalloc_scratch(stream, &scratch);
  if (rc) return rc;
  W4Args args = make_args(a, y, M, K, N, G, scratch);
  args.status = reinterpret_cast<int*>(scratch);
  args.counters = reinterpret_cast<int*>(scratch + kNoAllocCountersOff);
  args.partials = reinterpret_cast<float*>(scratch + kNoAllocPartialsOff);
  Plan pl;
  rc = plan_for<false>(args, kNoAllocMaxCtas, &pl);
  if (rc) return rc;
  if (pl.cs > 0)  // the cluster kernel uses none of the scratch: launched as b2_w4_gemm launches it
    return launch_plan<false>(args, qw, qz, sc, nullptr, pl, /*early=*/true, stream);
  // Stream-K: clear the status word and the counters this call uses first. The array keeps
  // whatever the last call left, and a call that gave up on a wait may have left counters behind.
  B2_CUDA_TRY(cudaMemsetAsync(scratch, 0, kNoAllocCountersOff + (size_t)tiles * 4, stream));
  return launch_plan<false>(args, qw, qz, sc, nullptr, pl, /*early=*/false, stream);
}

int noalloc_scratch_info(void** ptr, size_t* bytes) {
  unsigned char* p = nullptr;
  const int rc = noalloc_scratch(nullptr, &p);
  if (rc) return rc;
  *ptr = p;
  *bytes = kNoAllocBytes;
  return B2_OK;
}

// Checks and kernel arguments of one rank's fused launch. `residual` and `nw` non-null: the
// residual add + RMSNorm epilogue (see norm_rstd).
int fused_args(b2_nvar* h, const void* a, const void* qw, const void* qz, const void* sc, void* y,
               int M, int K, int N, int G, void* ws, size_t ws_bytes, void* residual,
               const void* nw, float eps, W4Args* out, ArView* view) {
  int rc = validate(a, qw, qz, sc, y, M, K, N, G, ws, ws_bytes);
  if (rc) return rc;
  const bool norm = residual || nw;
  if (norm) {
    if (!residual || !nw) return fail(B2_ERR_INVALID_ARG, "w4_allreduce_rmsnorm: null pointer");
    if ((reinterpret_cast<uintptr_t>(residual) & 7u) != 0 ||
        (reinterpret_cast<uintptr_t>(nw) & 7u) != 0)
      return fail(B2_ERR_INVALID_ARG,
                  "w4_allreduce_rmsnorm: residual and norm_weight must be 8-byte aligned");
    const uintptr_t yb = reinterpret_cast<uintptr_t>(y), rb = reinterpret_cast<uintptr_t>(residual);
    const uintptr_t wb = reinterpret_cast<uintptr_t>(nw);
    const uintptr_t mn = (uintptr_t)M * N * 2, nb = (uintptr_t)N * 2;
    if ((yb < rb + mn && rb < yb + mn) || (yb < wb + nb && wb < yb + mn) ||
        (rb < wb + nb && wb < rb + mn))
      return fail(B2_ERR_INVALID_ARG,
                  "w4_allreduce_rmsnorm: y, residual and norm_weight must not overlap");
    if (!(eps >= 0.f) || eps > 1.f)
      return fail(B2_ERR_INVALID_ARG, "w4_allreduce_rmsnorm: eps %g outside [0, 1]", (double)eps);
  }
  int tiles_cap = 0;
  rc = nvar_view(h, view, (size_t)M * N * sizeof(float), &tiles_cap);
  if (rc) return rc;
  if ((N + kTileN - 1) / kTileN > tiles_cap)
    return fail(B2_ERR_INVALID_ARG, "w4_allreduce: N=%d has more tiles than flags", N);
  W4Args args = make_args(a, y, M, K, N, G, ws);
  // the low-latency exchange needs 8 bytes per output element in each slot (the handle allocates
  // 4x the payload it was created for, so it always has them); B2_TUNE_AR_FLAGS selects the fp32
  // values + per-tile flags form instead
  args.ll = (view->slot_bytes >= (unsigned long long)M * N * 8 && tuning(B2_TUNE_AR_FLAGS) == 0)
                ? 1 : 0;
  // Two-shot moves 2 (P-1)/P of the payload per rank over NVLink instead of P-1 times it, for one
  // more hop of latency. Measured at 4 ranks on NVLink, one-shot is faster (config 4 step 3,298 µs
  // against 3,448; down_proj shard 16.5 against 17.9 µs), so two-shot is the choice from 8 ranks
  // up, where one-shot would move 7x the payload per rank (B2_TUNE_AR_TWO_SHOT: 1 on, 2 off).
  const int ts = tuning(B2_TUNE_AR_TWO_SHOT);
  args.two_shot = args.ll && (ts == 1 || (ts == 0 && view->world >= 8)) ? 1 : 0;
  if (norm) {
    args.norm = 1;
    args.eps = eps;
    args.res = static_cast<__half*>(residual);
    args.nw = static_cast<const __half*>(nw);
    args.npart = reinterpret_cast<float*>(static_cast<char*>(ws) + ws_norm_offset());
    args.norm_v16 = aligned16(y) && aligned16(residual) && aligned16(nw) ? 1 : 0;
  }
  *out = args;
  return B2_OK;
}

// The finishing launch of the split RMSNorm (norm_finish_kernel) after a fused launch of
// `nparts` CTAs. 128 threads per CTA, one vector per thread.
int launch_norm_finish(const W4Args& a, int nparts, cudaStream_t stream) {
  const int kH = a.norm_v16 ? 8 : 4;
  const int per = a.M * a.N / kH;
  const int grid = std::max(1, std::min((per + 127) / 128, kWsMaxCtas));
  if (a.norm_v16)
    return launch_kernel(norm_finish_kernel<uint4>, grid, 128, 0, stream, /*early=*/true, a,
                         nparts);
  return launch_kernel(norm_finish_kernel<uint2>, grid, 128, 0, stream, /*early=*/true, a, nparts);
}

// One rank's fused launch. With the RMSNorm the default is the split form (p.norm = 2): the
// fused launch stores the all-reduced rows and its CTAs' row sums, and norm_finish_kernel follows
// on the stream; B2_TUNE_NORM_IN_LAUNCH keeps all of it in the one launch (p.norm = 1).
// Early launch is safe here too: the generation is read after griddepcontrol.wait, and a
// dependent grid starts only once every CTA of this one is resident, so none of the CTAs that
// wait for peers in the second phase can be held back. (The cluster kernel's in-launch RMSNorm
// needs no co-residency either: its last cluster finishes the rows. The stream-K kernel's, with a
// grid-wide barrier, is launched without early start; see launch.)
int launch_fused(W4Args& args, const void* qw, const void* qz, const void* sc, const ArView& v,
                 cudaStream_t stream) {
  if (args.norm && tuning(B2_TUNE_NORM_IN_LAUNCH) == 0) args.norm = 2;
  if (args.norm != 2) return dispatch<true>(args, qw, qz, sc, &v, stream, /*early=*/true);
  Plan pl;
  int rc = plan_for<true>(args, kWsMaxCtas, &pl);
  if (rc) return rc;
  rc = launch_plan<true>(args, qw, qz, sc, &v, pl, /*early=*/true, stream);
  if (rc) return rc;
  return launch_norm_finish(args, pl.cs > 0 ? pl.cs * pl.nc : pl.sk.ctas, stream);
}

int launch_w4_allreduce(b2_nvar* h, const void* a, const void* qw, const void* qz, const void* sc,
                        void* y, int M, int K, int N, int G, void* ws, size_t ws_bytes,
                        cudaStream_t stream, void* residual = nullptr, const void* nw = nullptr,
                        float eps = 0.f) {
  W4Args args;
  ArView v;
  const int rc = fused_args(h, a, qw, qz, sc, y, M, K, N, G, ws, ws_bytes, residual, nw, eps,
                            &args, &v);
  if (rc) return rc;
  return launch_fused(args, qw, qz, sc, v, stream);
}

// The fused launch on weights repacked by w4_repack (`packed` in place of qw, qz, sc).
int launch_w4_allreduce_packed(b2_nvar* h, const void* a, const void* packed, void* y, int M,
                               int K, int N, int G, void* ws, size_t ws_bytes,
                               cudaStream_t stream, void* residual, const void* nw, float eps) {
  W4Args args;
  ArView v;
  const int rc = fused_args(h, a, packed, packed, packed, y, M, K, N, G, ws, ws_bytes, residual,
                            nw, eps, &args, &v);
  if (rc) return rc;
  args.pk = static_cast<const uint8_t*>(packed);
  args.pk_unit = packed_unit_bytes(G);
  return launch_fused(args, nullptr, nullptr, nullptr, v, stream);
}

// `R` ranks of one group in one cooperative launch on this GPU (grid.y = rank). Every rank gets
// 1/R of the GPU in the plan, and the cooperative attribute makes the launch fail rather than
// start with CTAs that cannot all be resident.
template <int GP>
int launch_emu(const W4Args* args, const ArView* views, const void* const* qw,
               const void* const* qz, const void* const* sc, int R, cudaStream_t stream) {
  using C = Cfg<GP>;
  Plan pl;
  int rc = make_plan<GP, true>(args[0], kWsMaxCtas, &pl, R);
  if (rc) return rc;
  W4Emu E;
  memset(&E, 0, sizeof(E));
  for (int r = 0; r < R; ++r) {
    W4Args a = args[r];
    a.sk = pl.sk;
    a.cl_size = pl.cs;
    a.cl_count = pl.nc;
    rc = encode_maps<C::RG>(a, qw[r], qz[r], sc[r], &E.qw[r], &E.sc[r], &E.qz[r], &E.x[r]);
    if (rc) return rc;
    E.p[r] = a;
    E.ar[r] = views[r];
  }
  auto kern = pl.cs > 0 ? w4c_kernel_emu<GP> : w4_kernel_emu<GP>;
  const int smem = pl.cs > 0 ? CfgC<GP>::kSmem : C::kSmem;
  B2_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  if (pl.cs > 8)
    B2_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(pl.cs > 0 ? pl.nc * pl.cs : pl.sk.ctas), (unsigned)R);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)pl.cs;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pl.cs > 0 ? 2 : 1;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, E));
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

int launch_w4_allreduce_emulated(b2_nvar* const* handles, int R, const void* const* a,
                                 const void* const* qw, const void* const* qz,
                                 const void* const* sc, void* const* residual,
                                 const void* const* nw, float eps, void* const* y, int M, int K,
                                 int N, int G, void* const* ws, size_t ws_bytes,
                                 cudaStream_t stream) {
  if (R < 1 || R > kEmuMaxRanks)
    return fail(B2_ERR_INVALID_ARG, "w4_allreduce_emulated: %d ranks (1..%d)", R, kEmuMaxRanks);
  if (!handles || !a || !qw || !qz || !sc || !y || !ws)
    return fail(B2_ERR_INVALID_ARG, "w4_allreduce_emulated: null array");
  if ((residual == nullptr) != (nw == nullptr))
    return fail(B2_ERR_INVALID_ARG, "w4_allreduce_emulated: residual and norm_weight go together");
  W4Args args[kEmuMaxRanks];
  ArView views[kEmuMaxRanks];
  for (int r = 0; r < R; ++r) {
    const int rc = fused_args(handles[r], a[r], qw[r], qz[r], sc[r], y[r], M, K, N, G, ws[r],
                              ws_bytes, residual ? residual[r] : nullptr, nw ? nw[r] : nullptr,
                              eps, &args[r], &views[r]);
    if (rc) return rc;
    if (views[r].rank != r || views[r].world != R)
      return fail(B2_ERR_STATE, "w4_allreduce_emulated: handle %d is rank %d of %d", r,
                  views[r].rank, views[r].world);
    if (args[r].ll != args[0].ll)
      return fail(B2_ERR_STATE, "w4_allreduce_emulated: the handles' slots differ in size");
  }
  switch (G) {
    case 32: return launch_emu<1>(args, views, qw, qz, sc, R, stream);
    case 64: return launch_emu<2>(args, views, qw, qz, sc, R, stream);
    default: return launch_emu<4>(args, views, qw, qz, sc, R, stream);
  }
}

}  // namespace b2

extern "C" int b2_w4_gemm(const void* a, const void* qw, const void* qz, const void* sc, void* y,
                          int M, int K, int N, int group_size, void* ws, size_t ws_bytes,
                          void* stream) {
  return b2::launch_w4(a, qw, qz, sc, y, M, K, N, group_size, ws, ws_bytes,
                       static_cast<cudaStream_t>(stream));
}

extern "C" size_t b2_w4_packed_bytes(int K, int N, int group_size) {
  return b2::w4_packed_bytes(K, N, group_size);
}

extern "C" int b2_w4_repack(const void* qw, const void* qz, const void* sc, int K, int N,
                            int group_size, void* out, size_t out_bytes, void* stream) {
  return b2::w4_repack(qw, qz, sc, K, N, group_size, out, out_bytes,
                       static_cast<cudaStream_t>(stream));
}

extern "C" int b2_w4_gemm_packed(const void* a, const void* packed, void* y, int M, int K, int N,
                                 int group_size, void* ws, size_t ws_bytes, void* stream) {
  return b2::launch_w4_packed(a, packed, y, M, K, N, group_size, ws, ws_bytes,
                              static_cast<cudaStream_t>(stream));
}

extern "C" int b2_w4_gemm_allreduce(b2_nvar* ar, const void* a, const void* qw, const void* qz,
                                    const void* sc, void* y, int M, int K, int N, int group_size,
                                    void* ws, size_t ws_bytes, void* stream) {
  if (!ar) return b2::fail(B2_ERR_STATE, "w4_allreduce: null all-reduce handle");
  return b2::launch_w4_allreduce(ar, a, qw, qz, sc, y, M, K, N, group_size, ws, ws_bytes,
                                 static_cast<cudaStream_t>(stream));
}

extern "C" int b2_w4_gemm_allreduce_rmsnorm(b2_nvar* ar, const void* a, const void* qw,
                                            const void* qz, const void* sc, void* residual,
                                            const void* norm_weight, float eps, void* y, int M,
                                            int K, int N, int group_size, void* ws,
                                            size_t ws_bytes, void* stream) {
  if (!ar) return b2::fail(B2_ERR_STATE, "w4_allreduce_rmsnorm: null all-reduce handle");
  if (!residual || !norm_weight)
    return b2::fail(B2_ERR_INVALID_ARG, "w4_allreduce_rmsnorm: null residual or norm_weight");
  return b2::launch_w4_allreduce(ar, a, qw, qz, sc, y, M, K, N, group_size, ws, ws_bytes,
                                 static_cast<cudaStream_t>(stream), residual, norm_weight, eps);
}

extern "C" int b2_w4_gemm_allreduce_packed(b2_nvar* ar, const void* a, const void* packed,
                                           void* y, int M, int K, int N, int group_size,
                                           void* ws, size_t ws_bytes, void* stream) {
  if (!ar) return b2::fail(B2_ERR_STATE, "w4_allreduce: null all-reduce handle");
  return b2::launch_w4_allreduce_packed(ar, a, packed, y, M, K, N, group_size, ws, ws_bytes,
                                        static_cast<cudaStream_t>(stream), nullptr, nullptr, 0.f);
}

extern "C" int b2_w4_gemm_allreduce_rmsnorm_packed(b2_nvar* ar, const void* a, const void* packed,
                                                   void* residual, const void* norm_weight,
                                                   float eps, void* y, int M, int K, int N,
                                                   int group_size, void* ws, size_t ws_bytes,
                                                   void* stream) {
  if (!ar) return b2::fail(B2_ERR_STATE, "w4_allreduce_rmsnorm: null all-reduce handle");
  if (!residual || !norm_weight)
    return b2::fail(B2_ERR_INVALID_ARG, "w4_allreduce_rmsnorm: null residual or norm_weight");
  return b2::launch_w4_allreduce_packed(ar, a, packed, y, M, K, N, group_size, ws, ws_bytes,
                                        static_cast<cudaStream_t>(stream), residual, norm_weight,
                                        eps);
}

// Ranks of one group emulated on one GPU in one cooperative launch; see include/b2_skinny.h.
extern "C" int b2_w4_gemm_allreduce_emulated(b2_nvar* const* handles, int ranks,
                                             const void* const* a, const void* const* qw,
                                             const void* const* qz, const void* const* sc,
                                             void* const* residual, const void* const* norm_weight,
                                             float eps, void* const* y, int M, int K, int N,
                                             int group_size, void* const* ws, size_t ws_bytes,
                                             void* stream) {
  return b2::launch_w4_allreduce_emulated(handles, ranks, a, qw, qz, sc, residual, norm_weight,
                                          eps, y, M, K, N, group_size, ws, ws_bytes,
                                          static_cast<cudaStream_t>(stream));
}

// The W4A16 GEMM without a caller-supplied workspace; see include/b2_skinny.h.
extern "C" int b2_w4_gemm_noalloc(const void* a, const void* qw, const void* qz, const void* sc,
                                  void* y, int M, int K, int N, int group_size, void* stream) {
  return b2::launch_w4_noalloc(a, qw, qz, sc, y, M, K, N, group_size,
                               static_cast<cudaStream_t>(stream));
}

// Address and size of the no-alloc scratch array on the current device; see include/b2_skinny.h.
extern "C" int b2_w4_noalloc_scratch(void** device_ptr, size_t* bytes) {
  if (!device_ptr || !bytes) return b2::fail(B2_ERR_INVALID_ARG, "w4_noalloc_scratch: null output");
  return b2::noalloc_scratch_info(device_ptr, bytes);
}

// The split-K plan of a W4 launch; see include/b2_skinny.h.
extern "C" int b2_w4_plan(int M, int K, int N, int group_size, int fused, int* path, int* cluster,
                          int* ctas) {
  if (!path || !cluster || !ctas) return b2::fail(B2_ERR_INVALID_ARG, "w4_plan: null output");
  const int fake = 256;  // validation needs aligned non-null pointers; nothing is dereferenced
  const void* p = reinterpret_cast<const void*>((uintptr_t)fake);
  int rc = b2::validate(p, p, p, p, p, M, K, N, group_size);
  if (rc) return rc;
  b2::W4Args a = b2::make_args(p, const_cast<void*>(p), M, K, N, group_size, nullptr);
  a.ll = fused ? 1 : 0;
  b2::Plan pl;
  rc = fused ? b2::plan_for<true>(a, b2::kWsMaxCtas, &pl)
             : b2::plan_for<false>(a, b2::kWsMaxCtas, &pl);
  if (rc) return rc;
  *path = pl.cs > 0 ? 2 : 1;
  *cluster = pl.cs;
  *ctas = pl.cs > 0 ? pl.cs * pl.nc : pl.sk.ctas;
  return B2_OK;
}

#ifdef B2_TRACE
// Copy the trace of the last traced launch to the host: units[5][4096] and ctas[4096][12] (64-bit
// nanoseconds; SM ids in ctas[i][2]); entries not written are 0 or hold an earlier launch's.
extern "C" int b2_trace_read(unsigned long long* units, unsigned long long* ctas) {
  if (cudaMemcpyFromSymbol(units, b2::g_trace_units, sizeof(b2::g_trace_units)) != cudaSuccess ||
      cudaMemcpyFromSymbol(ctas, b2::g_trace_ctas, sizeof(b2::g_trace_ctas)) != cudaSuccess)
    return B2_ERR_CUDA;
  return B2_OK;
}
extern "C" int b2_trace_clear() {
  static unsigned long long zero[4096 * 12];
  static_assert(sizeof(zero) >= sizeof(b2::g_trace_units) && sizeof(zero) >= sizeof(b2::g_trace_ctas),
                "one zero buffer clears both");
  if (cudaMemcpyToSymbol(b2::g_trace_units, zero, sizeof(b2::g_trace_units)) != cudaSuccess ||
      cudaMemcpyToSymbol(b2::g_trace_ctas, zero, sizeof(b2::g_trace_ctas)) != cudaSuccess)
    return B2_ERR_CUDA;
  return B2_OK;
}
#endif
