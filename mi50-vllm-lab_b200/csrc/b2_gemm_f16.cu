// fp16 skinny GEMM for sm_100a:  y[M,N] = x[M,K] @ w[N,K]^T,  1 <= M <= 8, fp32 accumulation.
//
// Replaces skinny_gemm / skinny_pipe_kernel of kernels/skinny.cu:224-328 (same op contract:
// row-major x and w with K contiguous, fp16 out). The weight matrix is streamed from HBM once:
//   - a producer warp moves 128-row x 64-k tiles (16 KB) of w into a ring of shared-memory
//     stages with TMA (cp.async.bulk.tensor, 128-byte swizzle, L2 evict-first);
//   - four consumer warps feed the tiles to mma.sync m16n8k16 (fp16 in, fp32 accumulate) with
//     the weights as the 16-row A operand and the <= 8 activation rows as the 8-column B
//     operand, so every weight is used for all M rows from one shared-memory read;
//   - the work (tiles x k-units) is split evenly over a persistent grid (stream-K); tiles that
//     straddle CTAs are summed by the last CTA to finish, in CTA order (deterministic), which
//     replaces the split-K reduce kernel of kernels/skinny.cu:181-188.
// Lane-to-k mapping: lane (g = lane/4, t = lane%4) reads the 16-byte chunks 2t and 2t+1 of a
// 128-byte weight row and the matching 16 bytes of x. A dot product may visit k in any order as
// long as A and B agree, so each chunk feeds two m16n8k16 steps directly (no ldmatrix), and the
// chunk pattern hits all 32 banks once per 8 lanes under the swizzle.
#include <cuda_fp16.h>

#include "b2_device.cuh"
#include "b2_internal.h"

namespace b2 {
namespace {

constexpr int kWarps = 4;                                // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;              // + one producer warp
constexpr int kUnitK = 64;                               // k per unit = one 128-byte row
constexpr int kStageBytes = kTileN * kUnitK * 2;         // 16 KB
constexpr int kStages = 6;
constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 2 * kStages * 8 + 16;
static_assert(kStageBytes % 1024 == 0, "swizzled TMA boxes start on 1024-byte boundaries");

struct F16Args {
  const __half* x;
  __half* y;
  int M, K, N;
  StreamK sk;
  float* partials;
  int* counters;
  int* status;
};

__device__ __forceinline__ void store_out(const F16Args& p, int tile, int warp, int g, int t,
                                          const float (&v)[2][4]) {
#pragma unroll
  for (int T = 0; T < 2; ++T)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = 2 * t + (i & 1);
      const int n = tile * kTileN + warp * 32 + T * 16 + g + (i >> 1) * 8;
      if (m < p.M && n < p.N) p.y[(size_t)m * p.N + n] = __float2half_rn(v[T][i]);
    }
}

__global__ void __launch_bounds__(kThreads) gemm_f16_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                            const F16Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  volatile int* s_abort = reinterpret_cast<volatile int*>(empty + kStages);
  volatile int* s_flag = s_abort + 1;

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
  // Programmatic dependent launch: until the previous grid on the stream has completed, its
  // stores may not be visible, so the producer only warms L2 with the first stages' weights
  // before it waits; every load into shared memory comes after.
  if (warp == kWarps) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      {
        UnitCursor cp(sk, u_lo, u_hi);
        for (int j = 0; j < kStages && cp.left > 0; ++j, cp.next(sk))
          tma_prefetch_l2_2d(&tm_w, cp.ku * kUnitK, cp.tile * kTileN);
      }
      grid_dep_wait();
      const uint64_t pol = l2_evict_first_policy();
      int st = 0;
      uint32_t ph = 0;
      uint32_t last_ph[kStages];
      bool used[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) used[s] = false, last_ph[s] = 0;
      for (UnitCursor cu(sk, u_lo, u_hi); cu.left > 0; cu.next(sk)) {
        if (!mbar_wait_backoff(&empty[st], ph ^ 1u, s_abort)) break;
        mbar_arrive_expect_tx(&full[st], kStageBytes);
        tma_load_2d(smem + st * kStageBytes, &tm_w, &full[st], cu.ku * kUnitK, cu.tile * kTileN,
                    pol);
        used[st] = true;
        last_ph[st] = ph;
        if (++st == kStages) st = 0, ph ^= 1u;
      }
      // Do not retire while copies this thread issued may still be landing in shared memory.
      for (int s = 0; s < kStages; ++s) {
        if (!used[s]) continue;
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_test(&full[s], last_ph[s]) && globaltimer_ns() - t0 < kPipeWaitNs) {
        }
      }
      if (*s_abort) atomicCAS(p.status, 0, B2_ERR_TIMEOUT);
    }
    return;
  }

  // ------------------------------------------------------------------ consumer warps
  grid_dep_wait();
  const int g = lane >> 2, t = lane & 3;
  const bool has_row = g < p.M;
  const __half* xrow = p.x + (size_t)(has_row ? g : 0) * p.K;
  float acc[2][2][4];
#pragma unroll
  for (int T = 0; T < 2; ++T)
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[T][h][i] = 0.f;

  int st = 0;
  uint32_t ph = 0;
  bool ok = true;
  for (UnitCursor cu(sk, u_lo, u_hi); cu.left > 0; cu.next(sk)) {
    const int tile = cu.tile, ku = cu.ku;
    uint4 xv[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int k = ku * kUnitK + 16 * t + 8 * h;
      xv[h] = (has_row && k < p.K) ? ldg_nc128(xrow + k) : make_uint4(0, 0, 0, 0);
    }
    if (ok) ok = mbar_wait(&full[st], ph, s_abort);
    // The lanes poll the barrier one by one and the activation loads above branch on the row,
    // so the warp may be diverged here; mma.sync.aligned needs all 32 lanes converged.
    __syncwarp();
    const uint32_t sb = smem_u32(smem + st * kStageBytes);
#pragma unroll
    for (int T = 0; T < 2; ++T) {
      const int ra = warp * 32 + T * 16 + g;  // A row g -> weight row ra; row g+8 -> ra+8
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t sw = (uint32_t)(((2 * t + h) ^ g) << 4);  // (ra & 7) == g
        const uint4 a = lds128(sb + ra * 128 + sw);
        const uint4 b = lds128(sb + (ra + 8) * 128 + sw);
        mma_16816(acc[T][h], a.x, b.x, a.y, b.y, xv[h].x, xv[h].y);
        mma_16816(acc[T][h], a.z, b.z, a.w, b.w, xv[h].z, xv[h].w);
      }
    }
    fence_proxy_async_smem();  // this lane's reads of the stage precede its next TMA fill
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (++st == kStages) st = 0, ph ^= 1u;

    if (!cu.segment_end(sk)) continue;
    // ---------------------------------------------------------------- end of a tile segment
    float v[2][4];
#pragma unroll
    for (int T = 0; T < 2; ++T)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[T][i] = acc[T][0][i] + acc[T][1][i];
        acc[T][0][i] = acc[T][1][i] = 0.f;
      }
    const long long ts = (long long)tile * sk.upt;
    const int first = sk_owner(sk, ts), last = sk_owner(sk, ts + sk.upt - 1);
    if (first == last) {
      store_out(p, tile, warp, g, t, v);
      continue;
    }
    float* slot =
        p.partials + ((size_t)blockIdx.x * 2 + sk_slot_from_begin(u_lo, ts)) * kSlotFloats;
#pragma unroll
    for (int T = 0; T < 2; ++T)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = 2 * t + (i & 1);
        const int r = warp * 32 + T * 16 + g + (i >> 1) * 8;
        if (m < p.M) __stcg(&slot[m * kTileN + r], v[T][i]);
      }
    // every writer makes its partials visible device-wide before the barrier; then one thread
    // counts the CTA's arrival
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
    if (!*s_flag) continue;
    // add the contributors' slots in CTA order, eight contributors' loads in flight at a time
    float s[2][4];
#pragma unroll
    for (int T = 0; T < 2; ++T)
#pragma unroll
      for (int i = 0; i < 4; ++i) s[T][i] = 0.f;
    const int first_slot = sk_slot_from_begin(sk_begin(sk, first), ts);
    for (int c0 = first; c0 <= last; c0 += 8) {
      float a[8][2][4];
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        const int c = c0 + b;
        const float* sl = p.partials + ((size_t)c * 2 + (c == first ? first_slot : 0)) * kSlotFloats;
#pragma unroll
        for (int T = 0; T < 2; ++T)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int m = 2 * t + (i & 1);
            const int r = warp * 32 + T * 16 + g + (i >> 1) * 8;
            a[b][T][i] = (c <= last && m < p.M) ? __ldcg(&sl[m * kTileN + r]) : 0.f;
          }
      }
#pragma unroll
      for (int b = 0; b < 8; ++b)
        if (c0 + b <= last)
#pragma unroll
          for (int T = 0; T < 2; ++T)
#pragma unroll
            for (int i = 0; i < 4; ++i) s[T][i] += a[b][T][i];
    }
    store_out(p, tile, warp, g, t, s);
  }
  if (!ok && lane == 0) atomicCAS(p.status, 0, B2_ERR_TIMEOUT);
}

struct KernelCache {
  bool configured = false;
  int occ = 0;
};
KernelCache g_cache[64];

}  // namespace

int launch_gemm_f16(const void* x, const void* w, void* y, int M, int K, int N, void* ws,
                    size_t ws_bytes, cudaStream_t stream) {
  if (!x || !w || !y) return fail(B2_ERR_INVALID_ARG, "gemm_f16: null pointer");
  if (M < 1 || M > kMaxM) return fail(B2_ERR_INVALID_ARG, "gemm_f16: M=%d outside 1..8", M);
  if (K < 8 || K % 8 != 0) return fail(B2_ERR_INVALID_ARG, "gemm_f16: K=%d must be a positive multiple of 8", K);
  if (N < 1) return fail(B2_ERR_INVALID_ARG, "gemm_f16: N=%d", N);
  if (!aligned16(x) || !aligned16(w))
    return fail(B2_ERR_INVALID_ARG, "gemm_f16: x and w must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(y) & 1u) != 0)
    return fail(B2_ERR_INVALID_ARG, "gemm_f16: y must be 2-byte aligned");
  if (!ws || ws_bytes < ws_total_bytes())
    return fail(B2_ERR_WORKSPACE, "gemm_f16: workspace of %zu B, need %zu B", ws_bytes, ws_total_bytes());
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  int dev = 0;
  B2_CUDA_TRY(cudaGetDevice(&dev));
  KernelCache& kc = g_cache[dev];
  if (!kc.configured) {
    B2_CUDA_TRY(cudaFuncSetAttribute(gemm_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes));
    B2_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&kc.occ, gemm_f16_kernel, kThreads,
                                                              kSmemBytes));
    if (kc.occ < 1) return fail(B2_ERR_UNSUPPORTED, "gemm_f16: kernel does not fit on an SM");
    kc.configured = true;
  }
  StreamK sk;
  sk.upt = (K + kUnitK - 1) / kUnitK;
  sk.tiles = (N + kTileN - 1) / kTileN;
  if (sk.tiles > kWsMaxTiles) return fail(B2_ERR_INVALID_ARG, "gemm_f16: N=%d too large", N);
  sk.total = (long long)sk.tiles * sk.upt;
  sk.ctas = streamk_ctas(sk.total, di.sm_count, kc.occ, 8);

  CUtensorMap tm;
  rc = encode_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w, (uint64_t)K, (uint64_t)N,
                 (uint64_t)K * 2, kUnitK, kTileN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;

  F16Args a;
  a.x = static_cast<const __half*>(x);
  a.y = static_cast<__half*>(y);
  a.M = M;
  a.K = K;
  a.N = N;
  a.sk = sk;
  char* wsb = static_cast<char*>(ws);
  a.status = reinterpret_cast<int*>(wsb);
  a.counters = reinterpret_cast<int*>(wsb + ws_counters_offset());
  a.partials = reinterpret_cast<float*>(wsb + ws_partials_offset());
  return launch_kernel(gemm_f16_kernel, sk.ctas, kThreads, kSmemBytes, stream, /*early=*/true, tm,
                       a);
}

}  // namespace b2

extern "C" int b2_gemm_f16(const void* x, const void* w, void* y, int M, int K, int N, void* ws,
                           size_t ws_bytes, void* stream) {
  return b2::launch_gemm_f16(x, w, y, M, K, N, ws, ws_bytes, static_cast<cudaStream_t>(stream));
}
