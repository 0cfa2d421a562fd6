// Device-side building blocks shared by the kernels: mbarrier pipeline, TMA, mma.sync,
// bounded waits, release/acquire flags and the stream-K work split.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2_skinny.h"

namespace b2 {

// Output tile width (columns of y) of both GEMMs and the M-rows capacity of a slot.
constexpr int kTileN = 128;
constexpr int kMaxM = 8;
constexpr int kSlotFloats = kMaxM * kTileN;  // one fp32 partial tile
constexpr int kStatusWords = 64;             // status region of the workspace (256 B)

// A device wait that has not finished after this long records B2_ERR_TIMEOUT and returns.
constexpr unsigned long long kPipeWaitNs = 2000000000ull;  // 2 s (data from HBM: microseconds)
constexpr unsigned int kMaxSpin = 1u << 30;                // iteration cap on top of the clock

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with an explicit suspend-time hint: a thread whose phase has not completed sleeps in
// hardware for up to `hint_ns` (waking early when the phase completes) instead of returning at
// once, so a waiting warp issues almost nothing while it waits.
__device__ __forceinline__ bool mbar_test_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` to complete. Gives up after kPipeWaitNs, or at once when
// another warp of the CTA already gave up (*abort != 0); then sets *abort and returns false.
// After the first test each poll suspends the thread (up to 20 us) until the phase completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (unsigned int it = 1; it < kMaxSpin; ++it) {
    if (mbar_test_hint(bar, parity, 20000u)) return true;
    if ((it & 7u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > kPipeWaitNs) break;
    }
  }
  *abort = 1;
  return false;
}

// The same wait for the producer thread, which backs off between polls so that its warp does not
// take issue slots from the consumer warps on the same scheduler while the ring is full.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (unsigned int it = 1; it < kMaxSpin; ++it) {
    __nanosleep(32);
    if (mbar_test(bar, parity)) return true;
    if ((it & 15u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > kPipeWaitNs) break;
    }
  }
  *abort = 1;
  return false;
}

// ---------------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor, no multicast) and L2 policy
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}
__device__ __forceinline__ uint64_t l2_evict_normal_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 2-D tiled load of the box at (c0 = innermost coordinate, c1) into shared memory, completing
// transaction bytes on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0,
                                            int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(m), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 3-D tiled load of the box at (c0 = innermost, c1, c2): one instruction for what would take
// several 2-D boxes (a producer thread issues only a few copy instructions per microsecond).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0,
                                            int c1, int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* m, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(m),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
// Contiguous bytes from global into shared memory (no tensor map), completing on `bar`. Both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Prefetch the box at (c0, c1) of a 2-D tensor into L2 (no shared memory, no barrier). Safe
// before griddepcontrol.wait: L2 is where the previous grid's late stores land, so a line
// fetched early is updated by them, while a copy into shared memory could keep stale data.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* m, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(m),
               "r"(c0), "r"(c1)
               : "memory");
}

// ---------------------------------------------------------------------------------------------
// Loads, stores, barriers
// ---------------------------------------------------------------------------------------------
// Volatile with a "memory" clobber: a stage may be read only between the wait on its full
// barrier and the arrival on its empty barrier, and these loads must stay in that window.
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
// The same at addr + 1024 (immediate offset: no address arithmetic).
__device__ __forceinline__ uint4 lds128_1k(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4+1024];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ uint4 ldg_nc128(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
// Orders this thread's earlier shared-memory accesses (generic proxy) before later accesses by
// the async proxy (TMA). A consumer issues it after its last read of a stage and before it
// releases the stage, whose next TMA fill must not land under those reads.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Named barrier over the first `threads` threads of the CTA (the consumer warps).
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Release store / acquire load of a 32-bit flag at GPU scope (flags read only by CTAs of the
// same GPU).
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// System-scope release store / acquire load of a 32-bit flag (peer memory over NVLink).
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Programmatic dependent launch. grid_dep_wait() returns once the grids this one depends on
// have completed and their memory is visible (at once when the launch has no such dependency);
// grid_dep_launch() lets the next grid on the stream start launching its CTAs early.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------
// Tensor cores: D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The same with C = 0: the first mma of an accumulation needs no zeroed registers.
__device__ __forceinline__ void mma_16816_first(float (&d)[4], uint32_t a0, uint32_t a1,
                                                uint32_t a2, uint32_t a3, uint32_t b0,
                                                uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f), "f"(0.f), "f"(0.f),
        "f"(0.f));
}

// ---------------------------------------------------------------------------------------------
// Thread-block clusters and distributed shared memory (no multicast)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrive on an mbarrier of another CTA of the cluster (release at cluster scope).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ bool mbar_test_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait (acquire at cluster scope) for arrivals made by other CTAs of the cluster; same
// give-up rule as mbar_wait.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort) {
  if (mbar_test_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (unsigned int it = 1; it < kMaxSpin; ++it) {
    if (mbar_test_cluster(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > kPipeWaitNs) break;
    }
  }
  *abort = 1;
  return false;
}
// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from this CTA's shared
// memory to another CTA of the cluster. The copy completes `bytes` transaction bytes on the
// destination CTA's mbarrier, so the receiver learns of the data from its own barrier; no fence
// and no remote arrival. dst_cluster and mbar_cluster are mapa_shared addresses.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta,
                                                  uint32_t bytes, uint32_t mbar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(dst_cluster), "r"(src_cta), "r"(bytes), "r"(mbar_cluster)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every bulk copy this thread committed has finished reading its source.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_dsmem_f32(uint32_t cluster_addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() {
  asm volatile("fence.acq_rel.cluster;" ::: "memory");
}
// Hardware barrier over every thread of the cluster (used once, right after the mbarriers are
// initialised, so that no CTA arrives on a peer's barrier before the peer has set it up).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// ---------------------------------------------------------------------------------------------
// Stream-K work split. The GEMM is cut into `tiles` output tiles of kTileN columns, each made
// of `upt` k-units. The total tiles*upt units are dealt to `ctas` CTAs as contiguous ranges:
// CTA i owns units [total*i/ctas, total*(i+1)/ctas). A tile touched by one CTA is written
// directly; a tile shared by several CTAs is summed by the last of them to finish, in CTA
// order, from fp32 slots (slot 0 = the CTA's first tile, slot 1 = its last tile).
// ---------------------------------------------------------------------------------------------
struct StreamK {
  long long total;  // tiles * upt
  int upt;          // k-units per tile
  int tiles;
  int ctas;         // grid size; ctas <= total so every CTA owns at least one unit
};

__host__ __device__ __forceinline__ long long sk_begin(const StreamK& s, int cta) {
  return s.total * (long long)cta / s.ctas;
}
// The CTA whose range contains unit u.
__host__ __device__ __forceinline__ int sk_owner(const StreamK& s, long long u) {
  return (int)(((u + 1) * (long long)s.ctas - 1) / s.total);
}
// Slot index (0 or 1) that CTA `cta` uses for its partial of tile `tile`.
__host__ __device__ __forceinline__ int sk_slot(const StreamK& s, int cta, int tile) {
  return (sk_begin(s, cta) / s.upt == tile) ? 0 : 1;
}

// The same rule without division, for the hot paths: a CTA whose range starts at unit `begin`
// uses slot 0 for the tile starting at unit `tile_start` iff it starts inside that tile. Of a
// tile's contributors first..last only `first` can start before the tile, so the reducer needs
// one sk_begin (for `first`) per tile instead of one per contributor.
__device__ __forceinline__ int sk_slot_from_begin(long long begin, long long tile_start) {
  return begin >= tile_start ? 0 : 1;
}

// Walks a CTA's unit range as (tile, k-unit) pairs without dividing in the loop.
struct UnitCursor {
  int tile, ku, left;
  __device__ __forceinline__ UnitCursor(const StreamK& s, long long lo, long long hi) {
    tile = (int)(lo / s.upt);
    ku = (int)(lo - (long long)tile * s.upt);
    left = (int)(hi - lo);
  }
  __device__ __forceinline__ bool segment_end(const StreamK& s) const {
    return ku == s.upt - 1 || left == 1;
  }
  __device__ __forceinline__ void next(const StreamK& s) {
    --left;
    if (++ku == s.upt) ku = 0, ++tile;
  }
};

}  // namespace b2
