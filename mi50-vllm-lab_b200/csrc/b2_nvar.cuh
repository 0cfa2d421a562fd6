// Layout of an NVLink all-reduce buffer and the device side of its protocol, shared by the
// standalone all-reduce kernel and the GEMM epilogue that fuses it.
//
// Every rank owns one buffer (cudaMalloc, exported with CUDA IPC, mapped by every peer):
//   [header 4 KB][flags: kArMaxWorld x kArMaxFlags u32][slots: 2 parities x world x slot_bytes]
// header.gen counts completed launches on this rank. A launch uses generation e = gen + 1 and
// slot parity e & 1. A rank writes its contribution for piece `idx` (a chunk or an output tile)
// into slot[e & 1][rank] of every rank, then stores flag[rank][idx] = e with release semantics on
// every rank. Readers acquire flag[src][idx] >= e for all src, then add the slots in rank order
// 0..world-1 in fp32, so all ranks produce bit-identical sums. A slot parity is reused only at
// e + 2, which a rank reaches only after every peer has published e + 1, which each peer does only
// after finishing launch e (stream order) - so no slot is overwritten while it is read
// (the argument of kernels/hostar.cu:9-14, for `world` ranks).
// When the slot has room (it is allocated at 4x the largest payload), the data instead travel as
// 64-bit (generation, fp32 value) words that need no flag and no fence (ll_store / ll_gather); the
// same reuse argument holds with "published e + 1" read as "wrote its words of e + 1".
#pragma once

#include "b2_device.cuh"

namespace b2 {

constexpr int kArMaxWorld = 8;
constexpr int kArMaxFlags = 4096;
constexpr size_t kArHeaderBytes = 4096;
constexpr size_t kArFlagsBytes = (size_t)kArMaxWorld * kArMaxFlags * sizeof(uint32_t);
constexpr size_t kArSlotsOffset = kArHeaderBytes + kArFlagsBytes;

// norm_count / norm_gen: the grid-wide barrier of a fused launch that normalises rows (residual
// add + RMSNorm). Every CTA adds 1 to norm_count; the last one resets it and stores the launch's
// generation in norm_gen, which the others wait for. Each sits on its own 128-byte line, so the
// waiters' polling does not slow the arrivals.
struct ArHeader {
  uint32_t gen;   // completed launches
  uint32_t done;  // CTAs of the running launch that finished
  int status;     // 0 or B2_ERR_TIMEOUT
  uint32_t pad0[29];
  uint32_t norm_gen;  // generation of the last launch whose CTAs all arrived
  uint32_t pad1[31];
  uint32_t norm_count;  // CTAs of the running launch that arrived
  uint32_t pad2[31];
};
static_assert(sizeof(ArHeader) <= kArHeaderBytes, "the header must fit its 4 KB");

// Kernel-parameter view of one all-reduce handle.
struct ArView {
  char* base[kArMaxWorld];  // base[r]: rank r's buffer as mapped in this process
  int rank;
  int world;
  unsigned long long slot_bytes;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ ArHeader* ar_header(const ArView& v) {
  return reinterpret_cast<ArHeader*>(v.base[v.rank]);
}
__device__ __forceinline__ uint32_t* ar_flag(const ArView& v, int owner, int src, int idx) {
  return reinterpret_cast<uint32_t*>(v.base[owner] + kArHeaderBytes) + (size_t)src * kArMaxFlags +
         idx;
}
__device__ __forceinline__ char* ar_slot(const ArView& v, int owner, int parity, int src) {
  return v.base[owner] + kArSlotsOffset + ((size_t)parity * v.world + src) * v.slot_bytes;
}

// Generation of the launch in progress (called by one thread).
__device__ __forceinline__ uint32_t ar_begin(const ArView& v) {
  return *reinterpret_cast<volatile uint32_t*>(&ar_header(v)->gen) + 1u;
}

// Publish piece `idx` of generation e on every rank, from one thread, after a CTA barrier that
// follows the CTA's data stores. The barrier orders the other threads' stores before this
// thread's system-scope release fence, which (being cumulative) makes all of them visible on every
// GPU before any flag is.
__device__ __forceinline__ void ar_publish(const ArView& v, int idx, uint32_t e) {
  __threadfence_system();
  for (int r = 0; r < v.world; ++r) st_relaxed_sys(ar_flag(v, r, v.rank, idx), e);
}

// Wait until every rank has published piece `idx` of generation e here. Bounded: after
// v.timeout_ns records B2_ERR_TIMEOUT in the header and returns false. One thread.
__device__ __forceinline__ bool ar_wait(const ArView& v, int idx, uint32_t e) {
  const unsigned long long t0 = globaltimer_ns();
  for (int src = 0; src < v.world; ++src) {
    const uint32_t* f = ar_flag(v, v.rank, src, idx);
    unsigned int it = 0;
    while ((int)(ld_acquire_sys(f) - e) < 0) {
      if (++it >= kMaxSpin || globaltimer_ns() - t0 > v.timeout_ns) {
        atomicCAS(&ar_header(v)->status, 0, B2_ERR_TIMEOUT);
        return false;
      }
      if ((it & 15u) == 0) __nanosleep(64);
    }
  }
  return true;
}

// Low-latency exchange: a 64-bit word carries an fp32 value in its low half and the generation
// in its high half, written with one single-copy-atomic 64-bit store, so the reader needs no flag
// and the writer no fence: a word whose high half equals e holds generation e's value. Slots start
// zeroed and e >= 1, and a slot parity is reused only at e + 2 (see above), so no stale word ever
// carries e.
__device__ __forceinline__ void ll_store(uint64_t* p, float v, uint32_t e) {
  const uint64_t w = ((uint64_t)e << 32) | (uint64_t)__float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ll_peek(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Generation e's values at p[0..n) (n <= N): all n loads are issued before any is checked, so the
// words that have already landed cost one round trip together; only the missing ones are polled
// again (bounded by the absolute deadline). Returns false if a word never arrived (its value
// reads as 0).
template <int N>
__device__ __forceinline__ bool ll_gather(const uint64_t* const (&p)[N], int n, uint32_t e,
                                          unsigned long long deadline_ns, float (&out)[N]) {
  uint64_t w[N];
#pragma unroll
  for (int k = 0; k < N; ++k)
    if (k < n) w[k] = ll_peek(p[k]);
  bool ok = true;
#pragma unroll
  for (int k = 0; k < N; ++k) {
    if (k >= n) continue;
    unsigned int it = 0;
    while ((uint32_t)(w[k] >> 32) != e) {
      if (++it >= kMaxSpin || ((it & 15u) == 0 && globaltimer_ns() > deadline_ns)) {
        ok = false;
        w[k] = 0;
        break;
      }
      __nanosleep(32);
      w[k] = ll_peek(p[k]);
    }
    out[k] = __uint_as_float((uint32_t)w[k]);
  }
  return ok;
}

// Count this CTA as finished; the last CTA of the launch advances the generation. One thread,
// after the CTA's last use of the buffer.
__device__ __forceinline__ void ar_finish(const ArView& v, uint32_t e) {
  ArHeader* h = ar_header(v);
  __threadfence();
  if (atomicAdd(&h->done, 1u) == gridDim.x - 1) {
    atomicExch(&h->done, 0u);
    atomicExch(&h->gen, e);
  }
}

}  // namespace b2
