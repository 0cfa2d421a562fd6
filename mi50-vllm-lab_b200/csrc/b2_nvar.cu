// One-shot all-reduce over NVLink peer memory for tensor-parallel ranks of one node.
//
// Replaces the two-GPU host-memory all-reduce of kernels/hostar.cu (hostar_create,
// hostar_allreduce, hostar_kernel). Where the reference writes each rank's slice into pinned host
// memory over PCIe and spins on a flag in host memory, here every rank stores its data straight
// into the peers' HBM over NVLink (CUDA IPC mappings), publishes a per-chunk flag with a
// system-scope release store, and reads the other ranks' data from its own HBM. The protocol
// (device generation counter, parity-alternating slots, fixed summation order) is described in
// b2_nvar.cuh. Waits are bounded and never trap: a peer that does not arrive within the handle's
// timeout leaves B2_ERR_TIMEOUT in the buffer header, which b2_nvar_status() reports.
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "b2_device.cuh"
#include "b2_internal.h"
#include "b2_nvar.cuh"

struct b2_nvar {
  int device;
  int rank;
  int world;
  size_t slot_bytes;  // largest payload per call (what the caller asked for)
  size_t slot_cap;    // bytes per slot as allocated: 4 x slot_bytes, room for the fused GEMM's
                      // 64-bit words
  size_t bytes;
  char* local;
  char* peers[b2::kArMaxWorld];
  bool opened[b2::kArMaxWorld];
  bool connected;
  unsigned long long timeout_ns;
};

namespace b2 {
namespace {

constexpr int kThreads = 512;
constexpr size_t kMinChunk = (size_t)kThreads * 16;  // one 16-byte vector per thread

__device__ __forceinline__ void add_vec(float (&acc)[8], const uint4& v, bool is_half) {
  if (is_half) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  } else {
    const float* f = reinterpret_cast<const float*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] += f[i];
  }
}

__device__ __forceinline__ uint4 pack_vec(const float (&acc)[8], bool is_half) {
  uint4 r;
  if (is_half) {
    __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
  } else {
    float* f = reinterpret_cast<float*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = acc[i];
  }
  return r;
}

// CTA c owns bytes [c*chunk, (c+1)*chunk) of the payload and flag index c. (The 64-bit word
// exchange of the fused GEMM epilogue measured slower here, 13.8 against ~10 us at 80 KB and
// P = 2: with one vector per thread the fence is cheaper than four times the bytes.)
__device__ __forceinline__ void nvar_body(const uint4* in, uint4* out, size_t nvec,
                                          size_t chunk_vec, int is_half, const ArView& v) {
  __shared__ uint32_t s_gen;
  if (threadIdx.x == 0) s_gen = ar_begin(v);
  __syncthreads();
  const uint32_t e = s_gen;
  const int par = (int)(e & 1u);
  const size_t lo = (size_t)blockIdx.x * chunk_vec;
  const size_t hi = (lo + chunk_vec < nvec) ? lo + chunk_vec : nvec;

  // 1. push this rank's chunk into slot[par][rank] of every rank
  for (size_t i = lo + threadIdx.x; i < hi; i += kThreads) {
    const uint4 val = in[i];
    for (int r = 0; r < v.world; ++r)
      reinterpret_cast<uint4*>(ar_slot(v, r, par, v.rank))[i] = val;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    ar_publish(v, blockIdx.x, e);
    ar_wait(v, blockIdx.x, e);
  }
  __syncthreads();
  __threadfence();

  // 2. add the `world` slots in rank order (fp32) and write the result
  for (size_t i = lo + threadIdx.x; i < hi; i += kThreads) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int src = 0; src < v.world; ++src)
      add_vec(acc, __ldcg(reinterpret_cast<const uint4*>(ar_slot(v, v.rank, par, src)) + i),
              is_half != 0);
    out[i] = pack_vec(acc, is_half != 0);
  }
  __syncthreads();
  if (threadIdx.x == 0) ar_finish(v, e);
}

__global__ void __launch_bounds__(kThreads) nvar_kernel(const uint4* in, uint4* out, size_t nvec,
                                                        size_t chunk_vec, int is_half,
                                                        const __grid_constant__ ArView v) {
  nvar_body(in, out, nvec, chunk_vec, is_half, v);
}

// Several ranks of one group on this GPU in one cooperative launch (grid.y = rank), for tests.
constexpr int kEmuMaxRanks = 4;
struct NvarEmu {
  const uint4* in[kEmuMaxRanks];
  uint4* out[kEmuMaxRanks];
  ArView ar[kEmuMaxRanks];
  size_t nvec, chunk_vec;
  int is_half;
};
__global__ void __launch_bounds__(kThreads) nvar_kernel_emu(const __grid_constant__ NvarEmu E) {
  const int r = blockIdx.y;
  nvar_body(E.in[r], E.out[r], E.nvec, E.chunk_vec, E.is_half, E.ar[r]);
}

unsigned long long default_timeout_ns() {
  const char* s = getenv("B2_NVAR_TIMEOUT_MS");
  if (s && *s) {
    const long long ms = atoll(s);
    if (ms > 0) return (unsigned long long)ms * 1000000ull;
  }
  return 10000000000ull;  // 10 s: tolerates host-side skew between ranks
}

class DeviceScope {
 public:
  explicit DeviceScope(int dev) {
    cudaGetDevice(&prev_);
    if (dev != prev_) cudaSetDevice(dev);
  }
  ~DeviceScope() { cudaSetDevice(prev_); }

 private:
  int prev_ = 0;
};

}  // namespace

int nvar_view(b2_nvar* h, ArView* out, size_t need_slot_bytes, int* tiles_cap) {
  if (!h) return fail(B2_ERR_STATE, "all-reduce: null handle");
  if (!h->connected) return fail(B2_ERR_STATE, "all-reduce: handle is not connected");
  if (need_slot_bytes > h->slot_bytes)
    return fail(B2_ERR_INVALID_ARG, "all-reduce: payload of %zu B exceeds the slot (%zu B)",
                need_slot_bytes, h->slot_bytes);
  int dev = 0;
  B2_CUDA_TRY(cudaGetDevice(&dev));
  if (dev != h->device)
    return fail(B2_ERR_STATE, "all-reduce: handle belongs to device %d, current device is %d",
                h->device, dev);
  ArView v;
  memset(&v, 0, sizeof(v));
  for (int r = 0; r < h->world; ++r) v.base[r] = h->peers[r];
  v.rank = h->rank;
  v.world = h->world;
  v.slot_bytes = h->slot_cap;  // the stride between slots
  v.timeout_ns = h->timeout_ns;
  *out = v;
  if (tiles_cap) *tiles_cap = kArMaxFlags;
  return B2_OK;
}

// Checks of one all-reduce call and its grid: one CTA per chunk of at least 8 KB.
int nvar_prepare(b2_nvar* h, const void* in, const void* out, size_t count, int dtype, ArView* v,
                 size_t* nvec, size_t* chunk_vec, size_t* grid) {
  if (!in || !out) return fail(B2_ERR_INVALID_ARG, "nvar_allreduce: null pointer");
  if (dtype != B2_DTYPE_F16 && dtype != B2_DTYPE_F32)
    return fail(B2_ERR_INVALID_ARG, "nvar_allreduce: dtype %d (0 = f16, 1 = f32)", dtype);
  const size_t bytes = count * (dtype == B2_DTYPE_F16 ? 2 : 4);
  if (bytes == 0 || bytes % 16 != 0)
    return fail(B2_ERR_INVALID_ARG, "nvar_allreduce: %zu bytes (must be a positive multiple of 16)",
                bytes);
  if (!aligned16(in) || !aligned16(out))
    return fail(B2_ERR_INVALID_ARG, "nvar_allreduce: buffers must be 16-byte aligned");
  int rc = nvar_view(h, v, bytes, nullptr);
  if (rc) return rc;
  *nvec = bytes / 16;
  size_t chunk = std::max(kMinChunk, (bytes + 147) / 148);
  chunk = (chunk + 15) & ~(size_t)15;
  *chunk_vec = chunk / 16;
  *grid = (*nvec + *chunk_vec - 1) / *chunk_vec;
  if (*grid > (size_t)kArMaxFlags)
    return fail(B2_ERR_INVALID_ARG, "nvar_allreduce: too many chunks");
  return B2_OK;
}

}  // namespace b2

using namespace b2;

extern "C" {

int b2_nvar_create(int device, int rank, int world, size_t slot_bytes, b2_nvar** out) {
  if (!out) return fail(B2_ERR_INVALID_ARG, "nvar_create: null output");
  if (world < 1 || world > kArMaxWorld || rank < 0 || rank >= world)
    return fail(B2_ERR_INVALID_ARG, "nvar_create: rank %d / world %d (world <= %d)", rank, world,
                kArMaxWorld);
  if (slot_bytes < 16) return fail(B2_ERR_INVALID_ARG, "nvar_create: slot of %zu B", slot_bytes);
  DeviceScope scope(device);
  slot_bytes = (slot_bytes + 255) & ~(size_t)255;
  b2_nvar* h = new b2_nvar;
  memset(h, 0, sizeof(*h));
  h->device = device;
  h->rank = rank;
  h->world = world;
  h->slot_bytes = slot_bytes;
  h->slot_cap = 4 * slot_bytes;  // an fp16 payload as 64-bit words takes 4x its bytes
  h->bytes = kArSlotsOffset + 2 * (size_t)world * h->slot_cap;
  h->timeout_ns = default_timeout_ns();
  cudaError_t e = cudaMalloc(&h->local, h->bytes);
  if (e == cudaSuccess) e = cudaMemset(h->local, 0, h->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (h->local) cudaFree(h->local);
    delete h;
    return fail(B2_ERR_CUDA, "nvar_create: %s", cudaGetErrorString(e));
  }
  h->peers[rank] = h->local;
  h->connected = (world == 1);
  *out = h;
  return B2_OK;
}

int b2_nvar_export(const b2_nvar* h, void* handle_out) {
  if (!h || !handle_out) return fail(B2_ERR_INVALID_ARG, "nvar_export: null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == B2_IPC_HANDLE_BYTES, "IPC handle size");
  DeviceScope scope(h->device);
  cudaIpcMemHandle_t ih;
  B2_CUDA_TRY(cudaIpcGetMemHandle(&ih, h->local));
  memcpy(handle_out, &ih, sizeof(ih));
  return B2_OK;
}

int b2_nvar_connect(b2_nvar* h, const void* handles) {
  if (!h || !handles) return fail(B2_ERR_INVALID_ARG, "nvar_connect: null argument");
  if (h->connected) return B2_OK;
  DeviceScope scope(h->device);
  const unsigned char* hb = static_cast<const unsigned char*>(handles);
  for (int r = 0; r < h->world; ++r) {
    if (r == h->rank || h->opened[r]) continue;
    cudaIpcMemHandle_t ih;
    memcpy(&ih, hb + (size_t)r * B2_IPC_HANDLE_BYTES, sizeof(ih));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, ih, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess)
      return fail(B2_ERR_CUDA, "nvar_connect: opening rank %d's buffer failed: %s", r,
                  cudaGetErrorString(e));
    h->peers[r] = static_cast<char*>(p);
    h->opened[r] = true;
  }
  h->connected = true;
  return B2_OK;
}

int b2_nvar_is_connected(const b2_nvar* h) { return h && h->connected ? 1 : 0; }

size_t b2_nvar_max_bytes(const b2_nvar* h) { return h ? h->slot_bytes : 0; }

int b2_nvar_set_timeout_ns(b2_nvar* h, uint64_t ns) {
  if (!h || ns == 0) return fail(B2_ERR_INVALID_ARG, "nvar_set_timeout_ns: bad argument");
  h->timeout_ns = ns;
  return B2_OK;
}

int b2_nvar_allreduce(b2_nvar* h, const void* in, void* out, size_t count, int dtype,
                      void* stream) {
  ArView v;
  size_t nvec = 0, chunk_vec = 0, grid = 0;
  int rc = nvar_prepare(h, in, out, count, dtype, &v, &nvec, &chunk_vec, &grid);
  if (rc) return rc;
  nvar_kernel<<<(unsigned)grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(in), static_cast<uint4*>(out), nvec, chunk_vec,
      dtype == B2_DTYPE_F16 ? 1 : 0, v);
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

int b2_nvar_connect_local(b2_nvar* const* handles, int ranks) {
  if (!handles || ranks < 1 || ranks > kEmuMaxRanks)
    return fail(B2_ERR_INVALID_ARG, "nvar_connect_local: %d ranks (1..%d)", ranks, kEmuMaxRanks);
  for (int r = 0; r < ranks; ++r) {
    const b2_nvar* h = handles[r];
    if (!h || h->rank != r || h->world != ranks || h->device != handles[0]->device)
      return fail(B2_ERR_INVALID_ARG,
                  "nvar_connect_local: handle %d must be rank %d of %d on device %d", r, r, ranks,
                  handles[0] ? handles[0]->device : -1);
    if (h->slot_cap != handles[0]->slot_cap)
      return fail(B2_ERR_INVALID_ARG, "nvar_connect_local: the handles' slots differ in size");
  }
  for (int r = 0; r < ranks; ++r) {
    for (int q = 0; q < ranks; ++q) handles[r]->peers[q] = handles[q]->local;
    handles[r]->connected = true;
  }
  return B2_OK;
}

int b2_nvar_allreduce_emulated(b2_nvar* const* handles, int ranks, const void* const* in,
                               void* const* out, size_t count, int dtype, void* stream) {
  if (!handles || !in || !out || ranks < 1 || ranks > kEmuMaxRanks)
    return fail(B2_ERR_INVALID_ARG, "nvar_allreduce_emulated: %d ranks (1..%d)", ranks,
                kEmuMaxRanks);
  NvarEmu E;
  memset(&E, 0, sizeof(E));
  size_t grid = 0;
  for (int r = 0; r < ranks; ++r) {
    int rc = nvar_prepare(handles[r], in[r], out[r], count, dtype, &E.ar[r], &E.nvec,
                          &E.chunk_vec, &grid);
    if (rc) return rc;
    if (E.ar[r].rank != r || E.ar[r].world != ranks)
      return fail(B2_ERR_STATE, "nvar_allreduce_emulated: handle %d is rank %d of %d", r,
                  E.ar[r].rank, E.ar[r].world);
    E.in[r] = static_cast<const uint4*>(in[r]);
    E.out[r] = static_cast<uint4*>(out[r]);
  }
  E.is_half = dtype == B2_DTYPE_F16 ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, (unsigned)ranks);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, nvar_kernel_emu, E));
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

int b2_nvar_status(b2_nvar* h, int clear, int* device_status) {
  if (!h || !device_status) return fail(B2_ERR_INVALID_ARG, "nvar_status: null argument");
  DeviceScope scope(h->device);
  ArHeader hdr;
  B2_CUDA_TRY(cudaDeviceSynchronize());
  B2_CUDA_TRY(cudaMemcpy(&hdr, h->local, sizeof(hdr), cudaMemcpyDeviceToHost));
  if (clear && hdr.status) {
    B2_CUDA_TRY(cudaMemset(h->local + offsetof(ArHeader, status), 0, sizeof(int)));
    // a launch that gave up may have left CTAs counted at its grid-wide barrier
    B2_CUDA_TRY(cudaMemset(h->local + offsetof(ArHeader, norm_count), 0, sizeof(uint32_t)));
  }
  *device_status = hdr.status;
  return B2_OK;
}

int b2_nvar_rank(const b2_nvar* h) { return h ? h->rank : -1; }
int b2_nvar_world(const b2_nvar* h) { return h ? h->world : -1; }

int b2_nvar_destroy(b2_nvar* h) {
  if (!h) return fail(B2_ERR_INVALID_ARG, "nvar_destroy: null handle");
  {
    DeviceScope scope(h->device);
    for (int r = 0; r < h->world; ++r)
      if (h->opened[r]) cudaIpcCloseMemHandle(h->peers[r]);
    cudaFree(h->local);
  }
  delete h;
  return B2_OK;
}

}  // extern "C"
