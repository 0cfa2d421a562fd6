// Host runtime of the library: status strings, error detail, device properties, tensor-map
// encoding, workspace management, tuning knobs and the shared-memory rendezvous registry.
#include <cudaTypedefs.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "b2_device.cuh"
#include "b2_internal.h"

namespace b2 {

static thread_local char g_last_error[512] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

// ----------------------------------------------------------------------------------------------
// Device properties
// ----------------------------------------------------------------------------------------------
static std::mutex g_dev_mu;
static DeviceInfo g_dev[64];

int device_info(DeviceInfo* out) {
  int dev = 0;
  B2_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(B2_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ok) {
    cudaDeviceProp p;
    B2_CUDA_TRY(cudaGetDeviceProperties(&p, dev));
    d.sm_count = p.multiProcessorCount;
    d.major = p.major;
    d.minor = p.minor;
    d.smem_optin = p.sharedMemPerBlockOptin;
    d.ok = true;
  }
  *out = d;
  if (d.major != 10)
    return fail(B2_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                d.major, d.minor);
  return B2_OK;
}

// ----------------------------------------------------------------------------------------------
// Tensor maps (driver entry point fetched through the runtime; no link-time libcuda dependency)
// ----------------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Encoding a tensor map costs microseconds of host time, comparable to a whole small GEMM, so
// maps are kept in a small per-thread cache keyed by everything they encode. A map depends only
// on these values, so a hit is always valid (even if the memory was freed and reallocated).
namespace {
struct MapKey {
  const void* base;
  int rank;
  uint64_t dims[3], strides[2];
  uint32_t box[3];
  int dtype, swizzle, device;
  bool operator==(const MapKey& o) const {
    if (base != o.base || rank != o.rank || dtype != o.dtype || swizzle != o.swizzle ||
        device != o.device)
      return false;
    for (int i = 0; i < rank; ++i)
      if (dims[i] != o.dims[i] || box[i] != o.box[i] || (i + 1 < rank && strides[i] != o.strides[i]))
        return false;
    return true;
  }
};
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool valid;
};
constexpr int kMapCache = 64;
thread_local MapEntry t_maps[kMapCache];

size_t map_hash(const MapKey& k) {
  size_t h = reinterpret_cast<uintptr_t>(k.base) >> 4;
  for (int i = 0; i < k.rank; ++i) {
    h = h * 1000003u ^ (size_t)k.dims[i];
    h = h * 1000003u ^ (size_t)k.box[i];
    if (i + 1 < k.rank) h = h * 1000003u ^ (size_t)k.strides[i];
  }
  h = h * 1000003u ^ (size_t)(k.dtype * 31 + k.swizzle * 7 + k.device + k.rank * 131);
  return h;
}

int encode_uncached(CUtensorMap* map, const MapKey& k) {
  auto fn = get_encode_fn();
  if (!fn) return fail(B2_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {0, 0, 0}, strides[2] = {0, 0};
  cuuint32_t box[3] = {0, 0, 0}, estr[3] = {1, 1, 1};
  for (int i = 0; i < k.rank; ++i) {
    dims[i] = k.dims[i];
    box[i] = k.box[i];
    if (i + 1 < k.rank) strides[i] = k.strides[i];
  }
  CUresult r = fn(map, (CUtensorMapDataType)k.dtype, (cuuint32_t)k.rank, const_cast<void*>(k.base),
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  (CUtensorMapSwizzle)k.swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B2_ERR_INVALID_ARG,
                "cuTensorMapEncodeTiled failed (%d): rank %d, dims %llu x %llu x %llu, strides "
                "%llu %llu B, box %u x %u x %u",
                (int)r, k.rank, (unsigned long long)dims[0], (unsigned long long)dims[1],
                (unsigned long long)dims[2], (unsigned long long)strides[0],
                (unsigned long long)strides[1], box[0], box[1], box[2]);
  return B2_OK;
}

int encode_cached(CUtensorMap* map, MapKey key) {
  cudaGetDevice(&key.device);
  MapEntry& e = t_maps[map_hash(key) % kMapCache];
  if (e.valid && e.key == key) {
    *map = e.map;
    return B2_OK;
  }
  const int rc = encode_uncached(map, key);
  if (rc == B2_OK) {
    e.key = key;
    e.map = *map;
    e.valid = true;
  }
  return rc;
}
}  // namespace

int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
              uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swizzle) {
  MapKey k = {};
  k.base = base;
  k.rank = 2;
  k.dims[0] = inner;
  k.dims[1] = outer;
  k.strides[0] = row_stride_bytes;
  k.box[0] = box_inner;
  k.box[1] = box_outer;
  k.dtype = (int)dtype;
  k.swizzle = (int)swizzle;
  return encode_cached(map, k);
}

int encode_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[3],
              const uint64_t strides_bytes[2], const uint32_t box[3], CUtensorMapSwizzle swizzle) {
  MapKey k = {};
  k.base = base;
  k.rank = 3;
  for (int i = 0; i < 3; ++i) {
    k.dims[i] = dims[i];
    k.box[i] = box[i];
  }
  k.strides[0] = strides_bytes[0];
  k.strides[1] = strides_bytes[1];
  k.dtype = (int)dtype;
  k.swizzle = (int)swizzle;
  return encode_cached(map, k);
}

// ----------------------------------------------------------------------------------------------
// Workspace
// ----------------------------------------------------------------------------------------------
size_t ws_counters_offset() { return kWsStatusBytes; }
size_t ws_partials_offset() {
  size_t off = kWsStatusBytes + (size_t)kWsMaxTiles * sizeof(int);
  return (off + 255) & ~(size_t)255;
}
size_t ws_norm_offset() {
  return ws_partials_offset() + (size_t)kWsMaxCtas * 2 * kSlotFloats * sizeof(float);
}
size_t ws_total_bytes() { return ws_norm_offset() + (size_t)kWsMaxCtas * kMaxM * sizeof(float); }

// ----------------------------------------------------------------------------------------------
// Tuning
// ----------------------------------------------------------------------------------------------
constexpr int kTuneKeys = 16;
static std::atomic<int> g_tune[kTuneKeys];

// B2_TUNE="key=value,key=value" in the environment presets tuning keys (read once, before the
// first use; b2_set_tuning overrides).
static void tuning_from_env() {
  static std::once_flag once;
  std::call_once(once, [] {
    const char* env = std::getenv("B2_TUNE");
    if (!env) return;
    const char* p = env;
    while (*p) {
      char* end = nullptr;
      const long k = std::strtol(p, &end, 10);
      if (end == p || *end != '=') break;
      p = end + 1;
      const long v = std::strtol(p, &end, 10);
      if (end == p) break;
      if (k >= 0 && k < kTuneKeys) g_tune[k].store((int)v);
      p = end;
      if (*p == ',') ++p;
    }
  });
}

int tuning(int key) {
  tuning_from_env();
  return (key >= 0 && key < kTuneKeys) ? g_tune[key].load() : 0;
}

int streamk_ctas(long long total, int sm_count, int occ, int min_units_default) {
  int cps = tuning(B2_TUNE_CTAS_PER_SM);
  if (cps <= 0 || cps > occ) cps = occ;
  int min_units = tuning(B2_TUNE_MIN_UNITS);
  if (min_units <= 0) min_units = min_units_default;
  long long cap = (long long)sm_count * cps;
  long long by_units = (total + min_units - 1) / min_units;
  long long c = std::min(std::min(cap, by_units), total);
  c = std::min<long long>(c, kWsMaxCtas);
  return (int)std::max<long long>(c, 1);
}

}  // namespace b2

using namespace b2;

extern "C" {

const char* b2_status_string(int status) {
  switch (status) {
    case B2_OK: return "ok";
    case B2_ERR_INVALID_ARG: return "invalid argument";
    case B2_ERR_UNSUPPORTED: return "unsupported device or configuration";
    case B2_ERR_CUDA: return "CUDA error";
    case B2_ERR_WORKSPACE: return "workspace missing or too small";
    case B2_ERR_TIMEOUT: return "device-side wait timed out";
    case B2_ERR_STATE: return "bad handle or state";
    default: return "unknown status";
  }
}

const char* b2_last_error(void) { return g_last_error; }

int b2_abi_version(void) { return B2_ABI_VERSION; }

size_t b2_workspace_bytes(int device) {
  (void)device;
  return ws_total_bytes();
}

int b2_workspace_init(void* ws, size_t ws_bytes, void* stream) {
  if (!ws || ws_bytes < ws_total_bytes())
    return fail(B2_ERR_WORKSPACE, "workspace of %zu B, need %zu B", ws_bytes, ws_total_bytes());
  // Only the status words and the counters must start at zero; the slots are overwritten.
  B2_CUDA_TRY(cudaMemsetAsync(ws, 0, ws_partials_offset(), (cudaStream_t)stream));
  return B2_OK;
}

int b2_workspace_status(void* ws, int clear, int* device_status) {
  if (!ws || !device_status) return fail(B2_ERR_INVALID_ARG, "null workspace or output");
  int v = 0;
  B2_CUDA_TRY(cudaDeviceSynchronize());
  B2_CUDA_TRY(cudaMemcpy(&v, ws, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear && v) B2_CUDA_TRY(cudaMemset(ws, 0, sizeof(int)));
  *device_status = v;
  return B2_OK;
}

int b2_set_tuning(int key, int value) {
  tuning_from_env();
  if (key < 0 || key >= kTuneKeys) return fail(B2_ERR_INVALID_ARG, "unknown tuning key %d", key);
  g_tune[key].store(value);
  return B2_OK;
}

int b2_get_tuning(int key) { return tuning(key); }

// ----------------------------------------------------------------------------------------------
// Rendezvous registry in POSIX shared memory
// ----------------------------------------------------------------------------------------------
}  // extern "C"

namespace {
constexpr uint32_t kRegMagic = 0x42325247u;  // "B2RG"
constexpr int kRegMaxWorld = 64;
struct RegLayout {
  uint32_t magic;
  uint32_t world;
  uint32_t present[kRegMaxWorld];
  unsigned char blob[kRegMaxWorld][B2_BLOB_BYTES];
};
}  // namespace

struct b2_registry {
  RegLayout* map;
  int world;
};

extern "C" {

int b2_registry_open(const char* name, int world, int create, b2_registry** out) {
  if (!name || !out || world < 1 || world > kRegMaxWorld)
    return fail(B2_ERR_INVALID_ARG, "registry: bad name/world (%d)", world);
  const int fd = shm_open(name, create ? (O_CREAT | O_RDWR) : O_RDWR, 0600);
  if (fd < 0) return fail(B2_ERR_STATE, "registry: shm_open(%s) failed", name);
  if (create && ftruncate(fd, sizeof(RegLayout)) != 0) {
    close(fd);
    return fail(B2_ERR_STATE, "registry: ftruncate(%s) failed", name);
  }
  void* p = mmap(nullptr, sizeof(RegLayout), PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return fail(B2_ERR_STATE, "registry: mmap(%s) failed", name);
  RegLayout* r = static_cast<RegLayout*>(p);
  if (create) {
    memset(r, 0, sizeof(RegLayout));
    r->world = (uint32_t)world;
    __atomic_store_n(&r->magic, kRegMagic, __ATOMIC_RELEASE);
  } else if (__atomic_load_n(&r->magic, __ATOMIC_ACQUIRE) != kRegMagic ||
             r->world != (uint32_t)world) {
    munmap(p, sizeof(RegLayout));
    return fail(B2_ERR_STATE, "registry %s is not initialised for world %d", name, world);
  }
  *out = new b2_registry{r, world};
  return B2_OK;
}

int b2_registry_put(b2_registry* reg, int rank, const void* blob) {
  if (!reg || !blob || rank < 0 || rank >= reg->world)
    return fail(B2_ERR_INVALID_ARG, "registry_put: bad rank %d", rank);
  memcpy(reg->map->blob[rank], blob, B2_BLOB_BYTES);
  __atomic_store_n(&reg->map->present[rank], 1u, __ATOMIC_RELEASE);
  return B2_OK;
}

int b2_registry_get(b2_registry* reg, int rank, void* blob_out) {
  if (!reg || !blob_out || rank < 0 || rank >= reg->world)
    return fail(B2_ERR_INVALID_ARG, "registry_get: bad rank %d", rank);
  if (__atomic_load_n(&reg->map->present[rank], __ATOMIC_ACQUIRE) != 1u)
    return fail(B2_ERR_STATE, "registry_get: rank %d has not published", rank);
  memcpy(blob_out, reg->map->blob[rank], B2_BLOB_BYTES);
  return B2_OK;
}

int b2_registry_close(b2_registry* reg) {
  if (!reg) return fail(B2_ERR_INVALID_ARG, "registry_close: null");
  munmap(reg->map, sizeof(RegLayout));
  delete reg;
  return B2_OK;
}

int b2_registry_unlink(const char* name) {
  if (!name) return fail(B2_ERR_INVALID_ARG, "registry_unlink: null name");
  shm_unlink(name);
  return B2_OK;
}

}  // extern "C"
