// Host-side helpers shared by the translation units of the library (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

#include "b2_skinny.h"

namespace b2 {

// Record a failure detail for b2_last_error() and return `status`.
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// Check a CUDA runtime call; on error record it and return B2_ERR_CUDA.
#define B2_CUDA_TRY(expr)                                                             \
  do {                                                                                \
    cudaError_t e_ = (expr);                                                          \
    if (e_ != cudaSuccess)                                                            \
      return ::b2::fail(B2_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

struct DeviceInfo {
  int sm_count = 0;
  int major = 0, minor = 0;
  size_t smem_optin = 0;
  bool ok = false;
};
// Cached properties of the current device (B2_ERR_UNSUPPORTED unless compute capability 10.x).
int device_info(DeviceInfo* out);

// Encode a 2-D tiled tensor map. dims/box: {inner, outer}; row_stride in bytes.
int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
              uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swizzle);
// Encode a 3-D tiled tensor map. dims/box innermost first; strides (bytes) of dims 1 and 2, in
// any order of size (a middle dimension may step further than the outer one).
int encode_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[3],
              const uint64_t strides_bytes[2], const uint32_t box[3], CUtensorMapSwizzle swizzle);

// Workspace layout: [status words][tile counters][partial slots][row sums of the fused RMSNorm,
// kMaxM floats per CTA].
constexpr size_t kWsStatusBytes = 256;
constexpr int kWsMaxTiles = 65536;
constexpr int kWsMaxCtas = 1024;
size_t ws_counters_offset();
size_t ws_partials_offset();
size_t ws_norm_offset();
size_t ws_total_bytes();

// Tuning knobs (b2_set_tuning).
int tuning(int key);

// Grid size of a stream-K launch over `total` units for a kernel with `occ` resident CTAs per SM.
int streamk_ctas(long long total, int sm_count, int occ, int min_units_default);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch `kernel` on `stream`. With `early` the launch is marked for programmatic dependent
// launch: its CTAs may start while the previous kernel on the stream is finishing, and they read
// nothing that kernel writes before grid_dep_wait(). B2_TUNE_NO_PDL != 0 turns this off.
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kernel)(KArgs...), int grid, int block, size_t smem, cudaStream_t stream,
                  bool early, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (early && tuning(B2_TUNE_NO_PDL) == 0) ? 1 : 0;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

// The same as a launch of thread-block clusters of `cluster` CTAs along x (grid % cluster == 0).
template <typename... KArgs, typename... Args>
int launch_kernel_clusters(void (*kernel)(KArgs...), int grid, int cluster, int block, size_t smem,
                           cudaStream_t stream, bool early, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (early && tuning(B2_TUNE_NO_PDL) == 0) ? 2 : 1;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}

}  // namespace b2
