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
// With `cooperative` the driver guarantees that every CTA is resident at once, or refuses the
// launch (for kernels with a grid-wide barrier).
template <typename... KArgs, typename... Args>
int launch_kernel_ex(void (*kernel)(KArgs...), int grid, int block, size_t smem,
                     cudaStream_t stream, bool early, bool cooperative, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cooperative) {
    attr[n].id = cudaLaunchAttributeCooperative;
    attr[n].val.cooperative = 1;
    ++n;
  }
  if (early && tuning(B2_TUNE_NO_PDL) == 0) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kernel)(KArgs...), int grid, int block, size_t smem, cudaStream_t stream,
                  bool early, Args&&... args) {
  return launch_kernel_ex(kernel, grid, block, smem, stream, early, false,
                          std::forward<Args>(args)...);
}

// A launch of thread-block clusters of `cluster` CTAs along x (grid % cluster == 0). With
// `cooperative` the driver guarantees that every CTA is resident at once, or refuses the launch
// (for kernels with a grid-wide barrier).
template <typename... KArgs, typename... Args>
int launch_kernel_clusters_ex(void (*kernel)(KArgs...), int grid, int cluster, int block,
                              size_t smem, cudaStream_t stream, bool early, bool cooperative,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[3];
  int n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = (unsigned)cluster;
  attr[n].val.clusterDim.y = 1;
  attr[n].val.clusterDim.z = 1;
  ++n;
  if (cooperative) {
    attr[n].id = cudaLaunchAttributeCooperative;
    attr[n].val.cooperative = 1;
    ++n;
  }
  if (early && tuning(B2_TUNE_NO_PDL) == 0) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  B2_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  B2_CUDA_TRY(cudaGetLastError());
  return B2_OK;
}
template <typename... KArgs, typename... Args>
int launch_kernel_clusters(void (*kernel)(KArgs...), int grid, int cluster, int block, size_t smem,
                           cudaStream_t stream, bool early, Args&&... args) {
  return launch_kernel_clusters_ex(kernel, grid, cluster, block, smem, stream, early, false,
                                   std::forward<Args>(args)...);
}

}  // namespace b2
