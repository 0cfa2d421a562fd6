// PyTorch operator library `gfx906_skinny` on top of the C ABI (include/b2_skinny.h).
//
// Registers the reference's operator names and schemas so that the vLLM call sites that load
// the reference's gfx906_skinny.so through torch.ops.load_library work unchanged:
//   gemm(Tensor x, Tensor w, int variant=0) -> Tensor                   kernels/skinny.cu:330-333
//   w4gemm(Tensor a, Tensor qw, Tensor qz, Tensor sc, int kw, int waves) kernels/w4.cu:506-509
//   hostar_create / hostar_unlink / hostar_max_bytes / hostar_allreduce kernels/hostar.cu:155-166
// plus operators the reference does not have (N-rank NVLink all-reduce, the W4 GEMM with the
// all-reduce fused into its epilogue, optionally followed by the residual add + RMSNorm, the
// load-time weight repack and the W4 GEMM on its image, status and tuning). Device operators
// are registered on the CUDA dispatch key and launch on the current stream; host operators on
// CompositeExplicitAutograd, as in the reference. Errors become RuntimeError via TORCH_CHECK.
//
// The tuning selectors of the reference (`variant` of gemm, `kw`/`waves` of w4gemm) are accepted
// and ignored: the sm_100a kernels size their grid from the shape and the SM count. The group
// size, which the reference's schema does not carry, is K / sc.size(0).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime_api.h>
#include <torch/library.h>

#include <mutex>
#include <string>
#include <vector>

#include "b2_skinny.h"

namespace {

std::string detail(int rc) {
  return std::string(b2_status_string(rc)) + ": " + b2_last_error();
}

// ------------------------------------------------------------------------------------------------
// Per-device workspace: allocated and zero-filled once, outside any stream capture. The kernels
// leave its counters at zero, so it is reused by every later call (and by graph replays).
// ------------------------------------------------------------------------------------------------
std::mutex g_ws_mu;
void* g_ws[64] = {nullptr};

void* workspace(int dev) {
  TORCH_CHECK(dev >= 0 && dev < 64, "gfx906_skinny: device ordinal ", dev);
  std::lock_guard<std::mutex> lk(g_ws_mu);
  if (g_ws[dev]) return g_ws[dev];
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(c10::cuda::getCurrentCUDAStream(dev).stream(), &cs);
  TORCH_CHECK(cs == cudaStreamCaptureStatusNone,
              "gfx906_skinny: the first GEMM call on a device allocates its workspace and must "
              "run before CUDA graph capture (warm up eagerly first)");
  const size_t bytes = b2_workspace_bytes(dev);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  TORCH_CHECK(e == cudaSuccess, "gfx906_skinny: workspace cudaMalloc failed: ",
              cudaGetErrorString(e));
  int rc = b2_workspace_init(p, bytes, nullptr);
  TORCH_CHECK(rc == B2_OK, "gfx906_skinny: workspace init: ", detail(rc));
  e = cudaDeviceSynchronize();
  TORCH_CHECK(e == cudaSuccess, "gfx906_skinny: workspace init: ", cudaGetErrorString(e));
  g_ws[dev] = p;
  return p;
}

void check_cuda_half(const at::Tensor& t, const char* op, const char* name) {
  TORCH_CHECK(t.is_cuda(), op, ": ", name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kHalf, op, ": ", name, " must be float16");
  TORCH_CHECK(t.is_contiguous(), op, ": ", name, " must be contiguous");
}

// ------------------------------------------------------------------------------------------------
// gemm: y[M, N] = x[M, K] @ w[N, K]^T   (kernels/skinny.cu:300-328)
// ------------------------------------------------------------------------------------------------
at::Tensor skinny_gemm(const at::Tensor& x, const at::Tensor& w, int64_t variant) {
  (void)variant;
  check_cuda_half(x, "gemm", "x");
  check_cuda_half(w, "gemm", "w");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2, "gemm: x and w must be 2-D");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && K % 8 == 0 && M >= 1 && M <= 8,
              "gemm: need x [M<=8, K], w [N, K], K % 8 == 0; got x ", x.sizes(), ", w ", w.sizes());
  TORCH_CHECK(x.device() == w.device(), "gemm: x and w on different devices");
  c10::cuda::CUDAGuard guard(x.device());
  auto y = at::empty({M, N}, x.options());
  const int dev = x.get_device();
  void* ws = workspace(dev);
  const int rc = b2_gemm_f16(x.data_ptr(), w.data_ptr(), y.data_ptr(), (int)M, (int)K, (int)N, ws,
                             b2_workspace_bytes(dev), c10::cuda::getCurrentCUDAStream(dev).stream());
  TORCH_CHECK(rc == B2_OK, "gfx906_skinny.gemm: ", detail(rc));
  return y;
}

at::Tensor skinny_gemm_meta(const at::Tensor& x, const at::Tensor& w, int64_t variant) {
  (void)variant;
  return at::empty({x.size(0), w.size(0)}, x.options());
}

// ------------------------------------------------------------------------------------------------
// w4gemm   (kernels/w4.cu:477-504)
// ------------------------------------------------------------------------------------------------
int check_w4(const at::Tensor& a, const at::Tensor& qw, const at::Tensor& qz, const at::Tensor& sc,
             const char* op) {
  check_cuda_half(a, op, "a");
  check_cuda_half(sc, op, "sc");
  TORCH_CHECK(qw.is_cuda() && qz.is_cuda(), op, ": qw and qz must be CUDA tensors");
  TORCH_CHECK(qw.scalar_type() == at::kInt && qz.scalar_type() == at::kInt, op,
              ": qw and qz must be int32");
  TORCH_CHECK(qw.is_contiguous() && qz.is_contiguous(), op, ": qw and qz must be contiguous");
  TORCH_CHECK(a.dim() == 2 && qw.dim() == 2 && qz.dim() == 2 && sc.dim() == 2, op,
              ": all operands must be 2-D");
  const int64_t M = a.size(0), K = a.size(1), N = qw.size(1);
  TORCH_CHECK(M >= 1 && M <= 8, op, ": M=", M, " outside 1..8");
  TORCH_CHECK(qw.size(0) * 8 == K, op, ": qw must be [K/8, N]; got ", qw.sizes(), " for K=", K);
  TORCH_CHECK(sc.size(0) > 0 && K % sc.size(0) == 0 && sc.size(1) == N, op,
              ": sc must be [K/G, N]; got ", sc.sizes());
  const int64_t G = K / sc.size(0);
  TORCH_CHECK(qz.size(0) == sc.size(0) && qz.size(1) * 8 == N, op, ": qz must be [K/G, N/8]; got ",
              qz.sizes());
  return (int)G;
}

at::Tensor w4_gemm(const at::Tensor& a, const at::Tensor& qw, const at::Tensor& qz,
                   const at::Tensor& sc, int64_t kw, int64_t waves) {
  (void)kw;
  (void)waves;
  const int G = check_w4(a, qw, qz, sc, "w4gemm");
  const int64_t M = a.size(0), K = a.size(1), N = qw.size(1);
  c10::cuda::CUDAGuard guard(a.device());
  auto y = at::empty({M, N}, a.options());
  const int dev = a.get_device();
  void* ws = workspace(dev);
  const int rc = b2_w4_gemm(a.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), y.data_ptr(),
                            (int)M, (int)K, (int)N, G, ws, b2_workspace_bytes(dev),
                            c10::cuda::getCurrentCUDAStream(dev).stream());
  TORCH_CHECK(rc == B2_OK, "gfx906_skinny.w4gemm: ", detail(rc));
  return y;
}

at::Tensor w4_gemm_meta(const at::Tensor& a, const at::Tensor& qw, const at::Tensor& qz,
                        const at::Tensor& sc, int64_t kw, int64_t waves) {
  (void)qz, (void)sc, (void)kw, (void)waves;
  return at::empty({a.size(0), qw.size(1)}, a.options());
}

// ------------------------------------------------------------------------------------------------
// Load-time repack (no counterpart in the reference). w4_repack(qw, qz, sc) returns the packed
// uint8 image of b2_w4_repack; w4gemm_packed(a, packed, N, group_size) is w4gemm on that image.
// The image is opaque, so N and the group size travel with the call; K is a.size(1).
// ------------------------------------------------------------------------------------------------
at::Tensor w4_repack(const at::Tensor& qw, const at::Tensor& qz, const at::Tensor& sc) {
  check_cuda_half(sc, "w4_repack", "sc");
  TORCH_CHECK(qw.is_cuda() && qz.is_cuda(), "w4_repack: qw and qz must be CUDA tensors");
  TORCH_CHECK(qw.scalar_type() == at::kInt && qz.scalar_type() == at::kInt,
              "w4_repack: qw and qz must be int32");
  TORCH_CHECK(qw.is_contiguous() && qz.is_contiguous(), "w4_repack: qw and qz must be contiguous");
  TORCH_CHECK(qw.dim() == 2 && qz.dim() == 2 && sc.dim() == 2, "w4_repack: operands must be 2-D");
  const int64_t K = qw.size(0) * 8, N = qw.size(1);
  TORCH_CHECK(sc.size(0) > 0 && K % sc.size(0) == 0 && sc.size(1) == N,
              "w4_repack: sc must be [K/G, N]; got ", sc.sizes());
  TORCH_CHECK(qz.size(0) == sc.size(0) && qz.size(1) * 8 == N,
              "w4_repack: qz must be [K/G, N/8]; got ", qz.sizes());
  const int G = (int)(K / sc.size(0));
  const size_t bytes = b2_w4_packed_bytes((int)K, (int)N, G);
  TORCH_CHECK(bytes > 0, "w4_repack: K=", K, " N=", N, " G=", G, " outside the W4 contract");
  c10::cuda::CUDAGuard guard(qw.device());
  auto out = at::empty({(int64_t)bytes}, qw.options().dtype(at::kByte));
  const int rc = b2_w4_repack(qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), (int)K, (int)N, G,
                              out.data_ptr(), bytes,
                              c10::cuda::getCurrentCUDAStream(qw.get_device()).stream());
  TORCH_CHECK(rc == B2_OK, "gfx906_skinny.w4_repack: ", detail(rc));
  return out;
}

void check_packed(const at::Tensor& a, const at::Tensor& packed, int64_t N, int64_t group_size,
                  const char* op) {
  check_cuda_half(a, op, "a");
  TORCH_CHECK(packed.is_cuda() && packed.scalar_type() == at::kByte && packed.is_contiguous() &&
                  packed.dim() == 1,
              op, ": packed must be the contiguous uint8 tensor w4_repack returns");
  TORCH_CHECK(packed.device() == a.device(), op, ": a and packed on different devices");
  TORCH_CHECK(a.dim() == 2, op, ": a must be 2-D");
  const int64_t M = a.size(0), K = a.size(1);
  TORCH_CHECK(M >= 1 && M <= 8, op, ": M=", M, " outside 1..8");
  const size_t bytes = b2_w4_packed_bytes((int)K, (int)N, (int)group_size);
  TORCH_CHECK(bytes > 0 && (size_t)packed.numel() >= bytes, op, ": packed holds ",
              packed.numel(), " bytes; K=", K, " N=", N, " G=", group_size, " needs ", bytes);
}

at::Tensor w4_gemm_packed(const at::Tensor& a, const at::Tensor& packed, int64_t N,
                          int64_t group_size) {
  check_packed(a, packed, N, group_size, "w4gemm_packed");
  const int64_t M = a.size(0), K = a.size(1);
  c10::cuda::CUDAGuard guard(a.device());
  auto y = at::empty({M, N}, a.options());
  const int dev = a.get_device();
  void* ws = workspace(dev);
  const int rc = b2_w4_gemm_packed(a.data_ptr(), packed.data_ptr(), y.data_ptr(), (int)M, (int)K,
                                   (int)N, (int)group_size, ws, b2_workspace_bytes(dev),
                                   c10::cuda::getCurrentCUDAStream(dev).stream());
  TORCH_CHECK(rc == B2_OK, "gfx906_skinny.w4gemm_packed: ", detail(rc));
  return y;
}

at::Tensor w4_repack_meta(const at::Tensor& qw, const at::Tensor& qz, const at::Tensor& sc) {
  (void)qz;
  const int64_t K = qw.size(0) * 8, N = qw.size(1);
  TORCH_CHECK(sc.size(0) > 0 && K % sc.size(0) == 0, "w4_repack: sc must be [K/G, N]");
  const size_t bytes = b2_w4_packed_bytes((int)K, (int)N, (int)(K / sc.size(0)));
  TORCH_CHECK(bytes > 0, "w4_repack: K=", K, " N=", N, " outside the W4 contract");
  return at::empty({(int64_t)bytes}, qw.options().dtype(at::kByte));
}

at::Tensor w4_gemm_packed_meta(const at::Tensor& a, const at::Tensor& packed, int64_t N,
                               int64_t group_size) {
  (void)packed, (void)group_size;
  return at::empty({a.size(0), N}, a.options());
}

// ------------------------------------------------------------------------------------------------
// All-reduce handles. hostar_* keep the reference's two-rank contract (kernels/hostar.cu:114-153,
// patches/vllm/gfx906_host_allreduce.py:22-48): the creator is rank 0, the process that attaches
// is rank 1, `rank` is passed again at every call. nvar_* generalise it to `world` ranks.
// Handles are indices into a process-wide table; the buffers live until the process exits.
// ------------------------------------------------------------------------------------------------
struct ArEntry {
  b2_nvar* ar = nullptr;
  b2_registry* reg = nullptr;
  int rank = 0;
  int world = 0;
};
std::mutex g_ar_mu;
std::vector<ArEntry> g_ars;

int64_t nvar_create_impl(const std::string& name, int64_t slot_bytes, int64_t rank, int64_t world,
                         bool create_registry) {
  TORCH_CHECK(world >= 1 && world <= 8 && rank >= 0 && rank < world, "nvar_create: rank ", rank,
              " world ", world);
  TORCH_CHECK(slot_bytes >= 16, "nvar_create: slot_bytes ", slot_bytes);
  int dev = 0;
  TORCH_CHECK(cudaGetDevice(&dev) == cudaSuccess, "nvar_create: no current CUDA device");
  ArEntry e;
  e.rank = (int)rank;
  e.world = (int)world;
  int rc = b2_registry_open(name.c_str(), (int)world, create_registry ? 1 : 0, &e.reg);
  TORCH_CHECK(rc == B2_OK, "nvar_create: ", detail(rc));
  rc = b2_nvar_create(dev, (int)rank, (int)world, (size_t)slot_bytes, &e.ar);
  TORCH_CHECK(rc == B2_OK, "nvar_create: ", detail(rc));
  unsigned char blob[B2_BLOB_BYTES];
  rc = b2_nvar_export(e.ar, blob);
  TORCH_CHECK(rc == B2_OK, "nvar_create: ", detail(rc));
  rc = b2_registry_put(e.reg, (int)rank, blob);
  TORCH_CHECK(rc == B2_OK, "nvar_create: ", detail(rc));
  std::lock_guard<std::mutex> lk(g_ar_mu);
  g_ars.push_back(e);
  return (int64_t)g_ars.size() - 1;
}

// Map every peer's buffer once all ranks have published (idempotent).
ArEntry& connected_entry(int64_t handle, const char* op) {
  std::lock_guard<std::mutex> lk(g_ar_mu);
  TORCH_CHECK(handle >= 0 && handle < (int64_t)g_ars.size(), op, ": bad handle ", handle);
  ArEntry& e = g_ars[handle];
  if (!b2_nvar_is_connected(e.ar)) {
    std::vector<unsigned char> all((size_t)e.world * B2_BLOB_BYTES);
    for (int r = 0; r < e.world; ++r) {
      const int rc = b2_registry_get(e.reg, r, all.data() + (size_t)r * B2_BLOB_BYTES);
      TORCH_CHECK(rc == B2_OK, op, ": rank ", r, " has not joined the all-reduce yet: ", detail(rc));
    }
    const int rc = b2_nvar_connect(e.ar, all.data());
    TORCH_CHECK(rc == B2_OK, op, ": ", detail(rc));
  }
  return e;
}

int64_t nvar_create(std::string name, int64_t slot_bytes, int64_t rank, int64_t world) {
  return nvar_create_impl(name, slot_bytes, rank, world, rank == 0);
}

void nvar_connect(int64_t handle) { (void)connected_entry(handle, "nvar_connect"); }

int64_t hostar_create(std::string name, int64_t slot_bytes, bool create) {
  // Two ranks: the creator is rank 0, the one that attaches is rank 1.
  const int64_t h = nvar_create_impl(name, slot_bytes, create ? 0 : 1, 2, create);
  if (!create) nvar_connect(h);  // rank 0 published before rank 1 attached
  return h;
}

void hostar_unlink(std::string name) { b2_registry_unlink(name.c_str()); }

int64_t hostar_max_bytes() { return 128 * 1024; }

at::Tensor nvar_allreduce_impl(const at::Tensor& inp, int64_t handle, const char* op) {
  TORCH_CHECK(inp.is_cuda() && inp.is_contiguous(), op, ": input must be a contiguous CUDA tensor");
  TORCH_CHECK(inp.scalar_type() == at::kHalf || inp.scalar_type() == at::kFloat, op,
              ": input must be float16 or float32");
  ArEntry& e = connected_entry(handle, op);
  c10::cuda::CUDAGuard guard(inp.device());
  auto out = at::empty_like(inp);
  const int dt = inp.scalar_type() == at::kHalf ? B2_DTYPE_F16 : B2_DTYPE_F32;
  const int rc = b2_nvar_allreduce(e.ar, inp.data_ptr(), out.data_ptr(), (size_t)inp.numel(), dt,
                                   c10::cuda::getCurrentCUDAStream(inp.get_device()).stream());
  TORCH_CHECK(rc == B2_OK, "gfx906_skinny.", op, ": ", detail(rc));
  return out;
}

at::Tensor hostar_allreduce(const at::Tensor& inp, int64_t handle, int64_t rank) {
  ArEntry& e = connected_entry(handle, "hostar_allreduce");
  TORCH_CHECK(rank == e.rank, "hostar_allreduce: rank ", rank, " does not match the handle's rank ",
              e.rank);
  return nvar_allreduce_impl(inp, handle, "hostar_allreduce");
}

at::Tensor nvar_allreduce(const at::Tensor& inp, int64_t handle) {
  return nvar_allreduce_impl(inp, handle, "nvar_allreduce");
}

at::Tensor w4gemm_ar(const at::Tensor& a, const at::Tensor& qw, const at::Tensor& qz,
                     const at::Tensor& sc, int64_t handle) {
  const int G = check_w4(a, qw, qz, sc, "w4gemm_ar");
  ArEntry& e = connected_entry(handle, "w4gemm_ar");
  const int64_t M = a.size(0), K = a.size(1), N = qw.size(1);
  c10::cuda::CUDAGuard guard(a.device());
  auto y = at::empty({M, N}, a.options());
  const int dev = a.get_device();
  void* ws = workspace(dev);
  const int rc = b2_w4_gemm_allreduce(e.ar, a.data_ptr(), qw.data_ptr(), qz.data_ptr(),
                                      sc.data_ptr(), y.data_ptr(), (int)M, (int)K, (int)N, G, ws,
                                      b2_workspace_bytes(dev),
                                      c10::cuda::getCurrentCUDAStream(dev).stream());
  TORCH_CHECK(rc == B2_OK, "gfx906_skinny.w4gemm_ar: ", detail(rc));
  return y;
}

// w4gemm_ar followed, in the same call, by vLLM's fused residual add + RMSNorm
// (b2_w4_gemm_allreduce_rmsnorm): `residual` becomes residual + all-reduced rows, in place, and
// the normalised rows are returned.
at::Tensor w4gemm_ar_rmsnorm(const at::Tensor& a, const at::Tensor& qw, const at::Tensor& qz,
                             const at::Tensor& sc, int64_t handle, at::Tensor& residual,
                             const at::Tensor& weight, double eps) {
  const char* op = "w4gemm_ar_rmsnorm";
  const int G = check_w4(a, qw, qz, sc, op);
  check_cuda_half(residual, op, "residual");
  check_cuda_half(weight, op, "weight");
  const int64_t M = a.size(0), K = a.size(1), N = qw.size(1);
  TORCH_CHECK(residual.dim() == 2 && residual.size(0) == M && residual.size(1) == N, op,
              ": residual must be [M, N]; got ", residual.sizes());
  TORCH_CHECK(weight.dim() == 1 && weight.size(0) == N, op, ": weight must be [N]; got ",
              weight.sizes());
  TORCH_CHECK(residual.device() == a.device() && weight.device() == a.device(), op,
              ": residual and weight must be on the input's device");
  ArEntry& e = connected_entry(handle, op);
  c10::cuda::CUDAGuard guard(a.device());
  auto y = at::empty({M, N}, a.options());
  const int dev = a.get_device();
  void* ws = workspace(dev);
  const int rc = b2_w4_gemm_allreduce_rmsnorm(
      e.ar, a.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), residual.data_ptr(),
      weight.data_ptr(), (float)eps, y.data_ptr(), (int)M, (int)K, (int)N, G, ws,
      b2_workspace_bytes(dev), c10::cuda::getCurrentCUDAStream(dev).stream());
  TORCH_CHECK(rc == B2_OK, "gfx906_skinny.w4gemm_ar_rmsnorm: ", detail(rc));
  return y;
}

// w4gemm_ar and w4gemm_ar_rmsnorm on weights repacked by w4_repack
at::Tensor w4gemm_ar_packed(const at::Tensor& a, const at::Tensor& packed, int64_t N,
                            int64_t group_size, int64_t handle) {
  check_packed(a, packed, N, group_size, "w4gemm_ar_packed");
  ArEntry& e = connected_entry(handle, "w4gemm_ar_packed");
  const int64_t M = a.size(0), K = a.size(1);
  c10::cuda::CUDAGuard guard(a.device());
  auto y = at::empty({M, N}, a.options());
  const int dev = a.get_device();
  void* ws = workspace(dev);
  const int rc = b2_w4_gemm_allreduce_packed(e.ar, a.data_ptr(), packed.data_ptr(), y.data_ptr(),
                                             (int)M, (int)K, (int)N, (int)group_size, ws,
                                             b2_workspace_bytes(dev),
                                             c10::cuda::getCurrentCUDAStream(dev).stream());
  TORCH_CHECK(rc == B2_OK, "gfx906_skinny.w4gemm_ar_packed: ", detail(rc));
  return y;
}

at::Tensor w4gemm_ar_rmsnorm_packed(const at::Tensor& a, const at::Tensor& packed, int64_t N,
                                    int64_t group_size, int64_t handle, at::Tensor& residual,
                                    const at::Tensor& weight, double eps) {
  const char* op = "w4gemm_ar_rmsnorm_packed";
  check_packed(a, packed, N, group_size, op);
  check_cuda_half(residual, op, "residual");
  check_cuda_half(weight, op, "weight");
  const int64_t M = a.size(0), K = a.size(1);
  TORCH_CHECK(residual.dim() == 2 && residual.size(0) == M && residual.size(1) == N, op,
              ": residual must be [M, N]; got ", residual.sizes());
  TORCH_CHECK(weight.dim() == 1 && weight.size(0) == N, op, ": weight must be [N]; got ",
              weight.sizes());
  TORCH_CHECK(residual.device() == a.device() && weight.device() == a.device(), op,
              ": residual and weight must be on the input's device");
  ArEntry& e = connected_entry(handle, op);
  c10::cuda::CUDAGuard guard(a.device());
  auto y = at::empty({M, N}, a.options());
  const int dev = a.get_device();
  void* ws = workspace(dev);
  const int rc = b2_w4_gemm_allreduce_rmsnorm_packed(
      e.ar, a.data_ptr(), packed.data_ptr(), residual.data_ptr(), weight.data_ptr(), (float)eps,
      y.data_ptr(), (int)M, (int)K, (int)N, (int)group_size, ws, b2_workspace_bytes(dev),
      c10::cuda::getCurrentCUDAStream(dev).stream());
  TORCH_CHECK(rc == B2_OK, "gfx906_skinny.w4gemm_ar_rmsnorm_packed: ", detail(rc));
  return y;
}

int64_t nvar_status(int64_t handle, bool clear) {
  ArEntry* e;
  {
    std::lock_guard<std::mutex> lk(g_ar_mu);
    TORCH_CHECK(handle >= 0 && handle < (int64_t)g_ars.size(), "nvar_status: bad handle ", handle);
    e = &g_ars[handle];
  }
  int st = 0;
  const int rc = b2_nvar_status(e->ar, clear ? 1 : 0, &st);
  TORCH_CHECK(rc == B2_OK, "nvar_status: ", detail(rc));
  return st;
}

void nvar_set_timeout_ms(int64_t handle, int64_t ms) {
  std::lock_guard<std::mutex> lk(g_ar_mu);
  TORCH_CHECK(handle >= 0 && handle < (int64_t)g_ars.size(), "nvar_set_timeout_ms: bad handle");
  const int rc = b2_nvar_set_timeout_ns(g_ars[handle].ar, (uint64_t)ms * 1000000ull);
  TORCH_CHECK(rc == B2_OK, "nvar_set_timeout_ms: ", detail(rc));
}

// Status word of the current device's GEMM workspace (synchronises the device).
int64_t workspace_status(bool clear) {
  int dev = 0;
  TORCH_CHECK(cudaGetDevice(&dev) == cudaSuccess, "workspace_status: no CUDA device");
  void* ws = workspace(dev);
  int st = 0;
  const int rc = b2_workspace_status(ws, clear ? 1 : 0, &st);
  TORCH_CHECK(rc == B2_OK, "workspace_status: ", detail(rc));
  return st;
}

void set_tuning(int64_t key, int64_t value) {
  const int rc = b2_set_tuning((int)key, (int)value);
  TORCH_CHECK(rc == B2_OK, "set_tuning: ", detail(rc));
}

}  // namespace

TORCH_LIBRARY(gfx906_skinny, m) {
  // reference schemas
  m.def("gemm(Tensor x, Tensor w, int variant=0) -> Tensor");
  m.def("w4gemm(Tensor a, Tensor qw, Tensor qz, Tensor sc, int kw, int waves) -> Tensor");
  m.def("hostar_create(str name, int slot_bytes, bool create) -> int");
  m.def("hostar_unlink(str name) -> ()");
  m.def("hostar_max_bytes() -> int");
  m.def("hostar_allreduce(Tensor inp, int handle, int rank) -> Tensor");
  // additions
  m.def("nvar_create(str name, int slot_bytes, int rank, int world) -> int");
  m.def("nvar_connect(int handle) -> ()");
  m.def("nvar_allreduce(Tensor inp, int handle) -> Tensor");
  m.def("w4gemm_ar(Tensor a, Tensor qw, Tensor qz, Tensor sc, int handle) -> Tensor");
  m.def("w4gemm_ar_rmsnorm(Tensor a, Tensor qw, Tensor qz, Tensor sc, int handle, "
        "Tensor(a!) residual, Tensor weight, float eps) -> Tensor");
  m.def("w4_repack(Tensor qw, Tensor qz, Tensor sc) -> Tensor");
  m.def("w4gemm_packed(Tensor a, Tensor packed, int N, int group_size) -> Tensor");
  m.def("w4gemm_ar_packed(Tensor a, Tensor packed, int N, int group_size, int handle) -> Tensor");
  m.def("w4gemm_ar_rmsnorm_packed(Tensor a, Tensor packed, int N, int group_size, int handle, "
        "Tensor(a!) residual, Tensor weight, float eps) -> Tensor");
  m.def("nvar_status(int handle, bool clear=False) -> int");
  m.def("nvar_set_timeout_ms(int handle, int ms) -> ()");
  m.def("workspace_status(bool clear=False) -> int");
  m.def("set_tuning(int key, int value) -> ()");
}

TORCH_LIBRARY_IMPL(gfx906_skinny, CUDA, m) {
  m.impl("gemm", &skinny_gemm);
  m.impl("w4gemm", &w4_gemm);
  m.impl("w4_repack", &w4_repack);
  m.impl("w4gemm_packed", &w4_gemm_packed);
  m.impl("hostar_allreduce", &hostar_allreduce);
  m.impl("nvar_allreduce", &nvar_allreduce);
  m.impl("w4gemm_ar", &w4gemm_ar);
  m.impl("w4gemm_ar_rmsnorm", &w4gemm_ar_rmsnorm);
  m.impl("w4gemm_ar_packed", &w4gemm_ar_packed);
  m.impl("w4gemm_ar_rmsnorm_packed", &w4gemm_ar_rmsnorm_packed);
}

TORCH_LIBRARY_IMPL(gfx906_skinny, Meta, m) {
  m.impl("gemm", &skinny_gemm_meta);
  m.impl("w4gemm", &w4_gemm_meta);
  m.impl("w4_repack", &w4_repack_meta);
  m.impl("w4gemm_packed", &w4_gemm_packed_meta);
}

TORCH_LIBRARY_IMPL(gfx906_skinny, CompositeExplicitAutograd, m) {
  m.impl("hostar_create", &hostar_create);
  m.impl("hostar_unlink", &hostar_unlink);
  m.impl("hostar_max_bytes", &hostar_max_bytes);
  m.impl("nvar_create", &nvar_create);
  m.impl("nvar_connect", &nvar_connect);
  m.impl("nvar_status", &nvar_status);
  m.impl("nvar_set_timeout_ms", &nvar_set_timeout_ms);
  m.impl("workspace_status", &workspace_status);
  m.impl("set_tuning", &set_tuning);
}
