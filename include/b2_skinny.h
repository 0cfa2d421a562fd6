/*
 * b2_skinny.h - C ABI of the B200 (sm_100a) skinny-GEMM library.
 *
 * Speculative decoding verifies k+1 <= 8 tokens per step, so the projections of a
 * verify step are GEMMs with M <= 8 activation rows. They are bound by HBM bandwidth.
 * This library provides, behind plain pointers and sizes:
 *   - an fp16 GEMM        y[M,N] = x[M,K] @ w[N,K]^T                      (b2_gemm_f16)
 *   - a W4A16 GEMM over GPTQ/Exllama-shuffled 4-bit weights                (b2_w4_gemm)
 *   - an all-reduce over NVLink peer memory (one-shot, two-shot from 8 ranks) (b2_nvar_*)
 *   - the W4A16 GEMM with that all-reduce fused into its epilogue          (b2_w4_gemm_allreduce)
 *   - the same, followed in the same launch by the residual add + RMSNorm
 *     of the decoder layer                                        (b2_w4_gemm_allreduce_rmsnorm)
 *   - a load-time repack of the W4 weights and the three W4 entry points above on it
 *     (b2_w4_repack, b2_w4_gemm_packed, b2_w4_gemm_allreduce(_rmsnorm)_packed)
 * Every compute entry point launches on the caller's stream, never synchronises and never
 * allocates, so it can be captured in a CUDA graph.
 *
 * Conventions
 *   - Pointers to device memory are plain `void*`; `stream` is a cudaStream_t (0 = legacy
 *     default stream).
 *   - Every entry point returns a b2 status code (B2_OK == 0). b2_last_error() gives a
 *     one-line detail of the last failure on the calling thread.
 *   - fp16 means IEEE binary16; int4 weights are packed 8 per 32-bit word.
 *
 * Reference interfaces (paths inside the reference project 0c33/mi50-vllm-lab):
 *   kernels/skinny.cu:300-333   gemm(Tensor x, Tensor w, int variant=0) -> Tensor
 *   kernels/w4.cu:477-509       w4gemm(Tensor a, Tensor qw, Tensor qz, Tensor sc, int kw, int waves)
 *   kernels/hostar.cu:114-166   hostar_create / hostar_unlink / hostar_max_bytes / hostar_allreduce
 */
#ifndef B2_SKINNY_H
#define B2_SKINNY_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2_ABI_VERSION 1

/* ------------------------------------------------------------------------------------------
 * Status codes
 * ---------------------------------------------------------------------------------------- */
#define B2_OK 0
#define B2_ERR_INVALID_ARG 1 /* shape, dtype, alignment or pointer outside the contract      */
#define B2_ERR_UNSUPPORTED 2 /* the device is not an sm_100 part, or a needed feature is off */
#define B2_ERR_CUDA 3        /* a CUDA runtime or driver call failed (detail in last_error)  */
#define B2_ERR_WORKSPACE 4   /* workspace missing or smaller than b2_workspace_bytes()       */
#define B2_ERR_TIMEOUT 5     /* a bounded device-side wait gave up (peer never arrived)      */
#define B2_ERR_STATE 6       /* bad handle, or an all-reduce handle that is not connected    */

/* Element types for the all-reduce. */
#define B2_DTYPE_F16 0
#define B2_DTYPE_F32 1

/* Short text for a status code (static storage). */
const char* b2_status_string(int status);
/* Detail of the last failure on this thread (thread-local storage, "" when none). */
const char* b2_last_error(void);
/* B2_ABI_VERSION of the loaded library. */
int b2_abi_version(void);

/* ------------------------------------------------------------------------------------------
 * Workspace
 *
 * The GEMMs split K across CTAs (stream-K). Partial sums go to fp32 slots in a workspace and
 * the last CTA to finish a tile adds them in a fixed order, so results are deterministic.
 * The workspace also holds one self-resetting arrival counter per output tile and a status
 * word. It must be zero-filled once (b2_workspace_init) before its first use; every call
 * leaves the counters at zero again. Calls that share a workspace must not overlap on the
 * GPU (issue them on one stream). Replaces the per-call at::empty split-K buffer of
 * kernels/w4.cu:330-334 and the separate w4_reduce_kernel launch (kernels/w4.cu:154-166).
 *
 * Early launch: b2_gemm_f16 and b2_w4_gemm use programmatic dependent launch. Their CTAs may
 * start while the previous kernel of this library on the stream is finishing; until it has
 * completed they only prefetch their first weight tiles into L2. Every read of operands into
 * the kernel and every write comes after it has completed, so stream order holds as for a plain
 * launch. b2_set_tuning(B2_TUNE_NO_PDL, 1) turns early launch off.
 * ---------------------------------------------------------------------------------------- */

/* Bytes of workspace that cover every supported shape on `device` (fixed per device). */
size_t b2_workspace_bytes(int device);
/* Zero-fill a workspace on `stream` (asynchronous). */
int b2_workspace_init(void* ws, size_t ws_bytes, void* stream);
/* Synchronously read the workspace status word: 0, or the B2_ERR_* code a kernel recorded
 * when one of its bounded waits gave up. Clears the word when `clear` is non-zero. */
int b2_workspace_status(void* ws, int clear, int* device_status);

/* ------------------------------------------------------------------------------------------
 * fp16 skinny GEMM          y[M,N] = x[M,K] @ w[N,K]^T, fp32 accumulation, fp16 output
 *
 * Replaces skinny_gemm (kernels/skinny.cu:300-328, op `gemm`, schema at :331).
 *   x : [M, K] fp16, row-major, 16-byte aligned          1 <= M <= 8
 *   w : [N, K] fp16, row-major (K contiguous), 16-byte aligned, K % 8 == 0
 *   y : [M, N] fp16, row-major (written)
 * ---------------------------------------------------------------------------------------- */
int b2_gemm_f16(const void* x, const void* w, void* y, int M, int K, int N, void* ws,
                size_t ws_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * W4A16 skinny GEMM         y[M,N] = a[M,K] @ dequant(qw, qz, sc)[K,N]
 *
 * Replaces w4_gemm (kernels/w4.cu:479-504, op `w4gemm`, schema at :507). Same layouts as the
 * reference (kernels/w4.cu:477-478, kernels/check_w4.py:11-18):
 *   a  : [M, K] fp16 row-major                                         1 <= M <= 8
 *   qw : [K/8, N] int32. Word (r, n) holds k = 8r..8r+7 of column n: nibble i (bits 4i..4i+3)
 *        is k = 8r+2i and nibble 4+i (bits 16+4i..) is k = 8r+2i+1, for i = 0..3.
 *   qz : [K/G, N/8] int32. Nibble c of word (g, j) is the zero point of column 8j+c ("v2"
 *        format: no +1 offset).
 *   sc : [K/G, N] fp16 scales.
 *   w[k][n] = (q[k][n] - z[k/G][n]) * sc[k/G][n]; fp32 accumulation; fp16 output.
 * Contract: K % 128 == 0, N % 32 == 0, G in {32, 64} or G a multiple of 128, K % G == 0,
 * all pointers 16-byte aligned.
 * ---------------------------------------------------------------------------------------- */
int b2_w4_gemm(const void* a, const void* qw, const void* qz, const void* sc, void* y, int M,
               int K, int N, int group_size, void* ws, size_t ws_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * W4A16 with weights repacked once at load time
 *
 * The reference's loader converts GPTQ checkpoints once, before the first forward
 * (gptq_shuffle at weight-load time); b2_w4_repack is the B200 step that may follow it. It
 * rewrites qw, qz and sc into one buffer in which each 128-column x 128-k unit is a single
 * contiguous run of bytes (its weights in the order the kernels' shared memory holds them, then
 * its scale and zero rows), so a unit is one sequential read from HBM instead of 16 rows of 512 B
 * set N * 4 bytes apart. The product is bit-identical to b2_w4_gemm on the original tensors.
 *   b2_w4_packed_bytes : size of the buffer (0 when K, N, G break b2_w4_gemm's contract).
 *   b2_w4_repack       : qw, qz, sc as for b2_w4_gemm -> out (16-byte aligned, >= that size).
 *                        Asynchronous on `stream`; the inputs may be freed once it completes.
 *   b2_w4_gemm_packed  : b2_w4_gemm with the repacked buffer in place of qw, qz, sc.
 * ---------------------------------------------------------------------------------------- */
size_t b2_w4_packed_bytes(int K, int N, int group_size);
int b2_w4_repack(const void* qw, const void* qz, const void* sc, int K, int N, int group_size,
                 void* out, size_t out_bytes, void* stream);
int b2_w4_gemm_packed(const void* a, const void* packed, void* y, int M, int K, int N,
                      int group_size, void* ws, size_t ws_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * W4A16 skinny GEMM that allocates nothing (no counterpart in the reference)
 *
 * Same operands, layouts, contract and results as b2_w4_gemm, but without the workspace
 * argument: its split-K scratch is a fixed 2,113,792-byte array in device memory that the
 * library reserves on every GPU it is loaded on and keeps until the process exits. It is for
 * callers that cannot allocate device memory at the point of the call: hosts whose device
 * memory belongs to a pool or allocator they cannot reach from where they call this (an FFI or
 * JNI binding, an embedded runtime), code that must not risk the device-wide synchronisation or
 * failure of a cudaMalloc in the middle of a decode step, and code that cannot keep a
 * workspace alive between calls. This entry point calls no cudaMalloc, cudaFree or other
 * allocating routine.
 *   - Limit: N <= 524288 (4096 output tiles of 128 columns); larger N is rejected with
 *     B2_ERR_INVALID_ARG. When the shape's plan is stream-K its grid is capped at 256 CTAs (the
 *     array's partial slots); when the plan is the thread-block-cluster kernel, which reduces
 *     through distributed shared memory and uses none of the array, the call launches exactly as
 *     b2_w4_gemm does.
 *   - The first call in a CUDA context (per device; for runtime-API callers the device's primary
 *     context) looks up the array's device address with cudaGetSymbolAddress. Make that first
 *     call before any CUDA graph capture: inside a capture it fails with B2_ERR_STATE. A call from
 *     another context, or after cudaDeviceReset, looks the address up again.
 *   - A stream-K call clears the array's status word and the tile counters it uses on `stream`
 *     (cudaMemsetAsync) before its kernel, so it never depends on what an earlier call left.
 *   - All calls on a device share the one array: calls that can overlap on the GPU (different
 *     streams, or graphs replayed concurrently) race and give wrong results. Issue them in order.
 *   - A device-side wait that gives up is recorded only in the array, which no entry point
 *     reads; use b2_w4_gemm with b2_workspace_status where that report is needed.
 * ---------------------------------------------------------------------------------------- */
int b2_w4_gemm_noalloc(const void* a, const void* qw, const void* qz, const void* sc, void* y,
                       int M, int K, int N, int group_size, void* stream);
/* Device address and size of that fixed array on the current device (the address
 * b2_w4_gemm_noalloc passes to its kernels), for diagnostics and tests. Same set-up rule as the
 * first b2_w4_gemm_noalloc call: not inside a stream capture. No counterpart in the reference. */
int b2_w4_noalloc_scratch(void** device_ptr, size_t* bytes);

/* ------------------------------------------------------------------------------------------
 * Host-side rendezvous registry (POSIX shared memory, no GPU needed)
 *
 * Ranks of one node publish fixed-size blobs (CUDA IPC handles) under a shared-memory name and
 * read each other's. Generalises the shm_open/mmap set-up of hostar_create
 * (kernels/hostar.cu:114-134) from two ranks to `world` ranks.
 * ---------------------------------------------------------------------------------------- */
#define B2_BLOB_BYTES 64
typedef struct b2_registry b2_registry;
int b2_registry_open(const char* name, int world, int create, b2_registry** out);
int b2_registry_put(b2_registry* reg, int rank, const void* blob);
/* B2_ERR_STATE when `rank` has not published yet. */
int b2_registry_get(b2_registry* reg, int rank, void* blob_out);
int b2_registry_close(b2_registry* reg);
/* Replaces hostar_unlink (kernels/hostar.cu:136). */
int b2_registry_unlink(const char* name);

/* ------------------------------------------------------------------------------------------
 * NVLink one-shot all-reduce (replaces the host-memory all-reduce of kernels/hostar.cu)
 *
 * Each rank owns a device buffer: a generation counter, per-rank flags and two
 * parity-alternating sets of `world` data slots (allocated at 4x `slot_bytes`). A call pushes
 * this rank's data into its slot on every peer over NVLink, publishes a flag with release
 * semantics, waits (bounded) for all peers' flags and sums the `world` slots in rank order
 * 0..world-1 in fp32. The fused GEMM (b2_w4_gemm_allreduce) instead sends 64-bit
 * (generation, fp32 value) words that need no flag and no fence. Every rank
 * therefore computes bit-identical results. The generation lives on the device, so calls can
 * be replayed from a CUDA graph (same protocol as kernels/hostar.cu:9-14, generalised to
 * `world` ranks). No TMA, no multicast.
 * ---------------------------------------------------------------------------------------- */
typedef struct b2_nvar b2_nvar;
#define B2_IPC_HANDLE_BYTES 64
/* Allocate this rank's buffer on `device` (`slot_bytes` = largest payload per call). */
int b2_nvar_create(int device, int rank, int world, size_t slot_bytes, b2_nvar** out);
/* Write this rank's CUDA IPC handle (B2_IPC_HANDLE_BYTES). */
int b2_nvar_export(const b2_nvar* ar, void* handle_out);
/* Map the peers' buffers; `handles` holds world * B2_IPC_HANDLE_BYTES in rank order. */
int b2_nvar_connect(b2_nvar* ar, const void* handles);
int b2_nvar_is_connected(const b2_nvar* ar);
/* Largest payload in bytes per call (replaces hostar_max_bytes, kernels/hostar.cu:138). */
size_t b2_nvar_max_bytes(const b2_nvar* ar);
/* Bound on each device-side wait for a peer, in nanoseconds (default 10 s). */
int b2_nvar_set_timeout_ns(b2_nvar* ar, uint64_t ns);
/* out = sum over ranks of in; `count` elements of `dtype`; count * size % 16 == 0.
 * Replaces hostar_allreduce (kernels/hostar.cu:140-153). `in` and `out` may alias. */
int b2_nvar_allreduce(b2_nvar* ar, const void* in, void* out, size_t count, int dtype,
                      void* stream);
/* Row-parallel W4A16 layer: y = allreduce_over_ranks(a_rank @ dequant(qw_rank, ...)), with the
 * all-reduce fused into the GEMM epilogue. Each rank passes its K-shard; M, N, G match on all
 * ranks, and so does the tuning (the ranks must choose the same split-K plan). The fp32 partial
 * sums cross NVLink as 64-bit (generation, value) words; they are added in rank order, so the
 * fp16 result is bit-identical on every rank. The handle's slot must hold M * N * 4 bytes. */
int b2_w4_gemm_allreduce(b2_nvar* ar, const void* a, const void* qw, const void* qz,
                         const void* sc, void* y, int M, int K, int N, int group_size, void* ws,
                         size_t ws_bytes, void* stream);
/* The same layer followed, in the same call, by the residual add + RMSNorm that the decoder
 * layer runs on the all-reduced output (vLLM's fused_add_rms_norm, vllm/ir/ops/layernorm.py:40-60
 * in vLLM 0.22; no counterpart in the reference's library):
 *   s        = allreduce_over_ranks(a_rank @ dequant(qw_rank, ...))     as b2_w4_gemm_allreduce
 *   x        = float(fp16(s)) + float(residual)                         fp32
 *   residual <- fp16(x)                                                 in place
 *   y        = fp16(fp16(x * rsqrt(sum_n(x^2) / N + eps)) * norm_weight[n])
 * residual : [M, N] fp16, read and written; norm_weight : [N] fp16; both 8-byte aligned, and
 * y, residual and norm_weight must not overlap. 0 <= eps <= 1. The row sums are added in a fixed
 * order, so y and residual are bit-identical on every rank and from call to call. Two launches on
 * `stream`: the fused GEMM + all-reduce, which also stores its CTAs' row sums of squares, then a
 * short kernel that adds them and writes residual and y (both may start early, as programmatic
 * dependent launches). B2_TUNE_NORM_IN_LAUNCH keeps it to one launch: the GEMM's last cluster
 * finishes the rows, or, in the stream-K kernel, one grid-wide barrier (bounded by the handle's
 * timeout; B2_ERR_TIMEOUT in the handle's status if it gives up) in a cooperative launch. */
int b2_w4_gemm_allreduce_rmsnorm(b2_nvar* ar, const void* a, const void* qw, const void* qz,
                                 const void* sc, void* residual, const void* norm_weight,
                                 float eps, void* y, int M, int K, int N, int group_size,
                                 void* ws, size_t ws_bytes, void* stream);
/* The two fused layers on weights repacked by b2_w4_repack (`packed` in place of qw, qz, sc);
 * the same contract and the same bits as the calls above on the original tensors. */
int b2_w4_gemm_allreduce_packed(b2_nvar* ar, const void* a, const void* packed, void* y, int M,
                                int K, int N, int group_size, void* ws, size_t ws_bytes,
                                void* stream);
int b2_w4_gemm_allreduce_rmsnorm_packed(b2_nvar* ar, const void* a, const void* packed,
                                        void* residual, const void* norm_weight, float eps,
                                        void* y, int M, int K, int N, int group_size, void* ws,
                                        size_t ws_bytes, void* stream);
/* Synchronously read the device error word of the handle (0 or B2_ERR_TIMEOUT). Clearing a
 * timeout also resets the grid-wide barrier count of b2_w4_gemm_allreduce_rmsnorm, which a
 * launch that gave up may have left behind: clear it before the next call. */
int b2_nvar_status(b2_nvar* ar, int clear, int* device_status);
int b2_nvar_rank(const b2_nvar* ar);
int b2_nvar_world(const b2_nvar* ar);
int b2_nvar_destroy(b2_nvar* ar);

/* ------------------------------------------------------------------------------------------
 * Several ranks of one tensor-parallel group emulated on one GPU (testing support; no counterpart
 * in the reference)
 *
 * The multi-rank exchange of the all-reduce and of the fused GEMM epilogues can be exercised on a
 * machine with one GPU: `ranks` handles created in one process on one device (b2_nvar_create with
 * rank r of world `ranks`, r = 0..ranks-1) are connected to one another's buffers directly, and
 * one launch runs every rank's CTAs (grid.y = rank), each rank with its own operands, workspace
 * and handle. The ranks' CTAs wait for one another, so the launch is cooperative: either all of
 * them are resident at once or the launch fails (B2_ERR_CUDA); each rank's grid is planned on
 * 1/ranks of the GPU. Results are those of `ranks` GPUs running the ordinary entry points, except
 * that the split-K plan (and so the fp32 rounding of the partial sums) is that of a GPU with
 * 1/ranks of the SMs. 1 <= ranks <= 4.
 * ---------------------------------------------------------------------------------------- */
/* Connect handles[0..ranks-1] (rank r = handles[r], all on one device) to one another. */
int b2_nvar_connect_local(b2_nvar* const* handles, int ranks);
/* b2_nvar_allreduce of every rank in one launch: out[r] = sum over ranks of in[q] (rank order). */
int b2_nvar_allreduce_emulated(b2_nvar* const* handles, int ranks, const void* const* in,
                               void* const* out, size_t count, int dtype, void* stream);
/* b2_w4_gemm_allreduce (residual == norm_weight == NULL) or b2_w4_gemm_allreduce_rmsnorm of every
 * rank in one launch; every array holds one pointer per rank. */
int b2_w4_gemm_allreduce_emulated(b2_nvar* const* handles, int ranks, const void* const* a,
                                  const void* const* qw, const void* const* qz,
                                  const void* const* sc, void* const* residual,
                                  const void* const* norm_weight, float eps, void* const* y, int M,
                                  int K, int N, int group_size, void* const* ws, size_t ws_bytes,
                                  void* stream);

/* ------------------------------------------------------------------------------------------
 * Tuning (process-wide; for measurement sweeps). B2_TUNE="key=value,..." in the environment
 * presets keys before first use; b2_set_tuning overrides them.
 * ---------------------------------------------------------------------------------------- */
#define B2_TUNE_CTAS_PER_SM 1     /* resident CTAs per SM the stream-K grid targets (0 = auto) */
#define B2_TUNE_MIN_UNITS 2       /* fewest k-units per CTA before the grid shrinks (0 = auto)  */
#define B2_TUNE_NO_PDL 3          /* nonzero: launch every kernel only after the previous one has
                                     finished (no programmatic dependent launch)                 */
#define B2_TUNE_W4_PATH 4         /* W4 split-K: 0 = choose per shape, 1 = stream-K with a global
                                     fix-up, 2 = thread-block clusters reducing through
                                     distributed shared memory                                   */
#define B2_TUNE_W4_CLUSTER 5      /* cluster path: CTAs per cluster (0 = chosen per shape)      */
#define B2_TUNE_AR_FLAGS 6        /* fused all-reduce: nonzero sends fp32 values published by
                                     per-tile flags instead of 64-bit (generation, value) words  */
#define B2_TUNE_AR_TWO_SHOT 7     /* fused all-reduce in the cluster kernel: 0 = two-shot from 8
                                     ranks up (each tile reduced at one owner rank, the result
                                     sent back), 1 = always two-shot, 2 = always one-shot        */
#define B2_TUNE_W4_NO_ALIAS 8     /* cluster path, G >= 128, no exchange: when every cluster has
                                     one output tile and every CTA at least 16 k-units, its
                                     reduction buffers take the place of the drained stage ring,
                                     which leaves room for a fifth stage; nonzero keeps them
                                     apart (four stages)                                         */
#define B2_TUNE_NORM_NO_COOP 9    /* nonzero: launch the stream-K kernel's fused RMSNorm (its
                                     grid-wide barrier) without the cooperative attribute, so
                                     that residency rests on the grid size alone                */
#define B2_TUNE_NORM_IN_LAUNCH 10  /* nonzero: the fused RMSNorm runs entirely inside the GEMM's
                                     launch (the last cluster, or the stream-K grid after a
                                     grid-wide barrier, finishes the rows) instead of in a short
                                     finishing launch that follows it on the stream             */
int b2_set_tuning(int key, int value);
int b2_get_tuning(int key);

/* The split-K plan that b2_w4_gemm (fused == 0) or b2_w4_gemm_allreduce with the 64-bit exchange
 * (fused != 0) would launch for this shape on the current device, under the current tuning:
 * *path = 1 (stream-K, kernel w4_kernel) or 2 (thread-block clusters, kernel w4c_kernel),
 * *cluster = CTAs per cluster (0 for stream-K), *ctas = CTAs of the grid. For benchmarks and
 * profiles, which name the kernel they time. No counterpart in the reference, whose grid is fixed
 * by its kw and waves arguments (kernels/w4.cu:489-500). */
int b2_w4_plan(int M, int K, int N, int group_size, int fused, int* path, int* cluster, int* ctas);

#ifdef __cplusplus
}
#endif

#endif /* B2_SKINNY_H */
