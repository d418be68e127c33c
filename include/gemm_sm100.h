/*
 * gemm_sm100.h -- C ABI of libgemm_sm100.so, the B200 (sm_100a) matmul
 * backend for php-gpu-tensors.
 *
 * The first block is a drop-in for the reference's native matmul boundary:
 * identical types, names, argument meaning and return conventions as
 *   src/backends/cuda/matmul_kernels.h:8-57   (launchers, precision, tuning)
 *   src/backends/cuda/backend_info.h:7-16     (cuda_backend_info, cuda_blas_info)
 * so src/cuda_array/ca_private.c:1127-1137,1195-1200, src/fusion_execute.c:
 * 159-173 and src/cuda.c:136-290 link against it unchanged.  The second block
 * is additive (FP64, fused epilogue, diagnostics, multi-GPU).
 *
 * Conventions (all entry points):
 *   - a, b, c, bias are DEVICE pointers owned by the caller; shape/stride
 *     arrays are HOST memory read during the call only (matmul_kernels.h:46).
 *   - strides are in ELEMENTS; a view's offset is folded into its pointer.
 *   - launchers return 1 on success and 0 on failure; on a CUDA failure
 *     cuda_blas_info().last_blas_status carries the cudaError_t (or a
 *     GEMM_SM100_STATUS_* code).  Degenerate extents (M or N or a batch extent
 *     of 0) return 1 without a launch; K == 0 writes zeros.
 *   - work is enqueued asynchronously on `stream` (NULL = legacy default
 *     stream); launchers never allocate, synchronise or read device memory,
 *     so they can be captured into CUDA graphs after the first call on a
 *     device (which performs one-time per-device set-up).
 *   - precision mode, counters and tuning plans are per host thread.
 *
 * When building inside the php-gpu-tensors extension, include the
 * extension's data_types.h, backend_info.h and matmul_kernels.h first; the
 * shared declarations below are then skipped by their include guards.
 */
#ifndef PT_GEMM_SM100_H
#define PT_GEMM_SM100_H

#include <stddef.h>
#include <cuda_runtime_api.h>

#ifndef DATA_TYPES_H
/* Same enumerators and values as the reference's dtype_t (src/data_types.h:8-27). */
typedef enum {
    DTYPE_FLOAT32,
    DTYPE_FLOAT64,
    DTYPE_INT8,
    DTYPE_INT16,
    DTYPE_INT32,
    DTYPE_INT64,
    DTYPE_UINT8,
    DTYPE_UINT16,
    DTYPE_UINT32,
    DTYPE_UINT64,
    DTYPE_BOOL,
    DTYPE_FLOAT16,
    DTYPE_BFLOAT16,
    DTYPE_UNKNOWN,
    DTYPE_COUNT,
    DTYPE_LIST,
    DTYPE_VOID
} dtype_t;
#endif

#ifndef MAX_DIMS
#define MAX_DIMS 10 /* src/tensor.h:16 */
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ */
/* Drop-in block: src/backends/cuda/backend_info.h:7-16               */
/* ------------------------------------------------------------------ */
#ifndef CUDA_BACKEND_INFO_H
#define CUDA_BACKEND_INFO_H
typedef struct {
    int cublas, cublas_lt, cudnn;
    unsigned long long blas_calls, lt_calls, builtin_matmul_calls;
    unsigned long long cub_calls, axis_calls, generic_reduce_calls;
    const char *last_matmul;
    const char *precision;
    int last_blas_status;
} cuda_backend_info;
#endif

/* Replaces backend_info.h:15.  Fills the matmul fields: cublas = cublas_lt =
 * 0 (this library contains no cuBLAS), builtin_matmul_calls counts launches,
 * last_matmul is "builtin" (float32), "builtin-low-precision" (float16 /
 * bfloat16) or "builtin-f64", precision is the thread's mode, last_blas_status
 * the last error code.  cudnn and the reduction counters are left untouched. */
void cuda_blas_info(cuda_backend_info *info);

/* ------------------------------------------------------------------ */
/* Drop-in block: src/backends/cuda/matmul_kernels.h:8-57             */
/* ------------------------------------------------------------------ */
#ifndef MATMUL_KERNELS_H
#define MATMUL_KERNELS_H

enum {
    CUDA_MATMUL_PRECISION_FP32_STRICT = 0, /* float32 via 3xTF32 tensor-core split */
    CUDA_MATMUL_PRECISION_TF32 = 1         /* float32 via one TF32 pass */
};

#define CUDA_MATMUL_TUNING_MAX_CANDIDATES 8

typedef struct {
    int algorithm_id;
    size_t workspace_bytes;
    double median_ms;
} cuda_matmul_tuning_candidate;

typedef struct {
    int candidate_count;
    int selected_candidate;
    cuda_matmul_tuning_candidate candidates[CUDA_MATMUL_TUNING_MAX_CANDIDATES];
} cuda_matmul_tuning_result;

#endif /* MATMUL_KERNELS_H */

/* matmul_kernels.h:31.  Clears this thread's counters and tuning plans. */
void cuda_blas_shutdown(void);

/* matmul_kernels.h:32.  Returns 1 and sets the thread's float32 mode, or 0
 * for an unknown mode.
 * Non-finite inputs in the strict mode: the tensor-core kernels form float32
 * products from split operands (hi*hi + hi*lo + lo*hi; for float32 x
 * bfloat16 gradients three bf16 parts of the float32 operand), so an infinite
 * element meets the zero low part of the other operand's element in a cross
 * term (inf * 0 = NaN): a dot product that involves an infinite input can
 * come out NaN where the IEEE float32 loop of HostArray::matmul gives +-Inf.
 * Finite inputs and NaN inputs behave as in that loop (within its error
 * bound; NaN propagates).  gemm_sm100_set_path(2) runs the CUDA-core kernel,
 * whose fma chains equal the loop bit for bit, for callers that need IEEE
 * infinities. */
int cuda_blas_set_precision(int precision);

/* matmul_kernels.h:33.  "fp32-strict" or "tf32". */
const char *cuda_blas_precision_name(void);

/* matmul_kernels.h:34-38.  Times this library's tile configurations for a
 * 2-D float32 product (2 warm-ups, median of 5, CUDA events on `stream`),
 * pins the fastest for this shape/layout/precision, and leaves the product
 * in c.  Returns 1 on success, 0 when the product is ineligible (null
 * pointer, a non-positive extent, rows*inner*cols < 1e7, or a layout the
 * tensor-core path cannot read), -1 on a CUDA error.  Synchronises `stream`;
 * not for use during graph capture.  algorithm_id values are listed by
 * gemm_sm100_algorithm_name(). */
int cuda_blas_tune_matmul(float *a, float *b, float *c,
                          int rows, int inner, int cols,
                          size_t a_stride0, size_t a_stride1,
                          size_t b_stride0, size_t b_stride1,
                          cudaStream_t stream, cuda_matmul_tuning_result *result);

/* matmul_kernels.h:40-44.  2-D float32 C = A.B.  NOTE the reference's
 * argument naming: m = rows of C, n = INNER extent, k = cols of C. */
int cuda_matmul_launcher(float *a, float *b, float *c,
                         int m, int n, int k,
                         size_t a_stride0, size_t a_stride1,
                         size_t b_stride0, size_t b_stride1,
                         size_t c_stride0, size_t c_stride1, cudaStream_t stream);

/* matmul_kernels.h:46-51.  Batched float32 C[...,M,N] = A[...,M,K] . B[...,K,N]
 * with NumPy batch broadcasting (right-aligned batch axes; an operand axis of
 * extent 1 or a missing axis is broadcast).  Shape and stride pointers refer
 * to host metadata. */
int cuda_batched_matmul_nd_launcher(
    float *a, float *b, float *c,
    int *shape_a, size_t *stride_a, int nd_a,
    int *shape_b, size_t *stride_b, int nd_b,
    int *shape_c, size_t *stride_c, int nd_c, cudaStream_t stream);

/* matmul_kernels.h:53-57.  As above for DTYPE_FLOAT16 / DTYPE_BFLOAT16
 * operands and result, FP32 accumulation, round-to-nearest-even output. */
int cuda_low_precision_matmul_nd_launcher(
    void *a, void *b, void *c, dtype_t dtype,
    int *shape_a, size_t *stride_a, int nd_a,
    int *shape_b, size_t *stride_b, int nd_b,
    int *shape_c, size_t *stride_c, int nd_c, cudaStream_t stream);

/* ------------------------------------------------------------------ */
/* Additive block (no counterpart in the reference's ABI)             */
/* ------------------------------------------------------------------ */

/* Error codes reported in last_blas_status besides cudaError_t values. */
#define GEMM_SM100_STATUS_TENSOR_MAP 9001  /* cuTensorMapEncodeTiled rejected a layout */
#define GEMM_SM100_STATUS_NO_DRIVER 9002   /* driver entry point unavailable */
#define GEMM_SM100_STATUS_NO_DEVICE 9003   /* no current CUDA device / not sm_100 */
#define GEMM_SM100_STATUS_NCCL 9004        /* NCCL failure (multi-GPU entry points) */
#define GEMM_SM100_STATUS_SCRATCH_LIMIT 9005 /* product larger than the library-owned buffer */
#define GEMM_SM100_STATUS_INVALID_ARGUMENT 9006 /* a multi-GPU entry point rejected its arguments */

/* float32 C = A.B where A and B are float32, float16 or bfloat16 (not float16
 * with bfloat16), with the batched launcher's shape/broadcast rules: the
 * gradient products of the autograd matmul node for 16-bit operands
 * (src/autograd.c:1547-1577 computes them in float32 on float32 copies made by
 * gradient_cast, src/autograd.c:683-712).  No copy is made here: a 16-bit
 * operand is read as it is, and with a float32 operand on the other side the
 * tensor-core kernel splits the float32 tile into three bfloat16 parts
 * (hi + mid + lo, 24+ significant bits) and accumulates the three exact
 * bf16 x bf16 products in float32.  float32 x float16 runs on the CUDA cores.
 * Returns 1 / 0 like the other launchers.  No counterpart in the reference. */
int cuda_mixed_matmul_nd_launcher(const void *a, dtype_t a_dtype, const void *b,
                                  dtype_t b_dtype, float *c,
                                  int *shape_a, size_t *stride_a, int nd_a,
                                  int *shape_b, size_t *stride_b, int nd_b,
                                  int *shape_c, size_t *stride_c, int nd_c,
                                  cudaStream_t stream);

/* FP64 C = A.B with the batched launcher's shape/broadcast rules.  New scope:
 * the reference rejects float64 matmul (src/cuda_array/ca_private.c:1099-1106). */
int cuda_f64_matmul_nd_launcher(
    double *a, double *b, double *c,
    int *shape_a, size_t *stride_a, int nd_a,
    int *shape_b, size_t *stride_b, int nd_b,
    int *shape_c, size_t *stride_c, int nd_c, cudaStream_t stream);

/* Activations a fused epilogue can apply (the Fusion plan unary ops). */
enum {
    CUDA_MATMUL_EPILOGUE_NONE = 0,
    CUDA_MATMUL_EPILOGUE_TANH = 1,
    CUDA_MATMUL_EPILOGUE_RELU = 2,
    CUDA_MATMUL_EPILOGUE_SIGMOID = 3
};

/* Fused native-matmul step: c = act(round(A.B) + bias[N]), the values the
 * unfused Fusion plan (matmul step, then the +bias / unary elementwise
 * kernel) produces: the product is rounded to the result dtype, the bias add
 * and activation run in float (double for float64) and round once.  dtype is
 * FLOAT32, FLOAT64, FLOAT16 or BFLOAT16; bias is a contiguous [N] vector of
 * that dtype or NULL; activation is a CUDA_MATMUL_EPILOGUE_* value. */
int cuda_matmul_epilogue_nd_launcher(
    void *a, void *b, void *c, dtype_t dtype,
    int *shape_a, size_t *stride_a, int nd_a,
    int *shape_b, size_t *stride_b, int nd_b,
    int *shape_c, size_t *stride_c, int nd_c,
    const void *bias, int activation, cudaStream_t stream);

/* Name of the kernel the last successful launch on this thread used, e.g.
 * "tc2-bf16-256x512", "tc2-bf16-256x256", "tc2-3xtf32-tmem-256x256",
 * "tc2-3xtf32-256x256", "tc-3xtf32-128x128",
 * "skinny-f32", "simt-f32"; "none" before any. */
const char *gemm_sm100_last_kernel(void);

/* Grid size (CTAs), CTA size (threads) and cluster size of the last
 * tensor-core or few-column launch on this thread (0 before any); any pointer
 * may be NULL. */
void gemm_sm100_last_launch(int *grid, int *block, int *cluster);

/* Selects the kernel family for this thread's later launches and returns the
 * previous setting: 0 = automatic, 1 = single-CTA tensor-core kernel whenever
 * the layout allows it (ignoring the size heuristic), 2 = CUDA-core kernel
 * only, 3 = 2-CTA tensor-core kernel whenever the layout allows it: 16-bit,
 * tf32 mode, strict float32 (3xTF32) and float32 x bf16 products, the split
 * kinds splitting K over clusters of 2 or 4 pairs when they have fewer tiles
 * than a quarter of the SMs (float64 and bf16/f16 x bf16/f16 -> float32 as 1),
 * 4 = few-column split-K CUDA-core kernel whenever N <= 32 and K >= 128
 * (otherwise as 0), 5 = 2-CTA kernel with 256 x 512 tiles for 16-bit
 * products with a 16-bit result whenever the layout allows it (other
 * products as 3), 6 = the same kernel running every tile as two 256-column
 * halves (the form its last round of clusters takes when the automatic
 * choice splits it; for tests). */
int gemm_sm100_set_path(int path);

/* Reads (and with clear != 0 resets) the device status word of `device`:
 * 0 = no kernel has reported a problem; 1..4 = a tensor-core kernel gave up a
 * bounded wait (producer, MMA, epilogue, split stage) and returned early;
 * 5 = gemm_sm100_selftest_wait_timeout ran.
 * Synchronises the device.  Returns -1 if the device cannot be queried. */
int gemm_sm100_device_status(int device, int clear);

/* Failure-detection self-test (no counterpart in the reference): launches on
 * `stream` one warp that waits, with the same bounded mbarrier wait every
 * tensor-core kernel uses, on a barrier nothing completes.  The wait gives up
 * after its 2 s limit, the kernel records status 5 in the device status word
 * and returns; the context stays usable.  Returns 1 if the launch was made. */
int gemm_sm100_selftest_wait_timeout(cudaStream_t stream);

/* Human-readable name of a tuning algorithm_id. */
const char *gemm_sm100_algorithm_name(int algorithm_id);

/* Library version, major * 10000 + minor * 100 + patch. */
int gemm_sm100_version(void);

/* ------------------------------------------------------------------ */
/* Multi-GPU, one process per GPU (new scope: the reference is        */
/* single-GPU).  Batched products shard along the batch axis with no  */
/* collective; a single large product splits along N and all-gathers  */
/* the column blocks with NCCL over NVLink.                           */
/* ------------------------------------------------------------------ */
typedef struct gemm_mgpu_comm gemm_mgpu_comm;
#define GEMM_MGPU_UNIQUE_ID_BYTES 128

/* Rank 0 creates the communicator id (128 bytes) and hands it to the other
 * ranks by any host channel.  Returns 1, or 0 when NCCL cannot be loaded. */
int gemm_mgpu_unique_id(unsigned char *id);

/* Joins the communicator on the CURRENT device.  Collective over all ranks. */
int gemm_mgpu_comm_init(const unsigned char *id, int nranks, int rank, gemm_mgpu_comm **comm);

void gemm_mgpu_comm_destroy(gemm_mgpu_comm *comm);

/* Gather-buffer bytes gemm_mgpu_nsplit_matmul needs (M * N elements), or 0
 * when N is not a multiple of nranks. */
size_t gemm_mgpu_nsplit_workspace_bytes(int nranks, dtype_t dtype, int M, int N);

/* C[M, N] = A[M, K] . B[K, N] split along N over the communicator's ranks:
 * every rank passes all of A and its column block b_local = B[:, r*N/G,
 * (r+1)*N/G) (both strided 2-D views, element strides), and receives the
 * whole row-major contiguous C.  Enqueued on `stream`: the rank's block is
 * computed into slot r of `workspace`, the slots are all-gathered in place
 * (ncclAllGather), and a permute kernel writes C.  dtype FLOAT64, FLOAT32,
 * FLOAT16 or BFLOAT16; N % nranks == 0.  Returns 1 / 0 (last_blas_status has
 * the CUDA error, GEMM_SM100_STATUS_NCCL, or GEMM_SM100_STATUS_INVALID_ARGUMENT
 * for a null pointer, a negative extent, N not divisible by the rank count or
 * a workspace smaller than M * N elements). */
int gemm_mgpu_nsplit_matmul(gemm_mgpu_comm *comm, dtype_t dtype,
                            const void *a, size_t a_s0, size_t a_s1,
                            const void *b_local, size_t b_s0, size_t b_s1,
                            void *c, int M, int N, int K,
                            void *workspace, size_t workspace_bytes, cudaStream_t stream);

/* A result buffer mapped into every rank (CUDA IPC over NVLink / NVSwitch)
 * for the fused N-split product.  Collective: each rank gets `bytes` of
 * device memory (returned in *local; freed by gemm_mgpu_window_destroy) that
 * every peer can store into.  At most 8 ranks. */
typedef struct gemm_mgpu_window gemm_mgpu_window;
int gemm_mgpu_window_create(gemm_mgpu_comm *comm, size_t bytes, gemm_mgpu_window **win,
                            void **local);
void gemm_mgpu_window_destroy(gemm_mgpu_window *win);

/* The float64 N-split product with the exchange fused into the GEMM: this
 * rank's column-block product puts every finished tile into all ranks'
 * windows at this rank's column offset while the remaining tiles compute
 * (see gemm_mgpu_window_set_exchange for the two ways), and no gather buffer
 * or permute exists.
 * After the call's work completes on `stream` (a one-element NCCL all-reduce
 * follows the kernel), every rank's window holds the whole row-major C
 * [M, N].  dtype FLOAT64; N divisible by the rank count with an even block
 * width; M * N * 8 <= the window's bytes.  Returns 1 / 0 (last_blas_status as
 * for gemm_mgpu_nsplit_matmul).
 *
 * Reuse of a window: the kernel of call k + 1 stores into every peer's
 * window, which a peer may still be reading from call k.  So every call first
 * runs a one-element NCCL all-reduce on `stream` and launches the kernel
 * behind it: no rank's stores of call k + 1 start before every rank's
 * `stream` has reached call k + 1.  A rank must therefore finish reading its
 * window (on `stream`, or on a stream that `stream` waits for) before it
 * makes the next call; reads on an unrelated stream are not ordered. */
int gemm_mgpu_nsplit_matmul_fused(gemm_mgpu_window *win, dtype_t dtype,
                                  const void *a, size_t a_s0, size_t a_s1,
                                  const void *b_local, size_t b_s0, size_t b_s1,
                                  int M, int N, int K, cudaStream_t stream);

/* How gemm_mgpu_nsplit_matmul_fused moves a finished tile into the other
 * ranks' windows (no counterpart in the reference):
 *   GEMM_MGPU_EXCHANGE_AUTO (default): epilogue stores (measured faster
 *     than the copies on 1, 2 and 8 B200s);
 *   GEMM_MGPU_EXCHANGE_STORE: the tile's epilogue stores its rows into every
 *     window (one CTA per tile);
 *   GEMM_MGPU_EXCHANGE_OVERLAP: the tile goes to this rank's window only;
 *     the next tile computed on the same SM copies it to the peers during its
 *     own math (a last short launch copies the final tiles).
 * Both give the same bits.  Returns 1, or 0 for an unknown mode or a null
 * window. */
#define GEMM_MGPU_EXCHANGE_AUTO 0
#define GEMM_MGPU_EXCHANGE_STORE 1
#define GEMM_MGPU_EXCHANGE_OVERLAP 2
int gemm_mgpu_window_set_exchange(gemm_mgpu_window *win, int mode);

/* Size of the library-owned gather buffer of gemm_mgpu_nsplit_matmul_noalloc:
 * 32 MiB of device memory on every GPU that loads the library, held until the
 * process exits. */
#define GEMM_MGPU_NSPLIT_SCRATCH_BYTES (32u << 20)

/* gemm_mgpu_nsplit_matmul for callers that cannot allocate device memory when
 * they multiply -- a thread that is capturing a CUDA graph (cudaMalloc is not
 * allowed there), or a program whose device memory all belongs to its own
 * pool and that must not call cudaMalloc/cudaFree (cudaFree synchronises the
 * device).  No counterpart in the reference; this entry point allocates
 * nothing.  Instead of a caller workspace it uses a buffer inside the library
 * (GEMM_MGPU_NSPLIT_SCRATCH_BYTES per device), so M * N elements of `dtype`
 * must fit in it; larger products return 0 with last_blas_status =
 * GEMM_SM100_STATUS_SCRATCH_LIMIT and enqueue nothing.  The first call on a
 * device looks up the buffer's device address (once per device, with the
 * communicator's device current): make that first call before any stream
 * capture.  All calls share the one buffer and it keeps the last call's
 * contents; every call overwrites the part it uses before reading it, so
 * nothing has to start at zero.  Calls whose work overlaps on the GPU (other
 * streams, or other threads on the same device) race on the buffer: issue
 * them on one stream.  With more than one rank the call runs an NCCL
 * all-gather on the communicator; NCCL sets up its connection buffers on a
 * communicator's first collective, so run one collective on it (e.g. one
 * gemm_mgpu_nsplit_matmul) at set-up time. */
int gemm_mgpu_nsplit_matmul_noalloc(gemm_mgpu_comm *comm, dtype_t dtype,
                                    const void *a, size_t a_s0, size_t a_s1,
                                    const void *b_local, size_t b_s0, size_t b_s1,
                                    void *c, int M, int N, int K, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PT_GEMM_SM100_H */
