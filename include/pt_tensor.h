/*
 * pt_tensor.h -- tensor-level matmul entry points of libgemm_sm100.so.
 *
 * The host layer above the launcher ABI (gemm_sm100.h), written in C++ in
 * place of the PHP extension's C dispatch, with the same argument meaning
 * and error behaviour as
 *   cuda_tensor_matmul / cuda_tensor_matmul_nd
 *       src/cuda_array/ca_private.c:1097-1213
 *   ZEND_METHOD(CudaArray, matmul)   src/cuda_array/cuda_array_ce.c:1568-1607
 *   fusion_native_submit (matmul)    src/fusion_execute.c:157-182
 *   AUTOGRAD_MATMUL backward GEMMs   src/autograd.c:1539-1585
 * A pt_tensor is the matmul-relevant part of the reference's tensor_t
 * (src/tensor.h:49-79): device data pointer with the view offset folded in,
 * dtype, rank, shape and ELEMENT strides.
 */
#ifndef PT_TENSOR_H
#define PT_TENSOR_H

#include "gemm_sm100.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    void *data;
    dtype_t dtype;
    int ndims;
    int shape[MAX_DIMS];
    size_t strides[MAX_DIMS];
} pt_tensor;

/* Status codes: PT_OK, or the PHP exception class the reference throws. */
enum {
    PT_OK = 0,
    PT_INVALID_ARGUMENT = 1, /* PhpTensors\InvalidArgumentException */
    PT_RUNTIME = 2           /* PhpTensors\RuntimeException */
};

/* Flags for pt_tensor_matmul_into. */
enum {
    PT_MATMUL_ALLOW_FLOAT64 = 1 /* accept float64 operands (the reference rejects them) */
};

/* Message of the last non-OK status on this thread (the reference's
 * exception text), "" when none. */
const char *pt_last_error(void);

/* Result shape of a matmul (src/operations.c:32-35 -> src/tensor_shape.h:46-59):
 * returns PT_OK, or PT_INVALID_ARGUMENT with "Matrix multiplication failed -
 * incompatible dimensions". */
int pt_matmul_result_shape(const pt_tensor *a, const pt_tensor *b, int *shape, int *ndims);

/* C = A . B into a preallocated, contiguous row-major result of the shape
 * pt_matmul_result_shape reports (the Fusion plan contract).  Checks, in the
 * reference's order: matching float32/float16/bfloat16 dtypes ("matmul
 * requires matching float32, float16 or bfloat16 operands"), the shape rule,
 * then dispatches -- 2-D float32 to cuda_matmul_launcher, other float32 to
 * cuda_batched_matmul_nd_launcher, float16/bfloat16 to
 * cuda_low_precision_matmul_nd_launcher, float64 (with
 * PT_MATMUL_ALLOW_FLOAT64) to cuda_f64_matmul_nd_launcher -- and reports a
 * launcher failure as PT_RUNTIME "Matmul backend submission failed (cuBLAS
 * status %d)".  Asynchronous on `stream`. */
int pt_tensor_matmul_into(const pt_tensor *a, const pt_tensor *b, const pt_tensor *result,
                          int flags, cudaStream_t stream);

/* As pt_tensor_matmul_into, but allocates the contiguous result with
 * cudaMallocAsync on `stream` (the eager CudaArray::matmul path).  Release
 * it with pt_tensor_release. */
int pt_tensor_matmul(const pt_tensor *a, const pt_tensor *b, pt_tensor *result, int flags,
                     cudaStream_t stream);

/* Frees a tensor allocated by pt_tensor_matmul (cudaFreeAsync on stream). */
void pt_tensor_release(pt_tensor *t, cudaStream_t stream);

/* The two GEMMs of the matmul backward node (src/autograd.c:1539-1585):
 * grad_a = grad_c . B^T and grad_b = A^T . grad_c, with B^T and A^T taken as
 * zero-copy transposed views (last two axes swapped).  A and B are float32,
 * float16 or bfloat16 (the same type); grad_c is float32 or their type; the
 * results are float32 (the reference's gradient dtype for 16-bit operands,
 * src/autograd.c:1547-1548), computed without the float32 copies the
 * reference makes (gradient_cast): cuda_mixed_matmul_nd_launcher reads the
 * 16-bit operands as they are.  Each result has either the batch-broadcast
 * shape of its product, or the shape of its operand when the product
 * broadcast that operand (src/autograd.c:714-760, gradient_unbroadcast):
 * the sum over the broadcast axes is then fused -- one GEMM over the folded
 * (batch..., inner) axis when the tensors' strides allow it, otherwise the
 * summed axes are walked inside the product kernel.  Either result may be
 * NULL to skip that GEMM.  With both requested, grad_b runs on a side stream
 * forked from `stream` and joined back into it with events (capture-safe);
 * on return every launch is ordered on `stream`. */
int pt_tensor_matmul_backward(const pt_tensor *a, const pt_tensor *b, const pt_tensor *grad_c,
                              const pt_tensor *grad_a, const pt_tensor *grad_b,
                              cudaStream_t stream);

/* Batched C = A . B between HOST buffers, streamed through the current
 * device: the batch axis is cut into `chunks` pieces whose host-to-device
 * copies, products and device-to-host copies overlap on three streams, so the
 * PCIe transfers in both directions run concurrently with each other and
 * with the tensor cores (the CudaArray::fromBuffer -> matmul -> toBuffer
 * sequence, pipelined).  A is [batches, M, K], B is [batches, K, N] (or one
 * [K, N] matrix shared by every batch when b_shared != 0), C is
 * [batches, M, N], all row-major contiguous host memory of `dtype`
 * (FLOAT32/FLOAT16/BFLOAT16, or FLOAT64 with PT_MATMUL_ALLOW_FLOAT64 in
 * flags).  Host buffers should be page-locked (cudaHostAlloc or
 * cudaHostRegister) for the copies to overlap.  The three streams and the
 * device staging (two chunk slots) are created on the first call and kept,
 * per host thread and device, for later calls; pt_host_release() frees them.
 * Blocks until C is on the host; returns PT_OK or a PT_* error with
 * pt_last_error() set. */
int pt_host_matmul(const void *a, const void *b, void *c, dtype_t dtype, int batches, int M,
                   int N, int K, int b_shared, int chunks, int flags);

/* pt_host_matmul over several devices of this process: the batch axis is cut
 * into ndev contiguous shards (sizes differing by at most one, shard g on
 * devices[g]), each streamed in `chunks` pieces through that device's own
 * pipeline as above, with chunk i enqueued on every device before chunk i+1
 * so that every device's PCIe link copies at the same time -- the
 * host-staged form of the batch-sharded product (toGpu / fromBuffer
 * transfers feeding the sharded path, src/cuda_array/tensor_transfer.c).  A
 * shared B is copied to every device.  Devices must be distinct; the
 * caller's current device is restored.  Blocks until C is on the host. */
int pt_host_matmul_sharded(const void *a, const void *b, void *c, dtype_t dtype, int batches,
                           int M, int N, int K, int b_shared, const int *devices, int ndev,
                           int chunks, int flags);

/* Frees this thread's pt_host_matmul streams and staging on every device
 * (synchronises them). */
void pt_host_release(void);

#ifdef __cplusplus
}
#endif

#endif /* PT_TENSOR_H */
