// Declarations shared by the library's translation units (not exported).
#pragma once

#include <cuda_runtime_api.h>
#include <cstddef>

// Records a status code for cuda_blas_info().last_blas_status (this thread).
void ptg_set_last_status(int code);

namespace ptg {

// Destinations of the fused N-split epilogue: this rank's column block is
// written into every rank's row-major [M, ldc] result at column col_off.
struct F64PeerOut {
    double *dst[8];
    int ndst;
    int rot;              // this rank: destination (rot + i) % ndst is stored i-th
    long long ldc;
    long long col_off;
    int exchange;         // GEMM_MGPU_EXCHANGE_*: store, overlap, or by rank count
    unsigned long long *slots;   // overlap: per-SM hand-off slots (device memory, zeroed)
    int nslots;
};

} // namespace ptg

// The float64 N-split block product whose epilogue writes into every rank's
// result: A is [M, K], B the [K, nb] block, both 2-D strided views; needs nb
// even and 16-byte aligned destinations.
cudaError_t ptg_launch_f64_peer(const double *a, size_t a_s0, size_t a_s1, const double *b,
                                size_t b_s0, size_t b_s1, int M, int nb, int K,
                                const ptg::F64PeerOut &po, cudaStream_t stream);

// float32 C = the sum over C's reduced batch axes of A . B: an axis where the
// broadcast batch shape of A and B has extent > 1 and C has extent 1 (or no
// axis) is summed inside the product kernel (the k loop runs over it), so the
// un-broadcast step of a gradient needs no scratch tensor and no second
// kernel.  Operand dtypes are dtype_t values: float32, float16, bfloat16 (not
// float16 with bfloat16).  Returns 1 / 0 like the launchers.
int ptg_reduced_matmul(const void *a, int a_dtype, const void *b, int b_dtype, float *c,
                       int *shape_a, size_t *stride_a, int nd_a, int *shape_b, size_t *stride_b,
                       int nd_b, int *shape_c, size_t *stride_c, int nd_c, cudaStream_t stream);
