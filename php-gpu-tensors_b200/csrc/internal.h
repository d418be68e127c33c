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
    long long ldc;
    long long col_off;
};

} // namespace ptg

// The float64 N-split block product whose epilogue writes into every rank's
// result: A is [M, K], B the [K, nb] block, both 2-D strided views; needs nb
// even and 16-byte aligned destinations.
cudaError_t ptg_launch_f64_peer(const double *a, size_t a_s0, size_t a_s1, const double *b,
                                size_t b_s0, size_t b_s1, int M, int nb, int K,
                                const ptg::F64PeerOut &po, cudaStream_t stream);

// Shape of a gradient's un-broadcast reduction: src is a contiguous float32
// tensor of extents ext[0..n); axes with keep[d] == 0 are summed (in
// row-major order of their coordinates, so the result is deterministic) and
// the sum lands at dst + sum over kept axes of coord * dst_stride[d].
struct PtgReduceDims {
    int n;
    int ext[10];
    int keep[10];
    long long dst_stride[10];
};

cudaError_t ptg_reduce_axes(const float *src, float *dst, const PtgReduceDims &d,
                            cudaStream_t stream);
