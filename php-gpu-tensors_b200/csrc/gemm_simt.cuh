// Generic strided batched GEMM on the CUDA cores.
//
// Serves the shapes the tensor-core kernel cannot describe with TMA: inner
// strides other than 1 (e.g. a `::2` slice), row strides that are not a
// multiple of 16 bytes (N = 10 in float32), unaligned view offsets, K = 0,
// and more than three non-mergeable batch axes.  It also carries FP64.
// Each output is accumulated with fma in k order starting from zero, the same
// sequence as the reference's host loop (src/contiguous_array_ce.c:1327-1333),
// so float32 and float64 results here are bit-identical to that loop.  Folded
// batch axes (a gradient summed over the axes its operand was broadcast
// along) are walked outside the k loop, in row-major order.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gemm_tc.cuh"

namespace ptg {

constexpr int kSimtMaxBatchDims = 8;

struct SimtParams {
    const void *a;
    const void *b;
    void *c;
    int M, N, K;
    long long batches;
    int nbd;
    int bshape[kSimtMaxBatchDims];
    long long a_bs[kSimtMaxBatchDims];   // element stride per C batch axis, 0 = broadcast
    long long b_bs[kSimtMaxBatchDims];
    long long c_bs[kSimtMaxBatchDims];
    long long a_sm, a_sk, b_sk, b_sn, c_sm, c_sn;
    const void *bias;
    int act;
    // batch axes summed into the product (gradient of a broadcast operand):
    // each output accumulates A[f] . B[f] over every fold coordinate f
    int nfd;
    int fshape[kSimtMaxBatchDims];
    long long a_fs[kSimtMaxBatchDims];
    long long b_fs[kSimtMaxBatchDims];
    long long folds;   // product of fshape (1 without folding)
};

template <typename T>
struct Elem;
template <>
struct Elem<float> {
    using Acc = float;
    __device__ static float load(const void *p, long long i) { return static_cast<const float *>(p)[i]; }
    __device__ static void store(void *p, long long i, float v) { static_cast<float *>(p)[i] = v; }
    __device__ static float round_trip(float v) { return v; }
    __device__ static float fma_(float a, float b, float c) { return fmaf(a, b, c); }
};
template <>
struct Elem<double> {
    using Acc = double;
    __device__ static double load(const void *p, long long i) { return static_cast<const double *>(p)[i]; }
    __device__ static void store(void *p, long long i, double v) { static_cast<double *>(p)[i] = v; }
    __device__ static double round_trip(double v) { return v; }
    __device__ static double fma_(double a, double b, double c) { return fma(a, b, c); }
};
template <>
struct Elem<__half> {
    using Acc = float;
    __device__ static float load(const void *p, long long i)
    {
        return __half2float(static_cast<const __half *>(p)[i]);
    }
    __device__ static void store(void *p, long long i, float v)
    {
        static_cast<__half *>(p)[i] = __float2half_rn(v);
    }
    __device__ static float round_trip(float v) { return __half2float(__float2half_rn(v)); }
    __device__ static float fma_(float a, float b, float c) { return fmaf(a, b, c); }
};
template <>
struct Elem<__nv_bfloat16> {
    using Acc = float;
    __device__ static float load(const void *p, long long i)
    {
        return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    }
    __device__ static void store(void *p, long long i, float v)
    {
        static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
    }
    __device__ static float round_trip(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
    __device__ static float fma_(float a, float b, float c) { return fmaf(a, b, c); }
};

__device__ __forceinline__ double apply_activation_d(double v, int act)
{
    switch (act) {
    case ACT_TANH: return tanh(v);
    case ACT_RELU: return v > 0.0 ? v : 0.0;
    case ACT_SIGMOID: return 1.0 / (1.0 + exp(-v));
    default: return v;
    }
}

constexpr int kSimtTile = 64;
constexpr int kSimtBK = 16;

// 16x16 threads, 64x64 output tile, 4x4 outputs per thread.  TA / TB are the
// operand element types (widened to the result's accumulator type on load),
// T the result's.
template <typename T, typename TA = T, typename TB = T>
__global__ void __launch_bounds__(256) simt_gemm_kernel(const SimtParams p)
{
    using E = Elem<T>;
    using Acc = typename E::Acc;
    __shared__ Acc sa[kSimtBK][kSimtTile + 1];
    __shared__ Acc sb[kSimtBK][kSimtTile + 1];

    // programmatic dependent launch: nothing global is touched before the
    // previous kernel in the stream has completed
    grid_dependency_wait();
    grid_launch_dependents();
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int n0 = blockIdx.x * kSimtTile;
    const int m_blocks = (p.M + kSimtTile - 1) / kSimtTile;

    for (long long batch = blockIdx.z; batch < p.batches; batch += gridDim.z)
    for (int mb = blockIdx.y; mb < m_blocks; mb += gridDim.y) {
        const int m0 = mb * kSimtTile;
        long long oa = 0, ob = 0, oc = 0, rem = batch;
        for (int d = p.nbd - 1; d >= 0; d--) {
            const long long coord = rem % p.bshape[d];
            rem /= p.bshape[d];
            oa += coord * p.a_bs[d];
            ob += coord * p.b_bs[d];
            oc += coord * p.c_bs[d];
        }
        Acc acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
                acc[i][j] = Acc(0);

        const long long oa0 = oa, ob0 = ob;
        for (long long f = 0; f < p.folds; f++) {
        oa = oa0;
        ob = ob0;
        long long frem = f;
        for (int d = p.nfd - 1; d >= 0; d--) {
            const long long coord = frem % p.fshape[d];
            frem /= p.fshape[d];
            oa += coord * p.a_fs[d];
            ob += coord * p.b_fs[d];
        }
        for (int k0 = 0; k0 < p.K; k0 += kSimtBK) {
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int e = threadIdx.x + 256 * r;    // 0..1023
                const int row = e >> 4, kk = e & 15;    // A: 64 rows x 16 k
                const int m = m0 + row, k = k0 + kk;
                sa[kk][row] = (m < p.M && k < p.K) ? Acc(Elem<TA>::load(p.a, oa + m * p.a_sm + k * p.a_sk))
                                                   : Acc(0);
                const int kr = e >> 6, col = e & 63;    // B: 16 k x 64 cols
                const int n = n0 + col, kb = k0 + kr;
                sb[kr][col] = (n < p.N && kb < p.K) ? Acc(Elem<TB>::load(p.b, ob + kb * p.b_sk + n * p.b_sn))
                                                    : Acc(0);
            }
            __syncthreads();
            const int kmax = p.K - k0 < kSimtBK ? p.K - k0 : kSimtBK;
            for (int kk = 0; kk < kmax; kk++) {
                Acc av[4], bv[4];
#pragma unroll
                for (int i = 0; i < 4; i++) av[i] = sa[kk][ty + 16 * i];
#pragma unroll
                for (int j = 0; j < 4; j++) bv[j] = sb[kk][tx + 16 * j];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        acc[i][j] = E::fma_(av[i], bv[j], acc[i][j]);
            }
            __syncthreads();
        }
        }   // folds
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int m = m0 + ty + 16 * i;
            if (m >= p.M) continue;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int n = n0 + tx + 16 * j;
                if (n >= p.N) continue;
                Acc v = acc[i][j];
                if (p.bias != nullptr || p.act != ACT_NONE) {
                    Acc x = E::round_trip(v);
                    if (p.bias != nullptr) x += Acc(E::load(p.bias, n));
                    if constexpr (sizeof(Acc) == 8)
                        v = apply_activation_d(x, p.act);
                    else
                        v = apply_activation(x, p.act);
                }
                E::store(p.c, oc + m * p.c_sm + n * p.c_sn, v);
            }
        }
    }
}

} // namespace ptg
