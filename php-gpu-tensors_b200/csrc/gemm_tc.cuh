// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[b] = epilogue(A[b] . B[b])      A: [M,K], B: [K,N], C: [M,N] per batch b
//
// Replaces the built-in tiled kernels and the cuBLAS calls of the reference
// (src/backends/cuda/matmul_kernels.cu:458-588, 612-672, 738-848).  Roles:
//   warp 0       TMA producer: fills a STAGES-deep shared-memory ring with
//                128-byte-swizzled A and B tiles (K-major or MN-major).
//   warp 1       allocates TMEM; one thread issues tcgen05.mma into one of two
//                TMEM accumulators (128 lanes x BN fp32 columns each).
//   warps 2..5   epilogue: tcgen05.ld the accumulator, optional bias +
//                activation, convert, stage 32x(128 B) boxes in swizzled shared
//                memory and write them with TMA stores.  Double-buffered TMEM
//                lets the epilogue of tile i overlap the mainloop of tile i+1.
//   warps 6..13  (split kinds only) F32X3: write lo = tf32(x - trunc(x)) of
//                each FP32 tile (the tensor core reads the tile itself as
//                hi = trunc(x)) so the MMA warp can issue hi*hi + hi*lo +
//                lo*hi (3xTF32).  MIX_A / MIX_B (one operand float32, the other
//                bfloat16): split the float32 tile into three bfloat16 parts
//                hi + mid + lo (24+ significant bits) so the MMA warp can
//                issue three exact bf16 x bf16 products per k16.
// Tiles (batch, m-block, n-block) are distributed round-robin over a grid of
// at most one CTA per SM.  Split-K (p.ksplit = G > 1, for problems with too
// few tiles to fill the GPU): a cluster of G CTAs shares one tile, CTA rank r
// taking the r-th contiguous range of k-blocks.  When its MMAs have drained,
// each CTA writes its FP32 partial tile into its (now idle) shared-memory
// ring; after a cluster barrier rank r adds the G partials of its BN/G
// columns over DSMEM in rank order and runs the epilogue on them, so the
// result is deterministic and needs no global workspace.  Batch is folded into the tile index and into rank-5
// tensor maps, so rows past M or columns past N of one batch are clipped by
// TMA and never touch a neighbouring batch.  Every wait is bounded; a timeout
// sets the CTA's abort flag and a device status word and the kernel drains
// its own copies and MMAs, frees TMEM and returns.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx_sm100.cuh"

namespace ptg {

enum InKind : int { IN_F16 = 0, IN_BF16 = 1, IN_TF32 = 2, IN_F32X3 = 3, IN_MIX_A = 4, IN_MIX_B = 5 };
enum OutKind : int { OUT_F32 = 0, OUT_F16 = 1, OUT_BF16 = 2 };
enum Activation : int { ACT_NONE = 0, ACT_TANH = 1, ACT_RELU = 2, ACT_SIGMOID = 3 };

// Status codes written to the device status word (first error wins).
enum DeviceStatus : int {
    DEV_OK = 0,
    DEV_TIMEOUT_PRODUCER = 1,
    DEV_TIMEOUT_MMA = 2,
    DEV_TIMEOUT_EPILOGUE = 3,
    DEV_TIMEOUT_SPLIT = 4,
    DEV_TIMEOUT_SELFTEST = 5,   // gemm_sm100_selftest_wait_timeout
};

struct TcParams {
    int M, N, K;
    int m_blocks, n_blocks, k_blocks;
    long long tiles;
    int nbd;          // merged batch dims (0..3)
    int bshape[3];    // their extents, outermost first
    int a_slot[3];    // tensor-map coordinate slot (2..4) of merged dim d in A, -1 = broadcast
    int b_slot[3];
    int a_mn_major;   // 1: A tile is M-contiguous (transposed view)
    int b_mn_major;   // 1: B tile is N-contiguous (row-major B)
    uint32_t idesc;   // tcgen05 instruction descriptor
    const void *bias; // [N] in the output dtype, or null
    int act;
    int *status;      // device status word
    int ksplit;       // CTAs per tile splitting K (cluster size), 1 = none
    // Batch axes summed into the product: k_blocks counts (fold, k-block)
    // pairs, k_per_fold k-blocks per fold coordinate; a_fslot / b_fslot give
    // the tensor-map slot (2..4) of each merged fold axis, -1 = broadcast.
    int nfd;
    int fshape[3];
    int a_fslot[3];
    int b_fslot[3];
    int k_per_fold;
    // 2-CTA 256 x 512 kernel: work items below wide_items are whole 256 x 512
    // tiles; each later item is one 256-column half of tile wide_items +
    // (item - wide_items) / 2 (tiles counts the items)
    long long wide_items;
};

__device__ __forceinline__ float apply_activation(float v, int act)
{
    switch (act) {
    case ACT_TANH: return tanhf(v);
    case ACT_RELU: return v > 0.0f ? v : 0.0f;
    case ACT_SIGMOID: return 1.0f / (1.0f + expf(-v));
    default: return v;
    }
}

template <int OUT>
struct OutTraits;
template <>
struct OutTraits<OUT_F32> {
    static constexpr int kBytes = 4;
    __device__ static float round_trip(float v) { return v; }
    __device__ static float load(const void *p, int i) { return static_cast<const float *>(p)[i]; }
};
template <>
struct OutTraits<OUT_F16> {
    static constexpr int kBytes = 2;
    __device__ static float round_trip(float v) { return __half2float(__float2half_rn(v)); }
    __device__ static float load(const void *p, int i)
    {
        return __half2float(static_cast<const __half *>(p)[i]);
    }
};
template <>
struct OutTraits<OUT_BF16> {
    static constexpr int kBytes = 2;
    __device__ static float round_trip(float v)
    {
        return __bfloat162float(__float2bfloat16_rn(v));
    }
    __device__ static float load(const void *p, int i)
    {
        return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    }
};

// Fused epilogue on one warp's row chunk: v[i] is column col0 + i of this
// lane's row.  The unfused plan's arithmetic: round to the output dtype, add
// bias[col] in float, apply the activation.  Lane l fetches the bias of
// columns col0 + l + 32 h (one coalesced load per 32 columns) and the values
// are broadcast with shuffles; the bias/activation choice is made once per
// chunk, outside the element loop.
template <int OUT, int COLS, int ACT, bool BIAS>
__device__ __forceinline__ void bias_act_chunk(float (&v)[COLS], const float (&bl)[COLS / 32])
{
#pragma unroll
    for (int i = 0; i < COLS; i++) {
        float x = OutTraits<OUT>::round_trip(v[i]);
        if constexpr (BIAS)
            x += __shfl_sync(0xffffffffu, bl[i >> 5], i & 31);
        if constexpr (ACT == ACT_TANH)
            x = tanhf(x);
        else if constexpr (ACT == ACT_RELU)
            x = x > 0.0f ? x : 0.0f;
        else if constexpr (ACT == ACT_SIGMOID)
            x = 1.0f / (1.0f + expf(-x));
        v[i] = x;
    }
}

template <int OUT, int COLS, bool BIAS>
__device__ __forceinline__ void bias_act_dispatch(float (&v)[COLS], const float (&bl)[COLS / 32],
                                                  int act)
{
    switch (act) {
    case ACT_TANH: bias_act_chunk<OUT, COLS, ACT_TANH, BIAS>(v, bl); break;
    case ACT_RELU: bias_act_chunk<OUT, COLS, ACT_RELU, BIAS>(v, bl); break;
    case ACT_SIGMOID: bias_act_chunk<OUT, COLS, ACT_SIGMOID, BIAS>(v, bl); break;
    default: bias_act_chunk<OUT, COLS, ACT_NONE, BIAS>(v, bl); break;
    }
}

template <int OUT, int COLS>
__device__ __forceinline__ void apply_epilogue(float (&v)[COLS], const void *bias, int act, int col0,
                                               int N, int lane)
{
    if (bias != nullptr) {
        float bl[COLS / 32];
#pragma unroll
        for (int h = 0; h < COLS / 32; h++) {
            const int col = col0 + h * 32 + lane;
            bl[h] = col < N ? OutTraits<OUT>::load(bias, col) : 0.0f;
        }
        bias_act_dispatch<OUT, COLS, true>(v, bl, act);
    } else {
        const float bl[COLS / 32] = {};
        bias_act_dispatch<OUT, COLS, false>(v, bl, act);
    }
}

// Compact form for the 3xTF32 kernel, whose 448 threads leave 128 registers
// each (the unrolled variants above spilled there): the same shuffled bias,
// the activation chosen per element.
template <int OUT, int COLS>
__device__ __forceinline__ void apply_epilogue_compact(float (&v)[COLS], const void *bias, int act,
                                                       int col0, int N, int lane)
{
    float bl[COLS / 32];
#pragma unroll
    for (int h = 0; h < COLS / 32; h++) {
        const int col = col0 + h * 32 + lane;
        bl[h] = bias != nullptr && col < N ? OutTraits<OUT>::load(bias, col) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < COLS; i++) {
        float x = OutTraits<OUT>::round_trip(v[i]);
        if (bias != nullptr)
            x += __shfl_sync(0xffffffffu, bl[i >> 5], i & 31);
        v[i] = apply_activation(x, act);
    }
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, int out)
{
    if (out == OUT_F16) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&h);
    }
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Inverse of pack2 (exact: every 16-bit value is a float).
__device__ __forceinline__ void unpack2(uint32_t q, float &lo, float &hi, int out)
{
    if (out == OUT_F16) {
        const __half2 h = *reinterpret_cast<const __half2 *>(&q);
        lo = __low2float(h);
        hi = __high2float(h);
    } else {
        lo = __uint_as_float(q << 16);
        hi = __uint_as_float(q & 0xffff0000u);
    }
}

// FP32 -> TF32 with round-to-nearest (ties away), low 13 bits cleared.
__device__ __forceinline__ float round_tf32(float x)
{
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// The TF32 value tcgen05.mma kind::tf32 takes from a float32 operand: the
// low 13 mantissa bits dropped (measured on B200: 1 + 2^-11 + 2^-12 and the
// exact half-ulp case both enter the product as 1).
__device__ __forceinline__ float trunc_tf32(float x)
{
    return __uint_as_float(__float_as_uint(x) & 0xffffe000u);
}

template <int IN_KIND, int BN_, int OUT>
struct TcConfig {
    static constexpr int BM = 128;
    static constexpr int BN = BN_;
    static constexpr bool kMix = IN_KIND == IN_MIX_A || IN_KIND == IN_MIX_B;
    static constexpr bool kMixA = IN_KIND == IN_MIX_A;   // the float32 operand is A
    // split warps, chunked accumulation and the TMEM running total
    static constexpr bool kSplit3 = IN_KIND == IN_F32X3 || kMix;
    static constexpr bool kTf32 = IN_KIND == IN_TF32 || IN_KIND == IN_F32X3;
    static constexpr int kInBytes = kTf32 ? 4 : 2;
    static constexpr int BK = 128 / kInBytes;            // one 128-byte swizzle row of K
    static constexpr int kMmaK = kTf32 ? 8 : 16;          // 32 bytes of K per instruction
    static constexpr int kKSteps = BK / kMmaK;            // 4
    static constexpr int kChunk = 128 / kInBytes;         // MN elements per 128-byte row
    static constexpr int kChunkBytes = 128 * BK;          // one MN-major box (chunk x BK)
    // MN-major tiles: 16-bit types use 8-row (1024 B) swizzle atoms; TF32 must
    // use the 32-byte-atom variant whose K groups are 4 rows (512 B).  The TMA
    // map of such a tile uses the matching CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.
    static constexpr uint32_t kMnLayout = kTf32 ? kLayoutSw128Base32B : kLayoutSw128;
    static constexpr uint32_t kMnSbo = kTf32 ? 512 : 1024;
    static constexpr int kATile = BM * BK * kInBytes;     // 16 KB
    static constexpr int kBTile = BN * BK * kInBytes;     // 16 or 32 KB
    // MIX: the float32 operand lands raw ([128][BK] floats, 32 KB, no swizzle)
    // at the stage start; the split rewrites it in place as the bf16 hi and
    // mid tiles and writes lo after it; the bf16 operand tile follows.
    static constexpr int kMixRawBytes = 128 * BK * 4;
    static constexpr int kMixLoOffset = kMixRawBytes;
    static constexpr int kMixOtherOffset = kMixRawBytes + 128 * BK * 2;
    static constexpr int kLoadBytes =
        kMix ? kMixRawBytes + 128 * BK * 2 : kATile + kBTile;   // bytes TMA lands per stage
    // F32X3: lo = tf32(x - trunc(x)) lives in its own 2-slot ring, needed only
    // from the split to the MMA, so the TMA ring of raw tiles gets 4 stages.
    static constexpr bool kLoRing = IN_KIND == IN_F32X3;
    static constexpr int kLoStages = kLoRing ? 2 : 0;
    static constexpr int kStageBytes =
        kMix ? kMixOtherOffset + 128 * BK * 2 : kLoadBytes * ((kSplit3 && !kLoRing) ? 2 : 1);
    static constexpr int kRawBudget = 196608 - kLoStages * kLoadBytes;
    static constexpr int kStages = (kRawBudget / kStageBytes) > 8 ? 8 : (kRawBudget / kStageBytes);
    static constexpr int kLoOffset = kStages * kStageBytes;
    static constexpr int kOutBytes = OutTraits<OUT>::kBytes;
    static constexpr int kEpiCols = 128 / kOutBytes;      // columns per staged box
    static constexpr int kEpiChunks = BN / kEpiCols;
    static constexpr int kEpiBufBytes = 32 * 128;         // 32 rows x 128 B
    static constexpr int kEpiWarps = 4;
    static constexpr int kSplitWarps = kSplit3 ? 8 : 0;
    static constexpr int kThreads = 32 * (2 + kEpiWarps + kSplitWarps);
    static constexpr int kAccCols = BN;
    // 3xTF32: k-blocks accumulated in a TMEM slot before the epilogue drains
    // it, with round-to-nearest float adds, into a running total kept in a
    // third TMEM region (columns [2 * BN, 3 * BN)).  This bounds the tensor
    // core's per-instruction accumulator rounding to 3 * kChunkKB * kKSteps
    // steps on a chunk-sized partial sum.  Other kinds keep one slot for the
    // whole tile.
    static constexpr int kChunkKB = kSplit3 ? 4 : (1 << 30);
    static constexpr int kTotalCol = 2 * kAccCols;
    static constexpr int kTmemUsed = (kSplit3 ? 3 : 2) * kAccCols;
    static constexpr int kTmemCols = kTmemUsed <= 256 ? 256 : 512;   // power of two
    static constexpr int kRingBytes = kStages * kStageBytes + kLoStages * kLoadBytes;
    static constexpr int kEpiOffset = kRingBytes;
    static constexpr int kBarOffset = kEpiOffset + kEpiWarps * 2 * kEpiBufBytes;
    // full, empty, ready per stage; tmem full/empty x2; drain
    static constexpr int kNumBars = 3 * kStages + 4 + 1 + kLoStages;
    static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
    // split-K partial tile [BM][BN + 4] floats at the start of the ring (the
    // 4-float pad keeps 16-byte row accesses of 8 lanes on distinct banks)
    static constexpr int kPartPitch = BN + 4;
    static_assert(BM * kPartPitch * 4 <= kRingBytes, "split-K partial tile fits in the ring");
    static_assert(kStages >= 2, "pipeline needs at least two stages");
    static_assert(BN % kEpiCols == 0, "epilogue box must divide BN");
    static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
    static_assert(kTmemUsed <= 512, "TMEM holds 512 columns");
    static_assert(!kMix || (BN == 128 && !kTf32), "mixed kinds use 128x128 bf16 tiles");
};

// x = hi + mid + lo in bfloat16 (round-to-nearest at each step; both
// differences are exact in float), so 24+ significant bits survive.  A
// non-finite hi carries the value alone.
__device__ __forceinline__ void split3_bf16(float x, __nv_bfloat16 &h, __nv_bfloat16 &m,
                                            __nv_bfloat16 &l)
{
    h = __float2bfloat16_rn(x);
    const float hf = __bfloat162float(h);
    if (!isfinite(hf)) {
        m = l = __float2bfloat16_rn(0.0f);
        return;
    }
    const float r = x - hf;
    m = __float2bfloat16_rn(r);
    l = __float2bfloat16_rn(r - __bfloat162float(m));
}

// Splits four consecutive floats into the hi/mid/lo bf16 tiles (8 bytes each
// at byte offset `off` of the three tiles, `part` bytes apart).
__device__ __forceinline__ void split3_store(const float4 &x, uint8_t *base, uint32_t off, int part)
{
    __nv_bfloat16 h[4], m[4], l[4];
    split3_bf16(x.x, h[0], m[0], l[0]);
    split3_bf16(x.y, h[1], m[1], l[1]);
    split3_bf16(x.z, h[2], m[2], l[2]);
    split3_bf16(x.w, h[3], m[3], l[3]);
    auto pack = [](const __nv_bfloat16 (&v)[4]) {
        uint2 u;
        __nv_bfloat162 lo2, hi2;
        lo2.x = v[0]; lo2.y = v[1];
        hi2.x = v[2]; hi2.y = v[3];
        u.x = *reinterpret_cast<uint32_t *>(&lo2);
        u.y = *reinterpret_cast<uint32_t *>(&hi2);
        return u;
    };
    *reinterpret_cast<uint2 *>(base + off) = pack(h);
    *reinterpret_cast<uint2 *>(base + part + off) = pack(m);
    *reinterpret_cast<uint2 *>(base + 2 * part + off) = pack(l);
}

__device__ __forceinline__ void decode_batch(long long b, const TcParams &p, int (&c)[3])
{
    c[0] = c[1] = c[2] = 0;
    for (int d = p.nbd - 1; d >= 0; d--) {
        c[d] = static_cast<int>(b % p.bshape[d]);
        b /= p.bshape[d];
    }
}

__device__ __forceinline__ void operand_coords(const int (&c)[3], const int (&slot)[3], int nbd,
                                               int (&o)[3])
{
    o[0] = o[1] = o[2] = 0;
    for (int d = 0; d < nbd; d++)
        if (slot[d] >= 2)
            o[slot[d] - 2] = c[d];
}

__device__ __forceinline__ void record_failure(volatile int *abort, int *status, int code)
{
    *abort = 1;
    atomicCAS(status, 0, code);
}

template <int IN_KIND, int BN, int OUT>
__global__ void __launch_bounds__(TcConfig<IN_KIND, BN, OUT>::kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                   const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ CUtensorMap tma_c, const TcParams p)
{
    using Cfg = TcConfig<IN_KIND, BN, OUT>;
    constexpr int S = Cfg::kStages;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kBarOffset);
    uint64_t *full = bars;
    uint64_t *empty = bars + S;
    uint64_t *ready = bars + 2 * S;
    uint64_t *tfull = bars + 3 * S;
    uint64_t *tempty = bars + 3 * S + 2;
    uint64_t *drain = bars + 3 * S + 4;
    uint64_t *lo_free = bars + 3 * S + 5;   // F32X3 lo ring: slot read by the MMAs
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + Cfg::kNumBars);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (warp == 0 && lane == 0) {
        prefetch_tensor_map(&tma_a);
        prefetch_tensor_map(&tma_b);
        prefetch_tensor_map(&tma_c);
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&ready[s], Cfg::kSplit3 ? Cfg::kSplitWarps * 32 : 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], Cfg::kEpiWarps);
        }
        mbar_init(drain, 1);
        for (int i = 0; i < Cfg::kLoStages; i++)
            mbar_init(&lo_free[i], 1);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Setup above overlaps the previous kernel's tail (programmatic dependent
    // launch); global memory is touched only after it has completed.  Every
    // CTA of this grid is resident from the start, so letting the next launch
    // begin its setup now cannot starve this grid of SMs.
    grid_dependency_wait();
    grid_launch_dependents();

    // Split-K: this CTA's tile and k-block range (one tile per cluster).
    const int G = p.ksplit;
    const int krank = G > 1 ? static_cast<int>(cluster_cta_rank()) : 0;
    const long long t_first = G > 1 ? blockIdx.x / G : blockIdx.x;
    const long long t_step = G > 1 ? p.tiles : gridDim.x;
    const int kb_per = (p.k_blocks + G - 1) / G;
    const int kb_begin = min(p.k_blocks, krank * kb_per);
    const int kb_end = min(p.k_blocks, kb_begin + kb_per);

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, parity_mask = 0;
            bool ok = true;
            for (long long t = t_first; ok && t < p.tiles; t += t_step) {
                const int nb = static_cast<int>(t % p.n_blocks);
                const long long r = t / p.n_blocks;
                const int mb = static_cast<int>(r % p.m_blocks);
                const long long batch = r / p.m_blocks;
                int c[3], ca[3], cb[3];
                decode_batch(batch, p, c);
                operand_coords(c, p.a_slot, p.nbd, ca);
                operand_coords(c, p.b_slot, p.nbd, cb);
                const int m0 = mb * Cfg::BM, n0 = nb * BN;
                for (int kbf = kb_begin; kbf < kb_end; kbf++) {
                    // (fold, k-block) of this step; the fold coordinates
                    // fill the operands' summed-axis map slots
                    int kb = kbf;
                    if (p.nfd > 0) {
                        int f = kbf / p.k_per_fold;
                        kb = kbf - f * p.k_per_fold;
                        for (int d = p.nfd - 1; d >= 0; d--) {
                            const int coord = f % p.fshape[d];
                            f /= p.fshape[d];
                            if (p.a_fslot[d] >= 2)
                                ca[p.a_fslot[d] - 2] = coord;
                            if (p.b_fslot[d] >= 2)
                                cb[p.b_fslot[d] - 2] = coord;
                        }
                    }
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort)) {
                        record_failure(abort, p.status, DEV_TIMEOUT_PRODUCER);
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + stage * Cfg::kStageBytes;
                    uint8_t *sb = sa + Cfg::kATile;
                    if constexpr (Cfg::kMix) {
                        // the float32 operand lands raw at the stage start
                        // (one unswizzled box), the bf16 one after lo
                        if constexpr (Cfg::kMixA)
                            sb = sa + Cfg::kMixOtherOffset;
                        else
                            sa = sa + Cfg::kMixOtherOffset, sb = smem + stage * Cfg::kStageBytes;
                    }
                    mbar_arrive_expect_tx(&full[stage], Cfg::kLoadBytes);
                    const int k0 = kb * Cfg::BK;
                    if (Cfg::kMixA) {
                        if (!p.a_mn_major)
                            tma_load_5d(sa, &tma_a, &full[stage], k0, m0, ca[0], ca[1], ca[2]);
                        else
                            tma_load_5d(sa, &tma_a, &full[stage], m0, k0, ca[0], ca[1], ca[2]);
                    } else if (!p.a_mn_major) {
                        tma_load_5d(sa, &tma_a, &full[stage], k0, m0, ca[0], ca[1], ca[2]);
                    } else {
#pragma unroll
                        for (int j = 0; j < Cfg::BM / Cfg::kChunk; j++)
                            tma_load_5d(sa + j * Cfg::kChunkBytes, &tma_a, &full[stage],
                                        m0 + j * Cfg::kChunk, k0, ca[0], ca[1], ca[2]);
                    }
                    if (Cfg::kMix && !Cfg::kMixA) {
                        if (!p.b_mn_major)
                            tma_load_5d(sb, &tma_b, &full[stage], k0, n0, cb[0], cb[1], cb[2]);
                        else
                            tma_load_5d(sb, &tma_b, &full[stage], n0, k0, cb[0], cb[1], cb[2]);
                    } else if (!p.b_mn_major) {
                        tma_load_5d(sb, &tma_b, &full[stage], k0, n0, cb[0], cb[1], cb[2]);
                    } else {
#pragma unroll
                        for (int j = 0; j < BN / Cfg::kChunk; j++)
                            tma_load_5d(sb + j * Cfg::kChunkBytes, &tma_b, &full[stage],
                                        n0 + j * Cfg::kChunk, k0, cb[0], cb[1], cb[2]);
                    }
                    issued_mask |= 1u << stage;
                    parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Let every copy this thread started land before shared memory
            // can be released (bounded, ignores the abort flag).
            for (int s = 0; s < S; s++) {
                if (issued_mask & (1u << s)) {
                    int no_abort = 0;
                    mbar_wait(&full[s], (parity_mask >> s) & 1u, &no_abort);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // An accumulator slot covers a whole tile, except for 3xTF32 where it
        // covers kChunkKB k-blocks and the epilogue drains it into registers.
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            long long iter = 0;   // accumulator slot uses
            int acc = 0;
            int lo_slot = 0;      // F32X3 lo ring slot of the current k-block
            uint32_t d_tmem = 0;
            bool ok = true;
            const uint32_t smem_base = smem_addr(smem);
            for (long long t = t_first; ok && t < p.tiles; t += t_step) {
                for (int kb = kb_begin; kb < kb_end; kb++) {
                    const int kc = (kb - kb_begin) % Cfg::kChunkKB;
                    if (kc == 0) {
                        acc = static_cast<int>(iter & 1);
                        const uint32_t acc_phase = static_cast<uint32_t>((iter >> 1) & 1);
                        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort)) {
                            record_failure(abort, p.status, DEV_TIMEOUT_MMA);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::kAccCols);
                    }
                    uint64_t *gate = Cfg::kSplit3 ? &ready[stage] : &full[stage];
                    if (!mbar_wait(gate, phase, abort)) {
                        record_failure(abort, p.status, DEV_TIMEOUT_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t stage_base = smem_base + stage * Cfg::kStageBytes;
                    // MIX: the float32 operand's hi, mid, lo bf16 tiles sit at
                    // 0, kATile, 2 * kATile of the stage, the other operand after
                    const uint32_t sa = Cfg::kMix && !Cfg::kMixA ? stage_base + Cfg::kMixOtherOffset
                                                                 : stage_base;
                    const uint32_t sb = Cfg::kMix ? (Cfg::kMixA ? stage_base + Cfg::kMixOtherOffset
                                                                : stage_base)
                                                  : stage_base + Cfg::kATile;
#pragma unroll
                    for (int k = 0; k < Cfg::kKSteps; k++) {
                        // one MMA consumes 32 bytes of K: a 32-byte column step
                        // in a K-major tile, kMmaK 128-byte rows in an MN-major one
                        const uint32_t a_off = p.a_mn_major ? k * Cfg::kMmaK * 128 : k * 32;
                        const uint32_t b_off = p.b_mn_major ? k * Cfg::kMmaK * 128 : k * 32;
                        const uint32_t a_lbo = p.a_mn_major ? Cfg::kChunkBytes : 16;
                        const uint32_t b_lbo = p.b_mn_major ? Cfg::kChunkBytes : 16;
                        const uint32_t a_sbo = p.a_mn_major ? Cfg::kMnSbo : 1024;
                        const uint32_t b_sbo = p.b_mn_major ? Cfg::kMnSbo : 1024;
                        const uint32_t a_lay = p.a_mn_major ? Cfg::kMnLayout : kLayoutSw128;
                        const uint32_t b_lay = p.b_mn_major ? Cfg::kMnLayout : kLayoutSw128;
                        const uint64_t ad = smem_desc(sa + a_off, a_lbo, a_sbo, a_lay);
                        const uint64_t bd = smem_desc(sb + b_off, b_lbo, b_sbo, b_lay);
                        const uint32_t accumulate = (kc | k) != 0;
                        if constexpr (Cfg::kTf32) {
                            umma_tf32(d_tmem, ad, bd, p.idesc, accumulate);
                            if constexpr (Cfg::kSplit3) {
                                // lo tiles: slot lo_slot of the lo ring, A then B
                                const uint32_t la = smem_base + Cfg::kLoOffset +
                                                    static_cast<uint32_t>(lo_slot * Cfg::kLoadBytes);
                                const uint32_t lb = la + Cfg::kATile;
                                const uint64_t ad_lo = smem_desc(la + a_off, a_lbo, a_sbo, a_lay);
                                const uint64_t bd_lo = smem_desc(lb + b_off, b_lbo, b_sbo, b_lay);
                                umma_tf32(d_tmem, ad, bd_lo, p.idesc, 1);
                                umma_tf32(d_tmem, ad_lo, bd, p.idesc, 1);
                            }
                        } else if constexpr (Cfg::kMix) {
                            // hi, mid and lo of the float32 operand against the
                            // bf16 operand: three exact products per k16
                            umma_f16(d_tmem, ad, bd, p.idesc, accumulate);
#pragma unroll
                            for (int part = 1; part < 3; part++) {
                                const uint32_t po = static_cast<uint32_t>(part * Cfg::kATile);
                                if constexpr (Cfg::kMixA)
                                    umma_f16(d_tmem, smem_desc(sa + po + a_off, a_lbo, a_sbo, a_lay),
                                             bd, p.idesc, 1);
                                else
                                    umma_f16(d_tmem, ad,
                                             smem_desc(sb + po + b_off, b_lbo, b_sbo, b_lay),
                                             p.idesc, 1);
                            }
                        } else {
                            umma_f16(d_tmem, ad, bd, p.idesc, accumulate);
                        }
                    }
                    umma_commit(&empty[stage]);
                    if constexpr (Cfg::kLoRing) {
                        umma_commit(&lo_free[lo_slot]);
                        if (++lo_slot == Cfg::kLoStages)
                            lo_slot = 0;
                    }
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                    if (kc == Cfg::kChunkKB - 1 || kb == kb_end - 1) {
                        umma_commit(&tfull[acc]);
                        iter++;
                    }
                }
            }
            // Wait until every MMA this thread issued has completed, so TMEM
            // and the shared-memory ring can be released safely.
            umma_commit(drain);
            int no_abort = 0;
            mbar_wait(drain, 0, &no_abort);
        }
    } else if (warp < 2 + Cfg::kEpiWarps) {
        // ------------------------------------------------------------ epilogue
        const int ew = warp - 2;                 // 0..3
        const int quad = warp & 3;               // TMEM lane quadrant this warp may access
        uint8_t *stage_buf = smem + Cfg::kEpiOffset + ew * 2 * Cfg::kEpiBufBytes;
        int buf = 0;
        long long iter = 0;   // accumulator slot uses
        bool ok = true;

        // Bias/activation, conversion, swizzled staging and the TMA store of
        // one 32-row x 128-byte box of this warp's rows.
        auto emit = [&](float (&v)[Cfg::kEpiCols], int col0, int row0, const int (&c)[3]) {
            if (p.bias != nullptr || p.act != ACT_NONE) {
                if constexpr (Cfg::kSplit3)
                    apply_epilogue_compact<OUT, Cfg::kEpiCols>(v, p.bias, p.act, col0, p.N, lane);
                else
                    apply_epilogue<OUT, Cfg::kEpiCols>(v, p.bias, p.act, col0, p.N, lane);
            }
            uint8_t *sbuf = stage_buf + buf * Cfg::kEpiBufBytes;
            if (lane == 0)
                bulk_wait_group_read<1>();   // the store that last used sbuf has read it
            __syncwarp();
            uint8_t *row = sbuf + lane * 128;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                uint4 q;
                if constexpr (OUT == OUT_F32) {
                    q.x = __float_as_uint(v[4 * j + 0]);
                    q.y = __float_as_uint(v[4 * j + 1]);
                    q.z = __float_as_uint(v[4 * j + 2]);
                    q.w = __float_as_uint(v[4 * j + 3]);
                } else {
                    q.x = pack2(v[8 * j + 0], v[8 * j + 1], OUT);
                    q.y = pack2(v[8 * j + 2], v[8 * j + 3], OUT);
                    q.z = pack2(v[8 * j + 4], v[8 * j + 5], OUT);
                    q.w = pack2(v[8 * j + 6], v[8 * j + 7], OUT);
                }
                // 128-byte swizzle: 16-byte chunk j of row r lives at j ^ (r % 8)
                *reinterpret_cast<uint4 *>(row + ((j ^ (lane & 7)) << 4)) = q;
            }
            fence_proxy_async_smem();
            __syncwarp();
            // boxes entirely past N or M hold nothing to write
            if (lane == 0 && col0 < p.N && row0 < p.M) {
                tma_store_5d(&tma_c, sbuf, col0, row0, c[0], c[1], c[2]);
                bulk_commit_group();
            }
            buf ^= 1;
        };

        // Split-K: this thread's row of the partial tile in the ring.
        float *part_row = reinterpret_cast<float *>(smem) + (quad * 32 + lane) * Cfg::kPartPitch;
        auto stash = [&](const float (&v)[Cfg::kEpiCols], int col) {
#pragma unroll
            for (int i = 0; i < Cfg::kEpiCols / 4; i++)
                *reinterpret_cast<float4 *>(part_row + col + 4 * i) =
                    make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        };
        int c_last[3] = {0, 0, 0};
        int n0_last = 0, row0_last = 0;

        for (long long t = t_first; ok && t < p.tiles; t += t_step) {
            const int nb = static_cast<int>(t % p.n_blocks);
            const long long r = t / p.n_blocks;
            const int mb = static_cast<int>(r % p.m_blocks);
            const long long batch = r / p.m_blocks;
            int c[3];
            decode_batch(batch, p, c);
            const int m0 = mb * Cfg::BM, n0 = nb * BN;
            const int row0 = m0 + quad * 32;
            const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
            c_last[0] = c[0];
            c_last[1] = c[1];
            c_last[2] = c[2];
            n0_last = n0;
            row0_last = row0;
            if constexpr (Cfg::kSplit3) {
                // Drain every K chunk, adding it with round-to-nearest float
                // adds into the running total in TMEM; the last chunk's sums
                // go straight to the output.
                static_assert(OUT == OUT_F32 && Cfg::kEpiCols == 32, "3xTF32 writes float32");
                const int nchunks = (kb_end - kb_begin + Cfg::kChunkKB - 1) / Cfg::kChunkKB;
                const uint32_t t_total = lane_base + static_cast<uint32_t>(Cfg::kTotalCol);
                for (int ck = 0; ck < nchunks; ck++, iter++) {
                    const int acc = static_cast<int>(iter & 1);
                    const uint32_t acc_phase = static_cast<uint32_t>((iter >> 1) & 1);
                    const bool got =
                        __all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, abort));
                    if (!got) {
                        if (lane == 0)
                            record_failure(abort, p.status, DEV_TIMEOUT_EPILOGUE);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t t_acc = lane_base + static_cast<uint32_t>(acc * Cfg::kAccCols);
                    const bool last = ck == nchunks - 1;
#pragma unroll 1
                    for (int h = 0; h < BN / 32; h++) {
                        uint32_t r32[32], t32[32];
                        tmem_ld_32x32b_x32(t_acc + h * 32, r32);
                        if (ck > 0)
                            tmem_ld_32x32b_x32(t_total + h * 32, t32);
                        tmem_ld_wait();
                        float v[32];
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            v[i] = (ck > 0 ? __uint_as_float(t32[i]) : 0.0f) +
                                   __uint_as_float(r32[i]);
                        if (!last) {
#pragma unroll
                            for (int i = 0; i < 32; i++)
                                t32[i] = __float_as_uint(v[i]);
                            tmem_st_32x32b_x32(t_total + h * 32, t32);
                        } else {
                            if (h == BN / 32 - 1) {
                                // slot fully read: hand it back to the MMA warp
                                tc_fence_before();
                                __syncwarp();
                                if (lane == 0)
                                    mbar_arrive(&tempty[acc]);
                            }
                            if (G > 1)
                                stash(v, h * 32);
                            else
                                emit(v, n0 + h * 32, row0, c);
                        }
                    }
                    if (!last) {
                        tmem_st_wait();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0)
                            mbar_arrive(&tempty[acc]);
                    }
                }
                if (!ok)
                    break;
            } else {
                const int acc = static_cast<int>(iter & 1);
                const uint32_t acc_phase = static_cast<uint32_t>((iter >> 1) & 1);
                iter++;
                // the whole warp must agree before the .sync.aligned TMEM loads
                const bool got = __all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, abort));
                if (!got) {
                    if (lane == 0)
                        record_failure(abort, p.status, DEV_TIMEOUT_EPILOGUE);
                    break;
                }
                tc_fence_after();
                const uint32_t t_acc = lane_base + static_cast<uint32_t>(acc * Cfg::kAccCols);
#pragma unroll 1
                for (int ch = 0; ch < Cfg::kEpiChunks; ch++) {
                    float v[Cfg::kEpiCols];
                    uint32_t r32[32];
#pragma unroll
                    for (int h = 0; h < Cfg::kEpiCols / 32; h++) {
                        tmem_ld_32x32b_x32(t_acc + ch * Cfg::kEpiCols + h * 32, r32);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            v[h * 32 + i] = __uint_as_float(r32[i]);
                    }
                    if (ch == Cfg::kEpiChunks - 1) {
                        // accumulator fully read: hand it back to the MMA warp
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0)
                            mbar_arrive(&tempty[acc]);
                    }
                    if (G > 1)
                        stash(v, ch * Cfg::kEpiCols);
                    else
                        emit(v, n0 + ch * Cfg::kEpiCols, row0, c);
                }
            }
        }
        if (G > 1) {
            // Every rank's partial tile is in its ring; rank r finishes the
            // columns [r * BN / G, (r + 1) * BN / G) of the tile.
            cluster_sync();
            if (ok && t_first < p.tiles) {
                const uint32_t row_s = smem_addr(part_row);
                constexpr int kSlice = BN / Cfg::kEpiCols;   // epilogue chunks per tile
                for (int ch = krank * kSlice / G; ch < (krank + 1) * kSlice / G; ch++) {
                    float v[Cfg::kEpiCols];
#pragma unroll
                    for (int i = 0; i < Cfg::kEpiCols / 4; i++) {
                        const uint32_t off = static_cast<uint32_t>((ch * Cfg::kEpiCols + 4 * i) * 4);
                        float4 s = ld_cluster_f4(map_to_cta(row_s + off, 0));
                        for (int q = 1; q < G; q++) {
                            const float4 x = ld_cluster_f4(map_to_cta(row_s + off, q));
                            s.x += x.x;
                            s.y += x.y;
                            s.z += x.z;
                            s.w += x.w;
                        }
                        v[4 * i] = s.x;
                        v[4 * i + 1] = s.y;
                        v[4 * i + 2] = s.z;
                        v[4 * i + 3] = s.w;
                    }
                    emit(v, n0_last + ch * Cfg::kEpiCols, row0_last, c_last);
                }
            }
            cluster_sync();   // peers are done reading this CTA's partial tile
        }
        if (lane == 0)
            bulk_wait_group<0>();
        __syncwarp();
    } else {
        // ------------------------------------------------------------ split warps
        if constexpr (Cfg::kMix) {
            // float32 operand -> bf16 hi/mid/lo tiles in the 128-byte-swizzled
            // layout a bf16 TMA load of the same operand would produce.  The
            // raw tile is read whole into registers, then (named barrier)
            // overwritten.  A failed wait sets the abort flag, after which
            // every wait returns at once; the loop still runs to the end so
            // that all 256 threads meet at every barrier.
            const int st = threadIdx.x - 32 * (2 + Cfg::kEpiWarps);   // 0..255
            const bool f_mn = Cfg::kMixA ? p.a_mn_major : p.b_mn_major;
            int stage = 0;
            uint32_t phase = 0;
            for (long long t = t_first; t < p.tiles; t += t_step) {
                for (int kb = kb_begin; kb < kb_end; kb++) {
                    if (!mbar_wait(&full[stage], phase, abort))
                        record_failure(abort, p.status, DEV_TIMEOUT_SPLIT);
                    uint8_t *base = smem + stage * Cfg::kStageBytes;
                    const float4 *raw = reinterpret_cast<const float4 *>(base);
                    constexpr int kPer = Cfg::kMixRawBytes / 16 / (Cfg::kSplitWarps * 32);   // 8
                    float4 x[kPer];
#pragma unroll
                    for (int j = 0; j < kPer; j++)
                        x[j] = raw[st + j * Cfg::kSplitWarps * 32];
                    named_barrier_sync(1, Cfg::kSplitWarps * 32);
#pragma unroll
                    for (int j = 0; j < kPer; j++) {
                        const int e = st + j * Cfg::kSplitWarps * 32;
                        uint32_t off;
                        if (!f_mn) {
                            // raw [128 rows][64 k]: row e/16, k 4*(e%16)
                            const int r = e >> 4, k4 = e & 15;
                            off = r * 128 + ((((k4 >> 1) ^ (r & 7))) << 4) + ((k4 & 1) << 3);
                        } else {
                            // raw [64 k][128 rows]: k e/32, rows 4*(e%32)
                            const int k = e >> 5, r4 = e & 31;
                            off = (r4 >> 4) * Cfg::kChunkBytes + k * 128 +
                                  ((((r4 & 15) >> 1) ^ (k & 7)) << 4) + ((r4 & 1) << 3);
                        }
                        split3_store(x[j], base, off, Cfg::kATile);
                    }
                    fence_proxy_async_smem();
                    mbar_arrive(&ready[stage]);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        } else if constexpr (Cfg::kSplit3) {
            const int st = threadIdx.x - 32 * (2 + Cfg::kEpiWarps);   // 0..255
            int stage = 0, lo_slot = 0;
            uint32_t phase = 0, lo_phase = 0;
            bool ok = true;
            constexpr int kVecs = Cfg::kLoadBytes / 16;
            constexpr int kPer = kVecs / (Cfg::kSplitWarps * 32);
            static_assert(kVecs % (Cfg::kSplitWarps * 32) == 0, "split covers the tile evenly");
            auto lo_of = [](float x) { return isfinite(x) ? round_tf32(x - trunc_tf32(x)) : 0.0f; };
            for (long long t = t_first; ok && t < p.tiles; t += t_step) {
                for (int kb = kb_begin; kb < kb_end; kb++) {
                    // hi is the landed tile itself (the tensor core truncates
                    // it to TF32); only lo = tf32(x - trunc(x)) is written, into
                    // the lo ring's slot.  lo is computed into registers as soon
                    // as the tile lands and stored once the slot is free, which
                    // keeps the loads and arithmetic off the slot-release chain.
                    if (!mbar_wait(&full[stage], phase, abort)) {
                        record_failure(abort, p.status, DEV_TIMEOUT_SPLIT);
                        ok = false;
                        break;
                    }
                    const float4 *raw =
                        reinterpret_cast<const float4 *>(smem + stage * Cfg::kStageBytes);
                    float4 l[kPer];
#pragma unroll
                    for (int j = 0; j < kPer; j++) {
                        const float4 x = raw[st + j * Cfg::kSplitWarps * 32];
                        l[j] = make_float4(lo_of(x.x), lo_of(x.y), lo_of(x.z), lo_of(x.w));
                    }
                    if (!mbar_wait(&lo_free[lo_slot], lo_phase ^ 1, abort)) {
                        record_failure(abort, p.status, DEV_TIMEOUT_SPLIT);
                        ok = false;
                        break;
                    }
                    float4 *lo = reinterpret_cast<float4 *>(smem + Cfg::kLoOffset +
                                                            lo_slot * Cfg::kLoadBytes);
#pragma unroll
                    for (int j = 0; j < kPer; j++)
                        lo[st + j * Cfg::kSplitWarps * 32] = l[j];
                    fence_proxy_async_smem();
                    mbar_arrive(&ready[stage]);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                    if (++lo_slot == Cfg::kLoStages) {
                        lo_slot = 0;
                        lo_phase ^= 1;
                    }
                }
            }
        }
    }

    if (G > 1 && !(warp >= 2 && warp < 2 + Cfg::kEpiWarps)) {
        // the epilogue warps' two split-K cluster barriers
        cluster_sync();
        cluster_sync();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

} // namespace ptg
