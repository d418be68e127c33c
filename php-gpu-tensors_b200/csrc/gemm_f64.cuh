// FP64 batched GEMM on the DMMA pipe (mma.sync.m16n8k4 .f64).
//
// New scope: the reference rejects float64 matmul.  Block tile 128 x 128 x 16,
// 8 warps in a 2 x 4 grid, each warp owning 64 x 32 outputs as 4 x 4 m16n8
// fragments (64 fp64 accumulators per thread).  Operand tiles move through a
// 3-stage cp.async ring into row-major shared tiles whose row pitches
// (20 doubles for A, 132 for B) make every fragment read of a half-warp hit
// distinct banks.  A K-contiguous A and an N-contiguous B with 16-byte aligned
// rows use 16-byte cp.async copies with zero fill at the edges; any other
// layout goes through the same ring with element loads.
//
// Tail: when the tiles of a launch leave the last wave of CTAs at most half
// full, its tiles run as two 128 x 64 halves each (8 warps in a 4 x 2 grid of
// 32 x 32 blocks), so that wave takes half as long.  Every output element
// sees the same sequence of k4 steps in either tile width, so the results are
// bit-identical.  (8192 x 1024 x 8192, the column block of one rank of an
// 8-way N-split, is 512 tiles: three full waves of 148 and 68 tiles left.)
#pragma once

#include "gemm_simt.cuh"
#include "internal.h"

namespace ptg {

constexpr int kF64BM = 128, kF64BN = 128, kF64BK = 16;
constexpr int kF64Stages = 3;
constexpr int kF64PitchA = kF64BK + 4;    // doubles per A row in shared memory
constexpr int kF64PitchB = kF64BN + 4;    // doubles per B row
constexpr int kF64StageA = kF64BM * kF64PitchA;
constexpr int kF64StageB = kF64BK * kF64PitchB;
constexpr int kF64SmemBytes = kF64Stages * (kF64StageA + kF64StageB) * 8;

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid)
{
    const uint32_t d = smem_addr(dst);
    const int n = valid ? 16 : 0;   // 0 source bytes: the 16 destination bytes are zero-filled
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n)
                 : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void dmma_16x8x4(double (&d)[4], const double (&a)[2], double b)
{
    asm volatile(
        "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64"
        " {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a[0]), "d"(a[1]), "d"(b));
}

// Tile geometry: WN warps along N (4: the full 128 x 128 tile, warps 2 x 4
// of 64 x 32; 2: the 128 x 64 half tile, warps 4 x 2 of 32 x 32).
template <int WN>
struct F64Tile {
    static constexpr int kWarpsM = 8 / WN;
    static constexpr int TJ = 4;                         // n8 fragments per warp
    static constexpr int kWarpN = TJ * 8;                // 32 columns per warp
    static constexpr int kWarpM = kF64BM / kWarpsM;      // 64 or 32 rows per warp
    static constexpr int TI = kWarpM / 16;               // m16 fragments per warp
    static constexpr int BN = WN * kWarpN;               // 128 or 64
};

// Fills one ring stage with the A tile [m0, m0+128) x [k0, k0+16) and the B
// tile [k0, k0+16) x [n0, n0+BN).
template <int BN>
__device__ __forceinline__ void f64_load_stage(const SimtParams &p, double *sa, double *sb,
                                               long long oa, long long ob, int m0, int n0, int k0,
                                               bool a_vec, bool b_vec)
{
    const double *A = static_cast<const double *>(p.a);
    const double *B = static_cast<const double *>(p.b);
    const int tid = threadIdx.x;
    if (a_vec) {
        // 128 rows x 8 pairs of k
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int e = tid + 256 * r;
            const int row = e >> 3, kp = (e & 7) * 2;
            const int m = m0 + row, k = k0 + kp;
            const bool ok = m < p.M && k < p.K;   // K even: a pair is all in or all out
            const double *src = ok ? A + oa + static_cast<long long>(m) * p.a_sm + k : A;
            cp_async16(sa + row * kF64PitchA + kp, src, ok);
        }
    } else {
#pragma unroll
        for (int r = 0; r < 8; r++) {
            const int e = tid + 256 * r;
            const int row = e >> 4, kk = e & 15;
            const int m = m0 + row, k = k0 + kk;
            sa[row * kF64PitchA + kk] =
                (m < p.M && k < p.K) ? A[oa + static_cast<long long>(m) * p.a_sm +
                                         static_cast<long long>(k) * p.a_sk]
                                     : 0.0;
        }
    }
    constexpr int kPairs = BN / 2;   // pairs of n per k row
    if (b_vec) {
        // 16 k rows x BN / 2 pairs of n
#pragma unroll
        for (int r = 0; r < kF64BK * kPairs / 256; r++) {
            const int e = tid + 256 * r;
            const int kr = e / kPairs, np = (e % kPairs) * 2;
            const int k = k0 + kr, n = n0 + np;
            const bool ok = k < p.K && n < p.N;   // N even: a pair is all in or all out
            const double *src = ok ? B + ob + static_cast<long long>(k) * p.b_sk + n : B;
            cp_async16(sb + kr * kF64PitchB + np, src, ok);
        }
    } else {
#pragma unroll
        for (int r = 0; r < kF64BK * BN / 256; r++) {
            const int e = tid + 256 * r;
            const int kr = e / BN, col = e % BN;
            const int k = k0 + kr, n = n0 + col;
            sb[kr * kF64PitchB + col] =
                (k < p.K && n < p.N) ? B[ob + static_cast<long long>(k) * p.b_sk +
                                         static_cast<long long>(n) * p.b_sn]
                                     : 0.0;
        }
    }
}

// One k-block of MMAs of a warp's block: 4 k4 steps of TI x TJ m16n8
// fragments.
template <int TI, int TJ>
__device__ __forceinline__ void f64_mma_kblock(double (&acc)[TI][TJ][4], const double *sa,
                                               const double *sb, int wm, int wn, int g, int t)
{
#pragma unroll
    for (int kk = 0; kk < kF64BK; kk += 4) {
        double af[TI][2], bf[TJ];
#pragma unroll
        for (int i = 0; i < TI; i++) {
            af[i][0] = sa[(wm + i * 16 + g) * kF64PitchA + kk + t];
            af[i][1] = sa[(wm + i * 16 + g + 8) * kF64PitchA + kk + t];
        }
#pragma unroll
        for (int j = 0; j < TJ; j++)
            bf[j] = sb[(kk + t) * kF64PitchB + wn + j * 8 + g];
#pragma unroll
        for (int i = 0; i < TI; i++)
#pragma unroll
            for (int j = 0; j < TJ; j++)
                dmma_16x8x4(acc[i][j], af[i], bf[j]);
    }
}

// A launch's work list: `full` tiles of 128 x 128 in row-major tile order
// (column block fastest, then row block, then batch), then, when the last
// wave is at most half full, its tiles as 2 x `tail` half tiles.
struct F64Work {
    long long full;
    long long tail;       // tiles run as two halves each (0 = none)
    int m_blocks, n_blocks;
};

__host__ __device__ inline F64Work f64_work(int M, int N, long long batches, long long ctas)
{
    F64Work w;
    w.m_blocks = (M + kF64BM - 1) / kF64BM;
    w.n_blocks = (N + kF64BN - 1) / kF64BN;
    const long long tiles = batches * w.m_blocks * w.n_blocks;
    const long long rem = ctas > 0 ? tiles % ctas : 0;
    w.tail = (rem > 0 && 2 * rem <= ctas) ? rem : 0;
    w.full = tiles - w.tail;
    return w;
}

// Runs the k loop of tile (batch, mb, nb) -- the half `half` of it when
// WN == 2 -- into acc, calling hook(kb) after each k-block's MMAs.
template <int WN, typename Hook>
__device__ __forceinline__ void f64_tile_mainloop(
    const SimtParams &p, double *sa_all, double *sb_all, long long oa, long long ob, int m0,
    int n0, bool a_vec, bool b_vec, double (&acc)[F64Tile<WN>::TI][F64Tile<WN>::TJ][4],
    Hook &&hook)
{
    using T = F64Tile<WN>;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int wm = (warp / WN) * T::kWarpM, wn = (warp % WN) * T::kWarpN;
    const int k_blocks = (p.K + kF64BK - 1) / kF64BK;
#pragma unroll
    for (int i = 0; i < T::TI; i++)
#pragma unroll
        for (int j = 0; j < T::TJ; j++)
#pragma unroll
            for (int r = 0; r < 4; r++)
                acc[i][j][r] = 0.0;
    __syncthreads();   // the previous tile's readers are done with the ring
#pragma unroll
    for (int s = 0; s < kF64Stages - 1; s++) {
        if (s < k_blocks)
            f64_load_stage<T::BN>(p, sa_all + s * kF64StageA, sb_all + s * kF64StageB, oa, ob,
                                  m0, n0, s * kF64BK, a_vec, b_vec);
        cp_async_commit();
    }
    for (int kb = 0; kb < k_blocks; kb++) {
        cp_async_wait<kF64Stages - 2>();
        __syncthreads();
        const int nxt = kb + kF64Stages - 1;
        if (nxt < k_blocks)
            f64_load_stage<T::BN>(p, sa_all + (nxt % kF64Stages) * kF64StageA,
                                  sb_all + (nxt % kF64Stages) * kF64StageB, oa, ob, m0, n0,
                                  nxt * kF64BK, a_vec, b_vec);
        cp_async_commit();
        f64_mma_kblock<T::TI, T::TJ>(acc, sa_all + (kb % kF64Stages) * kF64StageA,
                                     sb_all + (kb % kF64Stages) * kF64StageB, wm, wn, g, t);
        hook(kb, k_blocks);
    }
    cp_async_wait<0>();
}

// Origin of work unit u: a full tile for u < w.full, else half (u - full) % 2
// of tile full + (u - full) / 2.  Returns the tile width (128 or 64).
__device__ __forceinline__ int f64_unit(const F64Work &w, long long u, long long &batch, int &m0,
                                        int &n0)
{
    long long tile = u;
    int half = -1;
    if (u >= w.full) {
        tile = w.full + (u - w.full) / 2;
        half = static_cast<int>((u - w.full) % 2);
    }
    const long long per_batch = static_cast<long long>(w.m_blocks) * w.n_blocks;
    batch = tile / per_batch;
    const long long r = tile - batch * per_batch;
    m0 = static_cast<int>(r / w.n_blocks) * kF64BM;
    n0 = static_cast<int>(r % w.n_blocks) * kF64BN + (half > 0 ? kF64BN / 2 : 0);
    return half < 0 ? kF64BN : kF64BN / 2;
}

__device__ __forceinline__ void f64_batch_offsets(const SimtParams &p, long long batch,
                                                  long long &oa, long long &ob, long long &oc)
{
    oa = ob = oc = 0;
    long long rem = batch;
    for (int d = p.nbd - 1; d >= 0; d--) {
        const long long coord = rem % p.bshape[d];
        rem /= p.bshape[d];
        oa += coord * p.a_bs[d];
        ob += coord * p.b_bs[d];
        oc += coord * p.c_bs[d];
    }
}

// The plain product into p.c (optional bias / activation): one CTA per work
// unit of f64_work(M, N, batches, resident CTAs).
template <int WN>
__device__ __forceinline__ void f64_plain_unit(const SimtParams &p, double *sa_all,
                                               double *sb_all, long long batch, int m0, int n0,
                                               bool a_vec, bool b_vec)
{
    using T = F64Tile<WN>;
    long long oa, ob, oc;
    f64_batch_offsets(p, batch, oa, ob, oc);
    double acc[T::TI][T::TJ][4];
    f64_tile_mainloop<WN>(p, sa_all, sb_all, oa, ob, m0, n0, a_vec, b_vec, acc,
                          [](int, int) {});
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int wm = (warp / WN) * T::kWarpM, wn = (warp % WN) * T::kWarpN;
    double *C = static_cast<double *>(p.c);
    const double *bias = static_cast<const double *>(p.bias);
#pragma unroll
    for (int i = 0; i < T::TI; i++)
#pragma unroll
        for (int j = 0; j < T::TJ; j++)
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int m = m0 + wm + i * 16 + g + (r >> 1) * 8;
                const int n = n0 + wn + j * 8 + t * 2 + (r & 1);
                if (m < p.M && n < p.N) {
                    double v = acc[i][j][r];
                    if (bias != nullptr || p.act != ACT_NONE) {
                        if (bias != nullptr) v += bias[n];
                        v = apply_activation_d(v, p.act);
                    }
                    C[oc + static_cast<long long>(m) * p.c_sm + static_cast<long long>(n) * p.c_sn] = v;
                }
            }
}

// Full tiles: grid (column blocks, row blocks, batches), each CTA walking
// row blocks and batches by the grid's extents (more than 65535 of either);
// tiles from w.full on (row-major tile index) are left to the half-tile
// launch.  The loop form measured 1-3 % faster than one tile per CTA
// through f64_plain_unit on B200 (8192^3 and 4096^3).
// PEER = false: the plain product into p.c.  PEER = true: the N-split block
// product (rank-2, one batch) whose epilogue stages the tile in shared
// memory, half at a time, and stores its rows into every rank's window
// (16 bytes per thread, consecutive threads on consecutive columns).
template <bool PEER>
__global__ void __launch_bounds__(256, 1)
    f64_dmma_kernel(const SimtParams p, int a_vec, int b_vec, const F64Work w,
                    const F64PeerOut po)
{
    extern __shared__ __align__(16) double f64_smem[];
    double *sa_all = f64_smem;
    double *sb_all = f64_smem + kF64Stages * kF64StageA;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int wm = (warp >> 2) * 64, wn = (warp & 3) * 32;
    const int m_blocks = w.m_blocks;
    const int k_blocks = (p.K + kF64BK - 1) / kF64BK;
    const int n0 = blockIdx.x * kF64BN;

    for (long long batch = blockIdx.z; batch < p.batches; batch += gridDim.z)
    for (int mb = blockIdx.y; mb < m_blocks; mb += gridDim.y) {
        if ((batch * m_blocks + mb) * w.n_blocks + blockIdx.x >= w.full)
            continue;
        const int m0 = mb * kF64BM;
        long long oa, ob, oc;
        f64_batch_offsets(p, batch, oa, ob, oc);
        double acc[4][4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int r = 0; r < 4; r++)
                    acc[i][j][r] = 0.0;

        __syncthreads();   // the previous tile's readers are done with the ring
#pragma unroll
        for (int s = 0; s < kF64Stages - 1; s++) {
            if (s < k_blocks)
                f64_load_stage<kF64BN>(p, sa_all + s * kF64StageA, sb_all + s * kF64StageB, oa,
                                       ob, m0, n0, s * kF64BK, a_vec, b_vec);
            cp_async_commit();
        }
        for (int kb = 0; kb < k_blocks; kb++) {
            cp_async_wait<kF64Stages - 2>();
            __syncthreads();
            const int nxt = kb + kF64Stages - 1;
            if (nxt < k_blocks)
                f64_load_stage<kF64BN>(p, sa_all + (nxt % kF64Stages) * kF64StageA,
                                       sb_all + (nxt % kF64Stages) * kF64StageB, oa, ob, m0, n0,
                                       nxt * kF64BK, a_vec, b_vec);
            cp_async_commit();
            f64_mma_kblock<4, 4>(acc, sa_all + (kb % kF64Stages) * kF64StageA,
                                 sb_all + (kb % kF64Stages) * kF64StageB, wm, wn, g, t);
        }
        cp_async_wait<0>();

        if constexpr (PEER) {
            __syncthreads();   // every warp is done with the ring
            double *st = f64_smem;
            for (int h = 0; h < 2; h++) {
                if ((warp >> 2) == h) {
#pragma unroll
                    for (int i = 0; i < 4; i++)
#pragma unroll
                        for (int j = 0; j < 4; j++)
#pragma unroll
                            for (int r = 0; r < 4; r += 2)
                                *reinterpret_cast<double2 *>(
                                    st + (i * 16 + g + (r >> 1) * 8) * kF64PitchB + wn + j * 8 +
                                    t * 2) = make_double2(acc[i][j][r], acc[i][j][r + 1]);
                }
                __syncthreads();
                for (int idx = threadIdx.x; idx < 64 * (kF64BN / 2); idx += 256) {
                    const int row = idx / (kF64BN / 2), pair = idx % (kF64BN / 2);
                    const int m = m0 + h * 64 + row, n = n0 + 2 * pair;
                    if (m < p.M && n < p.N) {
                        const double2 v = *reinterpret_cast<const double2 *>(
                            st + row * kF64PitchB + 2 * pair);
                        const long long off = static_cast<long long>(m) * po.ldc + po.col_off + n;
                        for (int d = 0; d < po.ndst; d++)
                            *reinterpret_cast<double2 *>(po.dst[(po.rot + d) % po.ndst] + off) = v;
                    }
                }
                __syncthreads();
            }
            // make this thread's peer stores visible system-wide before the
            // kernel can be observed complete
            __threadfence_system();
            continue;
        }

        double *C = static_cast<double *>(p.c);
        const double *bias = static_cast<const double *>(p.bias);
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int r = 0; r < 4; r++) {
                    const int m = m0 + wm + i * 16 + g + (r >> 1) * 8;
                    const int n = n0 + wn + j * 8 + t * 2 + (r & 1);
                    if (m < p.M && n < p.N) {
                        double v = acc[i][j][r];
                        if (bias != nullptr || p.act != ACT_NONE) {
                            if (bias != nullptr) v += bias[n];
                            v = apply_activation_d(v, p.act);
                        }
                        C[oc + static_cast<long long>(m) * p.c_sm + static_cast<long long>(n) * p.c_sn] = v;
                    }
                }
    }
}

// The last wave's tiles as halves: one CTA per half tile, units
// w.full + [0, 2 w.tail); PEER as in f64_dmma_kernel (each thread stores its
// fragment pairs into every window).
template <bool PEER>
__global__ void __launch_bounds__(256, 1)
    f64_dmma_half_kernel(const SimtParams p, int a_vec, int b_vec, const F64Work w,
                         const F64PeerOut po)
{
    extern __shared__ __align__(16) double f64_smem[];
    long long batch;
    int m0, n0;
    f64_unit(w, w.full + blockIdx.x, batch, m0, n0);
    double *sa_all = f64_smem, *sb_all = f64_smem + kF64Stages * kF64StageA;
    if constexpr (!PEER) {
        f64_plain_unit<2>(p, sa_all, sb_all, batch, m0, n0, a_vec, b_vec);
    } else {
        using T = F64Tile<2>;
        double acc[T::TI][T::TJ][4];
        f64_tile_mainloop<2>(p, sa_all, sb_all, 0, 0, m0, n0, a_vec, b_vec, acc,
                             [](int, int) {});
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        const int g = lane >> 2, t = lane & 3;
        const int wm = (warp / 2) * T::kWarpM, wn = (warp % 2) * T::kWarpN;
#pragma unroll
        for (int i = 0; i < T::TI; i++)
#pragma unroll
            for (int j = 0; j < T::TJ; j++)
#pragma unroll
                for (int r = 0; r < 4; r += 2) {
                    const int m = m0 + wm + i * 16 + g + (r >> 1) * 8;
                    const int n = n0 + wn + j * 8 + t * 2;
                    if (m < p.M && n < p.N) {
                        const long long off = static_cast<long long>(m) * po.ldc + po.col_off + n;
                        for (int d = 0; d < po.ndst; d++)
                            *reinterpret_cast<double2 *>(po.dst[(po.rot + d) % po.ndst] + off) =
                                make_double2(acc[i][j][r], acc[i][j][r + 1]);
                    }
                }
        __threadfence_system();
    }
}

// ---------------------------------------------------------------------------
// The N-split block product with the exchange under the math (rank-2
// operands, one batch): one CTA per tile, as the plain kernel.  A CTA writes
// its tile into this rank's own window (local HBM) and leaves the tile's id
// in a slot for its SM (po.slots[%smid]); the next CTA to start on that SM
// claims the slot and, while its own k loop runs, copies a few 16-byte
// pieces of the claimed tile per k-block from the own window to the other
// ranks' windows (the next rank first, then around the ring).  So each
// tile's NVLink transfer runs under a later tile's DMMA work instead of
// holding its SM, and the hardware keeps scheduling the tiles.  A flush
// launch copies the tiles still in the slots when the last CTAs end.  The
// claims and hand-offs are atomic exchanges, never waits: a tile is copied
// once, by whoever takes it out of its slot.  (A persistent kernel doing the
// same with a fixed tile order lost 4-5 % of its math to the fixed order.)

// Pending remote copies of a claimed tile: its origin and width.
struct F64Pending {
    int m0, n0, width;
    int done, ops;
};

// Copy number e of a pending tile is piece e / peers of it (consecutive
// threads on consecutive 16-byte column pairs of a row) for destination rank
// (rot + 1 + e % peers) % ndst.  A piece read from the own window is stored
// one copy later, so the load's latency overlaps DMMA work instead of
// stalling a warp that feeds the tensor pipe.
struct F64Staged {
    double2 v;
    double *dst;
    bool valid;
};

__device__ __forceinline__ void f64_load_piece(const SimtParams &p, const F64PeerOut &po,
                                               const F64Pending &q, int e, F64Staged &sp)
{
    const int peers = po.ndst - 1;
    const int d = (po.rot + 1 + e % peers) % po.ndst;
    const int pairs = q.width / 2;
    const int idx = threadIdx.x + 256 * (e / peers);
    const int row = idx / pairs, pair = idx % pairs;
    const int m = q.m0 + row, n = q.n0 + 2 * pair;
    sp.valid = m < p.M && n < p.N;
    if (sp.valid) {
        const long long off = static_cast<long long>(m) * po.ldc + po.col_off + n;
        sp.v = __ldcg(reinterpret_cast<const double2 *>(po.dst[po.rot] + off));
        sp.dst = po.dst[d] + off;
    }
}

__device__ __forceinline__ void f64_store_piece(F64Staged &sp)
{
    if (sp.valid)
        *reinterpret_cast<double2 *>(sp.dst) = sp.v;
    sp.valid = false;
}

// Issues copies [q.done, q.ops) four at a time: four loads, then four
// stores, so a thread has several loads in flight.
__device__ __forceinline__ void f64_copy_rest(const SimtParams &p, const F64PeerOut &po,
                                              F64Pending &q)
{
    F64Staged sp[4];
    while (q.done < q.ops) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            sp[i].valid = false;
            if (q.done + i < q.ops)
                f64_load_piece(p, po, q, q.done + i, sp[i]);
        }
#pragma unroll
        for (int i = 0; i < 4; i++)
            f64_store_piece(sp[i]);
        q.done = min(q.done + 4, q.ops);
    }
}

// The copies owed for slot code `code` (work unit + 1; 0 = nothing).
__device__ __forceinline__ F64Pending f64_pending(const F64Work &w, const F64PeerOut &po,
                                                  unsigned long long code)
{
    F64Pending q;
    q.m0 = q.n0 = 0;
    q.width = kF64BN;
    q.done = q.ops = 0;
    if (code != 0) {
        long long batch;
        q.width = f64_unit(w, static_cast<long long>(code - 1), batch, q.m0, q.n0);
        q.ops = (po.ndst - 1) * (kF64BM * q.width / 2 / 256);
    }
    return q;
}

__device__ __forceinline__ uint32_t sm_id()
{
    uint32_t id;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(id));
    return id;
}

// WN = 4: full tiles (units [0, w.full)); WN = 2: half tiles (units
// w.full + [0, 2 w.tail)), launched after the full tiles.
template <int WN>
__global__ void __launch_bounds__(256, 1)
    f64_dmma_handoff_kernel(const SimtParams p, int a_vec, int b_vec, const F64Work w,
                            const F64PeerOut po)
{
    using T = F64Tile<WN>;
    // (no static shared memory: a static __shared__ word beside the dynamic
    // ring measured 13-14 % slower; the first ring word carries the slot
    // codes to the other threads instead, while the ring is idle)
    extern __shared__ __align__(16) double f64_smem[];
    unsigned long long *s_code = reinterpret_cast<unsigned long long *>(f64_smem);
    double *sa_all = f64_smem, *sb_all = f64_smem + kF64Stages * kF64StageA;
    const long long u = (WN == 4 ? 0 : w.full) + blockIdx.x;
    long long batch;
    int m0, n0;
    f64_unit(w, u, batch, m0, n0);
    const uint32_t sm = sm_id();
    const bool slotted = sm < static_cast<uint32_t>(po.nslots);
    // claim the tile the previous CTA on this SM left to be copied
    if (threadIdx.x == 0) {
        *s_code = slotted ? atomicExch(po.slots + sm, 0ull) : 0ull;
        __threadfence();
    }
    __syncthreads();
    F64Pending q = f64_pending(w, po, *s_code);
    // (f64_tile_mainloop's first barrier orders these reads before the ring
    // is filled)
    double acc[T::TI][T::TJ][4];
    // spread the q.ops copies evenly over the k blocks, Bresenham-style (a
    // division per k-block cost the DMMA warps measurable issue time); each
    // piece is loaded at one copy and stored at the next
    int credit = 0;
    F64Staged staged;
    staged.valid = false;
    f64_tile_mainloop<WN>(p, sa_all, sb_all, 0, 0, m0, n0, a_vec, b_vec, acc,
                          [&](int, int k_blocks) {
                              if (q.ops == 0)
                                  return;
                              credit += q.ops;
                              while (credit >= k_blocks && q.done < q.ops) {
                                  credit -= k_blocks;
                                  f64_store_piece(staged);
                                  f64_load_piece(p, po, q, q.done++, staged);
                              }
                          });
    f64_store_piece(staged);
    f64_copy_rest(p, po, q);
    // this tile into the own window
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int wm = (warp / WN) * T::kWarpM, wn = (warp % WN) * T::kWarpN;
    double *own = po.dst[po.rot];
#pragma unroll
    for (int i = 0; i < T::TI; i++)
#pragma unroll
        for (int j = 0; j < T::TJ; j++)
#pragma unroll
            for (int r = 0; r < 4; r += 2) {
                const int m = m0 + wm + i * 16 + g + (r >> 1) * 8;
                const int n = n0 + wn + j * 8 + t * 2;
                if (m < p.M && n < p.N)
                    *reinterpret_cast<double2 *>(own + static_cast<long long>(m) * po.ldc +
                                                 po.col_off + n) =
                        make_double2(acc[i][j][r], acc[i][j][r + 1]);
            }
    __syncthreads();   // every thread's part of the tile is written; the ring is idle
    // hand the tile to the next CTA on this SM; copy it here when there is
    // no slot, or copy what was left in the slot when two CTAs shared an SM
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned long long mine = static_cast<unsigned long long>(u) + 1;
        *s_code = slotted ? atomicExch(po.slots + sm, mine) : mine;
        __threadfence();
    }
    __syncthreads();
    const unsigned long long left = *s_code;
    if (left != 0) {
        q = f64_pending(w, po, left);
        f64_copy_rest(p, po, q);
    }
    // make this thread's peer stores visible system-wide before the kernel
    // can be observed complete
    __threadfence_system();
}

// Copies the tiles the last CTAs left in the slots (one CTA per slot) and
// empties the slots for the next call.
__global__ void __launch_bounds__(256)
    f64_handoff_flush_kernel(const SimtParams p, const F64Work w, const F64PeerOut po)
{
    __shared__ unsigned long long s_code;
    if (threadIdx.x == 0) {
        s_code = atomicExch(po.slots + blockIdx.x, 0ull);
        __threadfence();
    }
    __syncthreads();
    if (s_code == 0)
        return;
    F64Pending q = f64_pending(w, po, s_code);
    f64_copy_rest(p, po, q);
    __threadfence_system();
}

} // namespace ptg
