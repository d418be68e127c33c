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
#pragma once

#include "gemm_simt.cuh"
#include "internal.h"

namespace ptg {

constexpr int kF64BM = 128, kF64BN = 128, kF64BK = 16;
// Tiles run in groups of kF64GroupM row blocks, row block fastest: the CTAs
// resident at one time share a few A row blocks and B column blocks, so the
// operands of a large product come from DRAM a few times instead of once
// per resident row of tiles (8192^3 with the row-major tile order read
// 15.8 GB for 1.6 GB of operands).
constexpr int kF64GroupM = 16;
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

// Ring stage geometry for a k-block depth BK (16 for the plain kernel, 8
// for the N-split peer kernel): A rows pitched BK + 4 doubles and B rows
// kF64PitchB doubles, so every fragment read of a half-warp hits distinct
// banks.
template <int BK>
struct F64Stage {
    static constexpr int kPitchA = BK + 4;
    static constexpr int kA = kF64BM * kPitchA;   // doubles
    static constexpr int kB = BK * kF64PitchB;
};

// Fills one ring stage with the A tile [m0, m0+128) x [k0, k0+BK) and the B
// tile [k0, k0+BK) x [n0, n0+128).
template <int BK>
__device__ __forceinline__ void f64_load_stage_k(const SimtParams &p, double *sa, double *sb,
                                                 long long oa, long long ob, int m0, int n0,
                                                 int k0, bool a_vec, bool b_vec)
{
    constexpr int kPitchA = F64Stage<BK>::kPitchA;
    const double *A = static_cast<const double *>(p.a);
    const double *B = static_cast<const double *>(p.b);
    const int tid = threadIdx.x;
    if (a_vec) {
        // 128 rows x BK / 2 pairs of k
#pragma unroll
        for (int r = 0; r < BK / 4; r++) {
            const int e = tid + 256 * r;
            const int row = e / (BK / 2), kp = (e % (BK / 2)) * 2;
            const int m = m0 + row, k = k0 + kp;
            const bool ok = m < p.M && k < p.K;   // K even: a pair is all in or all out
            const double *src = ok ? A + oa + static_cast<long long>(m) * p.a_sm + k : A;
            cp_async16(sa + row * kPitchA + kp, src, ok);
        }
    } else {
#pragma unroll
        for (int r = 0; r < BK / 2; r++) {
            const int e = tid + 256 * r;
            const int row = e / BK, kk = e % BK;
            const int m = m0 + row, k = k0 + kk;
            sa[row * kPitchA + kk] =
                (m < p.M && k < p.K) ? A[oa + static_cast<long long>(m) * p.a_sm +
                                         static_cast<long long>(k) * p.a_sk]
                                     : 0.0;
        }
    }
    if (b_vec) {
        // BK k rows x 64 pairs of n
#pragma unroll
        for (int r = 0; r < BK / 4; r++) {
            const int e = tid + 256 * r;
            const int kr = e >> 6, np = (e & 63) * 2;
            const int k = k0 + kr, n = n0 + np;
            const bool ok = k < p.K && n < p.N;   // N even: a pair is all in or all out
            const double *src = ok ? B + ob + static_cast<long long>(k) * p.b_sk + n : B;
            cp_async16(sb + kr * kF64PitchB + np, src, ok);
        }
    } else {
#pragma unroll
        for (int r = 0; r < BK / 2; r++) {
            const int e = tid + 256 * r;
            const int kr = e >> 7, col = e & 127;
            const int k = k0 + kr, n = n0 + col;
            sb[kr * kF64PitchB + col] =
                (k < p.K && n < p.N) ? B[ob + static_cast<long long>(k) * p.b_sk +
                                         static_cast<long long>(n) * p.b_sn]
                                     : 0.0;
        }
    }
}

__device__ __forceinline__ void f64_load_stage(const SimtParams &p, double *sa, double *sb,
                                               long long oa, long long ob, int m0, int n0, int k0,
                                               bool a_vec, bool b_vec)
{
    f64_load_stage_k<kF64BK>(p, sa, sb, oa, ob, m0, n0, k0, a_vec, b_vec);
}

// One k-block of MMAs of a warp's 64 x 32 block: BK / 4 k4 steps of 4 x 4
// m16n8 fragments.
template <int BK = kF64BK>
__device__ __forceinline__ void f64_mma_kblock(double (&acc)[4][4][4], const double *sa,
                                               const double *sb, int wm, int wn, int g, int t)
{
    constexpr int kPitchA = F64Stage<BK>::kPitchA;
#pragma unroll
    for (int kk = 0; kk < BK; kk += 4) {
        double af[4][2], bf[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            af[i][0] = sa[(wm + i * 16 + g) * kPitchA + kk + t];
            af[i][1] = sa[(wm + i * 16 + g + 8) * kPitchA + kk + t];
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
            bf[j] = sb[(kk + t) * kF64PitchB + wn + j * 8 + g];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
                dmma_16x8x4(acc[i][j], af[i], bf[j]);
    }
}

// Tile (mb, nb) of tile index L in the grouped order: kF64GroupM row blocks
// per group, row block fastest.
__device__ __forceinline__ void f64_grouped_tile(long long L, int m_blocks, int n_blocks,
                                                 int &mb, int &nb)
{
    const long long per_group = static_cast<long long>(kF64GroupM) * n_blocks;
    const long long group = L / per_group;
    const int first_m = static_cast<int>(group) * kF64GroupM;
    const int gm = min(kF64GroupM, m_blocks - first_m);
    const long long r = L - group * per_group;
    mb = first_m + static_cast<int>(r % gm);
    nb = static_cast<int>(r / gm);
}

// The plain product into p.c (optional bias / activation).
__global__ void __launch_bounds__(256, 1)
    f64_dmma_kernel(const SimtParams p, int a_vec, int b_vec)
{
    extern __shared__ __align__(16) double f64_smem[];
    double *sa_all = f64_smem;
    double *sb_all = f64_smem + kF64Stages * kF64StageA;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int wm = (warp >> 2) * 64, wn = (warp & 3) * 32;
    const int m_blocks = (p.M + kF64BM - 1) / kF64BM;
    const int k_blocks = (p.K + kF64BK - 1) / kF64BK;
    // grouped tile order when the grid covers every row block (the launch
    // grid is (column blocks, row blocks, batches), x fastest)
    int mb_first = blockIdx.y, nb = blockIdx.x, mb_step = gridDim.y;
    if (static_cast<int>(gridDim.y) == m_blocks) {
        f64_grouped_tile(static_cast<long long>(blockIdx.y) * gridDim.x + blockIdx.x, m_blocks,
                         gridDim.x, mb_first, nb);
        mb_step = m_blocks;
    }
    const int n0 = nb * kF64BN;

    for (long long batch = blockIdx.z; batch < p.batches; batch += gridDim.z)
    for (int mb = mb_first; mb < m_blocks; mb += mb_step) {
        const int m0 = mb * kF64BM;
        long long oa = 0, ob = 0, oc = 0, rem = batch;
        for (int d = p.nbd - 1; d >= 0; d--) {
            const long long coord = rem % p.bshape[d];
            rem /= p.bshape[d];
            oa += coord * p.a_bs[d];
            ob += coord * p.b_bs[d];
            oc += coord * p.c_bs[d];
        }
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
                f64_load_stage(p, sa_all + s * kF64StageA, sb_all + s * kF64StageB, oa, ob, m0,
                               n0, s * kF64BK, a_vec, b_vec);
            cp_async_commit();
        }
        for (int kb = 0; kb < k_blocks; kb++) {
            cp_async_wait<kF64Stages - 2>();
            __syncthreads();
            const int nxt = kb + kF64Stages - 1;
            if (nxt < k_blocks)
                f64_load_stage(p, sa_all + (nxt % kF64Stages) * kF64StageA,
                               sb_all + (nxt % kF64Stages) * kF64StageB, oa, ob, m0, n0,
                               nxt * kF64BK, a_vec, b_vec);
            cp_async_commit();
            f64_mma_kblock(acc, sa_all + (kb % kF64Stages) * kF64StageA,
                           sb_all + (kb % kF64Stages) * kF64StageB, wm, wn, g, t);
        }
        cp_async_wait<0>();

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

// ---------------------------------------------------------------------------
// The N-split block product whose results go to every rank's window over
// NVLink (rank-2 operands, no batch).  Persistent: one CTA per SM walks the
// tiles in the grouped order with the plain kernel's ring.  When a tile's k
// loop ends, the CTA writes the tile into this rank's own window (local HBM,
// fragment layout), and during the NEXT tile's k loop every thread copies a
// few 16-byte pieces of it per k-block from there to the other ranks'
// windows, the next rank first and so on around the ring, so every rank
// spreads its traffic over all peers and the NVLink transfer runs under the
// DMMA work instead of after it.  (A non-persistent kernel that stored each
// tile to every window when it finished held each wave's SMs idle during the
// stores; staging the tile in shared memory instead left room only for a ring
// of 2 x 16-deep or 4 x 8-deep k-blocks, which slowed the math by 4-13 %.)
// Only the last tile of each CTA is copied after the math.
constexpr int kF64PeerSmemBytes = kF64SmemBytes;
// 16-byte pieces of one tile per thread
constexpr int kF64PeerPieces = kF64BM * (kF64BN / 2) / 256;

__global__ void __launch_bounds__(256, 1)
    f64_dmma_peer_kernel(const SimtParams p, int a_vec, int b_vec, const F64PeerOut po)
{
    extern __shared__ __align__(16) double f64_smem[];
    double *sa_all = f64_smem;
    double *sb_all = f64_smem + kF64Stages * kF64StageA;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int wm = (warp >> 2) * 64, wn = (warp & 3) * 32;
    const int m_blocks = (p.M + kF64BM - 1) / kF64BM;
    const int n_blocks = (p.N + kF64BN - 1) / kF64BN;
    const int k_blocks = (p.K + kF64BK - 1) / kF64BK;
    const long long tiles = static_cast<long long>(m_blocks) * n_blocks;
    double *own = po.dst[po.rot];
    const int peers = po.ndst - 1;
    const int ops = kF64PeerPieces * peers;   // remote copies per thread and tile

    // origin of the tile whose remote copies are pending, and how many of
    // them this thread has issued
    int pm0 = 0, pn0 = 0, done = ops;
    auto copy_op = [&](int e) {
        const int d = (po.rot + 1 + e % peers) % po.ndst;
        const int idx = threadIdx.x + 256 * (e / peers);
        const int row = idx / (kF64BN / 2), pair = idx % (kF64BN / 2);
        const int m = pm0 + row, n = pn0 + 2 * pair;
        if (m < p.M && n < p.N) {
            const long long off = static_cast<long long>(m) * po.ldc + po.col_off + n;
            const double2 v = __ldcg(reinterpret_cast<const double2 *>(own + off));
            *reinterpret_cast<double2 *>(po.dst[d] + off) = v;
        }
    };

    for (long long L = blockIdx.x; L < tiles; L += gridDim.x) {
        int mb, nb;
        f64_grouped_tile(L, m_blocks, n_blocks, mb, nb);
        const int m0 = mb * kF64BM, n0 = nb * kF64BN;
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
                f64_load_stage(p, sa_all + s * kF64StageA, sb_all + s * kF64StageB, 0, 0, m0,
                               n0, s * kF64BK, a_vec, b_vec);
            cp_async_commit();
        }
        for (int kb = 0; kb < k_blocks; kb++) {
            cp_async_wait<kF64Stages - 2>();
            __syncthreads();
            const int nxt = kb + kF64Stages - 1;
            if (nxt < k_blocks)
                f64_load_stage(p, sa_all + (nxt % kF64Stages) * kF64StageA,
                               sb_all + (nxt % kF64Stages) * kF64StageB, 0, 0, m0, n0,
                               nxt * kF64BK, a_vec, b_vec);
            cp_async_commit();
            f64_mma_kblock(acc, sa_all + (kb % kF64Stages) * kF64StageA,
                           sb_all + (kb % kF64Stages) * kF64StageB, wm, wn, g, t);
            // a share of the previous tile's remote copies, spread evenly
            // over the k loop
            const int target = static_cast<int>(
                (static_cast<long long>(kb + 1) * ops + k_blocks - 1) / k_blocks);
            for (; done < target; done++)
                copy_op(done);
        }
        cp_async_wait<0>();
        for (; done < ops; done++)
            copy_op(done);
        // this tile into the rank's own window
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int r = 0; r < 4; r += 2) {
                    const int m = m0 + wm + i * 16 + g + (r >> 1) * 8;
                    const int n = n0 + wn + j * 8 + t * 2;
                    if (m < p.M && n < p.N)
                        *reinterpret_cast<double2 *>(own + static_cast<long long>(m) * po.ldc +
                                                     po.col_off + n) =
                            make_double2(acc[i][j][r], acc[i][j][r + 1]);
                }
        __syncthreads();   // the tile is in the own window for every thread's copies
        pm0 = m0;
        pn0 = n0;
        done = 0;
    }
    for (; done < ops; done++)
        copy_op(done);
    // make this thread's peer stores visible system-wide before the kernel
    // can be observed complete
    __threadfence_system();
}

} // namespace ptg
