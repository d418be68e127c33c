// 2-CTA (cta_group::2) tcgen05 GEMM for 16-bit operands on sm_100a.
//
// A cluster of two CTAs on neighbouring SMs computes a 256 x 256 output tile:
// CTA r (r = 0, 1) loads rows [128 r, 128 r + 128) of the A tile and columns
// [128 r, 128 r + 128) of the B tile into its own shared memory, and one
// thread of CTA 0 issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16),
// which reads both CTAs' tiles and writes rows 128 r.. of D into CTA r's TMEM.
// Per FLOP each SM streams 2/3 of the bytes the single-CTA 128 x 256 tile
// needs (128 + 128 instead of 128 + 256 rows per K step).
//
// Protocol (no TMA multicast anywhere):
//   full[s]   lives in CTA 0; CTA 0 posts expect_tx for both CTAs' bytes and
//             both CTAs' TMA loads complete on it.
//   empty[s]  one per CTA; the MMA thread commits to its own and, through the
//             peer's shared::cluster address, to CTA 1's.
//   tfull[a]  one per CTA, committed the same way when accumulator a is done.
//   tempty[a] lives in CTA 0 with 8 arrivals: the 4 epilogue warps of each CTA
//             (CTA 1 arrives remotely).
// Waits are bounded as in gemm_tc.cuh.  Cluster barriers bracket the kernel
// so no barrier is used before the peer initialised it or after it exited.
#pragma once

#include "gemm_tc.cuh"

namespace ptg {

template <int IN_KIND, int OUT>
struct Tc2Config {
    static constexpr int BM = 256, BN = 256;          // per CTA pair
    static constexpr int kRowsCta = 128, kColsCta = 128;
    static constexpr int BK = 64;                      // 128 bytes of 16-bit K
    static constexpr int kMmaK = 16;
    static constexpr int kKSteps = BK / kMmaK;
    static constexpr int kChunk = 64;                  // MN elements per 128-byte row
    static constexpr int kChunkBytes = 128 * BK;       // one MN-major box (8 KB)
    static constexpr int kATile = kRowsCta * BK * 2;   // 16 KB
    static constexpr int kBTile = kColsCta * BK * 2;   // 16 KB
    static constexpr int kLoadBytes = kATile + kBTile; // per CTA and stage
    static constexpr int kStageBytes = kLoadBytes;
    static constexpr int kStages = 6;
    static constexpr int kEpiCols = 64;                // 128 bytes of 16-bit output
    static constexpr int kEpiChunks = BN / kEpiCols;
    static constexpr int kEpiBufBytes = 32 * 128;
    static constexpr int kEpiWarps = 4;
    static constexpr int kThreads = 32 * (2 + kEpiWarps);
    static constexpr int kAccCols = BN;
    static constexpr int kTmemCols = 2 * kAccCols;     // 512: double-buffered
    static constexpr int kRingBytes = kStages * kStageBytes;
    static constexpr int kEpiOffset = kRingBytes;
    static constexpr int kBarOffset = kEpiOffset + kEpiWarps * 2 * kEpiBufBytes;
    static constexpr int kNumBars = 2 * kStages + 4 + 1;
    static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
    static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
    static_assert(IN_KIND == IN_F16 || IN_KIND == IN_BF16, "16-bit operands only");
};

// Settle time for copies a CTA may still have in flight after it gave up a
// wait; only the abort path uses it.
constexpr uint64_t kAbortSettleNs = 200000ull;

__device__ __forceinline__ void settle_after_abort()
{
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < kAbortSettleNs) {
    }
}

template <int IN_KIND, int OUT>
__global__ void __launch_bounds__(Tc2Config<IN_KIND, OUT>::kThreads, 1)
    tc2_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                    const __grid_constant__ CUtensorMap tma_b,
                    const __grid_constant__ CUtensorMap tma_c, const TcParams p)
{
    using Cfg = Tc2Config<IN_KIND, OUT>;
    constexpr int S = Cfg::kStages;
    constexpr int BN = Cfg::BN;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kBarOffset);
    uint64_t *full = bars;
    uint64_t *empty = bars + S;
    uint64_t *tfull = bars + 2 * S;
    uint64_t *tempty = bars + 2 * S + 2;
    uint64_t *drain = bars + 2 * S + 4;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + Cfg::kNumBars);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_cta_rank();
    const long long cluster = blockIdx.x >> 1;
    const long long nclusters = gridDim.x >> 1;

    if (warp == 0 && lane == 0) {
        prefetch_tensor_map(&tma_a);
        prefetch_tensor_map(&tma_b);
        prefetch_tensor_map(&tma_c);
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 2 * Cfg::kEpiWarps);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // programmatic dependent launch, as in tc_gemm_kernel
    grid_dependency_wait();
    grid_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------------------ producer (both CTAs)
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, parity_mask = 0;
            bool ok = true;
            for (long long t = cluster; ok && t < p.tiles; t += nclusters) {
                const int nb = static_cast<int>(t % p.n_blocks);
                const long long r = t / p.n_blocks;
                const int mb = static_cast<int>(r % p.m_blocks);
                const long long batch = r / p.m_blocks;
                int c[3], ca[3], cb[3];
                decode_batch(batch, p, c);
                operand_coords(c, p.a_slot, p.nbd, ca);
                operand_coords(c, p.b_slot, p.nbd, cb);
                const int m0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::kRowsCta;
                const int n0 = nb * BN + static_cast<int>(rank) * Cfg::kColsCta;
                for (int kb = 0; kb < p.k_blocks; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort)) {
                        record_failure(abort, p.status, DEV_TIMEOUT_PRODUCER);
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + stage * Cfg::kStageBytes;
                    uint8_t *sb = sa + Cfg::kATile;
                    if (rank == 0)
                        mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kLoadBytes);
                    const uint32_t full0 = map_to_cta(smem_addr(&full[stage]), 0);
                    const int k0 = kb * Cfg::BK;
                    if (!p.a_mn_major) {
                        tma_load_5d_pair(sa, &tma_a, full0, k0, m0, ca[0], ca[1], ca[2]);
                    } else {
#pragma unroll
                        for (int j = 0; j < Cfg::kRowsCta / Cfg::kChunk; j++)
                            tma_load_5d_pair(sa + j * Cfg::kChunkBytes, &tma_a, full0,
                                             m0 + j * Cfg::kChunk, k0, ca[0], ca[1], ca[2]);
                    }
                    if (!p.b_mn_major) {
                        tma_load_5d_pair(sb, &tma_b, full0, k0, n0, cb[0], cb[1], cb[2]);
                    } else {
#pragma unroll
                        for (int j = 0; j < Cfg::kColsCta / Cfg::kChunk; j++)
                            tma_load_5d_pair(sb + j * Cfg::kChunkBytes, &tma_b, full0,
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
            if (rank == 0) {
                // CTA 0's full barriers count both CTAs' bytes of every stage
                // it posted: let them land (bounded, ignores the abort flag)
                for (int s = 0; s < S; s++) {
                    if (issued_mask & (1u << s)) {
                        int no_abort = 0;
                        mbar_wait(&full[s], (parity_mask >> s) & 1u, &no_abort);
                    }
                }
            }
            if (*abort)
                settle_after_abort();
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (CTA 0)
        if (lane == 0 && rank == 0) {
            int stage = 0;
            uint32_t phase = 0;
            long long iter = 0;
            bool ok = true;
            const uint32_t smem_base = smem_addr(smem);
            for (long long t = cluster; ok && t < p.tiles; t += nclusters, iter++) {
                const int acc = static_cast<int>(iter & 1);
                const uint32_t acc_phase = static_cast<uint32_t>((iter >> 1) & 1);
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort)) {
                    record_failure(abort, p.status, DEV_TIMEOUT_MMA);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::kAccCols);
                for (int kb = 0; kb < p.k_blocks; kb++) {
                    if (!mbar_wait(&full[stage], phase, abort)) {
                        record_failure(abort, p.status, DEV_TIMEOUT_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
                    const uint32_t sb = sa + Cfg::kATile;
#pragma unroll
                    for (int k = 0; k < Cfg::kKSteps; k++) {
                        const uint32_t a_off = p.a_mn_major ? k * Cfg::kMmaK * 128 : k * 32;
                        const uint32_t b_off = p.b_mn_major ? k * Cfg::kMmaK * 128 : k * 32;
                        const uint64_t ad = smem_desc(sa + a_off, p.a_mn_major ? Cfg::kChunkBytes : 16,
                                                      1024, kLayoutSw128);
                        const uint64_t bd = smem_desc(sb + b_off, p.b_mn_major ? Cfg::kChunkBytes : 16,
                                                      1024, kLayoutSw128);
                        umma_f16_pair(d_tmem, ad, bd, p.idesc, (kb | k) != 0);
                    }
                    const uint32_t e0 = smem_addr(&empty[stage]);
                    umma_commit_pair(e0);
                    umma_commit_pair(map_to_cta(e0, 1));
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok)
                    break;
                const uint32_t f0 = smem_addr(&tfull[acc]);
                umma_commit_pair(f0);
                umma_commit_pair(map_to_cta(f0, 1));
            }
            umma_commit_pair(smem_addr(drain));
            int no_abort = 0;
            mbar_wait(drain, 0, &no_abort);
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int ew = warp - 2;
        const int quad = warp & 3;
        uint8_t *stage_buf = smem + Cfg::kEpiOffset + ew * 2 * Cfg::kEpiBufBytes;
        int buf = 0;
        long long iter = 0;
        for (long long t = cluster; t < p.tiles; t += nclusters, iter++) {
            const int acc = static_cast<int>(iter & 1);
            const uint32_t acc_phase = static_cast<uint32_t>((iter >> 1) & 1);
            const bool got = __all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, abort));
            if (!got) {
                if (lane == 0)
                    record_failure(abort, p.status, DEV_TIMEOUT_EPILOGUE);
                break;
            }
            tc_fence_after();
            const int nb = static_cast<int>(t % p.n_blocks);
            const long long r = t / p.n_blocks;
            const int mb = static_cast<int>(r % p.m_blocks);
            const long long batch = r / p.m_blocks;
            int c[3];
            decode_batch(batch, p, c);
            const int row0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::kRowsCta + quad * 32;
            const int n0 = nb * BN;
            const uint32_t t_acc = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                   static_cast<uint32_t>(acc * Cfg::kAccCols);
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
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_cluster(map_to_cta(smem_addr(&tempty[acc]), 0));
                }
                const int col0 = n0 + ch * Cfg::kEpiCols;
                if (p.bias != nullptr || p.act != ACT_NONE)
                    apply_epilogue<OUT, Cfg::kEpiCols>(v, p.bias, p.act, col0, p.N, lane);
                uint8_t *sbuf = stage_buf + buf * Cfg::kEpiBufBytes;
                if (lane == 0)
                    bulk_wait_group_read<1>();
                __syncwarp();
                uint8_t *rowp = sbuf + lane * 128;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    uint4 q;
                    q.x = pack2(v[8 * j + 0], v[8 * j + 1], OUT);
                    q.y = pack2(v[8 * j + 2], v[8 * j + 3], OUT);
                    q.z = pack2(v[8 * j + 4], v[8 * j + 5], OUT);
                    q.w = pack2(v[8 * j + 6], v[8 * j + 7], OUT);
                    *reinterpret_cast<uint4 *>(rowp + ((j ^ (lane & 7)) << 4)) = q;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && col0 < p.N && row0 < p.M) {
                    tma_store_5d(&tma_c, sbuf, col0, row0, c[0], c[1], c[2]);
                    bulk_commit_group();
                }
                buf ^= 1;
            }
        }
        if (lane == 0)
            bulk_wait_group<0>();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    }
}

} // namespace ptg
