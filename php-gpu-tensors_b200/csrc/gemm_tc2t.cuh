// 2-CTA strict float32 (3xTF32) GEMM with the A operand in tensor memory.
//
// tc2x3_gemm_kernel reads both operands of its three MMAs per K step
// (hi*hi, hi*lo, lo*hi) from shared memory, next to the TMA writes of the raw
// tiles and the split warps' reads of them and writes of lo: per 32-deep
// k-block each CTA moves 192 KB through shared memory in the 1536 tensor
// cycles of its 12 MMAs, the whole 128 B/clk of the SM's shared-memory port.
// Here the split warps of the A operand write hi and lo of each CTA's 128 A
// rows into tensor memory (tcgen05.st, one TMEM lane per row, one column per
// element of K) and the MMAs take A from there (tcgen05.mma with [a_tmem]):
// shared memory carries only the raw tiles, their split reads, B's lo tile
// and B's three operand reads, 128 KB per k-block.
//
// TMEM per CTA: the accumulator (columns [0, 256)) and kLoStages slots of A
// hi (32 columns) and lo (32 columns) from column 256.  The running total of
// the finished 128-deep K chunks (the accumulator is restarted every 4
// k-blocks, since the tensor core's FP32 accumulation error over a long K
// would exceed the float32 bound) lives in the registers of the 8 epilogue
// warps, 128 columns each (warpgroup register reallocation gives them 160
// registers), and is added in the same order as tc2x3_gemm_kernel's TMEM
// total, so the two kernels' results are bit-identical.
//
// Warps: warpgroup 0: TMA producer, MMA issuer (TMEM owner), 2 B-split
// warps; warpgroup 1: 4 A-split warps (warp w writes TMEM lanes
// 32 (w mod 4) .. + 32, the rows it splits); warpgroups 2-3: epilogue.
// Only K-major A (one 128-byte row of K per A row in the raw tile), no
// split-K and no summed batch axes; other strict float32 pair products run
// tc2x3_gemm_kernel.
//
// Barriers (no TMA multicast anywhere):
//   full[s]      per CTA: its own TMA loads of stage s landed.
//   ready[s]     CTA 0, 2 x 6 arrivals: the split warps of both CTAs wrote
//                B lo and A hi / lo of stage s (release.cluster).
//   empty[s], lo_free[l], tfull
//                per CTA, committed by CTA 0's MMA thread to both CTAs.
//   tempty       CTA 0, 2 x 8 arrivals: the epilogue warps of both CTAs read
//                the accumulator chunk.
// Every wait is bounded; cluster barriers bracket the kernel.
#pragma once

#include "gemm_tc2.cuh"

namespace ptg {

struct Tc2tConfig {
    static constexpr int BM = 256, BN = 256;            // per CTA pair
    static constexpr int kRowsCta = 128, kColsCta = 128;
    static constexpr int BK = 32;                       // one 128-byte row of float32 K
    static constexpr int kMmaK = 8;
    static constexpr int kKSteps = BK / kMmaK;
    static constexpr int kChunk = 32;                   // MN elements per 128-byte row
    static constexpr int kChunkBytes = 128 * BK;        // one MN-major box
    static constexpr uint32_t kMnLayout = kLayoutSw128Base32B;
    static constexpr uint32_t kMnSbo = 512;
    static constexpr int kATile = kRowsCta * BK * 4;    // 16 KB
    static constexpr int kBTile = kColsCta * BK * 4;    // 16 KB
    static constexpr int kLoadBytes = kATile + kBTile;
#ifndef PTG_TC2T_STAGES
#define PTG_TC2T_STAGES 4
#endif
    static constexpr int kStages = PTG_TC2T_STAGES;     // raw A + B tiles
#ifndef PTG_TC2T_LO_STAGES
#define PTG_TC2T_LO_STAGES 3
#endif
    static constexpr int kLoStages = PTG_TC2T_LO_STAGES; // B lo tiles / A TMEM slots
    static constexpr int kLoOffset = kStages * kLoadBytes;
    static constexpr int kRingBytes = kLoOffset + kLoStages * kBTile;
    static constexpr int kEpiWarps = 8;
    static constexpr int kEpiCols = 32;                 // 128 bytes of float32 output
    static constexpr int kWarpCols = 128;               // columns per epilogue warp
    static constexpr int kEpiBufBytes = 32 * 128;
    static constexpr int kEpiOffset = kRingBytes;
    static constexpr int kBarOffset = kEpiOffset + kEpiWarps * kEpiBufBytes;
    // full, empty, ready per stage; lo_free per slot; tfull, tempty, drain
    static constexpr int kNumBars = 3 * kStages + kLoStages + 3;
    static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
    static constexpr int kBSplitWarps = 2, kASplitWarps = 4;
    static constexpr int kThreads = 512;                // four warpgroups
    static constexpr int kChunkKB = 4;                  // k-blocks per accumulator chunk
    static constexpr int kASlot0 = BN;                  // first TMEM column of the A slots
    static constexpr int kASlotCols = 2 * BK;           // hi, lo
    static constexpr int kTmemCols = 512;
    // 512 threads launch with 128 registers each; warpgroups 0 and 1 (the
    // A split holds 16 hi and 16 lo values per thread) drop to 96, the
    // epilogue warpgroups rise to 160 (the 128-float running total), which
    // adds up to the launch allocation exactly; an increase beyond it would
    // wait forever, so the launcher checks the compiled register count.
#ifndef PTG_TC2T_REGS
#define PTG_TC2T_REGS 96, 96, 160
#endif
    static constexpr int kRegsByWg[3] = {PTG_TC2T_REGS};
    static constexpr int kRegsWg0 = kRegsByWg[0], kRegsWg1 = kRegsByWg[1], kRegsEpi = kRegsByWg[2];
    static constexpr int kRegsTotal = 128 * kRegsWg0 + 128 * kRegsWg1 + 256 * kRegsEpi;
    static_assert(kRegsTotal <= 128 * kThreads, "register reallocation exceeds 128 per thread");
    static_assert(kASlot0 + kLoStages * kASlotCols <= kTmemCols, "TMEM budget");
    static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
};

// hi as the tensor core takes a float32 operand (low 13 mantissa bits
// dropped), keeping NaN a NaN; lo = tf32(x - hi), 0 for infinities and NaN.
__device__ __forceinline__ float tf32_hi(float x)
{
    return isnan(x) ? __int_as_float(0x7fffe000) : trunc_tf32(x);
}
__device__ __forceinline__ float tf32_lo(float x)
{
    return isfinite(x) ? round_tf32(x - trunc_tf32(x)) : 0.0f;
}

__global__ void __launch_bounds__(Tc2tConfig::kThreads, 1)
    tc2t_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                     const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_c, const TcParams p)
{
    using Cfg = Tc2tConfig;
    constexpr int S = Cfg::kStages;
    constexpr int L = Cfg::kLoStages;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kBarOffset);
    uint64_t *full = bars;
    uint64_t *empty = bars + S;
    uint64_t *ready = bars + 2 * S;
    uint64_t *lo_free = bars + 3 * S;
    uint64_t *tfull = bars + 3 * S + L;
    uint64_t *tempty = tfull + 1;
    uint64_t *drain = tfull + 2;
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
            mbar_init(&ready[s], 2 * (Cfg::kBSplitWarps + Cfg::kASplitWarps));
        }
        for (int l = 0; l < L; l++)
            mbar_init(&lo_free[l], 1);
        mbar_init(tfull, 1);
        mbar_init(tempty, 2 * Cfg::kEpiWarps);
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
    grid_dependency_wait();
    grid_launch_dependents();

    if (warp < 4) {
        warpgroup_reg_dealloc<Cfg::kRegsWg0>();
        if (warp == 0) {
            // -------------------------------------------------------- producer (both CTAs)
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
                    const int n0 = nb * Cfg::BN + static_cast<int>(rank) * Cfg::kColsCta;
                    for (int kb = 0; kb < p.k_blocks; kb++) {
                        if (!mbar_wait(&empty[stage], phase ^ 1, abort)) {
                            record_failure(abort, p.status, DEV_TIMEOUT_PRODUCER);
                            ok = false;
                            break;
                        }
                        uint8_t *sa = smem + stage * Cfg::kLoadBytes;
                        uint8_t *sb = sa + Cfg::kATile;
                        mbar_arrive_expect_tx(&full[stage], Cfg::kLoadBytes);
                        const int k0 = kb * Cfg::BK;
                        tma_load_5d(sa, &tma_a, &full[stage], k0, m0, ca[0], ca[1], ca[2]);
                        if (!p.b_mn_major) {
                            tma_load_5d(sb, &tma_b, &full[stage], k0, n0, cb[0], cb[1], cb[2]);
                        } else {
#pragma unroll
                            for (int j = 0; j < Cfg::kColsCta / Cfg::kChunk; j++)
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
                // every copy this thread started lands before shared memory
                // can be released (bounded, ignores the abort flag)
                for (int s = 0; s < S; s++) {
                    if (issued_mask & (1u << s)) {
                        int no_abort = 0;
                        mbar_wait(&full[s], (parity_mask >> s) & 1u, &no_abort);
                    }
                }
            }
        } else if (warp == 1) {
            // -------------------------------------------------------- MMA issuer (CTA 0)
            if (lane == 0 && rank == 0) {
                int stage = 0, slot = 0;
                uint32_t phase = 0;
                long long uses = 0;   // accumulator chunks issued
                bool ok = true;
                const uint32_t smem_base = smem_addr(smem);
                const uint32_t b_lbo = p.b_mn_major ? Cfg::kChunkBytes : 16;
                const uint32_t b_sbo = p.b_mn_major ? Cfg::kMnSbo : 1024;
                const uint32_t b_lay = p.b_mn_major ? Cfg::kMnLayout : kLayoutSw128;
                for (long long t = cluster; ok && t < p.tiles; t += nclusters) {
                    for (int kb = 0; kb < p.k_blocks; kb++) {
                        const int kc = kb % Cfg::kChunkKB;
                        if (kc == 0) {
                            if (!mbar_wait_cluster(tempty, static_cast<uint32_t>(uses & 1) ^ 1u,
                                                   abort)) {
                                record_failure(abort, p.status, DEV_TIMEOUT_MMA);
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                        }
                        if (!mbar_wait_cluster(&ready[stage], phase, abort)) {
                            record_failure(abort, p.status, DEV_TIMEOUT_MMA);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sb = smem_base + stage * Cfg::kLoadBytes + Cfg::kATile;
                        const uint32_t lb = smem_base + Cfg::kLoOffset + slot * Cfg::kBTile;
                        const int a_col = Cfg::kASlot0 + slot * Cfg::kASlotCols;
                        const uint32_t a_hi = tmem_base + static_cast<uint32_t>(a_col);
                        const uint32_t a_lo = a_hi + Cfg::BK;
#pragma unroll
                        for (int k = 0; k < Cfg::kKSteps; k++) {
                            const uint32_t b_off = p.b_mn_major ? k * Cfg::kMmaK * 128 : k * 32;
                            const uint64_t bd = smem_desc(sb + b_off, b_lbo, b_sbo, b_lay);
                            const uint64_t bd_lo = smem_desc(lb + b_off, b_lbo, b_sbo, b_lay);
                            const uint32_t ak = static_cast<uint32_t>(k * Cfg::kMmaK);
                            umma_tf32_pair_ts(tmem_base, a_hi + ak, bd, p.idesc, (kc | k) != 0);
                            umma_tf32_pair_ts(tmem_base, a_hi + ak, bd_lo, p.idesc, 1);
                            umma_tf32_pair_ts(tmem_base, a_lo + ak, bd, p.idesc, 1);
                        }
                        const uint32_t e0 = smem_addr(&empty[stage]);
                        umma_commit_pair(e0);
                        umma_commit_pair(map_to_cta(e0, 1));
                        const uint32_t l0 = smem_addr(&lo_free[slot]);
                        umma_commit_pair(l0);
                        umma_commit_pair(map_to_cta(l0, 1));
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1;
                        }
                        if (++slot == L)
                            slot = 0;
                        if (kc == Cfg::kChunkKB - 1 || kb == p.k_blocks - 1) {
                            const uint32_t f0 = smem_addr(tfull);
                            umma_commit_pair(f0);
                            umma_commit_pair(map_to_cta(f0, 1));
                            uses++;
                        }
                    }
                }
                umma_commit_pair(smem_addr(drain));
                int no_abort = 0;
                mbar_wait(drain, 0, &no_abort);
            }
        } else if (warp < 2 + Cfg::kBSplitWarps) {
            // -------------------------------------------------------- B split (both CTAs)
            // lo = tf32(x - trunc(x)) of this CTA's raw B tile into the lo
            // slot, in the raw tile's layout; computed into registers before
            // the slot is free.  Waits are warp-uniform.
            const int bt = threadIdx.x - 64;
            constexpr int kThr = 32 * Cfg::kBSplitWarps;
            constexpr int kPer = Cfg::kBTile / 16 / kThr;
            int stage = 0, slot = 0;
            uint32_t phase = 0, lo_phase = 0;
            bool ok = true;
            for (long long t = cluster; ok && t < p.tiles; t += nclusters) {
                for (int kb = 0; kb < p.k_blocks; kb++) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort))) {
                        if (lane == 0)
                            record_failure(abort, p.status, DEV_TIMEOUT_SPLIT);
                        ok = false;
                        break;
                    }
                    const float4 *raw = reinterpret_cast<const float4 *>(
                        smem + stage * Cfg::kLoadBytes + Cfg::kATile);
                    float4 l[kPer];
#pragma unroll
                    for (int j = 0; j < kPer; j++) {
                        const float4 x = raw[bt + j * kThr];
                        l[j] = make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
                    }
                    if (!__all_sync(0xffffffffu,
                                    mbar_wait(&lo_free[slot], lo_phase ^ 1, abort))) {
                        if (lane == 0)
                            record_failure(abort, p.status, DEV_TIMEOUT_SPLIT);
                        ok = false;
                        break;
                    }
                    float4 *lo =
                        reinterpret_cast<float4 *>(smem + Cfg::kLoOffset + slot * Cfg::kBTile);
#pragma unroll
                    for (int j = 0; j < kPer; j++)
                        lo[bt + j * kThr] = l[j];
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_cluster(map_to_cta(smem_addr(&ready[stage]), 0));
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                    if (++slot == L) {
                        slot = 0;
                        lo_phase ^= 1;
                    }
                }
            }
        }
    } else if (warp < 8) {
        warpgroup_reg_dealloc<Cfg::kRegsWg1>();
        {
            // -------------------------------------------------------- A split (both CTAs)
            // Thread = row 32 (warp mod 4) + lane of this CTA's A tile: its 32
            // raw values (K-major, 128-byte swizzle: 16-byte chunk j of row r
            // at chunk j ^ (r mod 8)) become hi and lo in TMEM slot columns.
            const int quad = warp & 3;
            const int row = quad * 32 + lane;
            const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
            int stage = 0, slot = 0;
            uint32_t phase = 0, lo_phase = 0;
            bool ok = true;
            for (long long t = cluster; ok && t < p.tiles; t += nclusters) {
                for (int kb = 0; kb < p.k_blocks; kb++) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort))) {
                        if (lane == 0)
                            record_failure(abort, p.status, DEV_TIMEOUT_SPLIT);
                        ok = false;
                        break;
                    }
                    // K columns [0, 16) are split before the slot is free,
                    // [16, 32) after their predecessors' stores
                    const uint8_t *ra = smem + stage * Cfg::kLoadBytes + row * 128;
                    uint32_t hi[16], lo[16];
                    auto split_half = [&](int h) {
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const int chunk = 4 * h + j;
                            const float4 x = *reinterpret_cast<const float4 *>(
                                ra + ((chunk ^ (row & 7)) << 4));
                            hi[4 * j + 0] = __float_as_uint(tf32_hi(x.x));
                            hi[4 * j + 1] = __float_as_uint(tf32_hi(x.y));
                            hi[4 * j + 2] = __float_as_uint(tf32_hi(x.z));
                            hi[4 * j + 3] = __float_as_uint(tf32_hi(x.w));
                            lo[4 * j + 0] = __float_as_uint(tf32_lo(x.x));
                            lo[4 * j + 1] = __float_as_uint(tf32_lo(x.y));
                            lo[4 * j + 2] = __float_as_uint(tf32_lo(x.z));
                            lo[4 * j + 3] = __float_as_uint(tf32_lo(x.w));
                        }
                    };
                    split_half(0);
                    if (!__all_sync(0xffffffffu,
                                    mbar_wait(&lo_free[slot], lo_phase ^ 1, abort))) {
                        if (lane == 0)
                            record_failure(abort, p.status, DEV_TIMEOUT_SPLIT);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t col =
                        lane_addr + static_cast<uint32_t>(Cfg::kASlot0 + slot * Cfg::kASlotCols);
                    tmem_st_32x32b_x16(col, hi);
                    tmem_st_32x32b_x16(col + Cfg::BK, lo);
                    tmem_st_wait();   // the registers are refilled below
                    split_half(1);
                    tmem_st_32x32b_x16(col + 16, hi);
                    tmem_st_32x32b_x16(col + Cfg::BK + 16, lo);
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_cluster(map_to_cta(smem_addr(&ready[stage]), 0));
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                    if (++slot == L) {
                        slot = 0;
                        lo_phase ^= 1;
                    }
                }
            }
        }
    } else {
        warpgroup_reg_alloc<Cfg::kRegsEpi>();
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int ew = warp - 8;
        const int quad = warp & 3;
        const int part = ew >> 2;   // its 128 of the 256 accumulator columns
        uint8_t *sbuf = smem + Cfg::kEpiOffset + ew * Cfg::kEpiBufBytes;
        const uint32_t t_acc = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                               static_cast<uint32_t>(part * Cfg::kWarpCols);
        const uint32_t tempty0 = map_to_cta(smem_addr(tempty), 0);
        const int nchunks = (p.k_blocks + Cfg::kChunkKB - 1) / Cfg::kChunkKB;
        const bool fused = p.bias != nullptr || p.act != ACT_NONE;
        long long uses = 0;
        bool ok = true;
        for (long long t = cluster; ok && t < p.tiles; t += nclusters) {
            const int nb = static_cast<int>(t % p.n_blocks);
            const long long r = t / p.n_blocks;
            const int mb = static_cast<int>(r % p.m_blocks);
            const long long batch = r / p.m_blocks;
            int c[3];
            decode_batch(batch, p, c);
            const int row0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::kRowsCta + quad * 32;
            const int n0 = nb * Cfg::BN + part * Cfg::kWarpCols;
            // running total of the finished chunks: 0 + chunk 0, then
            // total + chunk k, float adds with round-to-nearest
            float tot[Cfg::kWarpCols];
#pragma unroll
            for (int i = 0; i < Cfg::kWarpCols; i++)
                tot[i] = 0.0f;
            for (int ck = 0; ck < nchunks; ck++, uses++) {
                const bool got = __all_sync(
                    0xffffffffu, mbar_wait(tfull, static_cast<uint32_t>(uses & 1), abort));
                if (!got) {
                    if (lane == 0)
                        record_failure(abort, p.status, DEV_TIMEOUT_EPILOGUE);
                    ok = false;
                    break;
                }
                tc_fence_after();
                // 16 loads of 8 columns, each issued before the previous
                // one's values are added
                uint32_t b0[8], b1[8];
                tmem_ld_32x32b_x8(t_acc, b0);
                tmem_ld_wait_regs8(b0);
#pragma unroll
                for (int j = 0; j < Cfg::kWarpCols / 8; j++) {
                    uint32_t(&cur)[8] = (j & 1) ? b1 : b0;
                    uint32_t(&nxt)[8] = (j & 1) ? b0 : b1;
                    if (j + 1 < Cfg::kWarpCols / 8)
                        tmem_ld_32x32b_x8(t_acc + (j + 1) * 8, nxt);
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        tot[8 * j + i] = tot[8 * j + i] + __uint_as_float(cur[i]);
                    if (j + 1 < Cfg::kWarpCols / 8)
                        tmem_ld_wait_regs8(nxt);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive_cluster(tempty0);
            }
            if (!ok)
                break;
            // 4 boxes of 32 columns: bias / activation, staging, TMA store
#pragma unroll
            for (int bx = 0; bx < Cfg::kWarpCols / Cfg::kEpiCols; bx++) {
                const int col0 = n0 + bx * Cfg::kEpiCols;
                if (fused) {
                    const int bc = col0 + lane;
                    const float bl = p.bias != nullptr && bc < p.N
                                         ? static_cast<const float *>(p.bias)[bc]
                                         : 0.0f;
#pragma unroll
                    for (int i = 0; i < Cfg::kEpiCols; i++) {
                        float x = tot[bx * Cfg::kEpiCols + i];
                        if (p.bias != nullptr)
                            x += __shfl_sync(0xffffffffu, bl, i);
                        tot[bx * Cfg::kEpiCols + i] = apply_activation(x, p.act);
                    }
                }
                if (lane == 0)
                    bulk_wait_group_read<0>();
                __syncwarp();
                uint8_t *rowp = sbuf + lane * 128;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    uint4 q;
                    q.x = __float_as_uint(tot[bx * Cfg::kEpiCols + 4 * j + 0]);
                    q.y = __float_as_uint(tot[bx * Cfg::kEpiCols + 4 * j + 1]);
                    q.z = __float_as_uint(tot[bx * Cfg::kEpiCols + 4 * j + 2]);
                    q.w = __float_as_uint(tot[bx * Cfg::kEpiCols + 4 * j + 3]);
                    *reinterpret_cast<uint4 *>(rowp + ((j ^ (lane & 7)) << 4)) = q;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && col0 < p.N && row0 < p.M) {
                    tma_store_5d(&tma_c, sbuf, col0, row0, c[0], c[1], c[2]);
                    bulk_commit_group();
                }
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
