// 2-CTA (cta_group::2) tcgen05 GEMM with a 256 x 512 output tile per CTA pair:
// 16-bit operands, FP32 accumulation in TMEM, 16-bit output.
//
// The 256 x 256 pair tile of tc2_gemm_kernel streams 64 bytes per SM and
// tensor-core cycle (each CTA lands 128 rows of A and 128 columns of B per
// 64-deep k-block, 512 cycles of M = 256, N = 256 MMAs), and on B200 the
// L2-to-SM path does not sustain that across 148 SMs: the MMA thread waits
// for operand tiles while every ring stage is already in flight.  Here each
// CTA lands 128 rows of A and 2 x 128 columns of B per k-block, and CTA 0
// issues two M = 256, N = 256 MMAs per K step (tile columns [0, 256) and
// [256, 512)) on the same A descriptor: 48 bytes per SM and tensor cycle, a
// quarter fewer operand bytes per FLOP.
//
// The 128 x 512 FP32 accumulator of each CTA fills its 512 TMEM columns, so
// it is single-buffered.  To keep the tensor pipe busy across tiles, the 8
// epilogue warps (two per TMEM lane quadrant, each taking 128 columns of
// both accumulator halves; warpgroup register reallocation gives them 216
// registers each) first move the accumulator into registers, rounded to the
// output type (the unfused plan rounds the product before any bias or
// activation): half 0, which they release at once, then half 1.  The MMA
// thread starts the next tile's half-0 MMAs of its first k-block as soon as
// half 0 is released, so half 1's drain runs under them.  Only then do the
// warps apply the bias / activation, stage 32 x 64-column boxes in swizzled
// shared memory and TMA-store them while the next tile's k loop runs.
//
// Ring: 4 stages of 48 KB per CTA (A 16 KB, B 2 x 16 KB), the same 192 KB in
// flight as the 256 x 256 kernel's 6 stages of 32 KB.
//
// Work items (p.wide_items): the first wide_items items are whole 256 x 512
// tiles; every later item is one 256-column half of a tile, run through
// accumulator half 0 and B slot 0 only (half the loads, MMAs and stores).
// The launcher makes the whole tiles fill every full round of co-resident
// clusters and runs the remainder as halves, so a last round that would be
// half empty takes half as long.
//
// Protocol (no TMA multicast anywhere), as in tc2_gemm_kernel:
//   full[s]   lives in CTA 0; CTA 0 posts expect_tx for both CTAs' bytes and
//             both CTAs' TMA loads complete on it.
//   empty[s]  one per CTA, committed by CTA 0's MMA thread to both CTAs.
//   tfull     one per CTA, committed the same way when the tile's MMAs are done.
//   tempty[h] live in CTA 0 with 16 arrivals each: the 8 epilogue warps of
//             each CTA, once their TMEM loads of accumulator half h
//             completed (CTA 1 arrives remotely).
// Every wait is bounded; cluster barriers bracket the kernel.
#pragma once

#include "gemm_tc2.cuh"

namespace ptg {

template <int IN_KIND, int OUT>
struct Tc2wConfig {
    static constexpr int BM = 256, BN = 512;          // per CTA pair
    static constexpr int kRowsCta = 128;               // A rows per CTA
    static constexpr int kColsCta = 128;               // B columns per CTA and MMA half
    static constexpr int kHalfN = 256;                 // N of one MMA
    static constexpr int kInBytes = 2;
    static constexpr int BK = 64;                      // one 128-byte swizzle row of K
    static constexpr int kMmaK = 16;
    static constexpr int kKSteps = BK / kMmaK;
    static constexpr int kChunk = 64;                  // MN elements per 128-byte row
    static constexpr int kChunkBytes = 128 * BK;       // one MN-major box (kChunk x BK)
    static constexpr int kATile = kRowsCta * BK * kInBytes;   // 16 KB
    static constexpr int kBHalf = kColsCta * BK * kInBytes;   // 16 KB per MMA half
    static constexpr int kStageBytes = kATile + 2 * kBHalf;   // 48 KB
    static constexpr int kStages = 4;
    static constexpr int kEpiCols = 64;                // 128 bytes of 16-bit output
    static constexpr int kEpiWarps = 8;
    static constexpr int kWarpCols = BN / 2;           // columns per epilogue warp
    static constexpr int kPartCols = kWarpCols / 2;    // of them in each accumulator half
    static constexpr int kPacked = kWarpCols / 2;      // 32-bit registers of packed output
    static constexpr int kEpiBufBytes = 32 * 128;      // one 32 x 64 staging box per warp
    // warpgroup 0: producer (warp 0), MMA issuer and TMEM owner (warp 1), two
    // idle warps; warpgroups 1 and 2: the epilogue
    static constexpr int kThreads = 128 + 32 * kEpiWarps;
    // Registers: 384 threads launch with at most 168 each (four SM
    // sub-partitions of 16 K registers, three warps each).  Warpgroup 0 drops
    // to kRegsCtl and the epilogue warpgroups rise to kRegsEpi, which holds
    // the 128 packed output registers of a warp's 256 columns; the two
    // together must stay within the launch allocation, kRegsTotal, or the
    // increase would wait forever.  The launcher reads the kernel's register
    // count and does not launch it when threads x registers is below that.
    static constexpr int kRegsCtl = 56, kRegsEpi = 216;
    static constexpr int kRegsTotal = 128 * kRegsCtl + 32 * kEpiWarps * kRegsEpi;
    static_assert(kRegsTotal <= 168 * kThreads, "register reallocation exceeds 168 per thread");
    static constexpr int kTmemCols = 512;
    static constexpr int kRingBytes = kStages * kStageBytes;
    static constexpr int kEpiOffset = kRingBytes;
    static constexpr int kBarOffset = kEpiOffset + kEpiWarps * kEpiBufBytes;
    static constexpr int kNumBars = 2 * kStages + 4;   // full, empty, tfull, tempty[2], drain
    static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
    static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
    static_assert(IN_KIND == IN_F16 || IN_KIND == IN_BF16, "16-bit operands");
    static_assert(OUT == OUT_F16 || OUT == OUT_BF16, "16-bit output");
};

// Work item -> 256 x 512 tile index; hsel = -1 for the whole tile, else the
// one 256-column half the item covers.
__device__ __forceinline__ long long wide_item(const TcParams &p, long long i, int &hsel)
{
    if (i < p.wide_items) {
        hsel = -1;
        return i;
    }
    const long long j = i - p.wide_items;
    hsel = static_cast<int>(j & 1);
    return p.wide_items + (j >> 1);
}

template <int IN_KIND, int OUT>
__global__ void __launch_bounds__(Tc2wConfig<IN_KIND, OUT>::kThreads, 1)
    tc2w_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                     const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_c, const TcParams p)
{
    using Cfg = Tc2wConfig<IN_KIND, OUT>;
    constexpr int S = Cfg::kStages;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kBarOffset);
    uint64_t *full = bars;
    uint64_t *empty = bars + S;
    uint64_t *tfull = bars + 2 * S;
    uint64_t *tempty = bars + 2 * S + 1;   // [2]: one per accumulator half
    uint64_t *drain = bars + 2 * S + 3;
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
        mbar_init(tfull, 1);
        mbar_init(&tempty[0], 2 * Cfg::kEpiWarps);
        mbar_init(&tempty[1], 2 * Cfg::kEpiWarps);
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

    if (warp < 4) {
        warpgroup_reg_dealloc<Cfg::kRegsCtl>();
        if (warp == 0) {
            // ------------------------------------------------------------ producer (both CTAs)
            if (lane == 0) {
                int stage = 0;
                uint32_t phase = 0;
                uint32_t issued_mask = 0, parity_mask = 0;
                bool ok = true;
                for (long long t = cluster; ok && t < p.tiles; t += nclusters) {
                    int hsel;
                    const long long tile = wide_item(p, t, hsel);
                    const int nhalf = hsel < 0 ? 2 : 1;
                    const int nb = static_cast<int>(tile % p.n_blocks);
                    const long long r = tile / p.n_blocks;
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
                        uint8_t *sa = smem + stage * Cfg::kStageBytes;
                        uint8_t *sb = sa + Cfg::kATile;
                        if (rank == 0)
                            mbar_arrive_expect_tx(&full[stage],
                                                  2 * (Cfg::kATile + nhalf * Cfg::kBHalf));
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
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            if (h >= nhalf)
                                break;
                            // slot h holds the B columns of tile half h, or of
                            // the item's one half
                            uint8_t *sbh = sb + h * Cfg::kBHalf;
                            const int nh = n0 + (hsel < 0 ? h : hsel) * Cfg::kHalfN;
                            if (!p.b_mn_major) {
                                tma_load_5d_pair(sbh, &tma_b, full0, k0, nh, cb[0], cb[1], cb[2]);
                            } else {
#pragma unroll
                                for (int j = 0; j < Cfg::kColsCta / Cfg::kChunk; j++)
                                    tma_load_5d_pair(sbh + j * Cfg::kChunkBytes, &tma_b, full0,
                                                     nh + j * Cfg::kChunk, k0, cb[0], cb[1], cb[2]);
                            }
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
                    int hsel;
                    (void)wide_item(p, t, hsel);
                    const int nhalf = hsel < 0 ? 2 : 1;
                    const uint32_t acc_phase = static_cast<uint32_t>(iter & 1);
                    if (!mbar_wait(&tempty[0], acc_phase ^ 1, abort)) {
                        record_failure(abort, p.status, DEV_TIMEOUT_MMA);
                        break;
                    }
                    tc_fence_after();
                    for (int kb = 0; kb < p.k_blocks; kb++) {
                        if (!mbar_wait(&full[stage], phase, abort)) {
                            record_failure(abort, p.status, DEV_TIMEOUT_MMA);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
                        const uint32_t sb = sa + Cfg::kATile;
                        const uint32_t b_lbo = p.b_mn_major ? Cfg::kChunkBytes : 16;
                        // accumulator half 0, then half 1 (on the tile's first
                        // k-block, once the epilogue has read that half: its
                        // drain overlaps half 0's MMAs)
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            if (h == 1 && kb == 0) {
                                if (!mbar_wait(&tempty[1], acc_phase ^ 1, abort)) {
                                    record_failure(abort, p.status, DEV_TIMEOUT_MMA);
                                    ok = false;
                                    break;
                                }
                                tc_fence_after();
                            }
                            if (h >= nhalf)
                                break;
#pragma unroll
                            for (int k = 0; k < Cfg::kKSteps; k++) {
                                const uint32_t a_off = p.a_mn_major ? k * Cfg::kMmaK * 128 : k * 32;
                                const uint32_t b_off = p.b_mn_major ? k * Cfg::kMmaK * 128 : k * 32;
                                // 16-bit operands: the MN-major SBO and layout equal
                                // the K-major ones, only the LBO depends on the layout
                                const uint64_t ad = smem_desc(
                                    sa + a_off, p.a_mn_major ? Cfg::kChunkBytes : 16, 1024,
                                    kLayoutSw128);
                                const uint64_t bd =
                                    smem_desc(sb + h * Cfg::kBHalf + b_off, b_lbo, 1024,
                                              kLayoutSw128);
                                umma_f16_pair(tmem_base + h * Cfg::kHalfN, ad, bd, p.idesc,
                                              (kb | k) != 0);
                            }
                        }
                        if (!ok)
                            break;
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
                    const uint32_t f0 = smem_addr(tfull);
                    umma_commit_pair(f0);
                    umma_commit_pair(map_to_cta(f0, 1));
                }
                umma_commit_pair(smem_addr(drain));
                int no_abort = 0;
                mbar_wait(drain, 0, &no_abort);
            }
        }
    } else {
        warpgroup_reg_alloc<Cfg::kRegsEpi>();
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int ew = warp - 4;
        const int quad = warp & 3;           // TMEM lane quadrant this warp may read
        const int part = ew >> 2;            // its 128 columns of each accumulator half
        uint8_t *sbuf = smem + Cfg::kEpiOffset + ew * Cfg::kEpiBufBytes;
        const bool fused = p.bias != nullptr || p.act != ACT_NONE;
        long long iter = 0;
        for (long long t = cluster; t < p.tiles; t += nclusters, iter++) {
            const uint32_t acc_phase = static_cast<uint32_t>(iter & 1);
            const bool got = __all_sync(0xffffffffu, mbar_wait(tfull, acc_phase, abort));
            if (!got) {
                if (lane == 0)
                    record_failure(abort, p.status, DEV_TIMEOUT_EPILOGUE);
                break;
            }
            tc_fence_after();
            int hsel;
            const long long tile = wide_item(p, t, hsel);
            const int nhalf = hsel < 0 ? 2 : 1;
            const int nb = static_cast<int>(tile % p.n_blocks);
            const long long r = tile / p.n_blocks;
            const int mb = static_cast<int>(r % p.m_blocks);
            const long long batch = r / p.m_blocks;
            int c[3];
            decode_batch(batch, p, c);
            const int row0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::kRowsCta + quad * 32;
            // first column of this warp's part of accumulator half 0
            const int n0 =
                nb * Cfg::BN + (hsel < 0 ? 0 : hsel * Cfg::kHalfN) + part * Cfg::kPartCols;
            const uint32_t t_acc = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                   static_cast<uint32_t>(part * Cfg::kPartCols);

            // Drain: for each accumulator half, 8 loads of 16 columns, each
            // issued before the previous one's values are rounded and packed;
            // the half is released as soon as its loads completed.
            uint32_t pk[Cfg::kPacked];
            uint32_t buf0[16], buf1[16];
            constexpr int kLoads = Cfg::kPartCols / 16;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                if (h < nhalf) {
                    const uint32_t t_half = t_acc + h * Cfg::kHalfN;
                    tmem_ld_32x32b_x16(t_half, buf0);
                    tmem_ld_wait_regs(buf0);
#pragma unroll
                    for (int j = 0; j < kLoads; j++) {
                        uint32_t(&cur)[16] = (j & 1) ? buf1 : buf0;
                        uint32_t(&nxt)[16] = (j & 1) ? buf0 : buf1;
                        if (j + 1 < kLoads)
                            tmem_ld_32x32b_x16(t_half + (j + 1) * 16, nxt);
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            pk[(h * kLoads + j) * 8 + i] =
                                pack2(__uint_as_float(cur[2 * i]), __uint_as_float(cur[2 * i + 1]),
                                      OUT);
                        if (j + 1 < kLoads)
                            tmem_ld_wait_regs(nxt);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive_cluster(map_to_cta(smem_addr(&tempty[h]), 0));
            }

#pragma unroll
            for (int ch = 0; ch < Cfg::kWarpCols / Cfg::kEpiCols; ch++) {
                // chunks 0, 1: half 0; chunks 2, 3: half 1
                if ((ch >> 1) >= nhalf)
                    break;
                const int col0 = n0 + (ch >> 1) * Cfg::kHalfN + (ch & 1) * Cfg::kEpiCols;
                uint32_t *q32 = pk + ch * (Cfg::kEpiCols / 2);
                if (fused) {
                    float v[Cfg::kEpiCols];
#pragma unroll
                    for (int i = 0; i < Cfg::kEpiCols / 2; i++)
                        unpack2(q32[i], v[2 * i], v[2 * i + 1], OUT);
                    apply_epilogue<OUT, Cfg::kEpiCols>(v, p.bias, p.act, col0, p.N, lane);
#pragma unroll
                    for (int i = 0; i < Cfg::kEpiCols / 2; i++)
                        q32[i] = pack2(v[2 * i], v[2 * i + 1], OUT);
                }
                // the previous box's store must have read the staging buffer
                if (lane == 0)
                    bulk_wait_group_read<0>();
                __syncwarp();
                uint8_t *rowp = sbuf + lane * 128;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    uint4 q;
                    q.x = q32[4 * j + 0];
                    q.y = q32[4 * j + 1];
                    q.z = q32[4 * j + 2];
                    q.w = q32[4 * j + 3];
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
