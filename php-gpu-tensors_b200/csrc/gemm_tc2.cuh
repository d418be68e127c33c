// 2-CTA (cta_group::2) tcgen05 GEMMs on sm_100a: 16-bit operands and
// single-pass TF32 (float32 operands in the tf32 precision mode) in
// tc2_gemm_kernel, strict float32 (3xTF32) in tc2x3_gemm_kernel below.
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
    static constexpr bool kTf32 = IN_KIND == IN_TF32;
    static constexpr int kInBytes = kTf32 ? 4 : 2;
    static constexpr int BK = 128 / kInBytes;          // one 128-byte swizzle row of K
    static constexpr int kMmaK = 32 / kInBytes;        // 32 bytes of K per instruction
    static constexpr int kKSteps = BK / kMmaK;
    static constexpr int kChunk = 128 / kInBytes;      // MN elements per 128-byte row
    static constexpr int kChunkBytes = 128 * BK;       // one MN-major box (kChunk x BK)
    // MN-major TF32 tiles use the 32-byte-atom 128-byte swizzle (as in the
    // single-CTA kernel); everything else the 16-byte-atom one
    static constexpr uint32_t kMnLayout = kTf32 ? kLayoutSw128Base32B : kLayoutSw128;
    static constexpr uint32_t kMnSbo = kTf32 ? 512 : 1024;
    static constexpr int kATile = kRowsCta * BK * kInBytes;   // 16 KB
    static constexpr int kBTile = kColsCta * BK * kInBytes;   // 16 KB
    static constexpr int kLoadBytes = kATile + kBTile; // per CTA and stage
    static constexpr int kStageBytes = kLoadBytes;
    static constexpr int kStages = 6;
    static constexpr int kEpiCols = 128 / OutTraits<OUT>::kBytes;   // 128 bytes of output
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
    static_assert(IN_KIND == IN_F16 || IN_KIND == IN_BF16 || IN_KIND == IN_TF32,
                  "16-bit or single-pass TF32 operands");
    static_assert(kTf32 == (OUT == OUT_F32), "TF32 products write float32");
    static_assert(kATile == 16384 && kBTile == 16384, "one 128-byte row of K per tile row");
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
                        // (for 16-bit operands the MN-major SBO and layout equal
                        // the K-major ones, so only the LBO depends on the layout)
                        const uint64_t ad = smem_desc(sa + a_off, p.a_mn_major ? Cfg::kChunkBytes : 16,
                                                      p.a_mn_major ? Cfg::kMnSbo : 1024,
                                                      p.a_mn_major ? Cfg::kMnLayout : kLayoutSw128);
                        const uint64_t bd = smem_desc(sb + b_off, p.b_mn_major ? Cfg::kChunkBytes : 16,
                                                      p.b_mn_major ? Cfg::kMnSbo : 1024,
                                                      p.b_mn_major ? Cfg::kMnLayout : kLayoutSw128);
                        if constexpr (Cfg::kTf32)
                            umma_tf32_pair(d_tmem, ad, bd, p.idesc, (kb | k) != 0);
                        else
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

// ---------------------------------------------------------------------------
// 2-CTA split GEMMs: strict float32 (3xTF32, KIND = IN_F32X3) and float32 x
// bfloat16 products (bf16x3, KIND = IN_MIX_A / IN_MIX_B).
//
// A CTA pair computes a 256 x 256 tile with M = 256, N = 256
// tcgen05.mma.cta_group::2 instructions: CTA r holds rows [128 r, 128 r + 128)
// of the A tile and columns [128 r, 128 r + 128) of the B tile and computes a
// 128 x 256 output block, so per FLOP each SM streams and splits half the
// bytes of the single-CTA 128 x 128 kernels.
//
// 3xTF32, per CTA: a 3-stage ring of raw float32 tiles (A 16 KB + B 16 KB), a
// 3-slot lo ring (4 + 2 measured 4 % slower once the split was
// register-staged), 6 split warps writing lo = tf32(x - trunc(x)) of the
// CTA's own tiles and 8 epilogue warps (16 warps: 128 registers per thread).
// The lo of k-block kb can be stored only when the MMAs of k-block kb - L (L
// lo slots) have released its slot, and must be in place before the tensor
// core runs out of the k-blocks in between, a chain of barrier round trips
// that measured on B200 (L = 2) held the kernel to 188 of the 215 TFLOP/s it
// reached with the wait removed (8192^3, split skipped in both timing
// builds).  So each split thread loads its raw elements and computes lo into
// registers as soon as the tile lands, and only stores them once the slot is
// free.  (Stages of 16 K in the 64-byte swizzle, twice as many slots in the
// same bytes, ran slower: 130 against 154 TFLOP/s.)
//
// bf16x3, per CTA: 3 stages of 64 KB: the float32 operand's raw [128][64]
// box, split in place by the split warps into its bf16 hi, mid and lo tiles,
// then the bf16 operand's tile; three kind::f16 MMAs per k16.
//
// TMEM: the accumulator (columns [0, 256)) and the running total of the
// finished K chunks ([256, 512)); the accumulator is single-buffered, so the
// MMA thread waits for each chunk's drain, which two epilogue warps per TMEM
// lane quadrant share by columns (8192^3 on B200: 4 epilogue + 8 split warps
// 163 TFLOP/s, 8 + 6 169.5).
//
// Barriers (no TMA multicast anywhere), with "leader" the pair's even
// cluster rank (the only pair without split-K: ranks 0 and 1):
//   full[s]      per CTA: its own TMA loads of stage s landed.
//   ready[s]     leader, 2 x 6 arrivals: every split warp of both CTAs wrote
//                its part of stage s (remote arrive, release.cluster).
//   empty[s], lo_free[l], tfull
//                per CTA, committed by the leader's MMA thread to both CTAs.
//   tempty       leader, 2 x 8 arrivals: the epilogue warps of both CTAs
//                drained the accumulator.
template <int KIND, int CHUNK_KB>
struct Tc2x3Config {
    static constexpr bool kMix = KIND == IN_MIX_A || KIND == IN_MIX_B;
    static constexpr bool kMixA = KIND == IN_MIX_A;      // the float32 operand is A
    static_assert(KIND == IN_F32X3 || kMix, "3xTF32 or bf16x3 pair kernel");
    static constexpr int BM = 256, BN = 256;            // per CTA pair
    static constexpr int kRowsCta = 128, kColsCta = 128;
    // K per stage: one 128-byte row of the MMA operand type (float32 for
    // 3xTF32, bfloat16 for the mixed kinds)
    static constexpr int kOpBytes = kMix ? 2 : 4;
    static constexpr int BK = 128 / kOpBytes;
    static constexpr int kMmaK = 32 / kOpBytes;
    static constexpr int kKSteps = BK / kMmaK;
    static constexpr int kChunk = 128 / kOpBytes;        // MN elements per 128-byte row
    static constexpr int kChunkBytes = 128 * BK;         // one MN-major box
    static constexpr uint32_t kMnLayout = kMix ? kLayoutSw128 : kLayoutSw128Base32B;
    static constexpr uint32_t kMnSbo = kMix ? 1024 : 512;
    static constexpr uint32_t kKLayout = kLayoutSw128;
    static constexpr uint32_t kKSbo = 1024;
    static constexpr int kATile = kRowsCta * BK * kOpBytes;   // 16 KB
    static constexpr int kBTile = kColsCta * BK * kOpBytes;   // 16 KB
    // mixed: the float32 operand lands raw (one unswizzled [128][BK] box,
    // 32 KB) at the stage start and is split in place into its bf16 hi and
    // mid tiles, lo after them; the bf16 operand's tile follows
    static constexpr int kMixRawBytes = 128 * BK * 4;
    static constexpr int kMixOtherOffset = kMixRawBytes + kATile;
    static constexpr int kLoadBytes = kMix ? kMixRawBytes + kATile : kATile + kBTile;
    static constexpr int kStageBytes = kMix ? kMixOtherOffset + kATile : kLoadBytes;
#ifndef PTG_PAIR3_STAGES
#define PTG_PAIR3_STAGES 3
#endif
    static constexpr int kStages = kMix ? 3 : PTG_PAIR3_STAGES;
    static constexpr int kLoStages = kMix ? 0 : 6 - kStages;
    static constexpr int kLoOffset = kStages * kStageBytes;
    static constexpr int kRingBytes = kLoOffset + kLoStages * kLoadBytes;
    static constexpr int kEpiCols = 32;                  // 128 bytes of float32 output
    static constexpr int kEpiBufBytes = 32 * 128;
#ifndef PTG_PAIR3_EPI
#define PTG_PAIR3_EPI 8
#endif
    // epilogue warps: 4, or 8 (two per TMEM lane quadrant, each draining half
    // of the columns, with one staging buffer each)
    static constexpr int kEpiWarps = PTG_PAIR3_EPI;
    static constexpr int kEpiParts = kEpiWarps / 4;
    static constexpr int kEpiBufs = kEpiWarps == 4 ? 2 : 1;
#ifndef PTG_PAIR3_SPLIT
#define PTG_PAIR3_SPLIT 6
#endif
    static constexpr int kSplitWarps = PTG_PAIR3_SPLIT;
    static constexpr int kThreads = 32 * (2 + kEpiWarps + kSplitWarps);
    static constexpr int kEpiOffset = kRingBytes;
    static constexpr int kBarOffset = kEpiOffset + kEpiWarps * kEpiBufs * kEpiBufBytes;
    // full, empty, ready per stage; lo_free per lo slot; tfull, tempty, drain
    static constexpr int kNumBars = 3 * kStages + kLoStages + 3;
    static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
    static constexpr int kChunkKB = CHUNK_KB;            // k-blocks per accumulator chunk
    static constexpr int kTotalCol = BN;
    static constexpr int kTmemCols = 512;
    // split-K partial tile [128][BN + 4] floats at the start of the ring
    static constexpr int kPartPitch = BN + 4;
    static_assert(kRowsCta * kPartPitch * 4 <= kRingBytes, "partial tile fits in the ring");
    static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
};

template <int KIND, int CHUNK_KB>
__global__ void __launch_bounds__(Tc2x3Config<KIND, CHUNK_KB>::kThreads, 1)
    tc2x3_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                      const __grid_constant__ CUtensorMap tma_b,
                      const __grid_constant__ CUtensorMap tma_c, const TcParams p)
{
    using Cfg = Tc2x3Config<KIND, CHUNK_KB>;
    constexpr int S = Cfg::kStages;
    constexpr int BN = Cfg::BN;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kBarOffset);
    uint64_t *full = bars;
    uint64_t *empty = bars + S;
    uint64_t *ready = bars + 2 * S;
    uint64_t *lo_free = bars + 3 * S;
    uint64_t *tfull = bars + 3 * S + Cfg::kLoStages;
    uint64_t *tempty = tfull + 1;
    uint64_t *drain = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + Cfg::kNumBars);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // CTA pairs are the cluster ranks (2 q, 2 q + 1).  Split-K (p.ksplit =
    // G > 1): a cluster of G pairs shares one tile, pair q taking the q-th
    // contiguous range of k-blocks.
    const uint32_t crank = cluster_cta_rank();
    const uint32_t rank = crank & 1u;        // CTA within the pair
    const uint32_t leader = crank & ~1u;     // the pair's MMA-issuing CTA
    const int G = p.ksplit;
    const int krank = G > 1 ? static_cast<int>(crank >> 1) : 0;
    const long long t_first = G > 1 ? blockIdx.x / (2 * G) : blockIdx.x >> 1;
    const long long t_step = G > 1 ? p.tiles : gridDim.x >> 1;
    const int kb_per = (p.k_blocks + G - 1) / G;
    const int kb_begin = min(p.k_blocks, krank * kb_per);
    const int kb_end = min(p.k_blocks, kb_begin + kb_per);

    if (warp == 0 && lane == 0) {
        prefetch_tensor_map(&tma_a);
        prefetch_tensor_map(&tma_b);
        prefetch_tensor_map(&tma_c);
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&ready[s], 2 * Cfg::kSplitWarps);
        }
        for (int i = 0; i < Cfg::kLoStages; i++)
            mbar_init(&lo_free[i], 1);
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

    if (warp == 0) {
        // ------------------------------------------------------------ producer (both CTAs)
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
                const int m0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::kRowsCta;
                const int n0 = nb * BN + static_cast<int>(rank) * Cfg::kColsCta;
                for (int kbf = kb_begin; kbf < kb_end; kbf++) {
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
                        // the float32 operand raw at the stage start, the
                        // bf16 one after its three parts
                        if constexpr (Cfg::kMixA)
                            sb = sa + Cfg::kMixOtherOffset;
                        else
                            sa = sa + Cfg::kMixOtherOffset, sb = smem + stage * Cfg::kStageBytes;
                    }
                    mbar_arrive_expect_tx(&full[stage], Cfg::kLoadBytes);
                    const int k0 = kb * Cfg::BK;
                    // A: K-major one box, MN-major one box per 128-byte chunk
                    // of M (the raw float32 operand of a mixed kind is always
                    // one unswizzled box); B likewise
                    const bool a_raw = Cfg::kMixA, b_raw = Cfg::kMix && !Cfg::kMixA;
                    if (!p.a_mn_major) {
                        tma_load_5d(sa, &tma_a, &full[stage], k0, m0, ca[0], ca[1], ca[2]);
                    } else if (a_raw) {
                        tma_load_5d(sa, &tma_a, &full[stage], m0, k0, ca[0], ca[1], ca[2]);
                    } else {
#pragma unroll
                        for (int j = 0; j < Cfg::kRowsCta / Cfg::kChunk; j++)
                            tma_load_5d(sa + j * Cfg::kChunkBytes, &tma_a, &full[stage],
                                        m0 + j * Cfg::kChunk, k0, ca[0], ca[1], ca[2]);
                    }
                    if (!p.b_mn_major) {
                        tma_load_5d(sb, &tma_b, &full[stage], k0, n0, cb[0], cb[1], cb[2]);
                    } else if (b_raw) {
                        tma_load_5d(sb, &tma_b, &full[stage], n0, k0, cb[0], cb[1], cb[2]);
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
            // every copy this thread started lands before shared memory can
            // be released (bounded, ignores the abort flag)
            for (int s = 0; s < S; s++) {
                if (issued_mask & (1u << s)) {
                    int no_abort = 0;
                    mbar_wait(&full[s], (parity_mask >> s) & 1u, &no_abort);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (CTA 0)
        if (lane == 0 && rank == 0) {
            const uint32_t peer = leader + 1;
            int stage = 0, lo_slot = 0;
            uint32_t phase = 0;
            long long uses = 0;   // accumulator chunks issued
            bool ok = true;
            const uint32_t smem_base = smem_addr(smem);
            const uint32_t a_lbo = p.a_mn_major ? Cfg::kChunkBytes : 16;
            const uint32_t b_lbo = p.b_mn_major ? Cfg::kChunkBytes : 16;
            const uint32_t a_sbo = p.a_mn_major ? Cfg::kMnSbo : Cfg::kKSbo;
            const uint32_t b_sbo = p.b_mn_major ? Cfg::kMnSbo : Cfg::kKSbo;
            const uint32_t a_lay = p.a_mn_major ? Cfg::kMnLayout : Cfg::kKLayout;
            const uint32_t b_lay = p.b_mn_major ? Cfg::kMnLayout : Cfg::kKLayout;
            for (long long t = t_first; ok && t < p.tiles; t += t_step) {
                for (int kb = kb_begin; kb < kb_end; kb++) {
                    const int kc = (kb - kb_begin) % Cfg::kChunkKB;
                    if (kc == 0) {
                        if (!mbar_wait_cluster(tempty, static_cast<uint32_t>(uses & 1) ^ 1u, abort)) {
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
                    const uint32_t stage_base = smem_base + stage * Cfg::kStageBytes;
                    if constexpr (Cfg::kMix) {
                        // hi, mid and lo of the float32 operand (bf16 tiles at
                        // 0, 16 and 32 KB of the stage) against the bf16 operand
                        const uint32_t sa = Cfg::kMixA ? stage_base : stage_base + Cfg::kMixOtherOffset;
                        const uint32_t sb = Cfg::kMixA ? stage_base + Cfg::kMixOtherOffset : stage_base;
#pragma unroll
                        for (int k = 0; k < Cfg::kKSteps; k++) {
                            const uint32_t a_off = p.a_mn_major ? k * Cfg::kMmaK * 128 : k * 32;
                            const uint32_t b_off = p.b_mn_major ? k * Cfg::kMmaK * 128 : k * 32;
#pragma unroll
                            for (int part = 0; part < 3; part++) {
                                const uint32_t pa = Cfg::kMixA ? part * Cfg::kATile : 0;
                                const uint32_t pb = Cfg::kMixA ? 0 : part * Cfg::kATile;
                                umma_f16_pair(tmem_base, smem_desc(sa + pa + a_off, a_lbo, a_sbo, a_lay),
                                              smem_desc(sb + pb + b_off, b_lbo, b_sbo, b_lay), p.idesc,
                                              (kc | k | part) != 0);
                            }
                        }
                    } else {
                        const uint32_t sa = stage_base;
                        const uint32_t sb = sa + Cfg::kATile;
                        const uint32_t la = smem_base + Cfg::kLoOffset +
                                            static_cast<uint32_t>(lo_slot * Cfg::kLoadBytes);
                        const uint32_t lb = la + Cfg::kATile;
#pragma unroll
                        for (int k = 0; k < Cfg::kKSteps; k++) {
                            const uint32_t a_off = p.a_mn_major ? k * Cfg::kMmaK * 128 : k * 32;
                            const uint32_t b_off = p.b_mn_major ? k * Cfg::kMmaK * 128 : k * 32;
                            const uint64_t ad = smem_desc(sa + a_off, a_lbo, a_sbo, a_lay);
                            const uint64_t bd = smem_desc(sb + b_off, b_lbo, b_sbo, b_lay);
                            const uint64_t ad_lo = smem_desc(la + a_off, a_lbo, a_sbo, a_lay);
                            const uint64_t bd_lo = smem_desc(lb + b_off, b_lbo, b_sbo, b_lay);
                            umma_tf32_pair(tmem_base, ad, bd, p.idesc, (kc | k) != 0);
                            umma_tf32_pair(tmem_base, ad, bd_lo, p.idesc, 1);
                            umma_tf32_pair(tmem_base, ad_lo, bd, p.idesc, 1);
                        }
                    }
                    const uint32_t e0 = smem_addr(&empty[stage]);
                    umma_commit_pair(e0);
                    umma_commit_pair(map_to_cta(e0, peer));
                    if constexpr (!Cfg::kMix) {
                        const uint32_t l0 = smem_addr(&lo_free[lo_slot]);
                        umma_commit_pair(l0);
                        umma_commit_pair(map_to_cta(l0, peer));
                        if (++lo_slot == Cfg::kLoStages)
                            lo_slot = 0;
                    }
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                    if (kc == Cfg::kChunkKB - 1 || kb == kb_end - 1) {
                        const uint32_t f0 = smem_addr(tfull);
                        umma_commit_pair(f0);
                        umma_commit_pair(map_to_cta(f0, peer));
                        uses++;
                    }
                }
            }
            umma_commit_pair(smem_addr(drain));
            int no_abort = 0;
            mbar_wait(drain, 0, &no_abort);
        }
    } else if (warp < 2 + Cfg::kEpiWarps) {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int ew = warp - 2;
        const int quad = warp & 3;
        constexpr int kGroups = BN / 32 / Cfg::kEpiParts;   // 32-column groups per warp
        const int g0 = (ew >> 2) * kGroups;
        uint8_t *stage_buf = smem + Cfg::kEpiOffset + ew * Cfg::kEpiBufs * Cfg::kEpiBufBytes;
        const uint32_t tempty0 = map_to_cta(smem_addr(tempty), leader);
        int buf = 0;
        long long uses = 0;
        bool ok = true;
        auto emit = [&](float (&v)[Cfg::kEpiCols], int col0, int row0, const int (&c)[3]) {
            if (p.bias != nullptr || p.act != ACT_NONE)
                apply_epilogue_compact<OUT_F32, Cfg::kEpiCols>(v, p.bias, p.act, col0, p.N, lane);
            uint8_t *sbuf = stage_buf + buf * Cfg::kEpiBufBytes;
            if (lane == 0) {
                if constexpr (Cfg::kEpiBufs == 2)
                    bulk_wait_group_read<1>();
                else
                    bulk_wait_group_read<0>();
            }
            __syncwarp();
            uint8_t *rowp = sbuf + lane * 128;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                uint4 q;
                q.x = __float_as_uint(v[4 * j + 0]);
                q.y = __float_as_uint(v[4 * j + 1]);
                q.z = __float_as_uint(v[4 * j + 2]);
                q.w = __float_as_uint(v[4 * j + 3]);
                *reinterpret_cast<uint4 *>(rowp + ((j ^ (lane & 7)) << 4)) = q;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && col0 < p.N && row0 < p.M) {
                tma_store_5d(&tma_c, sbuf, col0, row0, c[0], c[1], c[2]);
                bulk_commit_group();
            }
            buf ^= Cfg::kEpiBufs - 1;
        };
        const int nchunks = (kb_end - kb_begin + Cfg::kChunkKB - 1) / Cfg::kChunkKB;
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
        const uint32_t t_total = lane_base + static_cast<uint32_t>(Cfg::kTotalCol);
        // split-K: this thread's row of the partial tile in the ring
        float *part_row = reinterpret_cast<float *>(smem) + (quad * 32 + lane) * Cfg::kPartPitch;
        int c_last[3] = {0, 0, 0};
        int n0_last = 0, row0_last = 0;
        for (long long t = t_first; ok && t < p.tiles; t += t_step) {
            const int nb = static_cast<int>(t % p.n_blocks);
            const long long r = t / p.n_blocks;
            const int mb = static_cast<int>(r % p.m_blocks);
            const long long batch = r / p.m_blocks;
            int c[3];
            decode_batch(batch, p, c);
            const int row0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::kRowsCta + quad * 32;
            const int n0 = nb * BN;
            c_last[0] = c[0];
            c_last[1] = c[1];
            c_last[2] = c[2];
            n0_last = n0;
            row0_last = row0;
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
                const bool last = ck == nchunks - 1;
#pragma unroll 1
                for (int h = g0; h < g0 + kGroups; h++) {
                    uint32_t r32[32], t32[32];
                    tmem_ld_32x32b_x32(lane_base + h * 32, r32);
                    if (ck > 0)
                        tmem_ld_32x32b_x32(t_total + h * 32, t32);
                    tmem_ld_wait();
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        v[i] = (ck > 0 ? __uint_as_float(t32[i]) : 0.0f) + __uint_as_float(r32[i]);
                    if (!last) {
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            t32[i] = __float_as_uint(v[i]);
                        tmem_st_32x32b_x32(t_total + h * 32, t32);
                    } else {
                        if (h == g0 + kGroups - 1) {
                            // accumulator fully read: hand it back to the MMA thread
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0)
                                mbar_arrive_cluster(tempty0);
                        }
                        if (G > 1) {
#pragma unroll
                            for (int i = 0; i < 8; i++)
                                *reinterpret_cast<float4 *>(part_row + h * 32 + 4 * i) =
                                    make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                        } else {
                            emit(v, n0 + h * 32, row0, c);
                        }
                    }
                }
                if (!last) {
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_cluster(tempty0);
                }
            }
        }
        if (G > 1) {
            // Every CTA's partial block is in its ring; CTA (q, c) of the
            // cluster finishes columns [q * BN / G, (q + 1) * BN / G) of its
            // 128 rows, adding the G partials of CTAs (0, c) .. (G - 1, c) in
            // that order over DSMEM.  The two warps of a lane quadrant share
            // the slice.
            cluster_sync();
            if (ok && t_first < p.tiles) {
                const uint32_t row_s = smem_addr(part_row);
                const int cols = BN / G, col_lo = krank * cols;
                for (int h = col_lo / 32 + (ew >> 2); h < (col_lo + cols) / 32; h += Cfg::kEpiParts) {
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const uint32_t off = static_cast<uint32_t>((h * 32 + 4 * i) * 4);
                        float4 acc4 = ld_cluster_f4(map_to_cta(row_s + off, rank));
                        for (int q = 1; q < G; q++) {
                            const float4 x = ld_cluster_f4(map_to_cta(row_s + off, 2 * q + rank));
                            acc4.x += x.x;
                            acc4.y += x.y;
                            acc4.z += x.z;
                            acc4.w += x.w;
                        }
                        v[4 * i] = acc4.x;
                        v[4 * i + 1] = acc4.y;
                        v[4 * i + 2] = acc4.z;
                        v[4 * i + 3] = acc4.w;
                    }
                    emit(v, n0_last + h * 32, row0_last, c_last);
                }
            }
            cluster_sync();   // peers are done reading this CTA's partial block
        }
        if (lane == 0)
            bulk_wait_group<0>();
        __syncwarp();
    } else {
        // ------------------------------------------------------------ split warps (both CTAs)
        if constexpr (Cfg::kMix) {
            // float32 operand -> bf16 hi/mid/lo tiles in the 128-byte-swizzled
            // layout a bf16 TMA load of it would produce, in place: every
            // split thread first reads its raw elements, then (named barrier)
            // the tiles are overwritten.  A failed wait sets the abort flag,
            // after which every wait returns at once; the loop runs to the
            // end so that all split threads meet at every barrier.
            constexpr int kThr = Cfg::kSplitWarps * 32;
            constexpr int kVecs = Cfg::kMixRawBytes / 16;
            constexpr int kPer = (kVecs + kThr - 1) / kThr;
            const int st = threadIdx.x - 32 * (2 + Cfg::kEpiWarps);
            const bool f_mn = Cfg::kMixA ? p.a_mn_major : p.b_mn_major;
            int stage = 0;
            uint32_t phase = 0;
            for (long long t = t_first; t < p.tiles; t += t_step) {
                for (int kb = kb_begin; kb < kb_end; kb++) {
                    if (!mbar_wait(&full[stage], phase, abort))
                        record_failure(abort, p.status, DEV_TIMEOUT_SPLIT);
                    uint8_t *base = smem + stage * Cfg::kStageBytes;
                    const float4 *raw = reinterpret_cast<const float4 *>(base);
                    float4 x[kPer];
#pragma unroll
                    for (int j = 0; j < kPer; j++) {
                        const int e = st + j * kThr;
                        if (kVecs % kThr == 0 || e < kVecs)
                            x[j] = raw[e];
                    }
                    named_barrier_sync(1, kThr);
#pragma unroll
                    for (int j = 0; j < kPer; j++) {
                        const int e = st + j * kThr;
                        if (kVecs % kThr != 0 && e >= kVecs)
                            continue;
                        uint32_t off;
                        if (!f_mn) {
                            // raw [128 rows][64 k]: row e / 16, k 4 * (e % 16)
                            const int r = e >> 4, k4 = e & 15;
                            off = r * 128 + ((((k4 >> 1) ^ (r & 7))) << 4) + ((k4 & 1) << 3);
                        } else {
                            // raw [64 k][128 rows]: k e / 32, rows 4 * (e % 32)
                            const int k = e >> 5, r4 = e & 31;
                            off = (r4 >> 4) * Cfg::kChunkBytes + k * 128 +
                                  ((((r4 & 15) >> 1) ^ (k & 7)) << 4) + ((r4 & 1) << 3);
                        }
                        split3_store(x[j], base, off, Cfg::kATile);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_cluster(map_to_cta(smem_addr(&ready[stage]), leader));
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        } else {
            // lo = tf32(x - trunc(x)) of this CTA's raw tiles into its lo ring;
            // each warp then arrives on CTA 0's ready barrier.  Waits are made
            // warp-uniform so a timeout leaves the warp together.
            const int st = threadIdx.x - 32 * (2 + Cfg::kEpiWarps);   // 0..255
            int stage = 0, lo_slot = 0;
            uint32_t phase = 0, lo_phase = 0;
            bool ok = true;
            constexpr int kVecs = Cfg::kLoadBytes / 16;
            constexpr int kPer = (kVecs + Cfg::kSplitWarps * 32 - 1) / (Cfg::kSplitWarps * 32);
            auto lo_of = [](float x) { return isfinite(x) ? round_tf32(x - trunc_tf32(x)) : 0.0f; };
            for (long long t = t_first; ok && t < p.tiles; t += t_step) {
                for (int kb = kb_begin; kb < kb_end; kb++) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort))) {
                        if (lane == 0)
                            record_failure(abort, p.status, DEV_TIMEOUT_SPLIT);
                        ok = false;
                        break;
                    }
                    const float4 *raw = reinterpret_cast<const float4 *>(smem + stage * Cfg::kStageBytes);
                    float4 l[kPer];
#pragma unroll
                    for (int j = 0; j < kPer; j++) {
                        const int i = st + j * Cfg::kSplitWarps * 32;
                        if (kVecs % (Cfg::kSplitWarps * 32) == 0 || i < kVecs) {
                            const float4 x = raw[i];
                            l[j] = make_float4(lo_of(x.x), lo_of(x.y), lo_of(x.z), lo_of(x.w));
                        }
                    }
                    if (!__all_sync(0xffffffffu, mbar_wait(&lo_free[lo_slot], lo_phase ^ 1, abort))) {
                        if (lane == 0)
                            record_failure(abort, p.status, DEV_TIMEOUT_SPLIT);
                        ok = false;
                        break;
                    }
                    float4 *lo = reinterpret_cast<float4 *>(smem + Cfg::kLoOffset +
                                                            lo_slot * Cfg::kLoadBytes);
#pragma unroll
                    for (int j = 0; j < kPer; j++) {
                        const int i = st + j * Cfg::kSplitWarps * 32;
                        if (kVecs % (Cfg::kSplitWarps * 32) == 0 || i < kVecs)
                            lo[i] = l[j];
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_cluster(map_to_cta(smem_addr(&ready[stage]), leader));
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
    cluster_sync();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    }
}

} // namespace ptg
