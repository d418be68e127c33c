// Batched GEMM for results with few columns (N <= 32) and a long inner axis:
// the classifier layer of an MLP (N = 10) and its weight gradient
// dW = h^T . dC.  The general kernels cover these with mostly empty 64- or
// 128-wide column tiles, and the weight gradient (M = fan_in, K = batch) gives
// them only a few dozen CTAs with a long serial K loop each.
//
// Here a CTA owns 32 rows and all NB (>= N) columns.  The K axis is cut into
// chunks of 32 that move through double-buffered shared tiles (A stored k-major
// [k][row] so each lane reads its own row; B [k][col]); the load mapping
// follows A's layout so global reads are coalesced whether A is K-contiguous
// (forward) or M-contiguous (the transposed view of the weight gradient).
// Inside the CTA, warp w = (column group, k group): lane = row, four columns
// per thread, the k group taking its own sub-range of every chunk.  Across
// CTAs, a thread-block cluster of C CTAs splits the chunks into C contiguous
// ranges.  Partial sums meet in shared memory and CTA rank 0 adds them over
// DSMEM in a fixed order (cluster rank, then k group), so results are
// deterministic, bit-identical from call to call.
//
// Two variants share that structure.  float32 and float64 stream their chunks
// through a multi-stage cp.async ring (one element per copy, zero-filled past
// the edges), so several chunks per CTA are in flight whatever the layout;
// the 16-bit types, which only come here when the tensor-core kernel cannot
// describe their layout, stage one chunk ahead in registers and widen to
// float on the way into shared memory.
#pragma once

#include "gemm_simt.cuh"
#include "ptx_sm100.cuh"

namespace ptg {

constexpr int kSkinnyMaxN = 32;
constexpr int kSkinnyBM = 32;      // rows per CTA (one per lane)
constexpr int kSkinnyKC = 32;      // k per staged chunk
constexpr int kSkinnyThreads = 256;
constexpr int kSkinnyMaxCluster = 8;
constexpr int kSkinnyRegChunks = 4;   // register-staged kernel: chunks loaded ahead

template <int NB>
struct SkinnyShape {
    static constexpr int kColGroups = NB / 4;                 // four columns per thread
    static constexpr int kKGroups = 8 / kColGroups;           // warps sharing a column group
    static constexpr int kKPerGroup = kSkinnyKC / kKGroups;   // k of a chunk per k group
    static constexpr int kAPitch = kSkinnyBM + 1;
    static constexpr int kAPerThread = kSkinnyBM * kSkinnyKC / kSkinnyThreads;   // 4
    static constexpr int kBElems = kSkinnyKC * NB;
    static constexpr int kBPerThread = (kBElems + kSkinnyThreads - 1) / kSkinnyThreads;
    static_assert(NB == 4 || NB == 8 || NB == 16 || NB == 32, "NB");
};

struct SkinnyArgs {
    int cluster;      // CTAs per cluster splitting K (1..8)
    int a_k_major;    // 1: A is K-contiguous (a_sk == 1)
    int b_n_major;    // 1: B is N-contiguous (b_sn == 1)
};

// Load of a peer CTA's shared memory (shared::cluster address from mapa).
__device__ __forceinline__ float ld_shared_cluster(uint32_t addr, float)
{
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ double ld_shared_cluster(uint32_t addr, double)
{
    double v;
    asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(addr) : "memory");
    return v;
}

// Four consecutive B values of a staged row (16-byte aligned).
__device__ __forceinline__ void load4(const float *s, float (&b)[4])
{
    const float4 v = *reinterpret_cast<const float4 *>(s);
    b[0] = v.x; b[1] = v.y; b[2] = v.z; b[3] = v.w;
}
__device__ __forceinline__ void load4(const double *s, double (&b)[4])
{
    const double2 v0 = *reinterpret_cast<const double2 *>(s);
    const double2 v1 = *reinterpret_cast<const double2 *>(s + 2);
    b[0] = v0.x; b[1] = v0.y; b[2] = v1.x; b[3] = v1.y;
}

// Output (m, n) of one batch with the optional bias and activation, rounded
// as the unfused plan rounds (product to the storage type first).
template <typename T>
__device__ __forceinline__ void skinny_store_out(const SimtParams &p, long long oc, int m, int n,
                                                 typename Elem<T>::Acc v)
{
    using E = Elem<T>;
    using Acc = typename E::Acc;
    if (p.bias != nullptr || p.act != ACT_NONE) {
        Acc x = E::round_trip(v);
        if (p.bias != nullptr) x += Acc(E::load(p.bias, n));
        if constexpr (sizeof(Acc) == 8)
            v = apply_activation_d(x, p.act);
        else
            v = apply_activation(x, p.act);
    }
    E::store(p.c, oc + static_cast<long long>(m) * p.c_sm + static_cast<long long>(n) * p.c_sn, v);
}

// TA / TB: operand element types (widened to float on load), T the result's.
template <typename T, int NB, typename TA = T, typename TB = T>
__global__ void __launch_bounds__(kSkinnyThreads) skinny_gemm_kernel(const SimtParams p,
                                                                      const SkinnyArgs sa)
{
    using E = Elem<T>;
    using Acc = typename E::Acc;
    using S = SkinnyShape<NB>;
    __shared__ __align__(16) Acc sA[2][kSkinnyKC][S::kAPitch];
    __shared__ __align__(16) Acc sB[2][kSkinnyKC][NB];
    __shared__ __align__(16) Acc red[S::kKGroups][kSkinnyBM][NB];

    // programmatic dependent launch: nothing global is touched before the
    // previous kernel in the stream has completed
    grid_dependency_wait();
    grid_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cg = warp % S::kColGroups, kg = warp / S::kColGroups;
    const int C = sa.cluster;
    const int rank = C > 1 ? static_cast<int>(cluster_cta_rank()) : 0;
    const int cluster_id = blockIdx.x / C, clusters = gridDim.x / C;
    const int m_blocks = (p.M + kSkinnyBM - 1) / kSkinnyBM;
    const int chunks = (p.K + kSkinnyKC - 1) / kSkinnyKC;
    const int per_rank = (chunks + C - 1) / C;
    const int c_begin = min(chunks, rank * per_rank);
    const int c_end = min(chunks, c_begin + per_rank);

    for (long long batch = blockIdx.z; batch < p.batches; batch += gridDim.z)
    for (int mb = cluster_id; mb < m_blocks; mb += clusters) {
        long long oa = 0, ob = 0, oc = 0, rem = batch;
        for (int d = p.nbd - 1; d >= 0; d--) {
            const long long coord = rem % p.bshape[d];
            rem /= p.bshape[d];
            oa += coord * p.a_bs[d];
            ob += coord * p.b_bs[d];
            oc += coord * p.c_bs[d];
        }
        const int m0 = mb * kSkinnyBM;

        // kSkinnyRegChunks chunks in flight in registers (a chunk is only
        // kAPerThread + kBPerThread values per thread), so the loop does not
        // wait a global-load round trip per chunk
        Acc ra_ring[kSkinnyRegChunks][S::kAPerThread], rb_ring[kSkinnyRegChunks][S::kBPerThread];
        auto load_chunk = [&](int c, Acc (&ra)[S::kAPerThread], Acc (&rb)[S::kBPerThread]) {
            const int k0 = c * kSkinnyKC;
#pragma unroll
            for (int i = 0; i < S::kAPerThread; i++) {
                const int e = threadIdx.x + kSkinnyThreads * i;
                const int row = sa.a_k_major ? e / kSkinnyKC : e % kSkinnyBM;
                const int kk = sa.a_k_major ? e % kSkinnyKC : e / kSkinnyBM;
                const int m = m0 + row, k = k0 + kk;
                ra[i] = (m < p.M && k < p.K)
                            ? Acc(Elem<TA>::load(p.a, oa + static_cast<long long>(m) * p.a_sm +
                                                          static_cast<long long>(k) * p.a_sk))
                            : Acc(0);
            }
#pragma unroll
            for (int i = 0; i < S::kBPerThread; i++) {
                const int e = threadIdx.x + kSkinnyThreads * i;
                const int n = sa.b_n_major ? e % NB : e / kSkinnyKC;
                const int kk = sa.b_n_major ? e / NB : e % kSkinnyKC;
                const int k = k0 + kk;
                rb[i] = (e < S::kBElems && n < p.N && k < p.K)
                            ? Acc(Elem<TB>::load(p.b, ob + static_cast<long long>(k) * p.b_sk +
                                                          static_cast<long long>(n) * p.b_sn))
                            : Acc(0);
            }
        };
        auto store_chunk = [&](int buf, const Acc (&ra)[S::kAPerThread],
                               const Acc (&rb)[S::kBPerThread]) {
#pragma unroll
            for (int i = 0; i < S::kAPerThread; i++) {
                const int e = threadIdx.x + kSkinnyThreads * i;
                const int row = sa.a_k_major ? e / kSkinnyKC : e % kSkinnyBM;
                const int kk = sa.a_k_major ? e % kSkinnyKC : e / kSkinnyBM;
                sA[buf][kk][row] = ra[i];
            }
#pragma unroll
            for (int i = 0; i < S::kBPerThread; i++) {
                const int e = threadIdx.x + kSkinnyThreads * i;
                if (e < S::kBElems) {
                    const int n = sa.b_n_major ? e % NB : e / kSkinnyKC;
                    const int kk = sa.b_n_major ? e / NB : e % kSkinnyKC;
                    sB[buf][kk][n] = rb[i];
                }
            }
        };

        Acc acc[4] = {Acc(0), Acc(0), Acc(0), Acc(0)};
#pragma unroll
        for (int j = 0; j < kSkinnyRegChunks; j++)
            if (c_begin + j < c_end)
                load_chunk(c_begin + j, ra_ring[j], rb_ring[j]);
        for (int c0 = c_begin; c0 < c_end; c0 += kSkinnyRegChunks) {
#pragma unroll
            for (int j = 0; j < kSkinnyRegChunks; j++) {   // static ring slot j
                const int c = c0 + j;
                if (c >= c_end)
                    break;   // uniform over the block
                const int buf = (c - c_begin) & 1;
                store_chunk(buf, ra_ring[j], rb_ring[j]);
                __syncthreads();
                if (c + kSkinnyRegChunks < c_end)   // refill the slot just stored
                    load_chunk(c + kSkinnyRegChunks, ra_ring[j], rb_ring[j]);
#pragma unroll
                for (int kk = kg * S::kKPerGroup; kk < (kg + 1) * S::kKPerGroup; kk++) {
                    const Acc a = sA[buf][kk][lane];
                    Acc b[4];
                    load4(&sB[buf][kk][cg * 4], b);
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        acc[q] = E::fma_(a, b[q], acc[q]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
            red[kg][lane][cg * 4 + j] = acc[j];
        if (C > 1)
            cluster_sync();   // every rank's partials are in its shared memory
        else
            __syncthreads();
        if (rank == 0) {
            for (int e = threadIdx.x; e < kSkinnyBM * p.N; e += kSkinnyThreads) {
                const int r = e / p.N, n = e % p.N;
                const int m = m0 + r;
                if (m >= p.M)
                    continue;
                Acc s = Acc(0);
                for (int q = 0; q < C; q++) {
#pragma unroll
                    for (int g = 0; g < S::kKGroups; g++) {
                        if (q == 0) {
                            s += red[g][r][n];
                        } else {
                            const uint32_t addr = map_to_cta(smem_addr(&red[g][r][n]), q);
                            s += ld_shared_cluster(addr, Acc(0));
                        }
                    }
                }
                skinny_store_out<T>(p, oc, m, n, s);
            }
        }
        if (C > 1)
            cluster_sync();   // rank 0 is done reading the peers' partials
        else
            __syncthreads();
    }
}

// ------------------------------------------------------------ cp.async ring
template <typename T>
__device__ __forceinline__ void cp_async_elem(uint32_t d, const T *src, bool valid)
{
    const int n = valid ? static_cast<int>(sizeof(T)) : 0;   // 0: zero-fill the element
    if constexpr (sizeof(T) == 4)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(n)
                     : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(d), "l"(src), "r"(n)
                     : "memory");
}

__device__ __forceinline__ void skinny_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void skinny_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// float32 / float64 variant: eight k groups (one per warp), lane = row, every
// thread accumulating all NB columns of its row, so each k costs a warp one
// conflict-free A read and NB/4 broadcast B reads for NB FMAs.
// AVEC (float32 only): A lands in 16-byte copies of four elements instead of
// one 4-byte copy per element, so a chunk costs each thread one copy instead
// of four.  An M-contiguous A keeps the [k][row] layout with the row pitch
// padded to 36 floats (16-byte aligned groups of four rows); a K-contiguous
// A is stored [row][k] with the 16-byte k-quads of row r at quad q ^ (r % 8),
// so each warp reads its k-quad as one float4 per lane without bank
// conflicts.
template <typename T, int NB, bool AVEC = false>
struct SkinnyRing {
    static constexpr int kStages = sizeof(T) == 4 ? 8 : 4;
    static constexpr int kKGroups = 8;
    static constexpr int kKPerGroup = kSkinnyKC / kKGroups;
    static constexpr int kAPitch = AVEC ? 36 : kSkinnyBM + 1;
    static_assert(!AVEC || (sizeof(T) == 4 && kKPerGroup == 4), "float32 k-quads");
    static constexpr int kAStage = kSkinnyKC * kAPitch;
    static constexpr int kBStage = kSkinnyKC * NB;
    static constexpr int kAPerThread = kSkinnyBM * kSkinnyKC / kSkinnyThreads;   // 4
    static constexpr int kBElems = kSkinnyKC * NB;
    static constexpr int kBPerThread = (kBElems + kSkinnyThreads - 1) / kSkinnyThreads;
    static_assert(NB % 4 == 0 && NB <= kSkinnyMaxN, "NB");
    static constexpr int kRedPitch = NB + 1;   // partials [warp][row][kRedPitch], aliasing the ring
    static constexpr int kRingElems = kStages * (kAStage + kBStage);
    static constexpr int kRedElems = kKGroups * kSkinnyBM * kRedPitch;
    static constexpr int kSmemBytes =
        (kRingElems > kRedElems ? kRingElems : kRedElems) * static_cast<int>(sizeof(T));
};

template <typename T, int NB, bool AVEC = false>
constexpr int skinny_async_smem_bytes()
{
    return SkinnyRing<T, NB, AVEC>::kSmemBytes;
}

__device__ __forceinline__ void cp_async_16(uint32_t d, const void *src, int bytes)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes)
                 : "memory");
}

// AKM: A is K-contiguous (loads walk k across the lanes) rather than
// M-contiguous or strided (loads walk m).
template <typename T, int NB, bool AKM, bool AVEC = false>
__global__ void __launch_bounds__(kSkinnyThreads) skinny_async_kernel(const SimtParams p,
                                                                       const SkinnyArgs sa)
{
    using E = Elem<T>;
    using R = SkinnyRing<T, NB, AVEC>;
    constexpr int kStages = R::kStages;
    extern __shared__ __align__(16) unsigned char skinny_smem[];
    T *ringA = reinterpret_cast<T *>(skinny_smem);
    T *ringB = ringA + kStages * R::kAStage;
    T *red = ringA;   // after the main loop
    grid_dependency_wait();   // programmatic dependent launch, as above
    grid_launch_dependents();

    const T *A = static_cast<const T *>(p.a);
    const T *B = static_cast<const T *>(p.b);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int C = sa.cluster;
    const int rank = C > 1 ? static_cast<int>(cluster_cta_rank()) : 0;
    const int cluster_id = blockIdx.x / C, clusters = gridDim.x / C;
    const int m_blocks = (p.M + kSkinnyBM - 1) / kSkinnyBM;
    const int chunks = (p.K + kSkinnyKC - 1) / kSkinnyKC;
    const int per_rank = (chunks + C - 1) / C;
    const int c_begin = min(chunks, rank * per_rank);
    const int c_end = min(chunks, c_begin + per_rank);
    const int n_chunks = c_end - c_begin;

    // This thread's fixed (row, k) slots of an A chunk and (k, n) slots of a
    // B chunk, and their shared-memory offsets inside a ring stage.
    const uint32_t ringA_s = smem_addr(ringA), ringB_s = smem_addr(ringB);
    int a_kk[R::kAPerThread];
    uint32_t a_dst[R::kAPerThread];   // byte offset inside a ring stage
    int b_kk[R::kBPerThread], b_n[R::kBPerThread];
    uint32_t b_dst[R::kBPerThread];
#pragma unroll
    for (int i = 0; i < R::kAPerThread; i++) {
        const int e = threadIdx.x + kSkinnyThreads * i;
        const int row = AKM ? e / kSkinnyKC : e % kSkinnyBM;
        a_kk[i] = AKM ? e % kSkinnyKC : e / kSkinnyBM;
        a_dst[i] = static_cast<uint32_t>((a_kk[i] * R::kAPitch + row) * sizeof(T));
    }
    // AVEC: this thread's one 16-byte slot (four rows at one k, or one row's
    // k-quad) and its byte offset inside a ring stage
    const int v_a = threadIdx.x >> 3, v_b = threadIdx.x & 7;   // 32 x 8 slots
    const int v_row = AKM ? v_a : 4 * v_b;                     // first row of the slot
    const int v_k = AKM ? 4 * v_b : v_a;                       // first k of the slot
    const uint32_t v_dst = static_cast<uint32_t>(
        (AKM ? v_a * kSkinnyKC + ((v_b ^ (v_a & 7)) << 2) : v_a * R::kAPitch + 4 * v_b) * 4);
#pragma unroll
    for (int i = 0; i < R::kBPerThread; i++) {
        const int e = threadIdx.x + kSkinnyThreads * i;
        b_n[i] = sa.b_n_major ? e % NB : e / kSkinnyKC;
        b_kk[i] = sa.b_n_major ? e / NB : e % kSkinnyKC;
        if (e >= R::kBElems)
            b_n[i] = NB;   // no slot: never valid
        b_dst[i] = static_cast<uint32_t>((b_kk[i] * NB + (b_n[i] < NB ? b_n[i] : 0)) * sizeof(T));
    }

    for (long long batch = blockIdx.z; batch < p.batches; batch += gridDim.z)
    for (int mb = cluster_id; mb < m_blocks; mb += clusters) {
        long long oa = 0, ob = 0, oc = 0, rem = batch;
        for (int d = p.nbd - 1; d >= 0; d--) {
            const long long coord = rem % p.bshape[d];
            rem /= p.bshape[d];
            oa += coord * p.a_bs[d];
            ob += coord * p.b_bs[d];
            oc += coord * p.c_bs[d];
        }
        const int m0 = mb * kSkinnyBM;

        // Running source of each slot, starting at this rank's first chunk and
        // advanced by one chunk per issue (rows past M and columns past N are
        // never read: their copies zero-fill from a valid address).
        const long long stepA = static_cast<long long>(kSkinnyKC) * p.a_sk;
        const long long stepB = static_cast<long long>(kSkinnyKC) * p.b_sk;
        const int kfirst = c_begin * kSkinnyKC;
        const T *pa[R::kAPerThread];
        bool va[R::kAPerThread];
#pragma unroll
        for (int i = 0; i < R::kAPerThread; i++) {
            const int e = threadIdx.x + kSkinnyThreads * i;
            const int m = m0 + (AKM ? e / kSkinnyKC : e % kSkinnyBM);
            va[i] = m < p.M;
            pa[i] = A + oa + static_cast<long long>(va[i] ? m : 0) * p.a_sm +
                    static_cast<long long>(kfirst + a_kk[i]) * p.a_sk;
        }
        // AVEC: the slot's source and how many of its four elements exist
        // (rows past M, or k past K in the last chunk, are zero-filled)
        const int v_rows = AKM ? (m0 + v_row < p.M ? 1 : 0) : max(0, min(4, p.M - (m0 + v_row)));
        const T *pav = v_rows ? A + oa + static_cast<long long>(m0 + v_row) * p.a_sm +
                                    static_cast<long long>(kfirst + v_k) * p.a_sk
                              : A;
        const T *pb[R::kBPerThread];
        bool vb[R::kBPerThread];
#pragma unroll
        for (int i = 0; i < R::kBPerThread; i++) {
            vb[i] = b_n[i] < p.N;
            pb[i] = B + ob + static_cast<long long>(kfirst + b_kk[i]) * p.b_sk +
                    static_cast<long long>(vb[i] ? b_n[i] : 0) * p.b_sn;
        }

        auto issue = [&](int j) {   // chunk c_begin + j into ring slot j % kStages
            if (j < n_chunks) {
                const int k0 = (c_begin + j) * kSkinnyKC;
                const uint32_t slot = static_cast<uint32_t>(j % kStages);
                const uint32_t sA = ringA_s + slot * (R::kAStage * sizeof(T));
                const uint32_t sB = ringB_s + slot * (R::kBStage * sizeof(T));
                if constexpr (AVEC) {
                    // bytes that exist: a row's k-quad cut at K, or four
                    // rows cut at M
                    const int n = AKM ? (v_rows ? 4 * min(4, max(0, p.K - (k0 + v_k))) : 0)
                                      : (k0 + v_k < p.K ? 4 * v_rows : 0);
                    cp_async_16(sA + v_dst, n ? pav : A, n);
                }
                if (k0 + kSkinnyKC <= p.K) {
#pragma unroll
                    for (int i = 0; i < (AVEC ? 0 : R::kAPerThread); i++)
                        cp_async_elem(sA + a_dst[i], va[i] ? pa[i] : A, va[i]);
#pragma unroll
                    for (int i = 0; i < R::kBPerThread; i++)
                        if (b_n[i] < NB)
                            cp_async_elem(sB + b_dst[i], vb[i] ? pb[i] : B, vb[i]);
                } else {   // the last chunk of K
#pragma unroll
                    for (int i = 0; i < (AVEC ? 0 : R::kAPerThread); i++) {
                        const bool ok = va[i] && k0 + a_kk[i] < p.K;
                        cp_async_elem(sA + a_dst[i], ok ? pa[i] : A, ok);
                    }
#pragma unroll
                    for (int i = 0; i < R::kBPerThread; i++) {
                        if (b_n[i] < NB) {
                            const bool ok = vb[i] && k0 + b_kk[i] < p.K;
                            cp_async_elem(sB + b_dst[i], ok ? pb[i] : B, ok);
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < R::kAPerThread; i++)
                    pa[i] += stepA;
                if (v_rows)
                    pav += stepA;
#pragma unroll
                for (int i = 0; i < R::kBPerThread; i++)
                    pb[i] += stepB;
            }
            skinny_commit();   // empty groups keep the wait_group count uniform
        };

        T acc[NB];
#pragma unroll
        for (int n = 0; n < NB; n++)
            acc[n] = T(0);
        __syncthreads();   // the previous tile is done with the ring (and the partials in it)
#pragma unroll 1
        for (int j = 0; j < kStages - 1; j++)
            issue(j);
#pragma unroll 1
        for (int j = 0; j < n_chunks; j++) {
            skinny_wait<kStages - 2>();
            __syncthreads();
            issue(j + kStages - 1);   // into the slot read at iteration j - 1
            const T *sA = ringA + (j % kStages) * R::kAStage;
            const T *sB = ringB + (j % kStages) * R::kBStage;
            const T *wA = sA + warp * R::kKPerGroup * R::kAPitch + lane;
            const T *wB = sB + warp * R::kKPerGroup * NB;
            T a4[R::kKPerGroup];
            if constexpr (AVEC && AKM) {
                // this lane's row, the warp's k-quad
                const float4 v = *reinterpret_cast<const float4 *>(
                    sA + lane * kSkinnyKC + ((warp ^ (lane & 7)) << 2));
                a4[0] = v.x;
                a4[1] = v.y;
                a4[2] = v.z;
                a4[3] = v.w;
            }
#pragma unroll
            for (int q = 0; q < R::kKPerGroup; q++) {
                const T a = AVEC && AKM ? a4[q] : wA[q * R::kAPitch];
#pragma unroll
                for (int n4 = 0; n4 < NB; n4 += 4) {
                    T b[4];
                    load4(wB + q * NB + n4, b);
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        acc[n4 + q] = E::fma_(a, b[q], acc[n4 + q]);
                }
            }
        }
        skinny_wait<0>();
        __syncthreads();   // every warp is done reading the ring
#pragma unroll
        for (int n = 0; n < NB; n++)
            red[(warp * kSkinnyBM + lane) * R::kRedPitch + n] = acc[n];
        __syncthreads();
        // this CTA's k groups, added in warp order into warp 0's slot
        for (int e = threadIdx.x; e < kSkinnyBM * p.N; e += kSkinnyThreads) {
            const int r = e / p.N, n = e % p.N;
            T s = red[r * R::kRedPitch + n];
#pragma unroll
            for (int w = 1; w < R::kKGroups; w++)
                s += red[(w * kSkinnyBM + r) * R::kRedPitch + n];
            red[r * R::kRedPitch + n] = s;
        }
        if (C > 1)
            cluster_sync();   // every rank's sums are in its shared memory
        if (rank == 0) {
            // thread e owns the same (r, n) as above, so its own sum needs no barrier
            for (int e = threadIdx.x; e < kSkinnyBM * p.N; e += kSkinnyThreads) {
                const int r = e / p.N, n = e % p.N;
                const int m = m0 + r;
                const uint32_t loc = smem_addr(red + r * R::kRedPitch + n);
                T v[kSkinnyMaxCluster];
#pragma unroll
                for (int q = 1; q < kSkinnyMaxCluster; q++)
                    v[q] = q < C ? ld_shared_cluster(map_to_cta(loc, q), T(0)) : T(0);
                T s = red[r * R::kRedPitch + n];
#pragma unroll
                for (int q = 1; q < kSkinnyMaxCluster; q++)
                    if (q < C)
                        s += v[q];
                if (m < p.M)
                    skinny_store_out<T>(p, oc, m, n, s);
            }
        }
        if (C > 1)
            cluster_sync();   // rank 0 is done reading the peers' sums
    }
}

} // namespace ptg
