// libgemm_sm100.so: the C ABI of include/gemm_sm100.h.
//
// Host-side dispatch that replaces src/backends/cuda/matmul_kernels.cu of
// lcmialichi/php-gpu-tensors.  For every call it
//   1. validates shapes and strides exactly as the reference launchers do
//      (matmul_kernels.cu:680-710, 856-875, 912-914), with NumPy batch
//      broadcasting (right-aligned axes, as src/tensor_shape.h:46-59 and the
//      host loop src/contiguous_array_ce.c:1280-1293 define it);
//   2. drops extent-1 batch axes and merges adjacent batch axes whose strides
//      compose, for all three operands at once;
//   3. when the layout can be described with TMA (unit stride in one of each
//      operand's matrix axes, 16-byte aligned pointer and strides, <= 3
//      merged batch axes, N-contiguous result) launches the persistent tcgen05
//      kernel (gemm_tc.cuh), otherwise the CUDA-core kernel (gemm_simt.cuh).
// Launches are asynchronous on the caller's stream and allocate nothing.
#include "gemm_sm100.h"

#include "gemm_f64.cuh"
#include "gemm_simt.cuh"
#include "gemm_skinny.cuh"
#include "gemm_tc.cuh"
#include "gemm_tc2.cuh"
#include "gemm_tc2w.cuh"
#include "gemm_tc2t.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <type_traits>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#define PT_API extern "C" __attribute__((visibility("default")))

using namespace ptg;

namespace {

// Device status word (one copy per device): first timeout code reported by a
// tensor-core kernel, 0 otherwise.
__device__ int g_device_status;

enum DType : int { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2, DT_F64 = 3 };

constexpr int kMaxBatchDims = kSimtMaxBatchDims;
constexpr double kTcMinWork = 4194304.0;   // M*N*K*batches below this: CUDA-core kernel
constexpr int kSkinnyMinK = 128;           // shortest K for the few-column kernel
constexpr int kStrictMinK = 64;            // shortest K for 3xTF32 (strict float32)
constexpr int kSplitMinKBlocks = 8;        // k-blocks per split-K rank, at least
#ifndef PTG_PAIR_CHUNK_KB
#define PTG_PAIR_CHUNK_KB 4
#endif
// 2-CTA 3xTF32: k-blocks (32 K each) per accumulator chunk, 128 K as in the
// single-CTA kernel
constexpr int kPairChunkKB = PTG_PAIR_CHUNK_KB;
// Time of one 256 x 256 tile of the 2-CTA 3xTF32 kernel in 128 x 128 tiles of
// the single-CTA one (B200, 4096 x 1024 x 1024: 64.0 us for one round of 64
// cluster tiles against 71.6 us for two waves of 256 tiles).  With it the
// choice matches the faster kernel on every measured shape (8192^3 pair,
// 4096^3 single-CTA, the config-4 layer products pair, their dW single-CTA).
constexpr double kPairTileCost = 1.79;
// The same for the 2-CTA strict float32 kernel with A in tensor memory
// (K-major A; B200: 4096 x 1024 x 1024 152 against 145 TFLOP/s for the
// shared-memory pair kernel, 4096^3 164-173 against 154-160): 1.79 scaled by
// those ratios.  With it 4096^3 (4 rounds of 74 pair tiles against 7 waves of
// 148 single-CTA tiles, 148-161 TFLOP/s) moves to the pair kernel.
constexpr double kPairTmemTileCost = 1.70;
// mixed kinds on the 2-CTA kernel: k-blocks (64 K each) per accumulator chunk,
// 256 K as in the single-CTA mixed kernel
constexpr int kMixPairChunkKB = 4;
// Time of one 256 x 512 tile of the wide 16-bit pair kernel in 256 x 256
// tiles of the plain one, and the shortest inner axis it is chosen for.
// Measured on B200 (TFLOP/s, plain -> wide, both with the same wave
// efficiency): bf16 [64,1024,1024]^2 1150 -> 1195, 8192^3 1447 -> 1609,
// [512,2048,2048]^2 (power-capped) 1141-1177 -> 1199-1228; with half as many
// waves' worth of padding lost the wide tile is slower (fp16 8192x4096x4096,
// 3.5 waves of wide tiles against 6.9: 1367 -> 1277).
constexpr double kWideTileCost = 1.9;
constexpr int kWideMinK = 1024;
constexpr double kTuneMinWork = 10000000.0; // matmul_kernels.cu:24 (MATMUL_LT_MIN_WORK)
// Fused float64 N-split: up to this many ranks each tile's epilogue stores
// it into every window; above it the persistent kernel copies a tile to the
// peers during the next tile's math.  Measured on B200 (8192^3, ms per step,
// compute alone / stores / copies): 1 GPU 34.88 / 34.93 / 36.55, 2 GPUs
// 17.46 / 17.66 / 18.58, 8 GPUs 4.45 / 5.10 / 5.16 -- the stores win at
// every rank count this library supports.
constexpr int kPeerStoreMaxRanks = 8;

struct Problem {
    int dt;
    const void *a, *b;
    void *c;
    int M, N, K;
    long long batches;
    int nbd;                       // C batch axes with extent > 1
    int bshape[kMaxBatchDims];
    long long a_bs[kMaxBatchDims]; // element strides, 0 = broadcast
    long long b_bs[kMaxBatchDims];
    long long c_bs[kMaxBatchDims];
    long long a_sm, a_sk, b_sk, b_sn, c_sm, c_sn;
    const void *bias;
    int act;
    int forced_bn;                 // 0 = heuristic / tuned plan
    int a_dt, b_dt;                // operand dtypes (dt is the result's; they differ only
                                   // for the float32-result gradient products)
    int nfd;                       // batch axes summed into the product (0 = none)
    int fshape[kMaxBatchDims];
    long long a_fs[kMaxBatchDims]; // element strides along the summed axes, 0 = broadcast
    long long b_fs[kMaxBatchDims];
    long long folds;               // product of fshape
};

// ------------------------------------------------------------ thread state
thread_local cuda_backend_info t_info = {};
thread_local int t_precision = CUDA_MATMUL_PRECISION_FP32_STRICT;
thread_local int t_path = 0;
thread_local const char *t_last_kernel = "none";
thread_local int t_last_grid = 0, t_last_block = 0, t_last_cluster = 0;

struct TunedPlan {
    int rows, inner, cols;
    size_t a_s0, a_s1, b_s0, b_s1;
    int precision;
    int algorithm;
};
constexpr size_t kMaxTunedPlans = 64;   // matmul_kernels.cu plan cache bound
thread_local std::vector<TunedPlan> t_plans;

// ------------------------------------------------------------ device state
constexpr int kMaxDevices = 64;
struct DeviceState {
    bool ready;
    int sms;
    int cc_major, cc_minor;
    int *status;                   // this device's copy of g_device_status
    unsigned long long attr_mask;  // kernels whose shared-memory limit has been raised
    int pair_clusters[12];         // co-resident 2-CTA clusters per pair kernel (0 = unknown)
};
std::mutex g_mutex;
DeviceState g_devices[kMaxDevices];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
bool g_encode_looked_up = false;

void set_status(int code) { t_info.last_blas_status = code; }

DeviceState *device_state()
{
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    DeviceState &d = g_devices[dev];
    if (!d.ready) {
        if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) !=
                cudaSuccess ||
            cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) !=
                cudaSuccess)
            return nullptr;
        void *status = nullptr;
        if (cudaGetSymbolAddress(&status, g_device_status) != cudaSuccess)
            return nullptr;
        d.status = static_cast<int *>(status);
        d.attr_mask = 0;
        d.ready = true;
    }
    if (!g_encode_looked_up) {
        g_encode_looked_up = true;
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    return &d;
}

// Raises the dynamic shared-memory limit of a kernel once per device.
template <typename K>
bool ensure_smem_attr(DeviceState *ds, int kernel_id, K kernel, int bytes)
{
    std::lock_guard<std::mutex> lock(g_mutex);
    if (ds->attr_mask & (1ull << kernel_id))
        return true;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
        cudaSuccess)
        return false;
    ds->attr_mask |= 1ull << kernel_id;
    return true;
}

// ------------------------------------------------------------ validation
// Returns 1 when there is work to launch, 2 when the call is a successful
// no-op (an M, N or batch extent of 0), 0 when the arguments are invalid.
int build_problem(int dt, const void *a, const void *b, void *c, const int *sa, const size_t *ta,
                  int na, const int *sb, const size_t *tb, int nb, const int *sc,
                  const size_t *tc, int nc, Problem *P)
{
    if (na < 2 || nb < 2 || nc < 2 || na > MAX_DIMS || nb > MAX_DIMS || nc > MAX_DIMS)
        return 0;
    if (!sa || !sb || !sc || !ta || !tb || !tc)
        return 0;
    const int rows = sa[na - 2], inner = sa[na - 1], cols = sb[nb - 1];
    if (inner != sb[nb - 2] || rows < 0 || inner < 0 || cols < 0 || sc[nc - 2] != rows ||
        sc[nc - 1] != cols)
        return 0;
    const int nbc = nc - 2, nba = na - 2, nbb = nb - 2;
    if (nba > nbc || nbb > nbc)
        return 0;
    std::memset(P, 0, sizeof(*P));
    P->dt = dt;
    P->a_dt = dt;
    P->b_dt = dt;
    P->folds = 1;
    P->a = a;
    P->b = b;
    P->c = c;
    P->M = rows;
    P->N = cols;
    P->K = inner;
    bool empty = rows == 0 || cols == 0;
    long long batches = 1;
    for (int d = 0; d < nbc; d++) {
        const int ext = sc[d];
        if (ext < 0)
            return 0;
        const int ia = d - (nbc - nba), ib = d - (nbc - nbb);
        const int ea = ia >= 0 ? sa[ia] : 1, eb = ib >= 0 ? sb[ib] : 1;
        if ((ea != 1 && ea != ext) || (eb != 1 && eb != ext) || ea < 0 || eb < 0)
            return 0;
        if (ext == 0) {
            empty = true;
            continue;
        }
        if (ext == 1)
            continue;
        if (batches > (1ll << 40) / ext)
            return 0;
        batches *= ext;
        const int k = P->nbd++;
        P->bshape[k] = ext;
        P->a_bs[k] = ea != 1 ? static_cast<long long>(ta[ia]) : 0;
        P->b_bs[k] = eb != 1 ? static_cast<long long>(tb[ib]) : 0;
        P->c_bs[k] = static_cast<long long>(tc[d]);
    }
    P->batches = batches;
    P->a_sm = static_cast<long long>(ta[na - 2]);
    P->a_sk = static_cast<long long>(ta[na - 1]);
    P->b_sk = static_cast<long long>(tb[nb - 2]);
    P->b_sn = static_cast<long long>(tb[nb - 1]);
    P->c_sm = static_cast<long long>(tc[nc - 2]);
    P->c_sn = static_cast<long long>(tc[nc - 1]);
    if (empty)
        return 2;
    if (!c || (inner > 0 && (!a || !b)))
        return 0;
    return 1;
}

// As build_problem, but C's batch axes may be a reduction of the broadcast
// batch shape of A and B: an axis where C has extent 1 (or no axis) while the
// product has extent > 1 is summed into the product (fshape, a_fs, b_fs).
int build_fold_problem(int dt, const void *a, const void *b, void *c, const int *sa,
                       const size_t *ta, int na, const int *sb, const size_t *tb, int nb,
                       const int *sc, const size_t *tc, int nc, Problem *P)
{
    if (na < 2 || nb < 2 || nc < 2 || na > MAX_DIMS || nb > MAX_DIMS || nc > MAX_DIMS)
        return 0;
    if (!sa || !sb || !sc || !ta || !tb || !tc)
        return 0;
    const int rows = sa[na - 2], inner = sa[na - 1], cols = sb[nb - 1];
    if (inner != sb[nb - 2] || rows < 0 || inner < 0 || cols < 0 || sc[nc - 2] != rows ||
        sc[nc - 1] != cols)
        return 0;
    const int nba = na - 2, nbb = nb - 2, nbc = nc - 2;
    const int nfull = nba > nbb ? nba : nbb;
    if (nbc > nfull)
        return 0;
    std::memset(P, 0, sizeof(*P));
    P->dt = P->a_dt = P->b_dt = dt;
    P->a = a;
    P->b = b;
    P->c = c;
    P->M = rows;
    P->N = cols;
    P->K = inner;
    bool empty = rows == 0 || cols == 0, fold_empty = false;
    long long batches = 1, folds = 1;
    for (int d = 0; d < nfull; d++) {
        const int ia = d - (nfull - nba), ib = d - (nfull - nbb), ic = d - (nfull - nbc);
        const int ea = ia >= 0 ? sa[ia] : 1, eb = ib >= 0 ? sb[ib] : 1;
        if (ea < 0 || eb < 0 || (ea != 1 && eb != 1 && ea != eb))
            return 0;
        const int ext = ea == 1 ? eb : ea;
        const int ec = ic >= 0 ? sc[ic] : 1;
        if (ec != ext && ec != 1)
            return 0;
        if (ext == 0) {
            if (ec == 0)
                empty = true;        // C itself is empty
            else
                fold_empty = true;   // a sum over nothing: C = 0
            continue;
        }
        if (ext == 1)
            continue;
        const long long as = ea != 1 ? static_cast<long long>(ta[ia]) : 0;
        const long long bs = eb != 1 ? static_cast<long long>(tb[ib]) : 0;
        if (ec == ext) {
            if (batches > (1ll << 40) / ext)
                return 0;
            batches *= ext;
            const int k = P->nbd++;
            P->bshape[k] = ext;
            P->a_bs[k] = as;
            P->b_bs[k] = bs;
            P->c_bs[k] = static_cast<long long>(tc[ic]);
        } else {
            if (folds > (1ll << 40) / ext)
                return 0;
            folds *= ext;
            const int k = P->nfd++;
            P->fshape[k] = ext;
            P->a_fs[k] = as;
            P->b_fs[k] = bs;
        }
    }
    P->batches = batches;
    P->folds = folds;
    P->a_sm = static_cast<long long>(ta[na - 2]);
    P->a_sk = static_cast<long long>(ta[na - 1]);
    P->b_sk = static_cast<long long>(tb[nb - 2]);
    P->b_sn = static_cast<long long>(tb[nb - 1]);
    P->c_sm = static_cast<long long>(tc[nc - 2]);
    P->c_sn = static_cast<long long>(tc[nc - 1]);
    if (empty)
        return 2;
    if (!c || (!fold_empty && inner > 0 && (!a || !b)))
        return 0;
    // a sum over an empty axis leaves C = 0: the CUDA-core kernel writes it
    if (fold_empty) {
        P->folds = 0;
        P->nfd = 0;
    }
    return 1;
}

// ------------------------------------------------------------ tensor maps
int element_bytes(int dt) { return dt == DT_F64 ? 8 : (dt == DT_F32 ? 4 : 2); }

CUtensorMapDataType tma_type(int dt)
{
    switch (dt) {
    case DT_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    case DT_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    }
}

struct MapDims {
    int rank = 0;            // used dims
    uint64_t ext[5];
    long long stride[5];     // element strides; stride[0] must be 1
};

// Encodes a rank-5, 128-byte-swizzled tiled tensor map.  Dims beyond `rank`
// and dims of extent 1 get a harmless 16-byte-multiple stride.  Returns false
// when TMA cannot describe the view.
bool encode_map(CUtensorMap *map, int dt, const void *base, const MapDims &m,
                const uint32_t (&box)[5], CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B)
{
    if (!g_encode)
        return false;
    const int es = element_bytes(dt);
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
        return false;
    cuuint64_t dims[5];
    cuuint64_t strides[4];
    cuuint32_t boxd[5], estr[5] = {1, 1, 1, 1, 1};
    const uint64_t filler = ((m.ext[0] * es + 15) / 16) * 16;
    for (int i = 0; i < 5; i++) {
        dims[i] = i < m.rank ? m.ext[i] : 1;
        boxd[i] = box[i];
        if (dims[i] == 0 || dims[i] > (1ull << 32))
            return false;
    }
    for (int i = 1; i < 5; i++) {
        uint64_t s = filler;
        if (i < m.rank && dims[i] > 1) {
            if (m.stride[i] <= 0)
                return false;
            s = static_cast<uint64_t>(m.stride[i]) * es;
            if (s % 16 != 0 || s >= (1ull << 40))
                return false;
        }
        strides[i - 1] = s;
    }
    const CUresult r = g_encode(map, tma_type(dt), 5, const_cast<void *>(base), dims, strides, boxd,
                                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Merged batch axes of a tensor-core launch.
struct TcBatch {
    int nbd;
    int bshape[3];
    long long a[3], b[3], c[3];
};

bool merge_batches(const Problem &P, TcBatch *out)
{
    int n = P.nbd;
    long long ext[kMaxBatchDims], sa[kMaxBatchDims], sb[kMaxBatchDims], sc[kMaxBatchDims];
    for (int d = 0; d < n; d++) {
        ext[d] = P.bshape[d];
        sa[d] = P.a_bs[d];
        sb[d] = P.b_bs[d];
        sc[d] = P.c_bs[d];
        if (sc[d] == 0)
            return false;   // distinct batches must not alias in the result
    }
    auto composable = [](long long outer, long long inner, long long inner_ext) {
        return (outer == 0 && inner == 0) || (outer != 0 && inner != 0 && outer == inner * inner_ext);
    };
    for (int d = n - 1; d > 0; d--) {
        if (composable(sa[d - 1], sa[d], ext[d]) && composable(sb[d - 1], sb[d], ext[d]) &&
            composable(sc[d - 1], sc[d], ext[d]) && ext[d - 1] * ext[d] < (1ll << 31)) {
            ext[d - 1] *= ext[d];
            sa[d - 1] = sa[d];
            sb[d - 1] = sb[d];
            sc[d - 1] = sc[d];
            for (int e = d; e < n - 1; e++) {
                ext[e] = ext[e + 1];
                sa[e] = sa[e + 1];
                sb[e] = sb[e + 1];
                sc[e] = sc[e + 1];
            }
            n--;
        }
    }
    if (n > 3)
        return false;
    out->nbd = n;
    for (int d = 0; d < 3; d++) {
        out->bshape[d] = d < n ? static_cast<int>(ext[d]) : 1;
        out->a[d] = d < n ? sa[d] : 0;
        out->b[d] = d < n ? sb[d] : 0;
        out->c[d] = d < n ? sc[d] : 0;
    }
    return true;
}

// Appends an operand's present batch axes to its map and records their slots.
// Merged summed (fold) axes of a tensor-core launch: as merge_batches, for A
// and B only.
struct TcFold {
    int nfd;
    int fshape[3];
    long long a[3], b[3];
};

bool merge_folds(const Problem &P, TcFold *out)
{
    int n = P.nfd;
    long long ext[kMaxBatchDims], sa[kMaxBatchDims], sb[kMaxBatchDims];
    for (int d = 0; d < n; d++) {
        ext[d] = P.fshape[d];
        sa[d] = P.a_fs[d];
        sb[d] = P.b_fs[d];
    }
    auto composable = [](long long outer, long long inner, long long inner_ext) {
        return (outer == 0 && inner == 0) || (outer != 0 && inner != 0 && outer == inner * inner_ext);
    };
    for (int d = n - 1; d > 0; d--) {
        if (composable(sa[d - 1], sa[d], ext[d]) && composable(sb[d - 1], sb[d], ext[d]) &&
            ext[d - 1] * ext[d] < (1ll << 31)) {
            ext[d - 1] *= ext[d];
            sa[d - 1] = sa[d];
            sb[d - 1] = sb[d];
            for (int e = d; e < n - 1; e++) {
                ext[e] = ext[e + 1];
                sa[e] = sa[e + 1];
                sb[e] = sb[e + 1];
            }
            n--;
        }
    }
    if (n > 3)
        return false;
    out->nfd = n;
    for (int d = 0; d < 3; d++) {
        out->fshape[d] = d < n ? static_cast<int>(ext[d]) : 1;
        out->a[d] = d < n ? sa[d] : 0;
        out->b[d] = d < n ? sb[d] : 0;
    }
    return true;
}

void add_fold_dims(MapDims &m, const TcFold &tf, const long long (&fs)[3], int (&slot)[3])
{
    for (int d = 0; d < 3; d++) {
        slot[d] = -1;
        if (d < tf.nfd && fs[d] != 0) {
            slot[d] = m.rank;
            m.ext[m.rank] = static_cast<uint64_t>(tf.fshape[d]);
            m.stride[m.rank] = fs[d];
            m.rank++;
        }
    }
}

void add_batch_dims(MapDims &m, const TcBatch &tb, const long long (&bs)[3], int (&slot)[3])
{
    for (int d = 0; d < 3; d++) {
        slot[d] = -1;
        if (d < tb.nbd && bs[d] != 0) {
            slot[d] = m.rank;
            m.ext[m.rank] = static_cast<uint64_t>(tb.bshape[d]);
            m.stride[m.rank] = bs[d];
            m.rank++;
        }
    }
}

uint32_t make_idesc(int fmt, int a_mn, int b_mn, int bn, int bm = 128)
{
    return (1u << 4)                                       // D: f32
           | (static_cast<uint32_t>(fmt) << 7)             // A format
           | (static_cast<uint32_t>(fmt) << 10)            // B format
           | (static_cast<uint32_t>(a_mn) << 15)           // A MN-major
           | (static_cast<uint32_t>(b_mn) << 16)           // B MN-major
           | (static_cast<uint32_t>(bn >> 3) << 17)        // N / 8
           | (static_cast<uint32_t>(bm >> 4) << 24);       // M / 16
}

enum KernelId : int {
    KID_BF16_128 = 0,
    KID_BF16_256,
    KID_F16_128,
    KID_F16_256,
    KID_TF32_128,
    KID_TF32_256,
    KID_F32X3_128,
    KID_BF16_PAIR,
    KID_F16_PAIR,
    KID_F64_DMMA,
    KID_F64_DMMA_PEER,
    KID_F32X3_PAIR,          // strict float32 on the 2-CTA 3xTF32 kernel
    KID_TF32_PAIR,           // tf32 precision mode on the 2-CTA kernel
    KID_MIX_A_PAIR,          // float32 A x bf16 B on the 2-CTA bf16x3 kernel
    KID_MIX_B_PAIR,          // bf16 A x float32 B on the 2-CTA bf16x3 kernel
    KID_SKINNY_ASYNC = 16,   // 24 ids: (float64 ? 12 : 0) + 2 * index of NB in {4,8,12,16,24,32} + A k-major
    KID_MIX_A = 40,          // float32 A (split into 3 bf16) x bf16 B -> float32
    KID_MIX_B,               // bf16 A x float32 B -> float32
    KID_BF16_F32,            // bf16 x bf16 -> float32
    KID_F16_F32,             // f16 x f16 -> float32
    KID_SKINNY_VEC,          // 12 ids: float32 few-column kernel with 16-byte A copies, 2 * NB index + A k-major
    KID_F64_DMMA_HALF = KID_SKINNY_VEC + 12,   // float64 half tiles of a launch's last wave
    KID_F64_DMMA_PEER_STORE,                   // N-split block, epilogue stores to every window
    KID_F64_DMMA_PEER_HALF,                    // its half tiles
    KID_F64_DMMA_HANDOFF_HALF,                 // half tiles of the hand-off kernel
    KID_BF16_WIDE,                             // bf16 on the 2-CTA 256 x 512 kernel
    KID_F16_WIDE,                              // f16 on the 2-CTA 256 x 512 kernel
    KID_F32X3_TPAIR,                           // strict float32, 2-CTA, A split into TMEM
};
static_assert(KID_F32X3_TPAIR < 64, "kernel ids index a 64-bit attribute mask");

const char *kernel_name(int kid)
{
    switch (kid) {
    case KID_BF16_128: return "tc-bf16-128x128";
    case KID_BF16_256: return "tc-bf16-128x256";
    case KID_F16_128: return "tc-f16-128x128";
    case KID_F16_256: return "tc-f16-128x256";
    case KID_TF32_128: return "tc-tf32-128x128";
    case KID_TF32_256: return "tc-tf32-128x256";
    case KID_F32X3_128: return "tc-3xtf32-128x128";
    case KID_BF16_PAIR: return "tc2-bf16-256x256";
    case KID_F16_PAIR: return "tc2-f16-256x256";
    case KID_BF16_WIDE: return "tc2-bf16-256x512";
    case KID_F16_WIDE: return "tc2-f16-256x512";
    case KID_F64_DMMA: return "dmma-f64-128x128";
    case KID_F32X3_PAIR: return "tc2-3xtf32-256x256";
    case KID_F32X3_TPAIR: return "tc2-3xtf32-tmem-256x256";
    case KID_TF32_PAIR: return "tc2-tf32-256x256";
    case KID_MIX_A_PAIR: return "tc2-f32xbf16-bf16x3-256x256";
    case KID_MIX_B_PAIR: return "tc2-bf16xf32-bf16x3-256x256";
    case KID_MIX_A: return "tc-f32xbf16-bf16x3-128x128";
    case KID_MIX_B: return "tc-bf16xf32-bf16x3-128x128";
    case KID_BF16_F32: return "tc-bf16-f32out-128x128";
    case KID_F16_F32: return "tc-f16-f32out-128x128";
    default: return "tc-unknown";
    }
}

// Tuning algorithm ids (cuda_blas_tune_matmul) -> kernel ids.
int algorithm_kernel(int algo)
{
    switch (algo) {
    case 1: return KID_F32X3_128;
    case 2: return KID_TF32_128;
    case 3: return KID_TF32_256;
    default: return -1;
    }
}

template <int IN, int BN, int OUT>
cudaError_t launch_tc_kernel(DeviceState *ds, int kid, const CUtensorMap &ma,
                             const CUtensorMap &mb, const CUtensorMap &mc, TcParams &p,
                             cudaStream_t stream)
{
    using Cfg = TcConfig<IN, BN, OUT>;
    auto kernel = tc_gemm_kernel<IN, BN, OUT>;
    if (!ensure_smem_attr(ds, kid, kernel, Cfg::kSmemBytes))
        return cudaErrorInvalidConfiguration;
    p.status = ds->status;
    // Split-K when the tiles fill less than half of the SMs: the largest G in
    // {4, 2} whose clusters still fit one CTA per SM, leaving every rank at
    // least kSplitMinKBlocks k-blocks and a whole number of epilogue boxes.
    int G = 1;
    if (p.tiles < ds->sms / 2) {
        for (int g : {4, 2}) {
            if (p.tiles * g <= ds->sms && p.k_blocks >= kSplitMinKBlocks * g &&
                (BN / g) % Cfg::kEpiCols == 0) {
                G = g;
                break;
            }
        }
    }
    p.ksplit = G;
    long long grid;
    cudaError_t err;
    grid = G > 1 ? p.tiles * G : std::min<long long>(p.tiles, ds->sms);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(G);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = G > 1 ? 2 : 1;
    err = cudaLaunchKernelEx(&cfg, kernel, ma, mb, mc, p);
    t_last_grid = static_cast<int>(grid);
    t_last_block = Cfg::kThreads;
    t_last_cluster = G;
    return err != cudaSuccess ? err : cudaGetLastError();
}

// Co-resident 2-CTA clusters of a pair kernel (the persistent, unsplit
// launch's grid), queried once per device and kernel slot.
template <typename Cfg, typename Kernel>
int pair_cluster_count(DeviceState *ds, int slot, Kernel kernel, cudaStream_t stream)
{
    int clusters = 0;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        clusters = ds->pair_clusters[slot];
    }
    if (clusters != 0)
        return clusters;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(Cfg::kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(ds->sms & ~1));
    // a failed query must not leave its error for a later launch check
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters < 1) {
        (void)cudaGetLastError();
        clusters = ds->sms / 2;
    }
    std::lock_guard<std::mutex> lock(g_mutex);
    ds->pair_clusters[slot] = clusters;
    return clusters;
}

// Cluster launch of the 2-CTA kernel: at most as many clusters as can be
// co-resident (one CTA per SM), two CTAs each.
template <typename Cfg, typename Kernel>
cudaError_t launch_pair_kernel(DeviceState *ds, int kid, int slot, Kernel kernel,
                               const CUtensorMap &ma, const CUtensorMap &mb,
                               const CUtensorMap &mc, TcParams &p, cudaStream_t stream)
{
    if (!ensure_smem_attr(ds, kid, kernel, Cfg::kSmemBytes))
        return cudaErrorInvalidConfiguration;
    // split-K (2-CTA split kernels only): clusters of G pairs, one tile each
    const int G = p.ksplit > 1 ? p.ksplit : 1;
    p.ksplit = G;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(2 * G);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(Cfg::kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const int clusters = pair_cluster_count<Cfg>(ds, slot, kernel, stream);
    p.status = ds->status;
    const long long n = G > 1 ? p.tiles * G : std::min<long long>(p.tiles, clusters);
    cfg.gridDim = dim3(static_cast<unsigned>(2 * n));
    const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, ma, mb, mc, p);
    t_last_grid = static_cast<int>(2 * n);
    t_last_block = Cfg::kThreads;
    t_last_cluster = 2 * G;
    if (err != cudaSuccess)
        return err;
    return cudaGetLastError();
}

template <int IN, int OUT>
cudaError_t launch_tc2_kernel(DeviceState *ds, int kid, int slot, const CUtensorMap &ma,
                              const CUtensorMap &mb, const CUtensorMap &mc, TcParams &p,
                              cudaStream_t stream)
{
    return launch_pair_kernel<Tc2Config<IN, OUT>>(ds, kid, slot, tc2_gemm_kernel<IN, OUT>, ma, mb,
                                                  mc, p, stream);
}

// Kernels that move registers between their warpgroups (setmaxnreg): an
// increase beyond the CTA's launch allocation (threads x registers per
// thread as compiled) would never complete, so the compiled register count
// is checked before every launch (read once per kernel).
template <typename Cfg, typename Kernel>
bool regs_cover_realloc(Kernel kernel)
{
    static const int regs = [&] {
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess) {
            (void)cudaGetLastError();
            return 0;
        }
        return fa.numRegs;
    }();
    return regs * Cfg::kThreads >= Cfg::kRegsTotal;
}

// The 256 x 512 kernel: register check, then its work items.
template <int IN, int OUT>
cudaError_t launch_wide_kernel(DeviceState *ds, int kid, int slot, const CUtensorMap &ma,
                               const CUtensorMap &mb, const CUtensorMap &mc, TcParams &p,
                               cudaStream_t stream)
{
    using Cfg = Tc2wConfig<IN, OUT>;
    auto kernel = tc2w_gemm_kernel<IN, OUT>;
    if (!regs_cover_realloc<Cfg>(kernel))
        return cudaErrorInvalidConfiguration;
    if (!ensure_smem_attr(ds, kid, kernel, Cfg::kSmemBytes))
        return cudaErrorInvalidConfiguration;
    // Work items: p.tiles holds the 256 x 512 tiles here.  wide_items < 0:
    // whole tiles for every full round of co-resident clusters, the rest as
    // 256-column halves (one more round of half-length items); 0: halves only.
    const long long tiles = p.tiles;
    if (p.wide_items < 0) {
        const long long clusters = pair_cluster_count<Cfg>(ds, slot, kernel, stream);
        p.wide_items = tiles / clusters * clusters;
    } else if (p.wide_items > tiles) {
        p.wide_items = tiles;
    }
    p.tiles = p.wide_items + 2 * (tiles - p.wide_items);
    return launch_pair_kernel<Cfg>(ds, kid, slot, kernel, ma, mb, mc, p, stream);
}

const TunedPlan *find_plan(const Problem &P)
{
    if (P.nbd != 0 || P.nfd != 0 || P.dt != DT_F32 || P.a_dt != DT_F32 || P.b_dt != DT_F32)
        return nullptr;
    for (const TunedPlan &t : t_plans)
        if (t.rows == P.M && t.inner == P.K && t.cols == P.N &&
            t.a_s0 == static_cast<size_t>(P.a_sm) && t.a_s1 == static_cast<size_t>(P.a_sk) &&
            t.b_s0 == static_cast<size_t>(P.b_sk) && t.b_s1 == static_cast<size_t>(P.b_sn) &&
            t.precision == t_precision)
            return &t;
    return nullptr;
}

// Tries the tensor-core kernel.  Returns 1 launched, 0 ineligible, -1 error.
int try_tc(const Problem &P, DeviceState *ds, cudaStream_t stream, int *kid_out)
{
    if (P.dt == DT_F64 || ds->cc_major != 10 || !g_encode)
        return 0;
    // Gradient products with a float32 result from 16-bit operand(s): the
    // MMA runs on the 16-bit type; a float32 operand (mix_side 0 = A, 1 = B)
    // is split into three bf16 parts by the kernel.
    const bool wide_out = P.a_dt != P.dt || P.b_dt != P.dt;
    const int op_dt = !wide_out ? P.dt : (P.a_dt != DT_F32 ? P.a_dt : P.b_dt);
    const int mix_side = !wide_out ? -1 : (P.a_dt == DT_F32 ? 0 : (P.b_dt == DT_F32 ? 1 : -1));
    if (wide_out && (P.K < kStrictMinK || (mix_side >= 0 && op_dt != DT_BF16) ||
                     (mix_side < 0 && P.a_dt != P.b_dt)))
        return 0;
    const int es = element_bytes(op_dt);
    TcBatch tb;
    if (!merge_batches(P, &tb))
        return 0;
    TcFold tf;
    tf.nfd = 0;
    if (P.nfd > 0 && (!merge_folds(P, &tf) || tb.nbd + tf.nfd > 3))
        return 0;
    const bool folded = P.nfd > 0;

    // A: K-major when K is contiguous, M-major for a transposed view.
    int a_mn;
    if (P.a_sk == 1 || P.K == 1)
        a_mn = 0;
    else if (P.a_sm == 1 || P.M == 1)
        a_mn = 1;
    else
        return 0;
    // B: N-major for a row-major B, K-major for a transposed view.
    int b_mn;
    if (P.b_sn == 1 || P.N == 1)
        b_mn = 1;
    else if (P.b_sk == 1 || P.K == 1)
        b_mn = 0;
    else
        return 0;
    if (!(P.c_sn == 1 || P.N == 1))
        return 0;

    // kernel selection
    int kid;
    const bool fp32 = P.dt == DT_F32 && !wide_out;
    // 3xTF32 (hi = the tensor core's truncation, lo rounded to TF32, lo*lo
    // dropped) errs by up to about 32 float32 ulps per product, inside the
    // K-ulp float32 dot-product bound with room to spare only for longer inner
    // axes; shorter ones run the exact-fma CUDA-core kernel.
    if (fp32 && t_precision == CUDA_MATMUL_PRECISION_FP32_STRICT && P.K < kStrictMinK)
        return 0;
    const long long m_blocks = (P.M + 127) / 128;
    int bn = P.forced_bn;
    if (fp32 && t_precision == CUDA_MATMUL_PRECISION_FP32_STRICT) {
        bn = 128;
    } else if (bn == 0) {
        const TunedPlan *plan = fp32 ? find_plan(P) : nullptr;
        if (plan) {
            bn = plan->algorithm == 3 ? 256 : 128;
        } else {
            const long long tiles256 = P.batches * m_blocks * ((P.N + 255) / 256);
            bn = (P.N <= 128 || tiles256 < ds->sms / 2) ? 128 : 256;
        }
    }
    // 16-bit products with enough 256x256 tiles to fill the co-resident
    // clusters run on the 2-CTA kernel (or whenever path 3 asks for it).
    bool pair = false;
    const bool strict = fp32 && t_precision == CUDA_MATMUL_PRECISION_FP32_STRICT;
    const long long tiles_pair = P.batches * ((P.M + 255) / 256) * ((P.N + 255) / 256);
    // 16-bit products and the tf32 precision mode: the 2-CTA kernel once it
    // has at least sms / 4 tiles of 256 x 256.  From there on it runs as
    // many CTAs as the single-CTA 128 x 256 kernel, each streaming a third
    // fewer bytes per FLOP (B200, tf32 4096x1024x1024 with 64 pair tiles:
    // 21.4 against 23.3 us); below it the 128 x 128 tiles fill more SMs.
    if ((!fp32 || !strict) && P.forced_bn == 0)
        pair = t_path == 3 || t_path >= 5 || (t_path != 1 && tiles_pair >= ds->sms / 4);
    if (wide_out || folded)
        bn = wide_out ? 128 : bn, pair = false;
    // Strict float32 and the mixed float32 x bf16 kinds: the 2-CTA split
    // kernel runs a 256 x 256 tile in kPairTileCost single-CTA 128 x 128 tile
    // times (measured on B200), so it is chosen when its rounds of
    // co-resident clusters take less time than the single-CTA kernel's waves
    // (or its split-K launch).
    // A forced pair launch (path 3) with fewer tiles than a quarter of the
    // SMs splits K over clusters of G pairs (G in {4, 2}, each pair keeping at
    // least kSplitMinKBlocks k-blocks).  The automatic choice never takes it:
    // clusters of 4 or 8 CTAs of 230 KB each need that many free SMs in one
    // GPC, and on B200 the config-4 dW products ran 153 us split over 8-CTA
    // clusters against 75 us on the single-CTA split-K kernel.
    const bool mix = mix_side >= 0;
    int pair_g = 1;
    if ((strict || mix) && P.forced_bn == 0) {
        const int bk1 = 128 / es;
        const long long kb1 = static_cast<long long>((P.K + bk1 - 1) / bk1) * P.folds;
        if (2 * tiles_pair < ds->sms / 2) {
            for (int g : {4, 2}) {
                if (2 * tiles_pair * g <= ds->sms && kb1 >= kSplitMinKBlocks * g) {
                    pair_g = g;
                    break;
                }
            }
        }
        if (t_path == 3 || t_path >= 5) {
            pair = true;
        } else if (t_path == 0) {
            const long long tiles1 = P.batches * m_blocks * ((P.N + 127) / 128);
            double t1 = std::ceil(static_cast<double>(tiles1) / ds->sms);
            if (tiles1 < ds->sms / 2) {
                for (int g : {4, 2}) {
                    if (tiles1 * g <= ds->sms && kb1 >= kSplitMinKBlocks * g) {
                        t1 = 1.0 / g;
                        break;
                    }
                }
            }
            const double t2 = std::ceil(static_cast<double>(tiles_pair) / (ds->sms / 2)) *
                              (strict && !a_mn && !folded ? kPairTmemTileCost : kPairTileCost);
            pair = pair_g == 1 && t2 < t1;
        }
    }
    if (pair)
        bn = 256;
    // 16-bit products on the 256 x 512 pair tile: path 5, or automatically
    // when its rounds of co-resident clusters, at kWideTileCost plain pair
    // tiles each, take less time than the plain pair kernel's rounds
    // (the whole tiles of every full round, the rest as 256-column halves,
    // when that costs less than whole tiles throughout)
    const long long tiles_wide = P.batches * ((P.M + 255) / 256) * ((P.N + 511) / 512);
    const long long clusters_est = ds->sms / 2;
    const double rounds_pair = std::ceil(static_cast<double>(tiles_pair) / clusters_est);
    const double cost_wide =
        std::ceil(static_cast<double>(tiles_wide) / clusters_est) * kWideTileCost;
    const long long full_rounds = tiles_wide / clusters_est;
    const double cost_mixed =
        full_rounds * kWideTileCost +
        std::ceil(2.0 * static_cast<double>(tiles_wide - full_rounds * clusters_est) /
                  clusters_est);
    // (the kernels that move registers between warpgroups are taken only
    // when their compiled register count covers the move; otherwise the
    // earlier kernel of the same kind runs)
    const bool wide = pair && !fp32 && !wide_out && !folded && P.forced_bn == 0 &&
                      (t_path == 5 || t_path == 6 ||
                       (t_path == 0 && P.K >= kWideMinK &&
                        std::min(cost_wide, cost_mixed) < rounds_pair)) &&
                      (P.dt == DT_BF16
                           ? regs_cover_realloc<Tc2wConfig<IN_BF16, OUT_BF16>>(
                                 tc2w_gemm_kernel<IN_BF16, OUT_BF16>)
                           : regs_cover_realloc<Tc2wConfig<IN_F16, OUT_F16>>(
                                 tc2w_gemm_kernel<IN_F16, OUT_F16>));
    const long long wide_items =
        t_path == 6 ? 0 : (t_path == 0 && cost_mixed < cost_wide) ? -1 : tiles_wide;
    if (wide_out)
        kid = mix_side == 0   ? (pair ? KID_MIX_A_PAIR : KID_MIX_A)
              : mix_side == 1 ? (pair ? KID_MIX_B_PAIR : KID_MIX_B)
                              : (op_dt == DT_BF16 ? KID_BF16_F32 : KID_F16_F32);
    else if (fp32)
        // the pair kernel with A in tensor memory takes K-major A without
        // split-K or summed batch axes
        kid = strict ? (pair ? (!a_mn && pair_g == 1 && !folded &&
                                        regs_cover_realloc<Tc2tConfig>(tc2t_gemm_kernel)
                                    ? KID_F32X3_TPAIR
                                    : KID_F32X3_PAIR)
                             : KID_F32X3_128)
                     : (pair ? KID_TF32_PAIR : (bn == 256 ? KID_TF32_256 : KID_TF32_128));
    else if (P.dt == DT_BF16)
        kid = wide   ? KID_BF16_WIDE
              : pair ? KID_BF16_PAIR
                     : (bn == 256 ? KID_BF16_256 : KID_BF16_128);
    else
        kid = wide   ? KID_F16_WIDE
              : pair ? KID_F16_PAIR
                     : (bn == 256 ? KID_F16_256 : KID_F16_128);

    const int bk = 128 / es;            // K elements per stage
    const int chunk = 128 / es;         // MN elements per 128-byte row
    const int out_es = P.dt == DT_F32 ? 4 : 2;
    const int epi_cols = 128 / out_es;

    TcParams p;
    std::memset(&p, 0, sizeof(p));
    MapDims ma, mb, mc;
    uint32_t box_a[5] = {1, 1, 1, 1, 1}, box_b[5] = {1, 1, 1, 1, 1}, box_c[5] = {1, 1, 1, 1, 1};
    if (!a_mn) {
        ma.ext[0] = P.K; ma.stride[0] = 1;
        ma.ext[1] = P.M; ma.stride[1] = P.a_sm;
        box_a[0] = bk; box_a[1] = 128;
    } else {
        ma.ext[0] = P.M; ma.stride[0] = 1;
        ma.ext[1] = P.K; ma.stride[1] = P.a_sk;
        box_a[0] = chunk; box_a[1] = bk;
    }
    ma.rank = 2;
    if (b_mn) {
        mb.ext[0] = P.N; mb.stride[0] = 1;
        mb.ext[1] = P.K; mb.stride[1] = P.b_sk;
        box_b[0] = chunk; box_b[1] = bk;
    } else {
        mb.ext[0] = P.K; mb.stride[0] = 1;
        mb.ext[1] = P.N; mb.stride[1] = P.b_sn;
        box_b[0] = bk; box_b[1] = pair ? bn / 2 : bn;   // each CTA of a pair loads half of N
    }
    mb.rank = 2;
    mc.ext[0] = P.N; mc.stride[0] = 1;
    mc.ext[1] = P.M; mc.stride[1] = P.c_sm;
    mc.rank = 2;
    box_c[0] = epi_cols; box_c[1] = 32;
    int c_slot[3];
    add_batch_dims(ma, tb, tb.a, p.a_slot);
    add_batch_dims(mb, tb, tb.b, p.b_slot);
    add_batch_dims(mc, tb, tb.c, c_slot);
    add_fold_dims(ma, tf, tf.a, p.a_fslot);
    add_fold_dims(mb, tf, tf.b, p.b_fslot);

    // TF32 operands stored MN-major need the 32-byte-atom 128-byte swizzle
    CUtensorMapSwizzle sw_a = (fp32 && a_mn) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                             : CU_TENSOR_MAP_SWIZZLE_128B;
    CUtensorMapSwizzle sw_b = (fp32 && b_mn) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                             : CU_TENSOR_MAP_SWIZZLE_128B;
    // The float32 operand of a mixed product lands as one unswizzled box of
    // 128 rows (or columns) x bk K: the kernel's split warps read it.
    if (mix_side == 0) {
        sw_a = CU_TENSOR_MAP_SWIZZLE_NONE;
        if (!a_mn) { box_a[0] = bk; box_a[1] = 128; } else { box_a[0] = 128; box_a[1] = bk; }
    } else if (mix_side == 1) {
        sw_b = CU_TENSOR_MAP_SWIZZLE_NONE;
        if (!b_mn) { box_b[0] = bk; box_b[1] = 128; } else { box_b[0] = 128; box_b[1] = bk; }
    }
    CUtensorMap tma_a, tma_b, tma_c;
    if (!encode_map(&tma_a, P.a_dt, P.a, ma, box_a, sw_a) ||
        !encode_map(&tma_b, P.b_dt, P.b, mb, box_b, sw_b) ||
        !encode_map(&tma_c, P.dt, P.c, mc, box_c))
        return 0;

    p.M = P.M;
    p.N = P.N;
    p.K = P.K;
    p.m_blocks = static_cast<int>(pair ? (P.M + 255) / 256 : m_blocks);
    p.n_blocks = (P.N + (wide ? 2 * bn : bn) - 1) / (wide ? 2 * bn : bn);
    p.k_per_fold = (P.K + bk - 1) / bk;
    if (static_cast<double>(p.k_per_fold) * P.folds > 2e9)
        return 0;
    p.k_blocks = static_cast<int>(p.k_per_fold * P.folds);
    p.nfd = tf.nfd;
    for (int d = 0; d < 3; d++)
        p.fshape[d] = tf.fshape[d];
    p.tiles = P.batches * p.m_blocks * p.n_blocks;
    p.wide_items = wide ? wide_items : 0;
    p.nbd = tb.nbd;
    for (int d = 0; d < 3; d++)
        p.bshape[d] = tb.bshape[d];
    p.a_mn_major = a_mn;
    p.b_mn_major = b_mn;
    const int fmt = fp32 ? 2 : (op_dt == DT_BF16 ? 1 : 0);
    p.idesc = make_idesc(fmt, a_mn, b_mn, bn, pair ? 256 : 128);
    p.bias = P.bias;
    p.act = P.act;
    p.ksplit = pair ? pair_g : 1;

    cudaError_t err;
    switch (kid) {
    case KID_BF16_128: err = launch_tc_kernel<IN_BF16, 128, OUT_BF16>(ds, kid, tma_a, tma_b, tma_c, p, stream); break;
    case KID_BF16_256: err = launch_tc_kernel<IN_BF16, 256, OUT_BF16>(ds, kid, tma_a, tma_b, tma_c, p, stream); break;
    case KID_F16_128: err = launch_tc_kernel<IN_F16, 128, OUT_F16>(ds, kid, tma_a, tma_b, tma_c, p, stream); break;
    case KID_F16_256: err = launch_tc_kernel<IN_F16, 256, OUT_F16>(ds, kid, tma_a, tma_b, tma_c, p, stream); break;
    case KID_TF32_128: err = launch_tc_kernel<IN_TF32, 128, OUT_F32>(ds, kid, tma_a, tma_b, tma_c, p, stream); break;
    case KID_TF32_256: err = launch_tc_kernel<IN_TF32, 256, OUT_F32>(ds, kid, tma_a, tma_b, tma_c, p, stream); break;
    case KID_BF16_PAIR: err = launch_tc2_kernel<IN_BF16, OUT_BF16>(ds, kid, 0, tma_a, tma_b, tma_c, p, stream); break;
    case KID_F16_PAIR: err = launch_tc2_kernel<IN_F16, OUT_F16>(ds, kid, 1, tma_a, tma_b, tma_c, p, stream); break;
    case KID_TF32_PAIR: err = launch_tc2_kernel<IN_TF32, OUT_F32>(ds, kid, 3, tma_a, tma_b, tma_c, p, stream); break;
    case KID_BF16_WIDE:
        err = launch_wide_kernel<IN_BF16, OUT_BF16>(ds, kid, 6, tma_a, tma_b, tma_c, p, stream);
        break;
    case KID_F16_WIDE:
        err = launch_wide_kernel<IN_F16, OUT_F16>(ds, kid, 7, tma_a, tma_b, tma_c, p, stream);
        break;
    case KID_F32X3_TPAIR:
        err = regs_cover_realloc<Tc2tConfig>(tc2t_gemm_kernel)
                  ? launch_pair_kernel<Tc2tConfig>(ds, kid, 8, tc2t_gemm_kernel, tma_a, tma_b,
                                                   tma_c, p, stream)
                  : cudaErrorInvalidConfiguration;
        break;
    case KID_F32X3_PAIR:
        err = launch_pair_kernel<Tc2x3Config<IN_F32X3, kPairChunkKB>>(
            ds, kid, 2, tc2x3_gemm_kernel<IN_F32X3, kPairChunkKB>, tma_a, tma_b, tma_c, p, stream);
        break;
    case KID_MIX_A_PAIR:
        err = launch_pair_kernel<Tc2x3Config<IN_MIX_A, kMixPairChunkKB>>(
            ds, kid, 4, tc2x3_gemm_kernel<IN_MIX_A, kMixPairChunkKB>, tma_a, tma_b, tma_c, p, stream);
        break;
    case KID_MIX_B_PAIR:
        err = launch_pair_kernel<Tc2x3Config<IN_MIX_B, kMixPairChunkKB>>(
            ds, kid, 5, tc2x3_gemm_kernel<IN_MIX_B, kMixPairChunkKB>, tma_a, tma_b, tma_c, p, stream);
        break;
    case KID_MIX_A: err = launch_tc_kernel<IN_MIX_A, 128, OUT_F32>(ds, kid, tma_a, tma_b, tma_c, p, stream); break;
    case KID_MIX_B: err = launch_tc_kernel<IN_MIX_B, 128, OUT_F32>(ds, kid, tma_a, tma_b, tma_c, p, stream); break;
    case KID_BF16_F32: err = launch_tc_kernel<IN_BF16, 128, OUT_F32>(ds, kid, tma_a, tma_b, tma_c, p, stream); break;
    case KID_F16_F32: err = launch_tc_kernel<IN_F16, 128, OUT_F32>(ds, kid, tma_a, tma_b, tma_c, p, stream); break;
    default: err = launch_tc_kernel<IN_F32X3, 128, OUT_F32>(ds, kid, tma_a, tma_b, tma_c, p, stream); break;
    }
    if (err != cudaSuccess) {
        set_status(static_cast<int>(err));
        return -1;
    }
    *kid_out = kid;
    return 1;
}

SimtParams simt_params(const Problem &P);

bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// FP64 on the DMMA pipe.  16-byte cp.async copies need a contiguous inner
// axis, an even extent along it, and even (16-byte) strides everywhere else.
cudaError_t launch_f64_dmma(const Problem &P, DeviceState *ds, cudaStream_t stream)
{
    const SimtParams s = simt_params(P);
    bool a_vec = P.a_sk == 1 && P.K % 2 == 0 && (P.a_sm % 2 == 0 || P.M == 1) && aligned16(P.a);
    bool b_vec = P.b_sn == 1 && P.N % 2 == 0 && (P.b_sk % 2 == 0 || P.K == 1) && aligned16(P.b);
    for (int d = 0; d < P.nbd; d++) {
        a_vec = a_vec && P.a_bs[d] % 2 == 0;
        b_vec = b_vec && P.b_bs[d] % 2 == 0;
    }
    if (!ensure_smem_attr(ds, KID_F64_DMMA, f64_dmma_kernel<false>, kF64SmemBytes) ||
        !ensure_smem_attr(ds, KID_F64_DMMA_HALF, f64_dmma_half_kernel<false>, kF64SmemBytes))
        return cudaErrorInvalidConfiguration;
    F64PeerOut none;
    std::memset(&none, 0, sizeof(none));
    // full tiles, one resident CTA per SM; then -- when the last wave would
    // be at most half full -- its tiles as half tiles in a second launch
    const F64Work w = f64_work(P.M, P.N, P.batches, ds->sms);
    if (w.full > 0) {
        dim3 grid(static_cast<unsigned>(w.n_blocks),
                  static_cast<unsigned>(std::min<long long>(w.m_blocks, 65535)),
                  static_cast<unsigned>(std::min<long long>(P.batches, 65535)));
        f64_dmma_kernel<false><<<grid, 256, kF64SmemBytes, stream>>>(s, a_vec ? 1 : 0,
                                                                     b_vec ? 1 : 0, w, none);
    }
    if (w.tail > 0)
        f64_dmma_half_kernel<false><<<static_cast<unsigned>(2 * w.tail), 256, kF64SmemBytes,
                                      stream>>>(s, a_vec ? 1 : 0, b_vec ? 1 : 0, w, none);
    return cudaGetLastError();
}

SimtParams simt_params(const Problem &P)
{
    SimtParams s;
    std::memset(&s, 0, sizeof(s));
    s.a = P.a;
    s.b = P.b;
    s.c = P.c;
    s.M = P.M;
    s.N = P.N;
    s.K = P.K;
    s.batches = P.batches;
    s.nbd = P.nbd;
    for (int d = 0; d < P.nbd; d++) {
        s.bshape[d] = P.bshape[d];
        s.a_bs[d] = P.a_bs[d];
        s.b_bs[d] = P.b_bs[d];
        s.c_bs[d] = P.c_bs[d];
    }
    s.a_sm = P.a_sm;
    s.a_sk = P.a_sk;
    s.b_sk = P.b_sk;
    s.b_sn = P.b_sn;
    s.c_sm = P.c_sm;
    s.c_sn = P.c_sn;
    s.bias = P.bias;
    s.act = P.act;
    s.nfd = P.nfd;
    s.folds = P.folds;
    for (int d = 0; d < P.nfd; d++) {
        s.fshape[d] = P.fshape[d];
        s.a_fs[d] = P.a_fs[d];
        s.b_fs[d] = P.b_fs[d];
    }
    return s;
}

template <typename T, typename TA = T, typename TB = T>
cudaError_t launch_simt(const Problem &P, cudaStream_t stream)
{
    const SimtParams s = simt_params(P);
    const long long mb = (P.M + kSimtTile - 1) / kSimtTile;
    const long long nb = (P.N + kSimtTile - 1) / kSimtTile;
    dim3 grid(static_cast<unsigned>(std::min<long long>(nb, 2147483647ll)),
              static_cast<unsigned>(std::min<long long>(mb, 65535)),
              static_cast<unsigned>(std::min<long long>(P.batches, 65535)));
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, simt_gemm_kernel<T, TA, TB>, s);
    return err != cudaSuccess ? err : cudaGetLastError();
}

// Few-column products (N <= 32) on the split-K CUDA-core kernel.  The
// cluster size C (1, 2, 4 or 8 CTAs splitting K) is the smallest that puts
// about 1.5 CTAs on every SM while each CTA keeps at least four chunks.
template <typename T, int NB, typename TA = T, typename TB = T>
cudaError_t launch_skinny_nb(const Problem &P, DeviceState *ds, cudaStream_t stream)
{
    const SimtParams s = simt_params(P);
    SkinnyArgs sa;
    sa.a_k_major = P.a_sk == 1 && P.a_sm != 1 ? 1 : 0;
    sa.b_n_major = P.b_sn == 1 ? 1 : 0;
    const long long m_blocks = (P.M + kSkinnyBM - 1) / kSkinnyBM;
    const long long zb = std::min<long long>(P.batches, 65535);
    const long long chunks = (P.K + kSkinnyKC - 1) / kSkinnyKC;
    // about 1.5 CTAs per SM: measured on B200 (graph-timed, N = 10) the
    // best split for 128 row blocks is C = 2 (11.3 us; C = 8: 14.3), for 32
    // row blocks C = 8 (11.0 us; C = 2: 20.2), for 2048 row blocks C = 1
    const long long target = 3ll * ds->sms / 2;
    int C = 1;
    while (C < kSkinnyMaxCluster && m_blocks * zb * C < target && chunks / (2 * C) >= 4)
        C *= 2;
    sa.cluster = C;
    const long long xc = std::min<long long>(m_blocks, 1 << 20);
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(xc * C), 1, static_cast<unsigned>(zb));
    cfg.blockDim = dim3(kSkinnyThreads, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(C);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = C > 1 ? 2 : 1;
    cudaError_t err;
    // float32 A in 16-byte copies: 16-byte aligned base, the non-contiguous
    // axes (the other matrix axis and the batch axes) in multiples of four
    bool a_vec = sizeof(T) == 4 && aligned16(P.a) &&
                 (sa.a_k_major ? (P.a_sm % 4 == 0 || P.M == 1) : (P.a_sm == 1 && P.a_sk % 4 == 0));
    for (int d = 0; d < P.nbd; d++)
        a_vec = a_vec && P.a_bs[d] % 4 == 0;
    if constexpr (sizeof(T) == 4 && std::is_same<T, TA>::value && std::is_same<T, TB>::value) {
        if (a_vec) {
            constexpr int smem = skinny_async_smem_bytes<T, NB, true>();
            const int base = KID_SKINNY_VEC + 2 * (NB <= 16 ? NB / 4 - 1 : NB == 24 ? 4 : 5);
            cfg.dynamicSmemBytes = smem;
            if (sa.a_k_major) {
                if (!ensure_smem_attr(ds, base + 1, skinny_async_kernel<T, NB, true, true>, smem))
                    return cudaErrorInvalidConfiguration;
                err = cudaLaunchKernelEx(&cfg, skinny_async_kernel<T, NB, true, true>, s, sa);
            } else {
                if (!ensure_smem_attr(ds, base, skinny_async_kernel<T, NB, false, true>, smem))
                    return cudaErrorInvalidConfiguration;
                err = cudaLaunchKernelEx(&cfg, skinny_async_kernel<T, NB, false, true>, s, sa);
            }
            t_last_grid = static_cast<int>(xc * C);
            t_last_block = kSkinnyThreads;
            t_last_cluster = C;
            return err != cudaSuccess ? err : cudaGetLastError();
        }
    }
    if constexpr (sizeof(T) >= 4 && std::is_same<T, TA>::value && std::is_same<T, TB>::value) {
        // float32 / float64: the cp.async ring variant
        constexpr int smem = skinny_async_smem_bytes<T, NB>();
        const int base = KID_SKINNY_ASYNC + (sizeof(T) == 8 ? 12 : 0) + 2 * (NB <= 16 ? NB / 4 - 1 : NB == 24 ? 4 : 5);
        cfg.dynamicSmemBytes = smem;
        if (sa.a_k_major) {
            if (!ensure_smem_attr(ds, base + 1, skinny_async_kernel<T, NB, true>, smem))
                return cudaErrorInvalidConfiguration;
            err = cudaLaunchKernelEx(&cfg, skinny_async_kernel<T, NB, true>, s, sa);
        } else {
            if (!ensure_smem_attr(ds, base, skinny_async_kernel<T, NB, false>, smem))
                return cudaErrorInvalidConfiguration;
            err = cudaLaunchKernelEx(&cfg, skinny_async_kernel<T, NB, false>, s, sa);
        }
    } else {
        err = cudaLaunchKernelEx(&cfg, skinny_gemm_kernel<T, NB, TA, TB>, s, sa);
    }
    t_last_grid = static_cast<int>(xc * C);
    t_last_block = kSkinnyThreads;
    t_last_cluster = C;
    return err != cudaSuccess ? err : cudaGetLastError();
}

// Mixed operand types (float32 result): the register-staged kernel, whose
// warp layout needs a power-of-two NB.
template <typename TA, typename TB>
cudaError_t launch_skinny_mixed(const Problem &P, DeviceState *ds, cudaStream_t stream)
{
    if (P.N <= 4) return launch_skinny_nb<float, 4, TA, TB>(P, ds, stream);
    if (P.N <= 8) return launch_skinny_nb<float, 8, TA, TB>(P, ds, stream);
    if (P.N <= 16) return launch_skinny_nb<float, 16, TA, TB>(P, ds, stream);
    return launch_skinny_nb<float, 32, TA, TB>(P, ds, stream);
}

// Column padding NB: 4, 8, 12, 16, 24 or 32 for float32/float64; the 16-bit
// kernel's warp layout needs a power of two.
template <typename T>
cudaError_t launch_skinny(const Problem &P, DeviceState *ds, cudaStream_t stream)
{
    if (P.N <= 4) return launch_skinny_nb<T, 4>(P, ds, stream);
    if (P.N <= 8) return launch_skinny_nb<T, 8>(P, ds, stream);
    if constexpr (sizeof(T) >= 4) {
        if (P.N <= 12) return launch_skinny_nb<T, 12>(P, ds, stream);
        if (P.N <= 16) return launch_skinny_nb<T, 16>(P, ds, stream);
        if (P.N <= 24) return launch_skinny_nb<T, 24>(P, ds, stream);
    } else {
        if (P.N <= 16) return launch_skinny_nb<T, 16>(P, ds, stream);
    }
    return launch_skinny_nb<T, 32>(P, ds, stream);
}

const char *family_name(int dt)
{
    switch (dt) {
    case DT_F32: return "builtin";
    case DT_F64: return "builtin-f64";
    default: return "builtin-low-precision";
    }
}

const char *simt_name(int dt)
{
    switch (dt) {
    case DT_F32: return "simt-f32";
    case DT_F64: return "simt-f64";
    case DT_F16: return "simt-f16";
    default: return "simt-bf16";
    }
}

const char *skinny_name(int dt)
{
    switch (dt) {
    case DT_F32: return "skinny-f32";
    case DT_F64: return "skinny-f64";
    case DT_F16: return "skinny-f16";
    default: return "skinny-bf16";
    }
}

// The few-column kernel.  The automatic choice takes it for float32 and
// float64 whenever N <= 32 and K >= 128 (ahead of 128-column tensor-core
// tiles that would be three-quarters empty and of the 3xTF32 / DMMA rates),
// and for float16/bfloat16 only where the tensor-core kernel cannot describe
// the layout: at full tensor-core rate even a mostly empty tile is faster
// than the CUDA cores.
int run_skinny(const Problem &P, DeviceState *ds, cudaStream_t stream)
{
    cudaError_t err;
    if (P.a_dt != P.dt || P.b_dt != P.dt) {
        auto code = [](int dt) { return dt == DT_F32 ? 0 : (dt == DT_BF16 ? 1 : 2); };
        switch (code(P.a_dt) * 3 + code(P.b_dt)) {
        case 1: err = launch_skinny_mixed<float, __nv_bfloat16>(P, ds, stream); break;
        case 2: err = launch_skinny_mixed<float, __half>(P, ds, stream); break;
        case 3: err = launch_skinny_mixed<__nv_bfloat16, float>(P, ds, stream); break;
        case 4: err = launch_skinny_mixed<__nv_bfloat16, __nv_bfloat16>(P, ds, stream); break;
        case 6: err = launch_skinny_mixed<__half, float>(P, ds, stream); break;
        case 8: err = launch_skinny_mixed<__half, __half>(P, ds, stream); break;
        default: err = cudaErrorInvalidValue; break;
        }
    } else switch (P.dt) {
    case DT_F32: err = launch_skinny<float>(P, ds, stream); break;
    case DT_F64: err = launch_skinny<double>(P, ds, stream); break;
    case DT_F16: err = launch_skinny<__half>(P, ds, stream); break;
    default: err = launch_skinny<__nv_bfloat16>(P, ds, stream); break;
    }
    if (err != cudaSuccess) {
        set_status(static_cast<int>(err));
        return 0;
    }
    t_info.builtin_matmul_calls++;
    t_info.last_matmul = family_name(P.dt);
    t_info.last_blas_status = 0;
    t_last_kernel = skinny_name(P.dt);
    return 1;
}

int run(Problem &P, cudaStream_t stream)
{
    DeviceState *ds = device_state();
    if (!ds) {
        set_status(GEMM_SM100_STATUS_NO_DEVICE);
        return 0;
    }
    if (P.nbd > kMaxBatchDims) {
        return 0;
    }
    const double work =
        static_cast<double>(P.M) * P.N * P.K * static_cast<double>(P.batches) * P.folds;
    const bool want_tc = P.K > 0 && P.folds > 0 && t_path != 2 &&
                         (t_path == 1 || t_path == 3 || t_path >= 5 || work >= kTcMinWork);
    const bool wide_out = P.a_dt != P.dt || P.b_dt != P.dt;   // float32 result, 16-bit operand(s)
    const bool folded = P.nfd > 0 || P.folds != 1;             // summed batch axes
    const bool skinny_fit = !folded && P.N > 0 && P.N <= kSkinnyMaxN && P.M > 0 &&
                            P.batches > 0 && P.K >= kSkinnyMinK;
    // float32 / float64 results, mixed-type gradient products included
    const bool wide_acc = P.dt == DT_F32 || P.dt == DT_F64;
    if (skinny_fit && (t_path == 4 || (t_path == 0 && wide_acc)))
        return run_skinny(P, ds, stream);
    if (want_tc && !folded && P.dt == DT_F64 && ds->cc_major == 10) {
        const cudaError_t err = launch_f64_dmma(P, ds, stream);
        if (err != cudaSuccess) {
            set_status(static_cast<int>(err));
            return 0;
        }
        t_info.builtin_matmul_calls++;
        t_info.last_matmul = family_name(P.dt);
        t_info.last_blas_status = 0;
        t_last_kernel = kernel_name(KID_F64_DMMA);
        return 1;
    }
    if (want_tc) {
        int kid = -1;
        const int r = try_tc(P, ds, stream, &kid);
        if (r < 0)
            return 0;
        if (r == 1) {
            t_info.builtin_matmul_calls++;
            t_info.last_matmul = family_name(P.dt);
            t_info.last_blas_status = 0;
            t_last_kernel = kernel_name(kid);
            return 1;
        }
    }
    if (skinny_fit && t_path == 0)
        return run_skinny(P, ds, stream);   // 16-bit layouts TMA cannot describe
    cudaError_t err;
    if (wide_out) {
        // float32 result: each operand widened to float on load
        auto code = [](int dt) { return dt == DT_F32 ? 0 : (dt == DT_BF16 ? 1 : 2); };
        switch (code(P.a_dt) * 3 + code(P.b_dt)) {
        case 1: err = launch_simt<float, float, __nv_bfloat16>(P, stream); break;
        case 2: err = launch_simt<float, float, __half>(P, stream); break;
        case 3: err = launch_simt<float, __nv_bfloat16, float>(P, stream); break;
        case 4: err = launch_simt<float, __nv_bfloat16, __nv_bfloat16>(P, stream); break;
        case 6: err = launch_simt<float, __half, float>(P, stream); break;
        case 8: err = launch_simt<float, __half, __half>(P, stream); break;
        default: err = cudaErrorInvalidValue; break;
        }
    } else switch (P.dt) {
    case DT_F32: err = launch_simt<float>(P, stream); break;
    case DT_F64: err = launch_simt<double>(P, stream); break;
    case DT_F16: err = launch_simt<__half>(P, stream); break;
    default: err = launch_simt<__nv_bfloat16>(P, stream); break;
    }
    if (err != cudaSuccess) {
        set_status(static_cast<int>(err));
        return 0;
    }
    t_info.builtin_matmul_calls++;
    t_info.last_matmul = family_name(P.dt);
    t_info.last_blas_status = 0;
    t_last_kernel = simt_name(P.dt);
    return 1;
}

int dtype_code(dtype_t dtype)
{
    switch (dtype) {
    case DTYPE_FLOAT32: return DT_F32;
    case DTYPE_FLOAT64: return DT_F64;
    case DTYPE_FLOAT16: return DT_F16;
    case DTYPE_BFLOAT16: return DT_BF16;
    default: return -1;
    }
}

int nd_entry(int dt, const void *a, const void *b, void *c, int *shape_a, size_t *stride_a,
             int nd_a, int *shape_b, size_t *stride_b, int nd_b, int *shape_c, size_t *stride_c,
             int nd_c, const void *bias, int act, cudaStream_t stream)
{
    Problem P;
    const int v = build_problem(dt, a, b, c, shape_a, stride_a, nd_a, shape_b, stride_b, nd_b,
                                shape_c, stride_c, nd_c, &P);
    if (v == 0)
        return 0;
    if (v == 2)
        return 1;
    P.bias = bias;
    P.act = act;
    return run(P, stream);
}

} // namespace

namespace {

// Failure-detection self-test: one warp waits, with the kernels' bounded
// mbar_wait, on a barrier that nothing ever completes; the wait gives up
// after its time limit and the kernel records DEV_TIMEOUT_SELFTEST.
__global__ void wait_selftest_kernel(int *status)
{
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncwarp();
    const bool got = __all_sync(0xffffffffu, mbar_wait(&bar, 0, &abort_flag));
    if (!got && threadIdx.x == 0)
        record_failure(&abort_flag, status, DEV_TIMEOUT_SELFTEST);
}

} // namespace

// Internal (hidden) hook for the other translation units of the library.
void ptg_set_last_status(int code) { set_status(code); }

// Internal (hidden, declared in internal.h), used by csrc/mgpu.cu.
cudaError_t ptg_launch_f64_peer(const double *a, size_t a_s0, size_t a_s1, const double *b,
                                size_t b_s0, size_t b_s1, int M, int nb, int K,
                                const F64PeerOut &po, cudaStream_t stream)
{
    DeviceState *ds = device_state();
    if (!ds)
        return cudaErrorNoDevice;
    int sa[2] = {M, K}, sb[2] = {K, nb}, sc[2] = {M, nb};
    size_t ta[2] = {a_s0, a_s1}, tb[2] = {b_s0, b_s1}, tc[2] = {static_cast<size_t>(nb), 1};
    Problem P;
    const int v = build_problem(DT_F64, a, b, po.dst[0], sa, ta, 2, sb, tb, 2, sc, tc, 2, &P);
    if (v == 0)
        return cudaErrorInvalidValue;
    if (v == 2)
        return cudaSuccess;
    const SimtParams s = simt_params(P);
    const bool a_vec = P.a_sk == 1 && P.K % 2 == 0 && (P.a_sm % 2 == 0 || P.M == 1) &&
                       reinterpret_cast<uintptr_t>(a) % 16 == 0;
    const bool b_vec = P.b_sn == 1 && P.N % 2 == 0 && (P.b_sk % 2 == 0 || P.K == 1) &&
                       reinterpret_cast<uintptr_t>(b) % 16 == 0;
    const F64Work w = f64_work(P.M, P.N, 1, ds->sms);
    const bool store = po.exchange == GEMM_MGPU_EXCHANGE_STORE ||
                       (po.exchange == GEMM_MGPU_EXCHANGE_AUTO && po.ndst <= kPeerStoreMaxRanks);
    if (store) {
        // few ranks: each tile's epilogue stores it into every window
        if (!ensure_smem_attr(ds, KID_F64_DMMA_PEER_STORE, f64_dmma_kernel<true>, kF64SmemBytes) ||
            !ensure_smem_attr(ds, KID_F64_DMMA_PEER_HALF, f64_dmma_half_kernel<true>,
                              kF64SmemBytes))
            return cudaErrorInvalidConfiguration;
        if (w.full > 0)
            f64_dmma_kernel<true><<<dim3(static_cast<unsigned>(w.n_blocks),
                                         static_cast<unsigned>(std::min(w.m_blocks, 65535))),
                                    256, kF64SmemBytes, stream>>>(s, a_vec ? 1 : 0, b_vec ? 1 : 0,
                                                                  w, po);
        if (w.tail > 0)
            f64_dmma_half_kernel<true><<<static_cast<unsigned>(2 * w.tail), 256, kF64SmemBytes,
                                         stream>>>(s, a_vec ? 1 : 0, b_vec ? 1 : 0, w, po);
    } else {
        // the remote copies under later tiles' math: per-SM hand-off, then a
        // flush of the tiles the last CTAs left behind
        if (!po.slots || po.nslots < 1 ||
            !ensure_smem_attr(ds, KID_F64_DMMA_PEER, f64_dmma_handoff_kernel<4>, kF64SmemBytes) ||
            !ensure_smem_attr(ds, KID_F64_DMMA_HANDOFF_HALF, f64_dmma_handoff_kernel<2>,
                              kF64SmemBytes))
            return cudaErrorInvalidConfiguration;
        if (w.full > 0)
            f64_dmma_handoff_kernel<4><<<static_cast<unsigned>(w.full), 256, kF64SmemBytes,
                                         stream>>>(s, a_vec ? 1 : 0, b_vec ? 1 : 0, w, po);
        if (w.tail > 0)
            f64_dmma_handoff_kernel<2><<<static_cast<unsigned>(2 * w.tail), 256, kF64SmemBytes,
                                         stream>>>(s, a_vec ? 1 : 0, b_vec ? 1 : 0, w, po);
        f64_handoff_flush_kernel<<<static_cast<unsigned>(po.nslots), 256, 0, stream>>>(s, w, po);
    }
    const cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) {
        t_info.builtin_matmul_calls++;
        t_info.last_matmul = "builtin-f64";
        t_info.last_blas_status = 0;
        t_last_kernel = "dmma-f64-128x128-peer";
    }
    return err;
}

// ============================================================ C ABI

PT_API void cuda_blas_shutdown(void)
{
    t_info = {};
    t_plans.clear();
    t_last_kernel = "none";
}

PT_API int cuda_blas_set_precision(int precision)
{
    if (precision != CUDA_MATMUL_PRECISION_FP32_STRICT && precision != CUDA_MATMUL_PRECISION_TF32)
        return 0;
    t_precision = precision;
    return 1;
}

PT_API const char *cuda_blas_precision_name(void)
{
    return t_precision == CUDA_MATMUL_PRECISION_TF32 ? "tf32" : "fp32-strict";
}

PT_API void cuda_blas_info(cuda_backend_info *info)
{
    if (!info)
        return;
    info->cublas = 0;
    info->cublas_lt = 0;
    info->blas_calls = t_info.blas_calls;
    info->lt_calls = t_info.lt_calls;
    info->builtin_matmul_calls = t_info.builtin_matmul_calls;
    info->last_matmul = t_info.last_matmul ? t_info.last_matmul : "none";
    info->last_blas_status = t_info.last_blas_status;
    info->precision = cuda_blas_precision_name();
}

PT_API int cuda_matmul_launcher(float *a, float *b, float *c, int m, int n, int k,
                                size_t a_stride0, size_t a_stride1, size_t b_stride0,
                                size_t b_stride1, size_t c_stride0, size_t c_stride1,
                                cudaStream_t stream)
{
    // reference argument naming: m = rows, n = inner, k = cols
    if (m < 0 || n < 0 || k < 0)
        return 0;
    if (!m || !k)
        return 1;
    int shape_a[2] = {m, n}, shape_b[2] = {n, k}, shape_c[2] = {m, k};
    size_t stride_a[2] = {a_stride0, a_stride1}, stride_b[2] = {b_stride0, b_stride1};
    size_t stride_c[2] = {c_stride0, c_stride1};
    return nd_entry(DT_F32, a, b, c, shape_a, stride_a, 2, shape_b, stride_b, 2, shape_c, stride_c,
                    2, nullptr, ACT_NONE, stream);
}

PT_API int cuda_batched_matmul_nd_launcher(float *a, float *b, float *c, int *shape_a,
                                           size_t *stride_a, int nd_a, int *shape_b,
                                           size_t *stride_b, int nd_b, int *shape_c,
                                           size_t *stride_c, int nd_c, cudaStream_t stream)
{
    return nd_entry(DT_F32, a, b, c, shape_a, stride_a, nd_a, shape_b, stride_b, nd_b, shape_c,
                    stride_c, nd_c, nullptr, ACT_NONE, stream);
}

PT_API int cuda_low_precision_matmul_nd_launcher(void *a, void *b, void *c, dtype_t dtype,
                                                 int *shape_a, size_t *stride_a, int nd_a,
                                                 int *shape_b, size_t *stride_b, int nd_b,
                                                 int *shape_c, size_t *stride_c, int nd_c,
                                                 cudaStream_t stream)
{
    if (dtype != DTYPE_FLOAT16 && dtype != DTYPE_BFLOAT16)
        return 0;
    return nd_entry(dtype_code(dtype), a, b, c, shape_a, stride_a, nd_a, shape_b, stride_b, nd_b,
                    shape_c, stride_c, nd_c, nullptr, ACT_NONE, stream);
}

PT_API int cuda_f64_matmul_nd_launcher(double *a, double *b, double *c, int *shape_a,
                                       size_t *stride_a, int nd_a, int *shape_b, size_t *stride_b,
                                       int nd_b, int *shape_c, size_t *stride_c, int nd_c,
                                       cudaStream_t stream)
{
    return nd_entry(DT_F64, a, b, c, shape_a, stride_a, nd_a, shape_b, stride_b, nd_b, shape_c,
                    stride_c, nd_c, nullptr, ACT_NONE, stream);
}

// Internal (hidden, declared in internal.h): float32 C = the sum over C's
// reduced batch axes of A . B (see build_fold_problem), operand types as for
// cuda_mixed_matmul_nd_launcher.
int ptg_reduced_matmul(const void *a, int a_dtype, const void *b, int b_dtype, float *c,
                       int *shape_a, size_t *stride_a, int nd_a, int *shape_b, size_t *stride_b,
                       int nd_b, int *shape_c, size_t *stride_c, int nd_c, cudaStream_t stream)
{
    const int da = dtype_code(static_cast<dtype_t>(a_dtype));
    const int db = dtype_code(static_cast<dtype_t>(b_dtype));
    if (da < 0 || db < 0 || da == DT_F64 || db == DT_F64 ||
        (da != DT_F32 && db != DT_F32 && da != db))
        return 0;
    Problem P;
    const int v = build_fold_problem(DT_F32, a, b, c, shape_a, stride_a, nd_a, shape_b, stride_b,
                                     nd_b, shape_c, stride_c, nd_c, &P);
    if (v == 0)
        return 0;
    if (v == 2)
        return 1;
    P.a_dt = da;
    P.b_dt = db;
    return run(P, stream);
}

PT_API int cuda_mixed_matmul_nd_launcher(const void *a, dtype_t a_dtype, const void *b,
                                         dtype_t b_dtype, float *c, int *shape_a,
                                         size_t *stride_a, int nd_a, int *shape_b,
                                         size_t *stride_b, int nd_b, int *shape_c,
                                         size_t *stride_c, int nd_c, cudaStream_t stream)
{
    const int da = dtype_code(a_dtype), db = dtype_code(b_dtype);
    if (da < 0 || db < 0 || da == DT_F64 || db == DT_F64)
        return 0;
    // at most one 16-bit type: float16 and bfloat16 do not meet in one product
    if (da != DT_F32 && db != DT_F32 && da != db)
        return 0;
    Problem P;
    const int v = build_problem(DT_F32, a, b, c, shape_a, stride_a, nd_a, shape_b, stride_b,
                                nd_b, shape_c, stride_c, nd_c, &P);
    if (v == 0)
        return 0;
    if (v == 2)
        return 1;
    P.a_dt = da;
    P.b_dt = db;
    return run(P, stream);
}

PT_API int cuda_matmul_epilogue_nd_launcher(void *a, void *b, void *c, dtype_t dtype,
                                            int *shape_a, size_t *stride_a, int nd_a,
                                            int *shape_b, size_t *stride_b, int nd_b,
                                            int *shape_c, size_t *stride_c, int nd_c,
                                            const void *bias, int activation, cudaStream_t stream)
{
    const int dt = dtype_code(dtype);
    if (dt < 0 || activation < CUDA_MATMUL_EPILOGUE_NONE ||
        activation > CUDA_MATMUL_EPILOGUE_SIGMOID)
        return 0;
    return nd_entry(dt, a, b, c, shape_a, stride_a, nd_a, shape_b, stride_b, nd_b, shape_c,
                    stride_c, nd_c, bias, activation, stream);
}

PT_API int cuda_blas_tune_matmul(float *a, float *b, float *c, int rows, int inner, int cols,
                                 size_t a_stride0, size_t a_stride1, size_t b_stride0,
                                 size_t b_stride1, cudaStream_t stream,
                                 cuda_matmul_tuning_result *result)
{
    if (!a || !b || !c || !result || rows <= 0 || inner <= 0 || cols <= 0 ||
        static_cast<double>(rows) * inner * cols < kTuneMinWork)
        return 0;
    int shape_a[2] = {rows, inner}, shape_b[2] = {inner, cols}, shape_c[2] = {rows, cols};
    size_t stride_a[2] = {a_stride0, a_stride1}, stride_b[2] = {b_stride0, b_stride1};
    size_t stride_c[2] = {static_cast<size_t>(cols), 1};
    Problem P;
    if (build_problem(DT_F32, a, b, c, shape_a, stride_a, 2, shape_b, stride_b, 2, shape_c,
                      stride_c, 2, &P) != 1)
        return 0;
    DeviceState *ds = device_state();
    if (!ds)
        return -1;

    const int strict_algos[] = {1};
    const int tf32_algos[] = {2, 3};
    const int *algos = t_precision == CUDA_MATMUL_PRECISION_TF32 ? tf32_algos : strict_algos;
    const int n_algos = t_precision == CUDA_MATMUL_PRECISION_TF32 ? 2 : 1;

    cudaEvent_t start = nullptr, stop = nullptr;
    if (cudaEventCreate(&start) != cudaSuccess || cudaEventCreate(&stop) != cudaSuccess) {
        if (start) cudaEventDestroy(start);
        return -1;
    }
    cuda_matmul_tuning_result measured = {};
    measured.selected_candidate = -1;
    int best_algo = -1;
    double best_ms = 0.0;
    int rc = 1;
    for (int i = 0; i < n_algos && rc == 1; i++) {
        const int algo = algos[i];
        const int kid = algorithm_kernel(algo);
        P.forced_bn = (kid == KID_TF32_256) ? 256 : 128;
        constexpr int kWarmups = 2, kSamples = 5;   // matmul_kernels.cu:373-374
        float times[kSamples];
        bool eligible = true;
        for (int s = -kWarmups; s < kSamples; s++) {
            if (s >= 0 && cudaEventRecord(start, stream) != cudaSuccess) { rc = -1; break; }
            int launched = -1;
            const int r = try_tc(P, ds, stream, &launched);
            if (r < 0) { rc = -1; break; }
            if (r == 0) { eligible = false; break; }
            if (s >= 0) {
                if (cudaEventRecord(stop, stream) != cudaSuccess ||
                    cudaEventSynchronize(stop) != cudaSuccess ||
                    cudaEventElapsedTime(&times[s], start, stop) != cudaSuccess) {
                    rc = -1;
                    break;
                }
            }
        }
        if (rc != 1 || !eligible)
            break;
        std::sort(times, times + kSamples);
        const double median = times[kSamples / 2];
        const int idx = measured.candidate_count++;
        measured.candidates[idx].algorithm_id = algo;
        measured.candidates[idx].workspace_bytes = 0;
        measured.candidates[idx].median_ms = median;
        if (best_algo < 0 || median < best_ms) {
            best_ms = median;
            best_algo = algo;
            measured.selected_candidate = idx;
        }
    }
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    if (rc < 0) {
        set_status(static_cast<int>(cudaGetLastError()));
        return -1;
    }
    if (best_algo < 0)
        return 0;

    // pin the winner, replacing an existing plan for the same key
    TunedPlan plan = {rows, inner, cols, a_stride0, a_stride1, b_stride0, b_stride1,
                      t_precision, best_algo};
    for (size_t i = 0; i < t_plans.size(); i++) {
        const TunedPlan &t = t_plans[i];
        if (t.rows == rows && t.inner == inner && t.cols == cols && t.a_s0 == a_stride0 &&
            t.a_s1 == a_stride1 && t.b_s0 == b_stride0 && t.b_s1 == b_stride1 &&
            t.precision == t_precision) {
            t_plans.erase(t_plans.begin() + static_cast<long>(i));
            break;
        }
    }
    if (t_plans.size() >= kMaxTunedPlans)
        t_plans.erase(t_plans.begin());
    t_plans.push_back(plan);
    // leave the product of the selected configuration in c
    P.forced_bn = best_algo == 3 ? 256 : 128;
    int kid = -1;
    if (try_tc(P, ds, stream, &kid) != 1)
        return -1;
    t_info.builtin_matmul_calls++;
    t_info.last_matmul = "builtin";
    t_last_kernel = kernel_name(kid);
    *result = measured;
    return 1;
}

PT_API const char *gemm_sm100_last_kernel(void) { return t_last_kernel; }

PT_API void gemm_sm100_last_launch(int *grid, int *block, int *cluster)
{
    if (grid) *grid = t_last_grid;
    if (block) *block = t_last_block;
    if (cluster) *cluster = t_last_cluster;
}

PT_API int gemm_sm100_set_path(int path)
{
    const int prev = t_path;
    if (path >= 0 && path <= 6)
        t_path = path;
    return prev;
}

PT_API int gemm_sm100_device_status(int device, int clear)
{
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess)
        return -1;
    if (device != prev && cudaSetDevice(device) != cudaSuccess)
        return -1;
    int value = -1;
    if (cudaDeviceSynchronize() == cudaSuccess &&
        cudaMemcpyFromSymbol(&value, g_device_status, sizeof(int)) == cudaSuccess && clear) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)) != cudaSuccess)
            value = -1;
    }
    if (device != prev)
        cudaSetDevice(prev);
    return value;
}

PT_API int gemm_sm100_selftest_wait_timeout(cudaStream_t stream)
{
    DeviceState *ds = device_state();
    if (!ds)
        return 0;
    wait_selftest_kernel<<<1, 32, 0, stream>>>(ds->status);
    return cudaGetLastError() == cudaSuccess ? 1 : 0;
}

PT_API const char *gemm_sm100_algorithm_name(int algorithm_id)
{
    const int kid = algorithm_kernel(algorithm_id);
    return kid < 0 ? "unknown" : kernel_name(kid);
}

PT_API int gemm_sm100_version(void) { return 100; }
