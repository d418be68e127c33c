// Multi-GPU entry points of libgemm_sm100.so (one process per GPU).
//
// The reference has no multi-GPU code; this is new scope.  A single large
// product is split along N: rank r holds all of A and the column block
// B[:, r*N/G, (r+1)*N/G) and computes C[:, block] with the ordinary launchers
// into slot r of a [G][M][N/G] gather buffer; an in-place NCCL all-gather over
// NVLink fills every slot on every rank, and an HBM-bound permute kernel lays
// the slots out as the row-major [M, N] result.  Batched products need no
// collective at all: ranks take disjoint batch ranges.
//
// NCCL is loaded at run time (the copy the process already mapped, e.g. the
// one PyTorch ships, else libnccl.so.2 from the loader path), so the library
// has no link-time NCCL dependency and single-GPU users never load it.
#include "gemm_sm100.h"
#include "internal.h"

#include <nccl.h>

#include <dlfcn.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#define PT_API extern "C" __attribute__((visibility("default")))



namespace {

struct NcclApi {
    bool loaded = false;
    void *handle = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                               ncclComm_t, cudaStream_t) = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_mutex;

bool nccl()
{
    std::lock_guard<std::mutex> lock(g_nccl_mutex);
    if (g_nccl.loaded)
        return g_nccl.handle != nullptr;
    g_nccl.loaded = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h)
        h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h)
        return false;
    g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    g_nccl.comm_init_rank = reinterpret_cast<decltype(g_nccl.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    g_nccl.comm_destroy = reinterpret_cast<decltype(g_nccl.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    g_nccl.all_gather = reinterpret_cast<decltype(g_nccl.all_gather)>(dlsym(h, "ncclAllGather"));
    g_nccl.all_reduce = reinterpret_cast<decltype(g_nccl.all_reduce)>(dlsym(h, "ncclAllReduce"));
    if (!g_nccl.get_unique_id || !g_nccl.comm_init_rank || !g_nccl.comm_destroy ||
        !g_nccl.all_gather || !g_nccl.all_reduce) {
        dlclose(h);
        return false;
    }
    g_nccl.handle = h;
    return true;
}

size_t element_bytes(dtype_t dt)
{
    switch (dt) {
    case DTYPE_FLOAT64: return 8;
    case DTYPE_FLOAT32: return 4;
    case DTYPE_FLOAT16:
    case DTYPE_BFLOAT16: return 2;
    default: return 0;
    }
}

// out[m][r * nb + j] = ws[r][m][j], in 16-byte units (vec) or elements.
template <typename T>
__global__ void nsplit_permute_kernel(const T *__restrict__ ws, T *__restrict__ out, int ranks,
                                      long long rows, long long nb)
{
    const long long total = static_cast<long long>(ranks) * rows * nb;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long j = i % nb;
        const long long m = (i / nb) % rows;
        const long long r = i / (nb * rows);
        out[m * (nb * ranks) + r * nb + j] = ws[i];
    }
}

} // namespace

struct gemm_mgpu_comm {
    ncclComm_t nccl;
    int nranks;
    int rank;
    int device;
};

PT_API int gemm_mgpu_unique_id(unsigned char *id)
{
    if (!id || !nccl()) {
        ptg_set_last_status(GEMM_SM100_STATUS_NCCL);
        return 0;
    }
    ncclUniqueId uid;
    if (g_nccl.get_unique_id(&uid) != ncclSuccess) {
        ptg_set_last_status(GEMM_SM100_STATUS_NCCL);
        return 0;
    }
    std::memcpy(id, uid.internal, GEMM_MGPU_UNIQUE_ID_BYTES);
    return 1;
}

PT_API int gemm_mgpu_comm_init(const unsigned char *id, int nranks, int rank,
                               gemm_mgpu_comm **comm)
{
    if (!id || !comm || nranks < 1 || rank < 0 || rank >= nranks || !nccl()) {
        ptg_set_last_status(GEMM_SM100_STATUS_NCCL);
        return 0;
    }
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess) {
        ptg_set_last_status(GEMM_SM100_STATUS_NO_DEVICE);
        return 0;
    }
    ncclUniqueId uid;
    std::memcpy(uid.internal, id, GEMM_MGPU_UNIQUE_ID_BYTES);
    ncclComm_t c = nullptr;
    if (g_nccl.comm_init_rank(&c, nranks, uid, rank) != ncclSuccess) {
        ptg_set_last_status(GEMM_SM100_STATUS_NCCL);
        return 0;
    }
    *comm = new gemm_mgpu_comm{c, nranks, rank, device};
    return 1;
}

PT_API void gemm_mgpu_comm_destroy(gemm_mgpu_comm *comm)
{
    if (!comm)
        return;
    if (comm->nccl && nccl())
        g_nccl.comm_destroy(comm->nccl);
    delete comm;
}

PT_API size_t gemm_mgpu_nsplit_workspace_bytes(int nranks, dtype_t dtype, int M, int N)
{
    if (nranks < 1 || M < 0 || N < 0 || N % nranks != 0)
        return 0;
    return static_cast<size_t>(M) * static_cast<size_t>(N) * element_bytes(dtype);
}

PT_API int gemm_mgpu_nsplit_matmul(gemm_mgpu_comm *comm, dtype_t dtype, const void *a,
                                   size_t a_s0, size_t a_s1, const void *b_local, size_t b_s0,
                                   size_t b_s1, void *c, int M, int N, int K, void *workspace,
                                   size_t workspace_bytes, cudaStream_t stream)
{
    const size_t es = element_bytes(dtype);
    if (!comm || es == 0 || M < 0 || N < 0 || K < 0 || N % comm->nranks != 0) {
        ptg_set_last_status(GEMM_SM100_STATUS_INVALID_ARGUMENT);
        return 0;
    }
    if (M == 0 || N == 0)
        return 1;
    const int G = comm->nranks;
    const int nb = N / G;
    const size_t slot = static_cast<size_t>(M) * nb;
    if (!workspace || !c || workspace_bytes < slot * G * es) {
        ptg_set_last_status(GEMM_SM100_STATUS_INVALID_ARGUMENT);
        return 0;
    }
    // 1. this rank's column block into its slot of the gather buffer
    void *mine = static_cast<char *>(workspace) + slot * comm->rank * es;
    int sa[2] = {M, K}, sb[2] = {K, nb}, sc[2] = {M, nb};
    size_t ta[2] = {a_s0, a_s1}, tb[2] = {b_s0, b_s1}, tc[2] = {static_cast<size_t>(nb), 1};
    int ok;
    if (dtype == DTYPE_FLOAT64)
        ok = cuda_f64_matmul_nd_launcher(static_cast<double *>(const_cast<void *>(a)),
                                         static_cast<double *>(const_cast<void *>(b_local)),
                                         static_cast<double *>(mine), sa, ta, 2, sb, tb, 2, sc,
                                         tc, 2, stream);
    else if (dtype == DTYPE_FLOAT32)
        ok = cuda_batched_matmul_nd_launcher(static_cast<float *>(const_cast<void *>(a)),
                                             static_cast<float *>(const_cast<void *>(b_local)),
                                             static_cast<float *>(mine), sa, ta, 2, sb, tb, 2, sc,
                                             tc, 2, stream);
    else
        ok = cuda_low_precision_matmul_nd_launcher(const_cast<void *>(a),
                                                   const_cast<void *>(b_local), mine, dtype, sa,
                                                   ta, 2, sb, tb, 2, sc, tc, 2, stream);
    if (!ok)
        return 0;
    // 2. in-place all-gather of every rank's block over NVLink
    if (G > 1) {
        if (!nccl() || g_nccl.all_gather(mine, workspace, slot * es, ncclUint8, comm->nccl,
                                         stream) != ncclSuccess) {
            ptg_set_last_status(GEMM_SM100_STATUS_NCCL);
            return 0;
        }
    }
    // 3. [G][M][nb] -> [M][G * nb]
    const long long total = static_cast<long long>(slot) * G;
    const int threads = 256;
    const long long want = (total + threads - 1) / threads;
    const int blocks = static_cast<int>(want < 148 * 16 ? want : 148 * 16);
    switch (es) {
    case 8:
        if ((nb % 2) == 0 && (reinterpret_cast<uintptr_t>(c) % 16) == 0)
            nsplit_permute_kernel<uint4><<<blocks, threads, 0, stream>>>(
                static_cast<const uint4 *>(workspace), static_cast<uint4 *>(c), G, M, nb / 2);
        else
            nsplit_permute_kernel<uint2><<<blocks, threads, 0, stream>>>(
                static_cast<const uint2 *>(workspace), static_cast<uint2 *>(c), G, M, nb);
        break;
    case 4:
        nsplit_permute_kernel<uint32_t><<<blocks, threads, 0, stream>>>(
            static_cast<const uint32_t *>(workspace), static_cast<uint32_t *>(c), G, M, nb);
        break;
    default:
        nsplit_permute_kernel<uint16_t><<<blocks, threads, 0, stream>>>(
            static_cast<const uint16_t *>(workspace), static_cast<uint16_t *>(c), G, M, nb);
        break;
    }
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
        ptg_set_last_status(static_cast<int>(err));
        return 0;
    }
    return 1;
}

// ---------------------------------------------------------------- no-alloc variant
//
// Some callers cannot allocate device memory at the moment they multiply:
// code that is being captured into a CUDA graph (cudaMalloc is not allowed
// from a capturing thread), or a host program whose device memory is entirely
// owned by its own pool allocator and must never see a cudaMalloc/cudaFree
// (cudaFree also synchronises the whole device).  For them the N-split
// product can use a gather buffer that lives in the library itself: a fixed
// array in device memory, reserved on every GPU that loads the library and
// held until the process exits.

namespace {

// The library-owned gather buffer (one copy per device).
static __device__ __align__(256) unsigned char g_nsplit_scratch[GEMM_MGPU_NSPLIT_SCRATCH_BYTES];

constexpr int kScratchDevices = 64;
void *g_scratch_addr[kScratchDevices];   // device address of g_nsplit_scratch, per device
std::mutex g_scratch_mutex;

// The host-side name g_nsplit_scratch is only a stand-in for the array, not a
// device address; the address a kernel or NCCL may use comes from
// cudaGetSymbolAddress, taken once per device with that device current.
void *scratch_address(int device)
{
    if (device < 0 || device >= kScratchDevices)
        return nullptr;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[device]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_nsplit_scratch) != cudaSuccess)
            return nullptr;
        g_scratch_addr[device] = p;
    }
    return g_scratch_addr[device];
}

} // namespace

PT_API int gemm_mgpu_nsplit_matmul_noalloc(gemm_mgpu_comm *comm, dtype_t dtype, const void *a,
                                           size_t a_s0, size_t a_s1, const void *b_local,
                                           size_t b_s0, size_t b_s1, void *c, int M, int N,
                                           int K, cudaStream_t stream)
{
    const size_t es = element_bytes(dtype);
    if (!comm || es == 0 || M < 0 || N < 0 || K < 0) {
        ptg_set_last_status(GEMM_SM100_STATUS_INVALID_ARGUMENT);
        return 0;
    }
    const size_t need = static_cast<size_t>(M) * static_cast<size_t>(N) * es;
    if (need > GEMM_MGPU_NSPLIT_SCRATCH_BYTES) {
        ptg_set_last_status(GEMM_SM100_STATUS_SCRATCH_LIMIT);
        return 0;
    }
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess || device != comm->device) {
        ptg_set_last_status(GEMM_SM100_STATUS_NO_DEVICE);
        return 0;
    }
    void *scratch = scratch_address(device);
    if (!scratch) {
        ptg_set_last_status(GEMM_SM100_STATUS_NO_DEVICE);
        return 0;
    }
    return gemm_mgpu_nsplit_matmul(comm, dtype, a, a_s0, a_s1, b_local, b_s0, b_s1, c, M, N, K,
                                   scratch, GEMM_MGPU_NSPLIT_SCRATCH_BYTES, stream);
}

// ---------------------------------------------------------------- fused N-split
//
// The N-split product with the exchange inside the GEMM: every rank's result
// buffer is mapped into every other rank (CUDA IPC over NVLink / NVSwitch), and
// the epilogue of the rank's column-block product stores each finished output
// row into all ranks' results directly.  No gather buffer, no permute; the
// peer stores overlap the remaining tiles' tensor-core work.  A one-element
// NCCL all-reduce after the kernel orders every rank's stores before any rank
// goes on to read its result, and another one before the kernel keeps a
// rank's stores of the next call out of a peer's window until that peer has
// reached the call (it may still be reading the previous result).

struct gemm_mgpu_window {
    gemm_mgpu_comm *comm;
    void *local;
    size_t bytes;
    void *peer[8];
    int *sync;   // one int for the ordering all-reduces
    int exchange;  // GEMM_MGPU_EXCHANGE_*
    unsigned long long *slots;   // the overlapped exchange's per-SM hand-off slots
};

namespace {
constexpr int kHandoffSlots = 1024;   // more than any %smid of a B200
}

PT_API int gemm_mgpu_window_create(gemm_mgpu_comm *comm, size_t bytes, gemm_mgpu_window **win,
                                   void **local)
{
    if (!comm || !win || !local || comm->nranks > 8 || bytes == 0 || !nccl()) {
        ptg_set_last_status(GEMM_SM100_STATUS_NCCL);
        return 0;
    }
    const int G = comm->nranks, rank = comm->rank;
    gemm_mgpu_window *w = new gemm_mgpu_window();
    w->comm = comm;
    w->bytes = bytes;
    unsigned char *xdev = nullptr;
    cudaStream_t s = nullptr;
    cudaIpcMemHandle_t mine;
    unsigned char all[8 * sizeof(cudaIpcMemHandle_t)];
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    bool good = cudaMalloc(&w->local, bytes) == cudaSuccess &&
                cudaMalloc(&w->sync, 16) == cudaSuccess &&
                cudaMemset(w->sync, 0, 16) == cudaSuccess &&
                cudaMalloc(&w->slots, kHandoffSlots * sizeof(unsigned long long)) == cudaSuccess &&
                cudaMemset(w->slots, 0, kHandoffSlots * sizeof(unsigned long long)) == cudaSuccess &&
                cudaIpcGetMemHandle(&mine, w->local) == cudaSuccess &&
                cudaMalloc(&xdev, hb * G) == cudaSuccess &&
                cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess &&
                cudaMemcpyAsync(xdev + hb * rank, &mine, hb, cudaMemcpyHostToDevice, s) ==
                    cudaSuccess;
    if (good && G > 1)
        good = g_nccl.all_gather(xdev + hb * rank, xdev, hb, ncclUint8, comm->nccl, s) ==
               ncclSuccess;
    good = good && cudaMemcpyAsync(all, xdev, hb * G, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
           cudaStreamSynchronize(s) == cudaSuccess;
    for (int g = 0; good && g < G; g++) {
        if (g == rank) {
            w->peer[g] = w->local;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, all + hb * g, hb);
        good = cudaIpcOpenMemHandle(&w->peer[g], h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    }
    if (s) cudaStreamDestroy(s);
    if (xdev) cudaFree(xdev);
    if (!good) {
        ptg_set_last_status(static_cast<int>(cudaGetLastError()));
        for (int g = 0; g < G; g++)
            if (g != rank && w->peer[g])
                cudaIpcCloseMemHandle(w->peer[g]);
        if (w->local) cudaFree(w->local);
        if (w->sync) cudaFree(w->sync);
        if (w->slots) cudaFree(w->slots);
        delete w;
        return 0;
    }
    *win = w;
    *local = w->local;
    return 1;
}

PT_API int gemm_mgpu_window_set_exchange(gemm_mgpu_window *win, int mode)
{
    if (!win || (mode != GEMM_MGPU_EXCHANGE_AUTO && mode != GEMM_MGPU_EXCHANGE_STORE &&
                 mode != GEMM_MGPU_EXCHANGE_OVERLAP)) {
        ptg_set_last_status(GEMM_SM100_STATUS_INVALID_ARGUMENT);
        return 0;
    }
    win->exchange = mode;
    return 1;
}

PT_API void gemm_mgpu_window_destroy(gemm_mgpu_window *win)
{
    if (!win)
        return;
    cudaDeviceSynchronize();
    for (int g = 0; g < win->comm->nranks; g++)
        if (g != win->comm->rank && win->peer[g])
            cudaIpcCloseMemHandle(win->peer[g]);
    cudaFree(win->local);
    cudaFree(win->sync);
    cudaFree(win->slots);
    delete win;
}

PT_API int gemm_mgpu_nsplit_matmul_fused(gemm_mgpu_window *win, dtype_t dtype, const void *a,
                                         size_t a_s0, size_t a_s1, const void *b_local,
                                         size_t b_s0, size_t b_s1, int M, int N, int K,
                                         cudaStream_t stream)
{
    if (!win || dtype != DTYPE_FLOAT64 || M < 0 || N < 0 || K < 0) {
        ptg_set_last_status(GEMM_SM100_STATUS_INVALID_ARGUMENT);
        return 0;
    }
    gemm_mgpu_comm *comm = win->comm;
    const int G = comm->nranks;
    if (N % G != 0 || (N / G) % 2 != 0 ||
        static_cast<size_t>(M) * static_cast<size_t>(N) * 8 > win->bytes) {
        ptg_set_last_status(GEMM_SM100_STATUS_INVALID_ARGUMENT);
        return 0;
    }
    if (M == 0 || N == 0)
        return 1;
    // Entry ordering: this call's kernel stores into every peer's window, and
    // a peer may still be reading the previous call's result there.  The
    // one-element all-reduce completes on this stream only once every rank's
    // stream has reached it, i.e. once every rank is done with call k.
    if (G > 1 && g_nccl.all_reduce(win->sync, win->sync, 1, ncclInt32, ncclSum, comm->nccl,
                                   stream) != ncclSuccess) {
        ptg_set_last_status(GEMM_SM100_STATUS_NCCL);
        return 0;
    }
    ptg::F64PeerOut po;
    std::memset(&po, 0, sizeof(po));
    for (int g = 0; g < G; g++)
        po.dst[g] = static_cast<double *>(win->peer[g]);
    po.ndst = G;
    po.rot = comm->rank;
    po.exchange = win->exchange;
    po.slots = win->slots;
    po.nslots = kHandoffSlots;
    po.ldc = N;
    po.col_off = static_cast<long long>(comm->rank) * (N / G);
    const cudaError_t err = ptg_launch_f64_peer(
        static_cast<const double *>(a), a_s0, a_s1, static_cast<const double *>(b_local), b_s0,
        b_s1, M, N / G, K, po, stream);
    if (err != cudaSuccess) {
        ptg_set_last_status(static_cast<int>(err));
        return 0;
    }
    if (G > 1 && g_nccl.all_reduce(win->sync, win->sync, 1, ncclInt32, ncclSum, comm->nccl,
                                   stream) != ncclSuccess) {
        ptg_set_last_status(GEMM_SM100_STATUS_NCCL);
        return 0;
    }
    return 1;
}
