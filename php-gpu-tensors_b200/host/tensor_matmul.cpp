// Tensor-level matmul dispatch (include/pt_tensor.h): the C++ host layer that
// sits where the PHP extension's C dispatch sits in the reference
// (src/cuda_array/ca_private.c:1097-1213, src/fusion_execute.c:157-182,
// src/autograd.c:1539-1585) and calls the launcher ABI of gemm_sm100.h.
#include "pt_tensor.h"

#include "internal.h"

#include <cstdio>
#include <cstring>

#define PT_API extern "C" __attribute__((visibility("default")))

namespace {

thread_local char t_error[256] = "";

int fail(int code, const char *fmt, int value = 0)
{
    std::snprintf(t_error, sizeof(t_error), fmt, value);
    return code;
}

int ok()
{
    t_error[0] = '\0';
    return PT_OK;
}

// src/tensor_shape.h:7-22
bool broadcast_shape(const int *a, int na, const int *b, int nb, int *out, int *nout)
{
    const int n = na > nb ? na : nb;
    for (int axis = 0; axis < n; axis++) {
        const int ia = axis - (n - na), ib = axis - (n - nb);
        const int ea = ia < 0 ? 1 : a[ia];
        const int eb = ib < 0 ? 1 : b[ib];
        if (ea != eb && ea != 1 && eb != 1)
            return false;
        out[axis] = ea == 1 ? eb : ea;
    }
    *nout = n;
    return true;
}

// src/tensor_shape.h:46-59
bool matmul_shape(const pt_tensor *a, const pt_tensor *b, int *shape, int *ndims)
{
    if (a->ndims < 2 || a->ndims > MAX_DIMS || b->ndims < 2 || b->ndims > MAX_DIMS ||
        a->shape[a->ndims - 1] != b->shape[b->ndims - 2])
        return false;
    int nb = 0;
    if (!broadcast_shape(a->shape, a->ndims - 2, b->shape, b->ndims - 2, shape, &nb))
        return false;
    shape[nb] = a->shape[a->ndims - 2];
    shape[nb + 1] = b->shape[b->ndims - 1];
    *ndims = nb + 2;
    return true;
}

size_t element_size(dtype_t dt)
{
    switch (dt) {
    case DTYPE_FLOAT64: return 8;
    case DTYPE_FLOAT32: return 4;
    case DTYPE_FLOAT16:
    case DTYPE_BFLOAT16: return 2;
    default: return 0;
    }
}

bool supported_dtype(dtype_t dt, int flags)
{
    return dt == DTYPE_FLOAT32 || dt == DTYPE_FLOAT16 || dt == DTYPE_BFLOAT16 ||
           (dt == DTYPE_FLOAT64 && (flags & PT_MATMUL_ALLOW_FLOAT64));
}

int submission_failed()
{
    cuda_backend_info info;
    std::memset(&info, 0, sizeof(info));
    cuda_blas_info(&info);
    return fail(PT_RUNTIME, "Matmul backend submission failed (cuBLAS status %d)",
                info.last_blas_status);
}

// Launcher choice of ca_private.c:1127-1137,1168-1200 and fusion_execute.c:159-173.
int dispatch(const pt_tensor *a, const pt_tensor *b, const pt_tensor *r, cudaStream_t stream)
{
    pt_tensor ca = *a, cb = *b, cr = *r;   // the launchers take non-const metadata
    int status;
    if (a->dtype == DTYPE_FLOAT32 && a->ndims == 2 && b->ndims == 2)
        status = cuda_matmul_launcher(static_cast<float *>(a->data), static_cast<float *>(b->data),
                                      static_cast<float *>(r->data), a->shape[0], a->shape[1],
                                      b->shape[1], a->strides[0], a->strides[1], b->strides[0],
                                      b->strides[1], r->strides[0], r->strides[1], stream);
    else if (a->dtype == DTYPE_FLOAT32)
        status = cuda_batched_matmul_nd_launcher(
            static_cast<float *>(a->data), static_cast<float *>(b->data),
            static_cast<float *>(r->data), ca.shape, ca.strides, a->ndims, cb.shape, cb.strides,
            b->ndims, cr.shape, cr.strides, r->ndims, stream);
    else if (a->dtype == DTYPE_FLOAT64)
        status = cuda_f64_matmul_nd_launcher(
            static_cast<double *>(a->data), static_cast<double *>(b->data),
            static_cast<double *>(r->data), ca.shape, ca.strides, a->ndims, cb.shape, cb.strides,
            b->ndims, cr.shape, cr.strides, r->ndims, stream);
    else
        status = cuda_low_precision_matmul_nd_launcher(
            a->data, b->data, r->data, a->dtype, ca.shape, ca.strides, a->ndims, cb.shape,
            cb.strides, b->ndims, cr.shape, cr.strides, r->ndims, stream);
    return status ? ok() : submission_failed();
}

int check_operands(const pt_tensor *a, const pt_tensor *b, int flags, int *shape, int *ndims)
{
    if (!a || !b || a->dtype != b->dtype || !supported_dtype(a->dtype, flags))
        return fail(PT_INVALID_ARGUMENT,
                    "matmul requires matching float32, float16 or bfloat16 operands");
    if (!matmul_shape(a, b, shape, ndims))
        return fail(PT_INVALID_ARGUMENT, "Matrix multiplication failed - incompatible dimensions");
    return PT_OK;
}

void contiguous_strides(const int *shape, int ndims, size_t *strides)
{
    size_t s = 1;
    for (int d = ndims - 1; d >= 0; d--) {
        strides[d] = s;
        s *= static_cast<size_t>(shape[d]);
    }
}

pt_tensor transposed_view(const pt_tensor *t)
{
    pt_tensor v = *t;
    const int n = t->ndims;
    v.shape[n - 2] = t->shape[n - 1];
    v.shape[n - 1] = t->shape[n - 2];
    v.strides[n - 2] = t->strides[n - 1];
    v.strides[n - 1] = t->strides[n - 2];
    return v;
}

} // namespace

PT_API const char *pt_last_error(void) { return t_error; }

PT_API int pt_matmul_result_shape(const pt_tensor *a, const pt_tensor *b, int *shape, int *ndims)
{
    if (!a || !b || !shape || !ndims)
        return fail(PT_INVALID_ARGUMENT, "Both operands must be valid tensor objects.");
    if (!matmul_shape(a, b, shape, ndims))
        return fail(PT_INVALID_ARGUMENT, "Matrix multiplication failed - incompatible dimensions");
    return ok();
}

PT_API int pt_tensor_matmul_into(const pt_tensor *a, const pt_tensor *b, const pt_tensor *result,
                                 int flags, cudaStream_t stream)
{
    int shape[MAX_DIMS], ndims = 0;
    const int v = check_operands(a, b, flags, shape, &ndims);
    if (v != PT_OK)
        return v;
    if (!result || result->dtype != a->dtype || result->ndims != ndims)
        return fail(PT_INVALID_ARGUMENT, "Matrix multiplication failed - incompatible dimensions");
    for (int d = 0; d < ndims; d++)
        if (result->shape[d] != shape[d])
            return fail(PT_INVALID_ARGUMENT,
                        "Matrix multiplication failed - incompatible dimensions");
    return dispatch(a, b, result, stream);
}

PT_API int pt_tensor_matmul(const pt_tensor *a, const pt_tensor *b, pt_tensor *result, int flags,
                            cudaStream_t stream)
{
    if (!result)
        return fail(PT_INVALID_ARGUMENT, "Both operands must be valid tensor objects.");
    int shape[MAX_DIMS], ndims = 0;
    const int v = check_operands(a, b, flags, shape, &ndims);
    if (v != PT_OK)
        return v;
    pt_tensor r;
    std::memset(&r, 0, sizeof(r));
    r.dtype = a->dtype;
    r.ndims = ndims;
    std::memcpy(r.shape, shape, sizeof(int) * static_cast<size_t>(ndims));
    contiguous_strides(shape, ndims, r.strides);
    size_t total = 1;
    for (int d = 0; d < ndims; d++)
        total *= static_cast<size_t>(shape[d]);
    const size_t bytes = total * element_size(a->dtype);
    if (bytes) {
        const cudaError_t err = cudaMallocAsync(&r.data, bytes, stream);
        if (err != cudaSuccess)
            return fail(PT_RUNTIME, "Failed to allocate the matmul result (CUDA error %d)",
                        static_cast<int>(err));
    }
    const int s = dispatch(a, b, &r, stream);
    if (s != PT_OK) {
        if (r.data)
            cudaFreeAsync(r.data, stream);
        return s;
    }
    *result = r;
    return PT_OK;
}

PT_API void pt_tensor_release(pt_tensor *t, cudaStream_t stream)
{
    if (t && t->data) {
        cudaFreeAsync(t->data, stream);
        t->data = nullptr;
    }
}

namespace {

// out (float32) = x . y where x and y are float32 or one 16-bit type each:
// float32 pairs take the reference's launchers, anything else the mixed
// launcher, which reads the 16-bit operands as they are.
int launch_product(const pt_tensor *x, const pt_tensor *y, const pt_tensor *out,
                   cudaStream_t stream)
{
    if (x->dtype == DTYPE_FLOAT32 && y->dtype == DTYPE_FLOAT32)
        return dispatch(x, y, out, stream);
    pt_tensor cx = *x, cy = *y, co = *out;
    const int st = cuda_mixed_matmul_nd_launcher(x->data, x->dtype, y->data, y->dtype,
                                                 static_cast<float *>(out->data), cx.shape,
                                                 cx.strides, x->ndims, cy.shape, cy.strides,
                                                 y->ndims, co.shape, co.strides, out->ndims,
                                                 stream);
    return st ? ok() : submission_failed();
}

// Whether the batch axes of t (aligned to the product's nb batch axes, all at
// full extent) chain onto its axis `inner` so that (batch..., inner) is one
// strided axis; returns its extent through *total.
bool folds_into(const pt_tensor *t, const int *full, int nb, int inner, long long *total)
{
    if (t->ndims - 2 != nb)
        return false;
    long long extent = t->shape[inner];
    long long stride = static_cast<long long>(t->strides[inner]);
    for (int d = nb - 1; d >= 0; d--) {
        if (t->shape[d] != full[d])
            return false;
        if (t->shape[d] == 1)
            continue;
        if (static_cast<long long>(t->strides[d]) != extent * stride)
            return false;
        extent *= t->shape[d];
    }
    *total = extent;
    return extent <= 0x7fffffffll;
}

// out = x . y, or -- when out has the shape of an operand that the product
// broadcast (extent 1 or no axis where the product has a batch axis) -- that
// product summed over the broadcast axes, the un-broadcast step of
// src/autograd.c:714-760 fused with the GEMM:
//   * every batch axis summed and both operands' batch axes chaining onto the
//     product's inner axis (contiguous tensors): one GEMM whose inner axis is
//     (batch..., K);
//   * otherwise: the product kernel itself walks the summed axes in its k
//     loop (ptg_reduced_matmul), writing the reduced gradient directly.
int gradient_product(const pt_tensor *x, const pt_tensor *y, const pt_tensor *out,
                     cudaStream_t stream)
{
    int full[MAX_DIMS], nf = 0;
    if (!matmul_shape(x, y, full, &nf) || out->ndims < 2 || out->ndims > nf ||
        out->shape[out->ndims - 2] != full[nf - 2] || out->shape[out->ndims - 1] != full[nf - 1])
        return fail(PT_INVALID_ARGUMENT, "Matrix multiplication failed - incompatible dimensions");
    if (out->dtype != DTYPE_FLOAT32)
        return fail(PT_INVALID_ARGUMENT, "matmul gradients are float32 tensors");
    const int nb = nf - 2;
    bool same = out->ndims == nf, all_reduced = true;
    for (int d = 0; d < nb; d++) {
        const int io = d - (nf - out->ndims);
        const int eo = io >= 0 ? out->shape[io] : 1;
        if (eo != full[d] && eo != 1)
            return fail(PT_INVALID_ARGUMENT,
                        "Gradient shape cannot be reduced to its operand shape at axis %d", io);
        same = same && eo == full[d];
        all_reduced = all_reduced && (full[d] == 1 || eo != full[d]);
    }
    if (same)
        return launch_product(x, y, out, stream);

    long long fx = 0, fy = 0;
    if (all_reduced && folds_into(x, full, nb, x->ndims - 1, &fx) &&
        folds_into(y, full, nb, y->ndims - 2, &fy) && fx == fy) {
        pt_tensor x2 = *x, y2 = *y, o2 = *out;
        x2.ndims = y2.ndims = o2.ndims = 2;
        x2.shape[0] = x->shape[x->ndims - 2];
        x2.shape[1] = static_cast<int>(fx);
        x2.strides[0] = x->strides[x->ndims - 2];
        x2.strides[1] = x->strides[x->ndims - 1];
        y2.shape[0] = static_cast<int>(fy);
        y2.shape[1] = y->shape[y->ndims - 1];
        y2.strides[0] = y->strides[y->ndims - 2];
        y2.strides[1] = y->strides[y->ndims - 1];
        o2.shape[0] = out->shape[out->ndims - 2];
        o2.shape[1] = out->shape[out->ndims - 1];
        o2.strides[0] = out->strides[out->ndims - 2];
        o2.strides[1] = out->strides[out->ndims - 1];
        return launch_product(&x2, &y2, &o2, stream);
    }

    // every other reduction: the summed axes run inside the product kernel
    pt_tensor cx = *x, cy = *y, co = *out;
    const int st = ptg_reduced_matmul(x->data, x->dtype, y->data, y->dtype,
                                      static_cast<float *>(out->data), cx.shape, cx.strides,
                                      x->ndims, cy.shape, cy.strides, y->ndims, co.shape,
                                      co.strides, out->ndims, stream);
    return st ? ok() : submission_failed();
}

} // namespace

namespace {

// The autograd node's side stream and fork/join events, per host thread and
// device (created on first use, kept for the thread's lifetime).
struct BackwardStreams {
    cudaStream_t side = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
constexpr int kMaxBackwardDevices = 64;
thread_local BackwardStreams t_backward[kMaxBackwardDevices];
thread_local cudaStream_t t_backward_side = nullptr;
thread_local cudaEvent_t t_backward_join = nullptr;

// Forks a side stream off `stream`: returns it with the fork recorded, or
// null when the stream or events cannot be made (the caller then runs both
// products on `stream`).
cudaStream_t backward_side_stream(cudaStream_t stream)
{
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxBackwardDevices)
        return nullptr;
    BackwardStreams &b = t_backward[dev];
    if (!b.side) {
        if (cudaStreamCreateWithFlags(&b.side, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&b.fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&b.join, cudaEventDisableTiming) != cudaSuccess) {
            (void)cudaGetLastError();
            if (b.side) cudaStreamDestroy(b.side);
            if (b.fork) cudaEventDestroy(b.fork);
            if (b.join) cudaEventDestroy(b.join);
            b = BackwardStreams();
            return nullptr;
        }
    }
    if (cudaEventRecord(b.fork, stream) != cudaSuccess ||
        cudaStreamWaitEvent(b.side, b.fork, 0) != cudaSuccess) {
        (void)cudaGetLastError();
        return nullptr;
    }
    t_backward_side = b.side;
    t_backward_join = b.join;
    return b.side;
}

// Joins the side stream back into `stream`.
int backward_join(cudaStream_t stream)
{
    if (cudaEventRecord(t_backward_join, t_backward_side) != cudaSuccess ||
        cudaStreamWaitEvent(stream, t_backward_join, 0) != cudaSuccess)
        return fail(PT_RUNTIME, "could not join the backward side stream");
    return PT_OK;
}

} // namespace

PT_API int pt_tensor_matmul_backward(const pt_tensor *a, const pt_tensor *b,
                                     const pt_tensor *grad_c, const pt_tensor *grad_a,
                                     const pt_tensor *grad_b, cudaStream_t stream)
{
    // src/autograd.c:1547-1551: float16/bfloat16 operands have float32
    // gradients; the upstream gradient is float32 or the operands' type
    if (!a || !b || !grad_c || a->dtype != b->dtype ||
        (a->dtype != DTYPE_FLOAT32 && a->dtype != DTYPE_FLOAT16 && a->dtype != DTYPE_BFLOAT16) ||
        (grad_c->dtype != DTYPE_FLOAT32 && grad_c->dtype != a->dtype))
        return fail(PT_INVALID_ARGUMENT,
                    "matmul backward requires float32, float16 or bfloat16 operands with a "
                    "float32 or same-typed upstream gradient");
    if (a->ndims < 2 || b->ndims < 2)
        return fail(PT_INVALID_ARGUMENT, "Autograd matmul requires operands with rank at least 2");
    const pt_tensor bt = transposed_view(b);
    const pt_tensor at = transposed_view(a);
    // Both gradients: dB runs on a side stream forked from and joined back
    // into the caller's stream (events, so graph capture records the fork
    // and join), letting the two products' launch tails, and small products
    // such as a classifier layer's, overlap.
    cudaStream_t side = grad_a && grad_b ? backward_side_stream(stream) : nullptr;
    if (side) {
        const int s1 = gradient_product(grad_c, &bt, grad_a, stream);
        const int s2 = s1 == PT_OK ? gradient_product(&at, grad_c, grad_b, side) : s1;
        const int sj = backward_join(stream);
        if (s1 != PT_OK)
            return s1;
        if (s2 != PT_OK)
            return s2;
        return sj;
    }
    if (grad_a) {
        const int s = gradient_product(grad_c, &bt, grad_a, stream);
        if (s != PT_OK)
            return s;
    }
    if (grad_b) {
        const int s = gradient_product(&at, grad_c, grad_b, stream);
        if (s != PT_OK)
            return s;
    }
    return ok();
}

namespace {

// Streams, events and device staging of the host-buffer pipeline, kept per
// host thread and device across calls (allocation and stream creation cost
// far more than a chunk's copies).
struct HostPipeline {
    int device = -1;
    cudaStream_t s_in = nullptr, s_comp = nullptr, s_out = nullptr;
    cudaEvent_t in_done[2] = {}, compute_done[2] = {}, out_done[2] = {};
    void *stage = nullptr;   // [slot 0: a | b | c][slot 1: a | b | c][shared b]
    size_t stage_bytes = 0;
};

constexpr int kMaxPipeDevices = 64;
thread_local HostPipeline t_pipes[kMaxPipeDevices];

// Frees one device's pipeline (switches to that device and back).
void release_pipeline(HostPipeline &p)
{
    if (p.device < 0)
        return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(p.device);
    if (p.s_in) cudaStreamSynchronize(p.s_in);
    if (p.s_comp) cudaStreamSynchronize(p.s_comp);
    if (p.s_out) cudaStreamSynchronize(p.s_out);
    if (p.stage) cudaFree(p.stage);
    for (int i = 0; i < 2; i++) {
        if (p.in_done[i]) cudaEventDestroy(p.in_done[i]);
        if (p.compute_done[i]) cudaEventDestroy(p.compute_done[i]);
        if (p.out_done[i]) cudaEventDestroy(p.out_done[i]);
    }
    if (p.s_in) cudaStreamDestroy(p.s_in);
    if (p.s_comp) cudaStreamDestroy(p.s_comp);
    if (p.s_out) cudaStreamDestroy(p.s_out);
    if (prev >= 0)
        cudaSetDevice(prev);
    p = HostPipeline();
}

// Makes device `dev`'s pipeline ready with at least `bytes` of staging; `dev`
// must be the current device.  Returns a cudaError_t.
cudaError_t prepare_pipeline(int dev, size_t bytes)
{
    if (dev < 0 || dev >= kMaxPipeDevices)
        return cudaErrorInvalidDevice;
    cudaError_t e;
    HostPipeline &p = t_pipes[dev];
    if (p.device != dev) {
        p.device = dev;
        if ((e = cudaStreamCreateWithFlags(&p.s_in, cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaStreamCreateWithFlags(&p.s_comp, cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaStreamCreateWithFlags(&p.s_out, cudaStreamNonBlocking)) != cudaSuccess)
            return e;
        for (int i = 0; i < 2; i++)
            if ((e = cudaEventCreateWithFlags(&p.in_done[i], cudaEventDisableTiming)) != cudaSuccess ||
                (e = cudaEventCreateWithFlags(&p.compute_done[i], cudaEventDisableTiming)) !=
                    cudaSuccess ||
                (e = cudaEventCreateWithFlags(&p.out_done[i], cudaEventDisableTiming)) != cudaSuccess)
                return e;
    }
    if (p.stage_bytes < bytes) {
        if (p.stage) {
            cudaStreamSynchronize(p.s_in);
            cudaStreamSynchronize(p.s_comp);
            cudaStreamSynchronize(p.s_out);
            cudaFree(p.stage);
            p.stage = nullptr;
            p.stage_bytes = 0;
        }
        if ((e = cudaMalloc(&p.stage, bytes)) != cudaSuccess)
            return e;
        p.stage_bytes = bytes;
    }
    return cudaSuccess;
}

size_t round256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// One device's share of a host-buffer product: batches [first, first +
// count) cut into chunks of `per`, double-buffered through two staging slots.
struct HostShard {
    int device;
    int first, count, per, chunks;
    HostPipeline *p;
};

struct HostJob {
    const void *a, *b;
    void *c;
    dtype_t dtype;
    int M, N, K, b_shared, flags;
    size_t a_b, b_b, c_b;   // bytes per batch
};

size_t slot_bytes_for(const HostJob &j, int per, size_t *sa, size_t *sb)
{
    *sa = round256(j.a_b * per);
    *sb = j.b_shared ? 0 : round256(j.b_b * per);
    return *sa + *sb + round256(j.c_b * per);
}

// Enqueues chunk i of a shard (its device is current): H2D of A (and B) on
// s_in, the product on s_comp, D2H of C on s_out, slots recycled through
// events only -- the host never waits here.  Returns PT_OK or an error.
int enqueue_chunk(const HostJob &j, const HostShard &sh, int i)
{
    HostPipeline &p = *sh.p;
    const int b0 = sh.first + i * sh.per;
    const int nb = (i + 1) * sh.per <= sh.count ? sh.per : sh.count - i * sh.per;
    if (nb <= 0)
        return PT_OK;
    size_t sa, sb;
    const size_t slot = slot_bytes_for(j, sh.per, &sa, &sb);
    const int k = i & 1;
    char *a_s = static_cast<char *>(p.stage) + k * slot, *b_s = a_s + sa, *c_s = b_s + sb;
    char *b_dev = static_cast<char *>(p.stage) + 2 * slot;
    auto err = [](cudaError_t e) {
        return fail(PT_RUNTIME, "Host matmul failed (CUDA error %d)", static_cast<int>(e));
    };
    cudaError_t e;
    if (i >= 2) {
        // slot reuse: the product of chunk i-2 has read its inputs and its
        // result has been copied out
        if ((e = cudaStreamWaitEvent(p.s_in, p.compute_done[k], 0)) != cudaSuccess ||
            (e = cudaStreamWaitEvent(p.s_comp, p.out_done[k], 0)) != cudaSuccess)
            return err(e);
    }
    if ((e = cudaMemcpyAsync(a_s, static_cast<const char *>(j.a) + j.a_b * b0, j.a_b * nb,
                             cudaMemcpyHostToDevice, p.s_in)) != cudaSuccess)
        return err(e);
    if (!j.b_shared &&
        (e = cudaMemcpyAsync(b_s, static_cast<const char *>(j.b) + j.b_b * b0, j.b_b * nb,
                             cudaMemcpyHostToDevice, p.s_in)) != cudaSuccess)
        return err(e);
    if ((e = cudaEventRecord(p.in_done[k], p.s_in)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(p.s_comp, p.in_done[k], 0)) != cudaSuccess)
        return err(e);
    pt_tensor ta, tb, tc;
    std::memset(&ta, 0, sizeof(ta));
    ta.data = a_s;
    ta.dtype = j.dtype;
    ta.ndims = 3;
    ta.shape[0] = nb; ta.shape[1] = j.M; ta.shape[2] = j.K;
    contiguous_strides(ta.shape, 3, ta.strides);
    tb = ta;
    if (j.b_shared) {
        tb.data = b_dev;
        tb.ndims = 2;
        tb.shape[0] = j.K; tb.shape[1] = j.N;
        contiguous_strides(tb.shape, 2, tb.strides);
    } else {
        tb.data = b_s;
        tb.shape[1] = j.K; tb.shape[2] = j.N;
        contiguous_strides(tb.shape, 3, tb.strides);
    }
    tc = ta;
    tc.data = c_s;
    tc.shape[1] = j.M; tc.shape[2] = j.N;
    contiguous_strides(tc.shape, 3, tc.strides);
    const int st = pt_tensor_matmul_into(&ta, &tb, &tc, j.flags, p.s_comp);
    if (st != PT_OK)
        return st;
    if ((e = cudaEventRecord(p.compute_done[k], p.s_comp)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(p.s_out, p.compute_done[k], 0)) != cudaSuccess ||
        (e = cudaMemcpyAsync(static_cast<char *>(j.c) + j.c_b * b0, c_s, j.c_b * nb,
                             cudaMemcpyDeviceToHost, p.s_out)) != cudaSuccess ||
        (e = cudaEventRecord(p.out_done[k], p.s_out)) != cudaSuccess)
        return err(e);
    return PT_OK;
}

// Shards the batch over `ndev` devices and runs their pipelines side by side
// from this thread; restores the caller's current device.
int host_matmul_devices(const void *a, const void *b, void *c, dtype_t dtype, int batches, int M,
                        int N, int K, int b_shared, const int *devices, int ndev, int chunks,
                        int flags)
{
    if (!supported_dtype(dtype, flags))
        return fail(PT_INVALID_ARGUMENT,
                    "matmul requires matching float32, float16 or bfloat16 operands");
    if (batches < 0 || M < 0 || N < 0 || K < 0 ||
        (!a && static_cast<long long>(M) * K != 0) || (!b && static_cast<long long>(K) * N != 0) ||
        (!c && static_cast<long long>(M) * N != 0))
        return fail(PT_INVALID_ARGUMENT, "Matrix multiplication failed - incompatible dimensions");
    if (ndev < 1 || ndev > kMaxPipeDevices || !devices)
        return fail(PT_INVALID_ARGUMENT, "host matmul needs between 1 and 64 devices");
    for (int g = 0; g < ndev; g++) {
        if (devices[g] < 0 || devices[g] >= kMaxPipeDevices)
            return fail(PT_INVALID_ARGUMENT, "host matmul device %d is out of range",
                        devices[g]);
        for (int h = 0; h < g; h++)
            if (devices[g] == devices[h])
                return fail(PT_INVALID_ARGUMENT, "host matmul devices must be distinct, got %d",
                            devices[g]);
    }
    if (batches == 0 || M == 0 || N == 0)
        return ok();
    HostJob j;
    j.a = a; j.b = b; j.c = c; j.dtype = dtype;
    j.M = M; j.N = N; j.K = K; j.b_shared = b_shared; j.flags = flags;
    const size_t es = element_size(dtype);
    j.a_b = static_cast<size_t>(M) * K * es;
    j.b_b = static_cast<size_t>(K) * N * es;
    j.c_b = static_cast<size_t>(M) * N * es;
    if (chunks < 1)
        chunks = 1;

    int prev = -1;
    cudaGetDevice(&prev);
    HostShard shards[kMaxPipeDevices];
    int nsh = 0, status = PT_OK, max_chunks = 0;
    const int base = batches / ndev, extra = batches % ndev;
    for (int g = 0, first = 0; g < ndev && status == PT_OK; g++) {
        HostShard &sh = shards[nsh];
        sh.device = devices[g];
        sh.first = first;
        sh.count = base + (g < extra ? 1 : 0);
        first += sh.count;
        if (sh.count == 0)
            continue;
        sh.chunks = chunks < sh.count ? chunks : sh.count;
        sh.per = (sh.count + sh.chunks - 1) / sh.chunks;
        size_t sa, sb;
        const size_t slot = slot_bytes_for(j, sh.per, &sa, &sb);
        cudaError_t e = cudaSetDevice(sh.device);
        if (e == cudaSuccess)
            e = prepare_pipeline(sh.device, 2 * slot + (b_shared ? round256(j.b_b) : 0));
        if (e == cudaSuccess && b_shared)
            e = cudaMemcpyAsync(static_cast<char *>(t_pipes[sh.device].stage) + 2 * slot, b, j.b_b,
                                cudaMemcpyHostToDevice, t_pipes[sh.device].s_comp);
        if (e != cudaSuccess) {
            status = fail(PT_RUNTIME, "Host matmul staging set-up failed (CUDA error %d)",
                          static_cast<int>(e));
            break;
        }
        sh.p = &t_pipes[sh.device];
        max_chunks = sh.chunks > max_chunks ? sh.chunks : max_chunks;
        nsh++;
    }
    // chunk i on every device before chunk i + 1, so all links copy at once
    for (int i = 0; i < max_chunks && status == PT_OK; i++)
        for (int g = 0; g < nsh && status == PT_OK; g++) {
            if (i >= shards[g].chunks)
                continue;
            const cudaError_t e = cudaSetDevice(shards[g].device);
            status = e == cudaSuccess ? enqueue_chunk(j, shards[g], i)
                                      : fail(PT_RUNTIME, "Host matmul failed (CUDA error %d)",
                                             static_cast<int>(e));
        }
    // drain every device's streams (also on the error path) before returning
    for (int g = 0; g < nsh; g++) {
        cudaSetDevice(shards[g].device);
        const cudaError_t e1 = cudaStreamSynchronize(shards[g].p->s_in);
        const cudaError_t e2 = cudaStreamSynchronize(shards[g].p->s_comp);
        const cudaError_t e3 = cudaStreamSynchronize(shards[g].p->s_out);
        const cudaError_t e = e1 != cudaSuccess ? e1 : (e2 != cudaSuccess ? e2 : e3);
        if (e != cudaSuccess && status == PT_OK)
            status = fail(PT_RUNTIME, "Host matmul failed (CUDA error %d)", static_cast<int>(e));
    }
    if (prev >= 0)
        cudaSetDevice(prev);
    return status == PT_OK ? ok() : status;
}

} // namespace

PT_API void pt_host_release(void)
{
    for (int d = 0; d < kMaxPipeDevices; d++)
        release_pipeline(t_pipes[d]);
}

PT_API int pt_host_matmul(const void *a, const void *b, void *c, dtype_t dtype, int batches, int M,
                          int N, int K, int b_shared, int chunks, int flags)
{
    int dev = -1;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return fail(PT_RUNTIME, "Host matmul staging set-up failed (CUDA error %d)",
                    static_cast<int>(e));
    return host_matmul_devices(a, b, c, dtype, batches, M, N, K, b_shared, &dev, 1, chunks,
                               flags);
}

PT_API int pt_host_matmul_sharded(const void *a, const void *b, void *c, dtype_t dtype,
                                  int batches, int M, int N, int K, int b_shared,
                                  const int *devices, int ndev, int chunks, int flags)
{
    return host_matmul_devices(a, b, c, dtype, batches, M, N, K, b_shared, devices, ndev, chunks,
                               flags);
}
