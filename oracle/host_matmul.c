/*
 * CPU oracle for the php-gpu-tensors matmul hot path -- TEST INFRASTRUCTURE.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load
 * this file's library, as the checker or as the timed CPU baseline; the
 * product library never links or calls it.
 *
 * Restates lcmialichi/php-gpu-tensors:
 *   - HostArray::matmul            src/contiguous_array_ce.c:1295-1343
 *   - batch offset rule            src/contiguous_array_ce.c:1280-1293
 *   - element read / result store  src/contiguous_array_ce.c:787-815
 *   - binary16/bfloat16 converters src/data_types.c:46-131 (IEEE 754 RNE)
 *   - shape rule                   src/tensor_shape.h:7-59
 * Pinned by tests/test_oracle.py against the reference's own converters and
 * shape rule (oracle/_ref, built from the reference sources when present) and
 * against the golden vectors in tests/golden/.
 */
#include "host_matmul.h"

#include <math.h>
#include <pthread.h>
#include <string.h>
#include <unistd.h>

static uint32_t float_bits(float v)
{
    uint32_t u;
    memcpy(&u, &v, sizeof u);
    return u;
}

static float bits_float(uint32_t u)
{
    float v;
    memcpy(&v, &u, sizeof v);
    return v;
}

/* IEEE 754 binary32 -> binary16, round to nearest, ties to even.  NaNs keep
 * the top ten payload bits (forced non-zero so they stay NaN), as the
 * reference converter does (src/data_types.c:53-58). */
uint16_t orc_float_to_float16_bits(float value)
{
    const uint32_t u = float_bits(value);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const int exp32 = (int)((u >> 23) & 0xffu);
    uint32_t frac = u & 0x7fffffu;

    if (exp32 == 0xff) {
        uint32_t payload = frac >> 13;
        if (frac != 0 && payload == 0)
            payload = 1;
        return (uint16_t)(sign | 0x7c00u | payload);
    }
    /* unbiased exponent, rebiased for binary16 */
    const int e16 = exp32 - 127 + 15;
    if (e16 >= 0x1f)
        return (uint16_t)(sign | 0x7c00u);
    if (e16 >= 1) {
        /* normal: keep 10 fraction bits, round on the 13 dropped bits; a
         * carry out of the fraction bumps the exponent (and may reach inf) */
        uint32_t q = ((uint32_t)e16 << 10) | (frac >> 13);
        const uint32_t rem = frac & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (q & 1u)))
            q += 1;
        return (uint16_t)(sign | q);
    }
    /* subnormal or underflow: value = 1.frac * 2^(exp32-127); the binary16
     * subnormal unit is 2^-24, so the significand (with hidden bit) is shifted
     * right by 14 - e16 places. */
    if (e16 < -10)
        return sign;
    const uint32_t sig = frac | 0x800000u;
    const int shift = 14 - e16;               /* 14 .. 24 */
    uint32_t q = sig >> shift;
    const uint32_t rem = sig & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u)))
        q += 1;
    return (uint16_t)(sign | q);
}

float orc_float16_bits_to_float(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t f = h & 0x3ffu;
    if (e == 0x1f)
        return bits_float(sign | 0x7f800000u | (f << 13));
    if (e != 0)
        return bits_float(sign | ((e + 112u) << 23) | (f << 13));
    if (f == 0)
        return bits_float(sign);
    /* subnormal: f * 2^-24 is exact in binary32 */
    const float mag = (float)f * 0x1p-24f;
    return sign ? -mag : mag;
}

/* binary32 -> bfloat16, RNE; NaNs become quiet NaNs with the top payload
 * (src/data_types.c:113-123). */
uint16_t orc_float_to_bfloat16_bits(float value)
{
    const uint32_t u = float_bits(value);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu) != 0)
        return (uint16_t)((u >> 16) | 0x40u);
    const uint32_t upper = u >> 16;
    const uint32_t lower = u & 0xffffu;
    uint32_t q = upper;
    if (lower > 0x8000u || (lower == 0x8000u && (upper & 1u)))
        q += 1;                               /* may carry into inf: correct */
    return (uint16_t)q;
}

float orc_bfloat16_bits_to_float(uint16_t h)
{
    return bits_float((uint32_t)h << 16);
}

void orc_floats_to_float16(const float *src, uint16_t *dst, size_t n)
{
    for (size_t i = 0; i < n; i++) dst[i] = orc_float_to_float16_bits(src[i]);
}

void orc_floats_to_bfloat16(const float *src, uint16_t *dst, size_t n)
{
    for (size_t i = 0; i < n; i++) dst[i] = orc_float_to_bfloat16_bits(src[i]);
}

void orc_float16_to_floats(const uint16_t *src, float *dst, size_t n)
{
    for (size_t i = 0; i < n; i++) dst[i] = orc_float16_bits_to_float(src[i]);
}

void orc_bfloat16_to_floats(const uint16_t *src, float *dst, size_t n)
{
    for (size_t i = 0; i < n; i++) dst[i] = orc_bfloat16_bits_to_float(src[i]);
}

int orc_broadcast_shape(const int *a, int a_dims, const int *b, int b_dims,
                        int *shape, int *ndims)
{
    const int n = a_dims > b_dims ? a_dims : b_dims;
    for (int axis = 0; axis < n; axis++) {
        /* right-align both shapes; a missing leading axis acts as extent 1 */
        const int ia = axis - (n - a_dims), ib = axis - (n - b_dims);
        const int ea = ia < 0 ? 1 : a[ia];
        const int eb = ib < 0 ? 1 : b[ib];
        if (ea != eb && ea != 1 && eb != 1)
            return 0;
        shape[axis] = ea == 1 ? eb : ea;
    }
    *ndims = n;
    return 1;
}

int orc_matmul_shape(const int *a, int a_dims, const int *b, int b_dims,
                     int *shape, int *ndims)
{
    if (a_dims < 2 || b_dims < 2 || a_dims > ORC_MAX_DIMS || b_dims > ORC_MAX_DIMS)
        return 0;
    if (a[a_dims - 1] != b[b_dims - 2])
        return 0;
    int batch_dims = 0;
    if (!orc_broadcast_shape(a, a_dims - 2, b, b_dims - 2, shape, &batch_dims))
        return 0;
    shape[batch_dims] = a[a_dims - 2];
    shape[batch_dims + 1] = b[b_dims - 1];
    *ndims = batch_dims + 2;
    return 1;
}

/* Element offset of flat batch index `batch` in operand t, for an output of
 * rank `ndims` and shape `shape`: broadcast (extent-1 or missing) axes add
 * nothing (src/contiguous_array_ce.c:1280-1293). */
static size_t batch_offset(const orc_tensor *t, size_t batch, const int *shape, int ndims)
{
    size_t off = 0;
    for (int d = ndims - 3; d >= 0; d--) {
        const size_t coord = batch % (size_t)shape[d];
        batch /= (size_t)shape[d];
        const int axis = d - (ndims - t->ndims);
        if (axis >= 0 && t->shape[axis] != 1)
            off += coord * t->strides[axis];
    }
    return off;
}

/* Element read widened to double (src/contiguous_array_ce.c:787-801). */
static double number_at(const orc_tensor *t, size_t off)
{
    switch (t->dtype) {
    case ORC_FLOAT32: return ((const float *)t->data)[off];
    case ORC_FLOAT64: return ((const double *)t->data)[off];
    case ORC_FLOAT16: return orc_float16_bits_to_float(((const uint16_t *)t->data)[off]);
    case ORC_BFLOAT16: return orc_bfloat16_bits_to_float(((const uint16_t *)t->data)[off]);
    default: return 0.0;
    }
}

static int dtype_ok_f32_path(int dt)
{
    return dt == ORC_FLOAT32 || dt == ORC_FLOAT16 || dt == ORC_BFLOAT16;
}

static size_t shape_total(const int *shape, int ndims)
{
    size_t n = 1;
    for (int i = 0; i < ndims; i++) n *= (size_t)shape[i];
    return n;
}

typedef struct {
    int shape[ORC_MAX_DIMS];
    int ndims;
    size_t rows, cols;
    int inner;
} plan_t;

static int make_plan(const orc_tensor *a, const orc_tensor *b, plan_t *p)
{
    if (!orc_matmul_shape(a->shape, a->ndims, b->shape, b->ndims, p->shape, &p->ndims))
        return 0;
    p->rows = (size_t)p->shape[p->ndims - 2];
    p->cols = (size_t)p->shape[p->ndims - 1];
    p->inner = a->shape[a->ndims - 1];
    return 1;
}

/* One output element of the reference loop: float operands, fmaf in k order
 * from zero (src/contiguous_array_ce.c:1320-1333). */
static float element_f32(const orc_tensor *a, const orc_tensor *b, const plan_t *p, size_t i)
{
    const size_t batch = i / p->cols / p->rows;
    const size_t oa = batch_offset(a, batch, p->shape, p->ndims) +
        (i / p->cols % p->rows) * a->strides[a->ndims - 2];
    const size_t ob = batch_offset(b, batch, p->shape, p->ndims) +
        (i % p->cols) * b->strides[b->ndims - 1];
    const size_t sak = a->strides[a->ndims - 1], sbk = b->strides[b->ndims - 2];
    float sum = 0.0f;
    for (int k = 0; k < p->inner; k++) {
        const float x = (float)number_at(a, oa + (size_t)k * sak);
        const float y = (float)number_at(b, ob + (size_t)k * sbk);
        sum = fmaf(x, y, sum);
    }
    return sum;
}

static double element_f64(const orc_tensor *a, const orc_tensor *b, const plan_t *p, size_t i)
{
    const size_t batch = i / p->cols / p->rows;
    const size_t oa = batch_offset(a, batch, p->shape, p->ndims) +
        (i / p->cols % p->rows) * a->strides[a->ndims - 2];
    const size_t ob = batch_offset(b, batch, p->shape, p->ndims) +
        (i % p->cols) * b->strides[b->ndims - 1];
    const size_t sak = a->strides[a->ndims - 1], sbk = b->strides[b->ndims - 2];
    double sum = 0.0;
    for (int k = 0; k < p->inner; k++)
        sum = fma(number_at(a, oa + (size_t)k * sak), number_at(b, ob + (size_t)k * sbk), sum);
    return sum;
}

/* Result store: the float sum cast to the operand dtype with RNE
 * (src/contiguous_array_ce.c:803-815 via cast_single_value). */
static void store(void *out, int dtype, size_t i, float v)
{
    if (dtype == ORC_FLOAT32) ((float *)out)[i] = v;
    else if (dtype == ORC_FLOAT16) ((uint16_t *)out)[i] = orc_float_to_float16_bits(v);
    else ((uint16_t *)out)[i] = orc_float_to_bfloat16_bits(v);
}

/* Work split for the multi-threaded variant: thread t computes a contiguous
 * block of output elements.  Each element's k-loop is the same as in the
 * single-threaded loop, so the result is bit-identical. */
typedef struct {
    const orc_tensor *a, *b;
    const plan_t *p;
    void *out;
    size_t out_base, lo, hi;
    int f64;
} job_t;

static void run_job(const job_t *j)
{
    if (j->f64) {
        for (size_t i = j->lo; i < j->hi; i++)
            ((double *)j->out)[i - j->out_base] = element_f64(j->a, j->b, j->p, i);
    } else {
        for (size_t i = j->lo; i < j->hi; i++)
            store(j->out, j->a->dtype, i - j->out_base, element_f32(j->a, j->b, j->p, i));
    }
}

static void *job_main(void *arg)
{
    run_job((const job_t *)arg);
    return NULL;
}

#define ORC_MAX_THREADS 256

static void run_range(const orc_tensor *a, const orc_tensor *b, const plan_t *p, void *out,
                      size_t out_base, size_t first, size_t count, int threads, int f64)
{
    if (threads > ORC_MAX_THREADS) threads = ORC_MAX_THREADS;
    if (threads <= 1 || count < (size_t)threads) {
        job_t j = {a, b, p, out, out_base, first, first + count, f64};
        run_job(&j);
        return;
    }
    pthread_t tid[ORC_MAX_THREADS];
    job_t jobs[ORC_MAX_THREADS];
    int started[ORC_MAX_THREADS];
    for (int t = 0; t < threads; t++) {
        jobs[t] = (job_t){a, b, p, out, out_base,
                          first + count * (size_t)t / (size_t)threads,
                          first + count * (size_t)(t + 1) / (size_t)threads, f64};
        started[t] = pthread_create(&tid[t], NULL, job_main, &jobs[t]) == 0;
        if (!started[t]) run_job(&jobs[t]);
    }
    for (int t = 0; t < threads; t++)
        if (started[t]) pthread_join(tid[t], NULL);
}

int orc_host_matmul(const orc_tensor *a, const orc_tensor *b, void *out,
                    int *out_shape, int *out_ndims, int threads)
{
    plan_t p;
    if (a->dtype != b->dtype || !dtype_ok_f32_path(a->dtype))
        return 0;
    if (!make_plan(a, b, &p))
        return 0;
    if (out_shape) memcpy(out_shape, p.shape, sizeof(int) * (size_t)p.ndims);
    if (out_ndims) *out_ndims = p.ndims;
    run_range(a, b, &p, out, 0, 0, shape_total(p.shape, p.ndims), threads, 0);
    return 1;
}

int orc_host_matmul_range(const orc_tensor *a, const orc_tensor *b, void *out,
                          size_t first, size_t count, int threads)
{
    plan_t p;
    if (a->dtype != b->dtype || !dtype_ok_f32_path(a->dtype))
        return 0;
    if (!make_plan(a, b, &p))
        return 0;
    const size_t total = shape_total(p.shape, p.ndims);
    if (first > total || count > total - first)
        return 0;
    run_range(a, b, &p, out, first, first, count, threads, 0);
    return 1;
}

int orc_host_matmul_f64(const orc_tensor *a, const orc_tensor *b, double *out,
                        int *out_shape, int *out_ndims, int threads)
{
    plan_t p;
    if (a->dtype != b->dtype ||
        (a->dtype != ORC_FLOAT64 && !dtype_ok_f32_path(a->dtype)))
        return 0;
    if (!make_plan(a, b, &p))
        return 0;
    if (out_shape) memcpy(out_shape, p.shape, sizeof(int) * (size_t)p.ndims);
    if (out_ndims) *out_ndims = p.ndims;
    run_range(a, b, &p, out, 0, 0, shape_total(p.shape, p.ndims), threads, 1);
    return 1;
}

int orc_host_matmul_f64_range(const orc_tensor *a, const orc_tensor *b, double *out,
                              size_t first, size_t count, int threads)
{
    plan_t p;
    if (a->dtype != b->dtype ||
        (a->dtype != ORC_FLOAT64 && !dtype_ok_f32_path(a->dtype)))
        return 0;
    if (!make_plan(a, b, &p))
        return 0;
    const size_t total = shape_total(p.shape, p.ndims);
    if (first > total || count > total - first)
        return 0;
    run_range(a, b, &p, out, first, first, count, threads, 1);
    return 1;
}

int orc_host_threads(void)
{
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) return 1;
    return n > ORC_MAX_THREADS ? ORC_MAX_THREADS : (int)n;
}
