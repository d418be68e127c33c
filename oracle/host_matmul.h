/*
 * CPU oracle for the php-gpu-tensors matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product library links or calls
 * this code; only tests/, __graft_entry__.smoke() and the cpu_baseline leg of
 * bench.py load it, and only as the checker or as the timed CPU baseline.
 *
 * It restates, in plain C, the reference's HostArray::matmul
 * (src/contiguous_array_ce.c:1280-1343 of lcmialichi/php-gpu-tensors), the
 * shape rule (src/tensor_shape.h:7-59) and the IEEE binary16 / bfloat16
 * converters (src/data_types.c:46-131).  Parity is pinned against the
 * reference's own converters and shape rule (compiled from its sources into
 * oracle/_ref/ where the reference tree is present) and against the golden
 * vectors of its matmul tests (tests/golden/).
 */
#ifndef PT_ORACLE_HOST_MATMUL_H
#define PT_ORACLE_HOST_MATMUL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes: same numbering as the reference's dtype_t (src/data_types.h:8-27). */
enum {
    ORC_FLOAT32 = 0,
    ORC_FLOAT64 = 1,
    ORC_FLOAT16 = 11,
    ORC_BFLOAT16 = 12
};

#define ORC_MAX_DIMS 10

/* A strided operand: strides are in ELEMENTS, the view offset is folded into
 * data (src/tensor.h:49-79). */
typedef struct {
    const void *data;
    int dtype;
    int ndims;
    int shape[ORC_MAX_DIMS];
    size_t strides[ORC_MAX_DIMS];
} orc_tensor;

uint16_t orc_float_to_float16_bits(float value);
float orc_float16_bits_to_float(uint16_t value);
uint16_t orc_float_to_bfloat16_bits(float value);
float orc_bfloat16_bits_to_float(uint16_t value);

/* Bulk converters used by tests to build fp16/bf16 inputs from float32. */
void orc_floats_to_float16(const float *src, uint16_t *dst, size_t n);
void orc_floats_to_bfloat16(const float *src, uint16_t *dst, size_t n);
void orc_float16_to_floats(const uint16_t *src, float *dst, size_t n);
void orc_bfloat16_to_floats(const uint16_t *src, float *dst, size_t n);

/* src/tensor_shape.h:7-22 */
int orc_broadcast_shape(const int *a, int a_dims, const int *b, int b_dims,
                        int *shape, int *ndims);
/* src/tensor_shape.h:46-59: 1 = ok, 0 = rejected. */
int orc_matmul_shape(const int *a, int a_dims, const int *b, int b_dims,
                     int *shape, int *ndims);

/*
 * HostArray::matmul (src/contiguous_array_ce.c:1295-1343).
 * Returns 1 on success, 0 when the reference would throw
 * InvalidArgumentException (dtype mismatch, FP64, rank < 2, inner mismatch,
 * non-broadcastable batches).  out must hold prod(out_shape) elements of the
 * operand dtype, row-major contiguous.  threads <= 1 runs the single-threaded
 * reference loop; threads > 1 splits output elements across pthreads,
 * which leaves every element's k-loop (and therefore every bit) unchanged.
 */
int orc_host_matmul(const orc_tensor *a, const orc_tensor *b, void *out,
                    int *out_shape, int *out_ndims, int threads);

/*
 * Double-precision twin of the same loop (fma in k order, no rounding to
 * float).  Accepts FLOAT64 operands (the new FP64 scope, which the reference
 * rejects) and also FLOAT32/FLOAT16/BFLOAT16 operands, which it widens to
 * double: that is the "FP64 reference" the float paths are compared against.
 * out is double, row-major contiguous.
 */
int orc_host_matmul_f64(const orc_tensor *a, const orc_tensor *b, double *out,
                        int *out_shape, int *out_ndims, int threads);

/* Row-range sample of the same loop for the timed CPU baseline: computes
 * output elements [first, first + count) of the flat row-major result. */
int orc_host_matmul_range(const orc_tensor *a, const orc_tensor *b, void *out,
                          size_t first, size_t count, int threads);

/* Same sample of the double twin (double output). */
int orc_host_matmul_f64_range(const orc_tensor *a, const orc_tensor *b, double *out,
                              size_t first, size_t count, int threads);

/* Online host cores (capped at 256): the thread count the CPU baseline uses. */
int orc_host_threads(void);

#ifdef __cplusplus
}
#endif

#endif
