/*
 * Exports the reference's header-only shape rule (src/tensor_shape.h, plain
 * C) under distinct names so tests can call it beside the oracle's
 * restatement.  Built only into oracle/_ref/libref.so, from the reference
 * tree, when that tree is present.
 */
#include "tensor_shape.h"

int ref_tensor_matmul_shape(const int *a, int a_dims, const int *b, int b_dims,
                            int *shape, int *ndims)
{
    return tensor_matmul_shape(a, a_dims, b, b_dims, shape, ndims);
}

int ref_tensor_broadcast_shape(const int *a, int a_dims, const int *b, int b_dims,
                               int *shape, int *ndims)
{
    return tensor_broadcast_shape(a, a_dims, b, b_dims, shape, ndims);
}

/* Bulk wrappers over the reference's own converters (src/data_types.c:46-131)
 * that move raw bits, so signaling-NaN payloads survive the comparison (a
 * float returned through ctypes is widened to a Python double, which quiets
 * it). */
#include <stdint.h>
#include <string.h>
#include "data_types.h"

void ref_bulk_half_to_float_bits(const uint16_t *src, uint32_t *dst, size_t n, int bf16)
{
    for (size_t i = 0; i < n; i++) {
        float f = bf16 ? bfloat16_bits_to_float(src[i]) : float16_bits_to_float(src[i]);
        memcpy(&dst[i], &f, sizeof f);
    }
}

void ref_bulk_float_bits_to_half(const uint32_t *src, uint16_t *dst, size_t n, int bf16)
{
    for (size_t i = 0; i < n; i++) {
        float f;
        memcpy(&f, &src[i], sizeof f);
        dst[i] = bf16 ? float_to_bfloat16_bits(f) : float_to_float16_bits(f);
    }
}
