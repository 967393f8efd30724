/*
 * hxq_affine.h -- affine group-quantized weights (B200 implementation).
 *
 * Drop-in for the reference header of the same name (hxq-native
 * include/hxq_affine.h).  Same struct layout (hxq_affine_tensor_t is 48 B
 * on x86-64) and the same function signatures.
 *
 *   W[o, i] = code[o, i] * scale[o, i / G] + offset[o, i / G]
 *   Y[n, o] = sum_g ( scale[o,g] * sum_{k in g} x[n,k] * code[o,k]
 *                   + offset[o,g] * sum_{k in g} x[n,k] ) + bias[o]
 *
 * The two *_ref functions are this library's CPU implementations.  The
 * GPU entry points run sm_100a kernels: an HBM-streaming dequant-GEMV for
 * small batches and a TMA + tcgen05 (TMEM accumulator) dequant-GEMM for
 * large ones, bias fused into the epilogue.
 */
#ifndef HXQ_AFFINE_H
#define HXQ_AFFINE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* reference include/hxq_affine.h:30-38.  For the GPU API every pointer is
 * device memory owned by the caller. */
typedef struct {
    uint8_t  *indices;        /* [out_features, in_features] codes          */
    float    *scales;         /* [out_features, n_groups]                   */
    float    *offsets;        /* [out_features, n_groups]                   */
    float    *bias;           /* [out_features] or NULL                     */
    uint32_t  out_features;
    uint32_t  in_features;
    uint32_t  group_size;     /* divides in_features (128 in practice)      */
} hxq_affine_tensor_t;

/* CPU fused matmul, sequential fp32 accumulation in n, o, g, k order.
 * x [N, in_f], output [N, out_f]; bias may be NULL.
 * reference include/hxq_affine.h:60-71, src/hxq_affine.c:23-66 */
void hxq_affine_group_matmul_ref(const float *x, const uint8_t *indices,
                                 const float *scales, const float *offsets,
                                 const float *bias, float *output, uint32_t N,
                                 uint32_t in_f, uint32_t out_f,
                                 uint32_t group_size);

/* CPU dense dequant, W[o,i] = code*scale + offset (rounded product, then
 * rounded add).  reference include/hxq_affine.h:86-94, hxq_affine.c:70-93 */
void hxq_affine_decompress_ref(const uint8_t *indices, const float *scales,
                               const float *offsets, float *output,
                               uint32_t out_f, uint32_t in_f,
                               uint32_t group_size);

/* GPU fused matmul on the library's stream; fp32 x [N, in_f] and fp32
 * output [N, out_f], all device pointers.  Returns 0 once the work is
 * enqueued, -1 on a CUDA error or an unsupported shape.  As in the
 * reference the call does not wait for the result: synchronise the
 * device (or use hxq_affine_group_matmul_async with your own stream).
 * reference include/hxq_affine.h:112-117, src/hxq_affine_cuda.cu:184-234 */
int hxq_affine_group_matmul(const float *d_x,
                            const hxq_affine_tensor_t *tensor,
                            float *d_output, uint32_t N);

/* Same with flat device pointers, for ctypes callers.  Exported but not
 * declared by the reference (src/hxq_affine_cuda.cu:252-294). */
int hxq_affine_matmul_flat(const float *d_x, const uint8_t *d_indices,
                           const float *d_scales, const float *d_offsets,
                           const float *d_bias, float *d_output, uint32_t N,
                           uint32_t in_f, uint32_t out_f, uint32_t group_size);

#ifdef __cplusplus
}
#endif

#if defined(__x86_64__) || defined(__aarch64__)
#ifdef __cplusplus
static_assert(sizeof(hxq_affine_tensor_t) == 48, "hxq_affine_tensor_t ABI");
#elif defined(__STDC_VERSION__) && __STDC_VERSION__ >= 201112L
_Static_assert(sizeof(hxq_affine_tensor_t) == 48, "hxq_affine_tensor_t ABI");
#endif
#endif

#endif /* HXQ_AFFINE_H */
