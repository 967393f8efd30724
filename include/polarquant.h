/*
 * polarquant.h -- PolarQuant KV-cache rotation (B200 implementation).
 *
 * Drop-in for the reference header of the same name (hxq-native
 * include/polarquant.h): same functions, error values and pq_layer_t
 * layout.
 *
 *   rotate:    head = head @ Q^T  (before scalar VQ of the KV cache)
 *   unrotate:  head = head @ Q    (after dequantization; Q is orthogonal)
 *
 * pq_generate_rotation runs on the host and gives the reference's matrix
 * bit for bit (MT19937 seeded like numpy.random.RandomState, polar
 * Box-Muller, fp32 Householder QR, sign of diag(R) made positive).
 * pq_rotate / pq_unrotate take host pointers as before and run the sm_100a
 * kernel of hxq_cuda_pq_rotate / hxq_cuda_pq_unrotate (hxq_cuda.h), which
 * keeps the reference's fp32 summation order, so results are bit-identical.
 * CUDA failures (and no GPU) are reported as PQ_ERR_ALLOC_FAILED.
 */
#ifndef POLARQUANT_H
#define POLARQUANT_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PQ_VERSION_MAJOR 0
#define PQ_VERSION_MINOR 1
#define PQ_VERSION_PATCH 0
#define PQ_VERSION_STRING "0.1.0"

/* reference include/polarquant.h:51-57 (values by declaration order) */
typedef enum {
    PQ_OK = 0,
    PQ_ERR_NULL_PTR,
    PQ_ERR_INVALID_DIM,
    PQ_ERR_ALLOC_FAILED,
    PQ_ERR_NOT_DIVISIBLE,
} pq_error_t;

/* Q [dim * dim] row-major; dim in [1, 1024].  reference polarquant.h:77. */
pq_error_t pq_generate_rotation(uint32_t dim, uint32_t seed, float *Q);

/* values [n_heads * head_dim] in place; Q [head_dim * head_dim].
 * reference polarquant.h:94-99, 114-119. */
pq_error_t pq_rotate(float *values, const float *Q, uint32_t n_heads, uint32_t head_dim);
pq_error_t pq_unrotate(float *values, const float *Q, uint32_t n_heads, uint32_t head_dim);

/* n_heads_hint > 0: entry_size / hint; else the first of head_dim 128, 64,
 * 32 that divides entry_size.  reference polarquant.h:132-137. */
pq_error_t pq_infer_head_geometry(uint32_t entry_size, uint32_t n_heads_hint, uint32_t *out_n_heads,
                                  uint32_t *out_head_dim);

/* reference polarquant.h:146-152 */
typedef struct {
    float   *Q;           /* [head_dim * head_dim], host memory */
    uint32_t head_dim;
    uint32_t n_heads;
    uint32_t seed;        /* base_seed + layer_idx */
    int      initialized;
} pq_layer_t;

pq_error_t pq_layer_init(pq_layer_t *layer, uint32_t head_dim, uint32_t n_heads, uint32_t base_seed,
                         uint32_t layer_idx);
pq_error_t pq_layer_rotate(pq_layer_t *layer, float *values);
pq_error_t pq_layer_unrotate(pq_layer_t *layer, float *values);
void pq_layer_free(pq_layer_t *layer);

#ifdef __cplusplus
}
#endif

#endif /* POLARQUANT_H */
