/*
 * hxq_lloyd.h -- one iteration of Lloyd's algorithm on grouped VQ
 * codebooks (B200 implementation).
 *
 * Drop-in for the reference header of the same name (hxq-native
 * include/hxq_lloyd.h): same function signatures and error values.  The
 * reference runs on the host with OpenMP; here both functions take host
 * pointers as before, copy to the GPU, run the sm_100a kernels of
 * hxq_cuda_lloyd_reassign / hxq_cuda_lloyd_assign (hxq_cuda.h) and copy the
 * results back.  Without a usable GPU they return HXQ_LLOYD_ERR_CUDA
 * (additive; the reference never returns it).
 *
 *   1. assign:  index[i] = argmin_j ||w_i||^2 + ||c_j||^2 - 2 w_i . c_j
 *               (fp32, sums in component order, first minimum wins)
 *   2. update:  c_j = mean of the vectors assigned to j (counts > 0)
 *   3. reinit:  every centroid left without vectors moves to the member
 *               of the largest cluster farthest from its (updated) centroid,
 *               times 1.001
 */
#ifndef HXQ_LLOYD_H
#define HXQ_LLOYD_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HXQ_LLOYD_OK         0
#define HXQ_LLOYD_ERR_NULL  -1
#define HXQ_LLOYD_ERR_K     -2   /* k outside [1, 256]        */
#define HXQ_LLOYD_ERR_DIM   -3   /* d not one of 1, 2, 4, 8   */
#define HXQ_LLOYD_ERR_ALLOC -4
#define HXQ_LLOYD_ERR_CUDA  -5   /* additive: a CUDA call failed (or no GPU) */

/* weights [n_vectors * d] fp32, codebook [k * d] fp32 (updated), indices
 * [n_vectors] (written); n_dead (may be NULL) receives the number of
 * centroids that had no vectors.  reference include/hxq_lloyd.h:63-71. */
int hxq_lloyd_reassign(const float *weights, float *codebook, uint8_t *indices, size_t n_vectors, int k, int d,
                       int *n_dead);

/* Phase 1 only.  reference include/hxq_lloyd.h:86-93. */
int hxq_lloyd_assign_only(const float *weights, const float *codebook, uint8_t *indices, size_t n_vectors, int k,
                          int d);

#ifdef __cplusplus
}
#endif

#endif /* HXQ_LLOYD_H */
