/*
 * hxq.h -- HXQ weight codec, public C99 API (B200 implementation).
 *
 * Drop-in for the reference header of the same name (hxq-native
 * include/hxq.h).  Every type, enum value, struct layout and function
 * signature here is ABI-identical to the reference so existing callers
 * relink without source changes; the static asserts at the bottom pin the
 * x86-64 layout (hxq_tensor_t 96 B with sidecar_l2_norm at offset 92,
 * hxq_shared_buffer_t 24 B, hxq_result_t 24 B).
 *
 * What changes is behind the API: HXQ_BACKEND_CUDA (and an output pointer
 * or shared buffer that lives in device memory) runs hand-written sm_100a
 * kernels; the CPU backend is this library's own C code.  There is no
 * silent fallback from CUDA to CPU.  Additive entry points (device arena,
 * bf16 output, batched and sharded decompress) are in hxq_cuda.h.
 *
 * Weight model (reference src/hxq.c:354-389):
 *     W[i][j] = codebook[index(i, j)] (+ sidecar delta at (i, j))
 * and the "confidence" of a decompress is sqrt(sum of squared in-range
 * sidecar deltas), stored into tensor->sidecar_l2_norm.
 */
#ifndef HXQ_H
#define HXQ_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* API level implemented (reference include/hxq.h:36-39). */
#define HXQ_VERSION_MAJOR 0
#define HXQ_VERSION_MINOR 4
#define HXQ_VERSION_PATCH 0
#define HXQ_VERSION_STRING "0.4.0"

/* Status codes; numbering fixed by the reference (include/hxq.h:43-52).
 * HXQ_ERR_SIDECAR_OOB is declared but, as in the reference, never
 * returned: out-of-range sidecar entries are skipped. */
typedef enum {
    HXQ_OK = 0,
    HXQ_ERR_NULL_PTR,
    HXQ_ERR_INVALID_K,
    HXQ_ERR_INVALID_DIM,
    HXQ_ERR_ALLOC_FAILED,
    HXQ_ERR_INDEX_OOB,
    HXQ_ERR_PACK_FORMAT,
    HXQ_ERR_SIDECAR_OOB,
} hxq_error_t;

/* Index encodings (reference include/hxq.h:56-61).  HXQ_VQ2D_8BIT is
 * declared only; decompressing it reports HXQ_ERR_INVALID_DIM. */
typedef enum {
    HXQ_SCALAR_VQ,      /* k = 256 codebook, one uint8 index per weight     */
    HXQ_VQ2D_8BIT,      /* reserved, not implemented                        */
    HXQ_VQ2D_12BIT,     /* k = 4096 x dim 2; two 12-bit indices per 3 bytes */
    HXQ_AFFINE_G128,    /* uint8 code * group scale + group offset          */
} hxq_mode_t;

/* Compressed tensor (reference include/hxq.h:65-96).  All pointers are
 * host memory owned by the descriptor (the loaders deep-copy).  The CUDA
 * backend keeps its device copy in a side table keyed by the descriptor
 * address; a loader call or hxq_tensor_free drops that copy. */
typedef struct {
    float       *codebook;          /* [k * vector_dim] fp32                 */
    uint32_t     k;                 /* 256 or 4096                           */
    uint32_t     vector_dim;        /* 1 (scalar) or 2 (pairs)               */

    uint8_t     *indices_raw;       /* packed index bytes                    */
    size_t       indices_len;       /* bytes in indices_raw                  */

    uint32_t    *sidecar_rows;      /* COO corrections, array order matters  */
    uint32_t    *sidecar_cols;
    float       *sidecar_vals;
    uint32_t     sidecar_nnz;

    uint32_t     out_features;      /* rows                                  */
    uint32_t     in_features;       /* columns                               */

    hxq_mode_t   mode;

    float       *affine_scales;     /* [out_features * n_groups]             */
    float       *affine_offsets;    /* [out_features * n_groups]             */
    uint32_t     affine_group_size;

    float        sidecar_l2_norm;   /* confidence of the last decompress     */
} hxq_tensor_t;

/* Materialisation buffer shared across tensors (reference
 * include/hxq.h:100-104).  capacity and high_water count floats.  When
 * created by hxq_shared_buffer_init it is host memory; when created by
 * hxq_cuda_arena_init (hxq_cuda.h) `data` is device memory and the buffer
 * is a device arena that the CUDA backend grows with cudaMalloc. */
typedef struct {
    float   *data;
    size_t   capacity;
    size_t   high_water;
} hxq_shared_buffer_t;

/* -- Descriptor lifecycle and loaders (reference src/hxq.c:19-214) ------ */

/* Zero the descriptor (mode becomes HXQ_SCALAR_VQ).  reference hxq.h:111 */
hxq_error_t hxq_tensor_init(hxq_tensor_t *t);

/* Copy a [k, vdim] fp32 codebook; k must be 256 or 4096, vdim 1 or 2.
 * reference hxq.h:121-126, hxq.c:39-61 */
hxq_error_t hxq_tensor_load_codebook(hxq_tensor_t *t, const float *data,
                                     uint32_t k, uint32_t vdim);

/* Copy out_f*in_f uint8 indices; sets mode HXQ_SCALAR_VQ.
 * reference hxq.h:134-139, hxq.c:65-87 */
hxq_error_t hxq_tensor_load_indices_8bit(hxq_tensor_t *t,
                                         const uint8_t *indices,
                                         uint32_t out_f, uint32_t in_f);

/* Copy `len` packed bytes; sets mode HXQ_VQ2D_12BIT.  Byte layout of a
 * pair (a, b): b0 = a[11:4], b1 = a[3:0] << 4 | b[11:8], b2 = b[7:0].
 * Each row holds ceil((in_f/2)/2) triples and rows follow each other with
 * no padding.  `len` is not checked here; a short buffer is reported by
 * the decompress as HXQ_ERR_PACK_FORMAT.
 * reference hxq.h:149-155, hxq.c:91-128 */
hxq_error_t hxq_tensor_load_indices_12bit(hxq_tensor_t *t,
                                          const uint8_t *packed, size_t len,
                                          uint32_t out_f, uint32_t in_f);

/* Copy codes/scales/offsets; sets mode HXQ_AFFINE_G128.  group_size must
 * divide in_f.  reference hxq.h:169-177, hxq.c:172-214 */
hxq_error_t hxq_tensor_load_affine(hxq_tensor_t *t, const uint8_t *indices,
                                   const float *scales, const float *offsets,
                                   uint32_t out_f, uint32_t in_f,
                                   uint32_t group_size);

/* Copy nnz COO corrections.  nnz == 0 clears the count and keeps the old
 * arrays, exactly as the reference does.  reference hxq.h:186-192,
 * hxq.c:132-168 */
hxq_error_t hxq_tensor_load_sidecar(hxq_tensor_t *t, const uint32_t *rows,
                                    const uint32_t *cols, const float *vals,
                                    uint32_t nnz);

/* Reconstruct all out_f*in_f weights into `output`, then add in-range
 * sidecar deltas in array order and set t->sidecar_l2_norm.  `output` may
 * be host memory (CPU backend) or device memory (CUDA backend; the call
 * returns with the weights written and the confidence stored).  On error
 * the output may be partly written and the confidence is left unchanged.
 * reference hxq.h:209-212, hxq.c:354-389 */
hxq_error_t hxq_tensor_decompress(hxq_tensor_t *t, float *output);

/* Decompress into a shared buffer, growing it to out_f*in_f floats if
 * needed, and return buf->data in *out.  A device arena stays on the
 * device.  reference hxq.h:223-227, hxq.c:393-420 */
hxq_error_t hxq_tensor_decompress_shared(hxq_tensor_t *t,
                                         hxq_shared_buffer_t *buf,
                                         float **out);

/* Release everything the descriptor owns (host and device copies) and
 * zero it.  reference hxq.h:232, hxq.c:25-35 */
void hxq_tensor_free(hxq_tensor_t *t);

/* Host shared buffer of `initial_capacity` zeroed floats.
 * reference hxq.h:236-237, hxq.c:424-442 */
hxq_error_t hxq_shared_buffer_init(hxq_shared_buffer_t *buf,
                                   size_t initial_capacity);
/* Frees a host buffer or a device arena, whichever `buf` is. */
void        hxq_shared_buffer_free(hxq_shared_buffer_t *buf);

/* -- 12-bit pair helpers (reference include/hxq.h:245-265) -------------- */

static inline void hxq_unpack_12bit_pair(const uint8_t *packed,
                                         uint16_t *idx_a, uint16_t *idx_b)
{
    uint16_t b0 = packed[0], b1 = packed[1], b2 = packed[2];
    *idx_a = (uint16_t)((b0 << 4) | (b1 >> 4));
    *idx_b = (uint16_t)(((b1 & 0x0Fu) << 8) | b2);
}

static inline void hxq_pack_12bit_pair(uint16_t idx_a, uint16_t idx_b,
                                       uint8_t *packed)
{
    packed[0] = (uint8_t)(idx_a >> 4);
    packed[1] = (uint8_t)(((idx_a & 0x0Fu) << 4) | (idx_b >> 8));
    packed[2] = (uint8_t)(idx_b & 0xFFu);
}

/* Confidence of the last successful decompress (reference hxq.h:274-276). */
static inline float hxq_get_sidecar_confidence(const hxq_tensor_t *t)
{
    return t->sidecar_l2_norm;
}

/* -- Meta-kernel (reference include/hxq.h:285-333, src/hxq.c:446-468) ---- */

typedef struct {
    float       *weights;        /* aliases buf->data until the next call  */
    float        confidence;     /* sidecar L2 norm of this decompress     */
    uint32_t     out_features;
    uint32_t     in_features;
} hxq_result_t;

typedef enum {
    HXQ_BACKEND_AUTO,     /* CUDA when `buf` is a device arena, else CPU   */
    HXQ_BACKEND_CPU,      /* this library's C path, host buffer            */
    HXQ_BACKEND_CUDA,     /* sm_100a kernels; never falls back to the CPU  */
    HXQ_BACKEND_METAL,    /* not provided: HXQ_ERR_BACKEND_UNAVAILABLE     */
    HXQ_BACKEND_VULKAN,   /* not provided: HXQ_ERR_BACKEND_UNAVAILABLE     */
} hxq_backend_t;

/* Decompress `tensor` into the shared buffer and report weights pointer,
 * confidence and shape.  With HXQ_BACKEND_CUDA and a host buffer the
 * weights are computed on the GPU and copied into the host buffer; with
 * a device arena they stay on the device.  The call returns with the
 * result complete (it synchronises its own stream). */
hxq_error_t hxq_dequant(hxq_tensor_t *tensor, hxq_shared_buffer_t *buf,
                        hxq_backend_t backend, hxq_result_t *result);

#ifdef __cplusplus
}
#endif

/* Layout pins for the drop-in ABI on LP64 targets. */
#if defined(__x86_64__) || defined(__aarch64__)
#ifdef __cplusplus
static_assert(sizeof(hxq_tensor_t) == 96, "hxq_tensor_t ABI");
static_assert(offsetof(hxq_tensor_t, mode) == 68, "hxq_tensor_t ABI");
static_assert(offsetof(hxq_tensor_t, sidecar_l2_norm) == 92, "hxq_tensor_t ABI");
static_assert(sizeof(hxq_shared_buffer_t) == 24, "hxq_shared_buffer_t ABI");
static_assert(sizeof(hxq_result_t) == 24, "hxq_result_t ABI");
#elif defined(__STDC_VERSION__) && __STDC_VERSION__ >= 201112L
_Static_assert(sizeof(hxq_tensor_t) == 96, "hxq_tensor_t ABI");
_Static_assert(offsetof(hxq_tensor_t, mode) == 68, "hxq_tensor_t ABI");
_Static_assert(offsetof(hxq_tensor_t, sidecar_l2_norm) == 92, "hxq_tensor_t ABI");
_Static_assert(sizeof(hxq_shared_buffer_t) == 24, "hxq_shared_buffer_t ABI");
_Static_assert(sizeof(hxq_result_t) == 24, "hxq_result_t ABI");
#endif
#endif

#endif /* HXQ_H */
