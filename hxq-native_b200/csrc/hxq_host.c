/*
 * hxq_host.c -- C99 host side of the HXQ codec: descriptor lifecycle,
 * loaders, the CPU backend and the backend dispatch of the public API in
 * include/hxq.h and the CPU functions of include/hxq_affine.h.
 *
 * Behaviour (error codes, their order, ownership, what is written on
 * error) follows the reference library (hxq-native src/hxq.c and
 * src/hxq_affine.c); the CPU arithmetic keeps the reference's fp32 order so
 * both backends are bit-exact with it.  The CUDA backend is reached through
 * hxq_internal.h and never falls back to the CPU code below.
 */
#include "hxq.h"
#include "hxq_affine.h"
#include "hxq_cuda.h"
#include "hxq_internal.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- descriptor lifecycle (reference src/hxq.c:19-35) ------------------ */

hxq_error_t hxq_tensor_init(hxq_tensor_t *t)
{
    if (!t) return HXQ_ERR_NULL_PTR;
    hxqi_cuda_forget_tensor(t);
    memset(t, 0, sizeof(*t));
    return HXQ_OK;
}

void hxq_tensor_free(hxq_tensor_t *t)
{
    if (!t) return;
    hxqi_cuda_forget_tensor(t);
    free(t->codebook);
    free(t->indices_raw);
    free(t->sidecar_rows);
    free(t->sidecar_cols);
    free(t->sidecar_vals);
    free(t->affine_scales);
    free(t->affine_offsets);
    memset(t, 0, sizeof(*t));
}

/* malloc + memcpy of n bytes (n may be 0). */
static void *dup_bytes(const void *src, size_t n)
{
    void *p = malloc(n ? n : 1);
    if (p && n) memcpy(p, src, n);
    return p;
}

/* ---- loaders (reference src/hxq.c:39-214) ------------------------------ */

hxq_error_t hxq_tensor_load_codebook(hxq_tensor_t *t, const float *data,
                                     uint32_t k, uint32_t vdim)
{
    if (!t || !data) return HXQ_ERR_NULL_PTR;
    if (k != 256u && k != 4096u) return HXQ_ERR_INVALID_K;
    if (vdim < 1u || vdim > 2u) return HXQ_ERR_INVALID_DIM;
    float *cb = (float *)dup_bytes(data, (size_t)k * vdim * sizeof(float));
    if (!cb) return HXQ_ERR_ALLOC_FAILED;
    hxqi_cuda_forget_tensor(t);
    free(t->codebook);
    t->codebook = cb;
    t->k = k;
    t->vector_dim = vdim;
    return HXQ_OK;
}

hxq_error_t hxq_tensor_load_indices_8bit(hxq_tensor_t *t, const uint8_t *indices,
                                         uint32_t out_f, uint32_t in_f)
{
    if (!t || !indices) return HXQ_ERR_NULL_PTR;
    const size_t n = (size_t)out_f * in_f;
    uint8_t *buf = (uint8_t *)dup_bytes(indices, n);
    if (!buf) return HXQ_ERR_ALLOC_FAILED;
    hxqi_cuda_forget_tensor(t);
    free(t->indices_raw);
    t->indices_raw = buf;
    t->indices_len = n;
    t->out_features = out_f;
    t->in_features = in_f;
    t->mode = HXQ_SCALAR_VQ;
    return HXQ_OK;
}

hxq_error_t hxq_tensor_load_indices_12bit(hxq_tensor_t *t, const uint8_t *packed,
                                          size_t len, uint32_t out_f, uint32_t in_f)
{
    if (!t || !packed) return HXQ_ERR_NULL_PTR;
    uint8_t *buf = (uint8_t *)dup_bytes(packed, len);
    if (!buf) return HXQ_ERR_ALLOC_FAILED;
    hxqi_cuda_forget_tensor(t);
    free(t->indices_raw);
    t->indices_raw = buf;
    t->indices_len = len;
    t->out_features = out_f;
    t->in_features = in_f;
    t->mode = HXQ_VQ2D_12BIT;
    return HXQ_OK;
}

hxq_error_t hxq_tensor_load_sidecar(hxq_tensor_t *t, const uint32_t *rows,
                                    const uint32_t *cols, const float *vals,
                                    uint32_t nnz)
{
    if (!t) return HXQ_ERR_NULL_PTR;
    if (nnz == 0) {            /* count cleared, arrays kept (src/hxq.c:140-143) */
        hxqi_cuda_forget_tensor(t);
        t->sidecar_nnz = 0;
        return HXQ_OK;
    }
    if (!rows || !cols || !vals) return HXQ_ERR_NULL_PTR;
    uint32_t *r = (uint32_t *)dup_bytes(rows, (size_t)nnz * sizeof(uint32_t));
    uint32_t *c = (uint32_t *)dup_bytes(cols, (size_t)nnz * sizeof(uint32_t));
    float *v = (float *)dup_bytes(vals, (size_t)nnz * sizeof(float));
    if (!r || !c || !v) {
        free(r);
        free(c);
        free(v);
        return HXQ_ERR_ALLOC_FAILED;
    }
    hxqi_cuda_forget_tensor(t);
    free(t->sidecar_rows);
    free(t->sidecar_cols);
    free(t->sidecar_vals);
    t->sidecar_rows = r;
    t->sidecar_cols = c;
    t->sidecar_vals = v;
    t->sidecar_nnz = nnz;
    return HXQ_OK;
}

hxq_error_t hxq_tensor_load_affine(hxq_tensor_t *t, const uint8_t *indices,
                                   const float *scales, const float *offsets,
                                   uint32_t out_f, uint32_t in_f, uint32_t group_size)
{
    if (!t || !indices || !scales || !offsets) return HXQ_ERR_NULL_PTR;
    if (group_size == 0 || in_f % group_size != 0) return HXQ_ERR_INVALID_DIM;
    const size_t n = (size_t)out_f * in_f;
    const size_t ng = (size_t)out_f * (in_f / group_size);
    uint8_t *q = (uint8_t *)dup_bytes(indices, n);
    float *s = (float *)dup_bytes(scales, ng * sizeof(float));
    float *o = (float *)dup_bytes(offsets, ng * sizeof(float));
    if (!q || !s || !o) {
        free(q);
        free(s);
        free(o);
        return HXQ_ERR_ALLOC_FAILED;
    }
    hxqi_cuda_forget_tensor(t);
    free(t->indices_raw);
    free(t->affine_scales);
    free(t->affine_offsets);
    t->indices_raw = q;
    t->indices_len = n;
    t->affine_scales = s;
    t->affine_offsets = o;
    t->out_features = out_f;
    t->in_features = in_f;
    t->affine_group_size = group_size;
    t->mode = HXQ_AFFINE_G128;
    return HXQ_OK;
}

/* ---- CPU backend -------------------------------------------------------- */

static void cpu_scalar(const hxq_tensor_t *t, float *out)
{
    const size_t n = (size_t)t->out_features * t->in_features;
    const float *cb = t->codebook;
    const uint8_t *q = t->indices_raw;
    for (size_t i = 0; i < n; i++) out[i] = cb[q[i]];
}

/* Row r holds ceil((in_f/2)/2) triples; the byte cursor never resets, so the
 * stream is consumed front to back and checked triple by triple. */
static hxq_error_t cpu_vq12(const hxq_tensor_t *t, float *out)
{
    if (t->vector_dim != 2u) return HXQ_ERR_INVALID_DIM;  /* see hxq_cuda_rt.cu */
    const uint32_t in_f = t->in_features;
    const uint32_t pairs = in_f / 2u;
    const float *cb = t->codebook;
    const uint8_t *src = t->indices_raw;
    size_t at = 0;
    for (uint32_t r = 0; r < t->out_features; r++) {
        float *row = out + (size_t)r * in_f;
        for (uint32_t p = 0; p < pairs; p += 2u) {
            if (at + 3u > t->indices_len) return HXQ_ERR_PACK_FORMAT;
            uint16_t a, b;
            hxq_unpack_12bit_pair(src + at, &a, &b);
            at += 3u;
            if (a >= t->k || b >= t->k) return HXQ_ERR_INDEX_OOB;
            const uint32_t col = 2u * p;
            if (col + 1u < in_f) {
                row[col] = cb[2u * a];
                row[col + 1u] = cb[2u * a + 1u];
            }
            if (col + 3u < in_f) {
                row[col + 2u] = cb[2u * b];
                row[col + 3u] = cb[2u * b + 1u];
            }
        }
    }
    return HXQ_OK;
}

static void cpu_affine(const hxq_tensor_t *t, float *out)
{
    hxq_affine_decompress_ref(t->indices_raw, t->affine_scales, t->affine_offsets,
                              out, t->out_features, t->in_features,
                              t->affine_group_size);
}

/* In-range corrections in array order; fp32 running sum of squares. */
static float cpu_sidecar(const hxq_tensor_t *t, float *out)
{
    float sum = 0.0f;
    if (!t->sidecar_rows || !t->sidecar_cols || !t->sidecar_vals) return 0.0f;
    for (uint32_t s = 0; s < t->sidecar_nnz; s++) {
        const uint32_t r = t->sidecar_rows[s], c = t->sidecar_cols[s];
        if (r >= t->out_features || c >= t->in_features) continue;
        const float v = t->sidecar_vals[s];
        out[(size_t)r * t->in_features + c] += v;
        const float sq = v * v;
        sum += sq;
    }
    return sqrtf(sum);
}

static hxq_error_t cpu_decompress(hxq_tensor_t *t, float *out)
{
    hxq_error_t err;
    switch (t->mode) {
    case HXQ_SCALAR_VQ:
        cpu_scalar(t, out);
        err = HXQ_OK;
        break;
    case HXQ_VQ2D_12BIT:
        err = cpu_vq12(t, out);
        break;
    case HXQ_AFFINE_G128:
        if (!t->affine_scales || !t->affine_offsets || t->affine_group_size == 0)
            return HXQ_ERR_NULL_PTR;
        cpu_affine(t, out);
        err = HXQ_OK;
        break;
    default:
        return HXQ_ERR_INVALID_DIM;
    }
    if (err != HXQ_OK) return err;
    t->sidecar_l2_norm = 0.0f;
    if (t->sidecar_nnz > 0) t->sidecar_l2_norm = cpu_sidecar(t, out);
    return HXQ_OK;
}

/* NULL checks of src/hxq.c:358-361. */
static hxq_error_t check_tensor(const hxq_tensor_t *t)
{
    if (!t->indices_raw) return HXQ_ERR_NULL_PTR;
    if (t->mode != HXQ_AFFINE_G128 && !t->codebook) return HXQ_ERR_NULL_PTR;
    return HXQ_OK;
}

static hxq_error_t gpu_into_device(hxq_tensor_t *t, float *d_out)
{
    float l2 = 0.0f;
    hxq_error_t err = hxqi_cuda_decompress(t, d_out, 0, &l2);
    if (err == HXQ_OK) t->sidecar_l2_norm = l2;
    return err;
}

/* ---- public decompress entry points ------------------------------------ */

hxq_error_t hxq_tensor_decompress(hxq_tensor_t *t, float *output)
{
    if (!t || !output) return HXQ_ERR_NULL_PTR;
    hxq_error_t err = check_tensor(t);
    if (err != HXQ_OK) return err;
    if (hxqi_cuda_ptr_is_device(output)) return gpu_into_device(t, output);
    return cpu_decompress(t, output);
}

/* Host buffer growth exactly as src/hxq.c:400-413. */
static hxq_error_t grow_host(hxq_shared_buffer_t *buf, size_t needed)
{
    if (needed > buf->capacity) {
        float *nd = (float *)realloc(buf->data, needed * sizeof(float));
        if (!nd) return HXQ_ERR_ALLOC_FAILED;
        buf->data = nd;
        buf->capacity = needed;
    }
    if (needed > buf->high_water) buf->high_water = needed;
    return HXQ_OK;
}

hxq_error_t hxq_tensor_decompress_shared(hxq_tensor_t *t, hxq_shared_buffer_t *buf,
                                         float **out)
{
    if (!t || !buf || !out) return HXQ_ERR_NULL_PTR;
    const size_t needed = (size_t)t->out_features * t->in_features;
    hxq_error_t err;
    if (hxqi_cuda_is_arena(buf)) {
        if ((err = hxqi_cuda_arena_reserve(buf, needed)) != HXQ_OK) return err;
        if (needed > buf->high_water) buf->high_water = needed;
        if (!buf->data) return HXQ_ERR_NULL_PTR;
        if ((err = check_tensor(t)) != HXQ_OK) return err;
        if ((err = gpu_into_device(t, buf->data)) != HXQ_OK) return err;
    } else {
        if ((err = grow_host(buf, needed)) != HXQ_OK) return err;
        if (!buf->data) return HXQ_ERR_NULL_PTR;
        if ((err = check_tensor(t)) != HXQ_OK) return err;
        if ((err = cpu_decompress(t, buf->data)) != HXQ_OK) return err;
    }
    *out = buf->data;
    return HXQ_OK;
}

hxq_error_t hxq_shared_buffer_init(hxq_shared_buffer_t *buf, size_t initial_capacity)
{
    if (!buf) return HXQ_ERR_NULL_PTR;
    hxqi_cuda_arena_forget(buf);
    buf->data = (float *)calloc(initial_capacity, sizeof(float));
    if (!buf->data && initial_capacity > 0) return HXQ_ERR_ALLOC_FAILED;
    buf->capacity = initial_capacity;
    buf->high_water = 0;
    return HXQ_OK;
}

void hxq_shared_buffer_free(hxq_shared_buffer_t *buf)
{
    if (!buf) return;
    if (hxqi_cuda_is_arena(buf)) {
        hxqi_cuda_arena_release(buf);
        return;
    }
    free(buf->data);
    buf->data = NULL;
    buf->capacity = 0;
    buf->high_water = 0;
}

hxq_error_t hxq_dequant(hxq_tensor_t *tensor, hxq_shared_buffer_t *buf,
                        hxq_backend_t backend, hxq_result_t *result)
{
    if (!tensor || !buf || !result) return HXQ_ERR_NULL_PTR;
    const int arena = hxqi_cuda_is_arena(buf);
    int use_cuda;
    switch (backend) {
    case HXQ_BACKEND_AUTO: use_cuda = arena; break;
    case HXQ_BACKEND_CPU:
        if (arena) return HXQ_ERR_INVALID_ARG;  /* the CPU cannot write HBM */
        use_cuda = 0;
        break;
    case HXQ_BACKEND_CUDA: use_cuda = 1; break;
    default: return HXQ_ERR_BACKEND_UNAVAILABLE;
    }

    hxq_error_t err;
    float *out = NULL;
    if (!use_cuda || arena) {
        err = hxq_tensor_decompress_shared(tensor, buf, &out);
        if (err != HXQ_OK) return err;
    } else {
        /* CUDA backend with a host buffer: grow it as the reference does,
         * compute on the GPU, copy the weights back. */
        const size_t needed = (size_t)tensor->out_features * tensor->in_features;
        if ((err = grow_host(buf, needed)) != HXQ_OK) return err;
        if (!buf->data) return HXQ_ERR_NULL_PTR;
        if ((err = check_tensor(tensor)) != HXQ_OK) return err;
        float l2 = 0.0f;
        if ((err = hxqi_cuda_decompress_to_host(tensor, buf->data, &l2)) != HXQ_OK) return err;
        tensor->sidecar_l2_norm = l2;
        out = buf->data;
    }
    result->weights = out;
    result->confidence = tensor->sidecar_l2_norm;
    result->out_features = tensor->out_features;
    result->in_features = tensor->in_features;
    return HXQ_OK;
}

/* ---- affine CPU functions (reference src/hxq_affine.c) ----------------- */

void hxq_affine_group_matmul_ref(const float *x, const uint8_t *indices,
                                 const float *scales, const float *offsets,
                                 const float *bias, float *output, uint32_t N,
                                 uint32_t in_f, uint32_t out_f, uint32_t group_size)
{
    const uint32_t ng = in_f / group_size;
    for (uint32_t n = 0; n < N; n++) {
        const float *xr = x + (size_t)n * in_f;
        for (uint32_t o = 0; o < out_f; o++) {
            const uint8_t *qr = indices + (size_t)o * in_f;
            const float *so = scales + (size_t)o * ng;
            const float *fo = offsets + (size_t)o * ng;
            float acc = 0.0f;
            for (uint32_t g = 0; g < ng; g++) {
                const uint32_t base = g * group_size;
                float dot = 0.0f, xs = 0.0f;
                for (uint32_t k = 0; k < group_size; k++) {
                    const float xv = xr[base + k];
                    const float pr = xv * (float)qr[base + k];
                    dot += pr;
                    xs += xv;
                }
                const float a = so[g] * dot;
                const float b = fo[g] * xs;
                acc += a + b;
            }
            if (bias) acc += bias[o];
            output[(size_t)n * out_f + o] = acc;
        }
    }
}

void hxq_affine_decompress_ref(const uint8_t *indices, const float *scales,
                               const float *offsets, float *output,
                               uint32_t out_f, uint32_t in_f, uint32_t group_size)
{
    const uint32_t ng = in_f / group_size;
    for (uint32_t o = 0; o < out_f; o++)
        for (uint32_t g = 0; g < ng; g++) {
            const float s = scales[(size_t)o * ng + g];
            const float f = offsets[(size_t)o * ng + g];
            const size_t base = (size_t)o * in_f + (size_t)g * group_size;
            for (uint32_t k = 0; k < group_size; k++) {
                const float pr = (float)indices[base + k] * s;
                output[base + k] = pr + f;
            }
        }
}
