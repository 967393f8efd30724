/* pq_host.c -- host side of PolarQuant: the rotation matrix, head geometry
 * and the per-layer context (reference hxq-native src/polarquant.c).
 *
 * The rotation must equal the reference's bit for bit, so that a KV cache
 * rotated by the reference unrotates here: the generator and the
 * factorisation below perform the reference's floating-point operations in
 * the reference's order (compiled, like it, as C99 without contraction).
 *   - MT19937 (Matsumoto-Nishimura), seeded as numpy.random.RandomState;
 *   - uniform doubles from 53 bits of two draws (27 + 26 bits);
 *   - Gaussians by the polar Box-Muller method, the second value of each
 *     pair cached (numpy's legacy normal generator);
 *   - Householder QR in fp32: each column's reflector from the column's
 *     norm with the sign of the diagonal element, applied to the trailing
 *     columns, stored scaled by its first element; Q accumulated from the
 *     identity by the reflectors in reverse order; columns of Q negated
 *     where R's diagonal is negative.
 * pq_rotate / pq_unrotate (polarquant.cu) run on the GPU.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "polarquant.h"

/* ---- MT19937 ----------------------------------------------------------- */

enum { MT_STATE = 624, MT_SHIFT = 397 };

typedef struct {
    uint32_t state[MT_STATE];
    int pos;
    int have_spare;      /* a second Gaussian of the last pair is waiting */
    double spare;
} pq_rng;

static void rng_seed(pq_rng *r, uint32_t seed)
{
    r->state[0] = seed;
    for (int i = 1; i < MT_STATE; ++i)
        r->state[i] = 1812433253u * (r->state[i - 1] ^ (r->state[i - 1] >> 30)) + (uint32_t)i;
    r->pos = MT_STATE;
    r->have_spare = 0;
    r->spare = 0.0;
}

static uint32_t twist_word(uint32_t hi_src, uint32_t lo_src, uint32_t far)
{
    const uint32_t y = (hi_src & 0x80000000u) | (lo_src & 0x7fffffffu);
    return far ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
}

static uint32_t rng_u32(pq_rng *r)
{
    if (r->pos >= MT_STATE) {
        uint32_t *s = r->state;
        for (int i = 0; i < MT_STATE; ++i)
            s[i] = twist_word(s[i], s[(i + 1) % MT_STATE], s[(i + MT_SHIFT) % MT_STATE]);
        r->pos = 0;
    }
    uint32_t y = r->state[r->pos++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

static double rng_uniform53(pq_rng *r)
{
    const uint32_t hi = rng_u32(r) >> 5, lo = rng_u32(r) >> 6;
    return ((double)hi * 67108864.0 + (double)lo) / 9007199254740992.0;
}

static double rng_gauss(pq_rng *r)
{
    if (r->have_spare) {
        r->have_spare = 0;
        return r->spare;
    }
    double u, v, q;
    do {
        u = 2.0 * rng_uniform53(r) - 1.0;
        v = 2.0 * rng_uniform53(r) - 1.0;
        q = u * u + v * v;
    } while (q >= 1.0 || q == 0.0);
    const double f = sqrt(-2.0 * log(q) / q);
    r->spare = f * u;
    r->have_spare = 1;
    return f * v;
}

/* ---- Householder QR (fp32) -------------------------------------------- */

/* a [n x n] row-major, overwritten; q [n x n] receives Q; rdiag [n] the
 * diagonal of R.  work: 2n floats. */
static void qr_householder(float *a, float *q, float *rdiag, float *work, int n)
{
    float *v = work, *tau = work + n;
    for (int c = 0; c < n; ++c) {
        float nsq = 0.0f;
        for (int i = c; i < n; ++i) {
            v[i] = a[i * n + c];
            nsq += v[i] * v[i];
        }
        const float nrm = sqrtf(nsq);
        tau[c] = 0.0f;
        if (nrm < 1e-30f) continue;
        v[c] += (a[c * n + c] >= 0.0f ? 1.0f : -1.0f) * nrm;
        float vsq = 0.0f;
        for (int i = c; i < n; ++i) vsq += v[i] * v[i];
        if (vsq < 1e-30f) continue;
        const float t = 2.0f / vsq;
        tau[c] = t;
        for (int col = c; col < n; ++col) {
            float dot = 0.0f;
            for (int i = c; i < n; ++i) dot += v[i] * a[i * n + col];
            for (int i = c; i < n; ++i) a[i * n + col] -= t * v[i] * dot;
        }
        for (int i = c + 1; i < n; ++i) a[i * n + c] = v[i] / v[c];
    }
    for (int i = 0; i < n; ++i) rdiag[i] = a[i * n + i];

    for (int i = 0; i < n * n; ++i) q[i] = 0.0f;
    for (int i = 0; i < n; ++i) q[i * n + i] = 1.0f;
    for (int c = n - 1; c >= 0; --c) {
        if (tau[c] == 0.0f) continue;
        v[c] = 1.0f;
        for (int i = c + 1; i < n; ++i) v[i] = a[i * n + c];
        float vsq = 0.0f;
        for (int i = c; i < n; ++i) vsq += v[i] * v[i];
        const float t = 2.0f / vsq;
        for (int col = 0; col < n; ++col) {
            float dot = 0.0f;
            for (int i = c; i < n; ++i) dot += v[i] * q[i * n + col];
            for (int i = c; i < n; ++i) q[i * n + col] -= t * v[i] * dot;
        }
    }
}

/* ---- public API -------------------------------------------------------- */

pq_error_t pq_generate_rotation(uint32_t dim, uint32_t seed, float *Q)
{
    if (!Q) return PQ_ERR_NULL_PTR;
    if (dim == 0 || dim > 1024) return PQ_ERR_INVALID_DIM;
    const size_t n = dim;
    float *a = (float *)malloc(n * n * sizeof(float));
    float *extra = (float *)malloc(3 * n * sizeof(float));   /* rdiag | work (2n) */
    pq_rng *r = (pq_rng *)malloc(sizeof(pq_rng));
    if (!a || !extra || !r) {
        free(a);
        free(extra);
        free(r);
        return PQ_ERR_ALLOC_FAILED;
    }
    rng_seed(r, seed);
    for (size_t i = 0; i < n * n; ++i) a[i] = (float)rng_gauss(r);
    qr_householder(a, Q, extra, extra + n, (int)dim);
    for (size_t c = 0; c < n; ++c)
        if (extra[c] < 0.0f)
            for (size_t i = 0; i < n; ++i) Q[i * n + c] = -Q[i * n + c];
    free(a);
    free(extra);
    free(r);
    return PQ_OK;
}

pq_error_t pq_infer_head_geometry(uint32_t entry_size, uint32_t n_heads_hint, uint32_t *out_n_heads,
                                  uint32_t *out_head_dim)
{
    if (!out_n_heads || !out_head_dim) return PQ_ERR_NULL_PTR;
    if (n_heads_hint > 0) {
        if (entry_size % n_heads_hint != 0) return PQ_ERR_NOT_DIVISIBLE;
        *out_n_heads = n_heads_hint;
        *out_head_dim = entry_size / n_heads_hint;
        return PQ_OK;
    }
    static const uint32_t dims[3] = {128u, 64u, 32u};
    for (int i = 0; i < 3; ++i) {
        if (entry_size % dims[i] == 0) {
            *out_n_heads = entry_size / dims[i];
            *out_head_dim = dims[i];
            return PQ_OK;
        }
    }
    return PQ_ERR_NOT_DIVISIBLE;
}

pq_error_t pq_layer_init(pq_layer_t *layer, uint32_t head_dim, uint32_t n_heads, uint32_t base_seed,
                         uint32_t layer_idx)
{
    if (!layer) return PQ_ERR_NULL_PTR;
    layer->head_dim = head_dim;
    layer->n_heads = n_heads;
    layer->seed = base_seed + layer_idx;
    layer->Q = (float *)malloc((size_t)head_dim * head_dim * sizeof(float));
    if (!layer->Q) return PQ_ERR_ALLOC_FAILED;
    const pq_error_t e = pq_generate_rotation(head_dim, layer->seed, layer->Q);
    if (e != PQ_OK) {
        free(layer->Q);
        layer->Q = NULL;
        return e;
    }
    layer->initialized = 1;
    return PQ_OK;
}

pq_error_t pq_layer_rotate(pq_layer_t *layer, float *values)
{
    if (!layer || !layer->initialized) return PQ_ERR_NULL_PTR;
    return pq_rotate(values, layer->Q, layer->n_heads, layer->head_dim);
}

pq_error_t pq_layer_unrotate(pq_layer_t *layer, float *values)
{
    if (!layer || !layer->initialized) return PQ_ERR_NULL_PTR;
    return pq_unrotate(values, layer->Q, layer->n_heads, layer->head_dim);
}

void pq_layer_free(pq_layer_t *layer)
{
    if (layer && layer->Q) {
        free(layer->Q);
        layer->Q = NULL;
        layer->initialized = 0;
    }
}
