/*
 * hxq_oracle.c -- CPU oracle for the HXQ decompress and affine matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, in plain C99, the
 * algorithm of the reference C library (hxq-native: src/hxq.c and
 * src/hxq_affine.c) so that the CUDA path can be checked against it.
 * Only tests, the smoke check and the CPU-baseline leg of the benchmark
 * may load it; the product library never links or calls it.
 *
 * Every function names the reference lines it follows.  Floating-point
 * order is kept exactly: sequential fp32 accumulation, no FMA contraction
 * (build with -ffp-contract=off, as the reference's -O2 -std=c99 x86-64
 * build has no FMA), so outputs are bit-identical to the reference.
 *
 * Pinning: tests/test_oracle.py checks this file against the reference's
 * own known-answer tests (test/test_hxq.c, test/test_affine.c) and against
 * golden vectors produced by the reference library itself
 * (tests/golden/make_golden.py, built by oracle/Makefile into oracle/_ref).
 */
#include <stdint.h>
#include <stddef.h>
#include <math.h>

/* Error codes, same numbering as the reference enum (include/hxq.h:43-52). */
enum {
    ORC_OK = 0,
    ORC_ERR_NULL_PTR = 1,
    ORC_ERR_INVALID_K = 2,
    ORC_ERR_INVALID_DIM = 3,
    ORC_ERR_ALLOC_FAILED = 4,
    ORC_ERR_INDEX_OOB = 5,
    ORC_ERR_PACK_FORMAT = 6,
    ORC_ERR_SIDECAR_OOB = 7
};

/* Modes, same numbering as include/hxq.h:56-61. */
enum { ORC_SCALAR = 0, ORC_VQ2D_8BIT = 1, ORC_VQ2D_12BIT = 2, ORC_AFFINE = 3 };

/* 12-bit pair layout, include/hxq.h:245-252 (the code, not the :143 comment):
 * a = b0 << 4 | b1 >> 4 ; b = (b1 & 15) << 8 | b2. */
void orc_unpack12(const uint8_t *p, uint16_t *a, uint16_t *b)
{
    uint16_t hi = p[0], mid = p[1], lo = p[2];
    *a = (uint16_t)((hi << 4) | (mid >> 4));
    *b = (uint16_t)(((mid & 0x0Fu) << 8) | lo);
}

/* Inverse of the above, include/hxq.h:257-265. */
void orc_pack12(uint16_t a, uint16_t b, uint8_t *p)
{
    p[0] = (uint8_t)(a >> 4);
    p[1] = (uint8_t)(((a & 0x0Fu) << 4) | (b >> 8));
    p[2] = (uint8_t)(b & 0xFFu);
}

/* Pack an index stream laid out exactly as the reference decoder consumes
 * it (src/hxq.c:256-268): per row, ceil(pairs_per_row/2) byte triples; an
 * odd final pair gets a zero partner.  idx has out_f * (in_f/2) entries. */
size_t orc_pack_rows12(const uint16_t *idx, uint32_t out_f, uint32_t in_f,
                       uint8_t *packed)
{
    uint32_t ppr = in_f / 2u;
    size_t pos = 0;
    for (uint32_t r = 0; r < out_f; r++) {
        for (uint32_t p = 0; p < ppr; p += 2) {
            uint16_t a = idx[(size_t)r * ppr + p];
            uint16_t b = (p + 1 < ppr) ? idx[(size_t)r * ppr + p + 1] : 0;
            if (packed) orc_pack12(a, b, packed + pos);
            pos += 3;
        }
    }
    return pos;
}

/* Scalar VQ, src/hxq.c:218-235: out[i*in_f+j] = cb[idx[i*in_f+j]]. */
static void scalar_vq(const float *cb, const uint8_t *idx, uint32_t out_f,
                      uint32_t in_f, float *out)
{
    size_t n = (size_t)out_f * in_f;
    for (size_t g = 0; g < n; g++) out[g] = cb[idx[g]];
}

/* 12-bit 2D VQ, src/hxq.c:239-298.  The byte cursor runs continuously
 * across rows (:257,:268); a short buffer is PACK_FORMAT (:262), an index
 * >= k is INDEX_OOB (:271); only column pairs inside the row are written
 * (:277,:284).  Outputs written before an error stay written.
 * vdim must be 2 here: the reference reads cb[2*idx+1] regardless of vdim,
 * which for vdim == 1 reads past the codebook (undefined behaviour); the
 * oracle reports INVALID_DIM instead of reproducing it. */
static int vq2d_12bit(const float *cb, uint32_t k, uint32_t vdim,
                      const uint8_t *raw, size_t len, uint32_t out_f,
                      uint32_t in_f, float *out)
{
    if (vdim != 2) return ORC_ERR_INVALID_DIM;
    uint32_t ppr = in_f / 2u;
    size_t cur = 0;
    for (uint32_t r = 0; r < out_f; r++) {
        float *row = out + (size_t)r * in_f;
        for (uint32_t p = 0; p < ppr; p += 2) {
            if (cur + 3 > len) return ORC_ERR_PACK_FORMAT;
            uint16_t a, b;
            orc_unpack12(raw + cur, &a, &b);
            cur += 3;
            if (a >= k || b >= k) return ORC_ERR_INDEX_OOB;
            uint32_t ca = 2u * p, cb2 = ca + 2u;
            if (ca + 1u < in_f) { row[ca] = cb[2u * a]; row[ca + 1u] = cb[2u * a + 1u]; }
            if (cb2 + 1u < in_f) { row[cb2] = cb[2u * b]; row[cb2 + 1u] = cb[2u * b + 1u]; }
        }
    }
    return ORC_OK;
}

/* Affine dense dequant, src/hxq.c:302-326 and src/hxq_affine.c:70-93:
 * W[o,i] = (float)q * s + off, a rounded product then a rounded add. */
void orc_affine_decompress(const uint8_t *idx, const float *scales,
                           const float *offsets, float *out, uint32_t out_f,
                           uint32_t in_f, uint32_t gs)
{
    uint32_t ng = in_f / gs;
    for (uint32_t o = 0; o < out_f; o++)
        for (uint32_t g = 0; g < ng; g++) {
            float s = scales[(size_t)o * ng + g];
            float f = offsets[(size_t)o * ng + g];
            for (uint32_t kk = 0; kk < gs; kk++) {
                size_t i = (size_t)o * in_f + (size_t)g * gs + kk;
                float prod = (float)idx[i] * s;
                out[i] = prod + f;
            }
        }
}

/* Sidecar, src/hxq.c:330-350: in array order, entries with r < out_f and
 * c < in_f add v to out[r*in_f+c] and v*v to a sequential fp32 sum;
 * out-of-range entries are skipped and excluded.  Returns sqrtf(sum). */
float orc_apply_sidecar(const uint32_t *rows, const uint32_t *cols,
                        const float *vals, uint32_t nnz, uint32_t out_f,
                        uint32_t in_f, float *out)
{
    float sum = 0.0f;
    for (uint32_t s = 0; s < nnz; s++) {
        uint32_t r = rows[s], c = cols[s];
        float v = vals[s];
        if (r < out_f && c < in_f) {
            if (out) out[(size_t)r * in_f + c] += v;
            float sq = v * v;
            sum += sq;
        }
    }
    return sqrtf(sum);
}

/* The same confidence computed exactly: v*v is exact in double and the
 * double sum of at most a few million such terms is far below fp32
 * resolution.  Used to judge how far the reference's own fp32 order is
 * from the true value. */
double orc_sidecar_l2_exact(const uint32_t *rows, const uint32_t *cols,
                            const float *vals, uint32_t nnz, uint32_t out_f,
                            uint32_t in_f)
{
    double sum = 0.0;
    for (uint32_t s = 0; s < nnz; s++)
        if (rows[s] < out_f && cols[s] < in_f)
            sum += (double)vals[s] * (double)vals[s];
    return sqrt(sum);
}

/* Whole decompress, src/hxq.c:354-389: validate, reconstruct by mode,
 * then (only on success) apply the sidecar and set the confidence.
 * *l2 is written only on success, as t->sidecar_l2_norm is. */
int orc_decompress(int mode, const float *cb, uint32_t k, uint32_t vdim,
                   const uint8_t *idx, size_t idx_len, uint32_t out_f,
                   uint32_t in_f, const float *aff_s, const float *aff_o,
                   uint32_t gs, const uint32_t *sr, const uint32_t *sc,
                   const float *sv, uint32_t nnz, float *out, float *l2)
{
    if (!out || !idx) return ORC_ERR_NULL_PTR;
    if (mode != ORC_AFFINE && !cb) return ORC_ERR_NULL_PTR;
    int err;
    switch (mode) {
    case ORC_SCALAR:
        scalar_vq(cb, idx, out_f, in_f, out);
        err = ORC_OK;
        break;
    case ORC_VQ2D_12BIT:
        err = vq2d_12bit(cb, k, vdim, idx, idx_len, out_f, in_f, out);
        break;
    case ORC_AFFINE:
        if (!aff_s || !aff_o || gs == 0) return ORC_ERR_NULL_PTR;
        orc_affine_decompress(idx, aff_s, aff_o, out, out_f, in_f, gs);
        err = ORC_OK;
        break;
    default:
        return ORC_ERR_INVALID_DIM;
    }
    if (err != ORC_OK) return err;
    float norm = 0.0f;
    if (nnz > 0) norm = orc_apply_sidecar(sr, sc, sv, nnz, out_f, in_f, out);
    if (l2) *l2 = norm;
    return ORC_OK;
}

/* Fused affine group matmul, src/hxq_affine.c:23-66, loop order n, o, g, k:
 * partial and x_sum accumulate sequentially in fp32; acc += s*partial +
 * off*x_sum; bias added last.  Rows [n0, n1) of x only, so tests can
 * sample large batches. */
void orc_affine_matmul_rows(const float *x, const uint8_t *idx,
                            const float *scales, const float *offsets,
                            const float *bias, float *out, uint32_t n0,
                            uint32_t n1, uint32_t in_f, uint32_t out_f,
                            uint32_t gs)
{
    uint32_t ng = in_f / gs;
    for (uint32_t n = n0; n < n1; n++) {
        const float *xr = x + (size_t)n * in_f;
        for (uint32_t o = 0; o < out_f; o++) {
            const uint8_t *qr = idx + (size_t)o * in_f;
            float acc = 0.0f;
            for (uint32_t g = 0; g < ng; g++) {
                float s = scales[(size_t)o * ng + g];
                float off = offsets[(size_t)o * ng + g];
                float partial = 0.0f, xsum = 0.0f;
                for (uint32_t kk = 0; kk < gs; kk++) {
                    uint32_t i = g * gs + kk;
                    float xv = xr[i];
                    float prod = xv * (float)qr[i];
                    partial += prod;
                    xsum += xv;
                }
                float t1 = s * partial;
                float t2 = off * xsum;
                acc += t1 + t2;
            }
            if (bias) acc += bias[o];
            out[(size_t)n * out_f + o] = acc;
        }
    }
}

void orc_affine_matmul(const float *x, const uint8_t *idx, const float *scales,
                       const float *offsets, const float *bias, float *out,
                       uint32_t N, uint32_t in_f, uint32_t out_f, uint32_t gs)
{
    orc_affine_matmul_rows(x, idx, scales, offsets, bias, out, 0, N, in_f,
                           out_f, gs);
}

/* Dense naive matmul of the reference's tests (test/test_affine.c:51-65):
 * y[n,o] = sum_i x[n,i]*W[o,i] in ascending i, fp32, then + bias.  With
 * W from orc_decompress this is the CPU restatement of "decompress, then
 * multiply" used to check the fused VQ matmul. */
void orc_dense_matmul_rows(const float *x, const float *W, const float *bias,
                           float *out, uint32_t n0, uint32_t n1, uint32_t in_f,
                           uint32_t out_f)
{
    for (uint32_t n = n0; n < n1; n++)
        for (uint32_t o = 0; o < out_f; o++) {
            float acc = 0.0f;
            for (uint32_t i = 0; i < in_f; i++) {
                float prod = x[(size_t)n * in_f + i] * W[(size_t)o * in_f + i];
                acc += prod;
            }
            if (bias) acc += bias[o];
            out[(size_t)n * out_f + o] = acc;
        }
}

/* Same product accumulated in double, for judging fp32 rounding noise. */
void orc_dense_matmul_rows_f64(const float *x, const float *W, double *out,
                               uint32_t n0, uint32_t n1, uint32_t in_f,
                               uint32_t out_f)
{
    for (uint32_t n = n0; n < n1; n++)
        for (uint32_t o = 0; o < out_f; o++) {
            double acc = 0.0;
            for (uint32_t i = 0; i < in_f; i++)
                acc += (double)x[(size_t)n * in_f + i] * (double)W[(size_t)o * in_f + i];
            out[(size_t)(n - n0) * out_f + o] = acc;
        }
}

/* ---- Lloyd's algorithm, src/hxq_lloyd.c:41-308 ------------------------- */

/* Phase 1, src/hxq_lloyd.c:41-95: squared centroid norms, then per vector
 * its squared norm, each centroid's dot product (sums in component order)
 * and dist = w_sq + c_sq - 2 dot; the first strict minimum wins. */
void orc_lloyd_assign(const float *w, const float *cb, uint8_t *idx, size_t n, int k, int d)
{
    float csq[256];
    for (int j = 0; j < k; j++) {
        float s = 0.0f;
        for (int p = 0; p < d; p++) s += cb[j * d + p] * cb[j * d + p];
        csq[j] = s;
    }
    for (size_t i = 0; i < n; i++) {
        const float *wi = w + i * (size_t)d;
        float wsq = 0.0f;
        for (int p = 0; p < d; p++) wsq += wi[p] * wi[p];
        float best = 3.402823466e38f;
        int bj = 0;
        for (int j = 0; j < k; j++) {
            float dot = 0.0f;
            for (int p = 0; p < d; p++) dot += wi[p] * cb[j * d + p];
            float dist = wsq + csq[j] - 2.0f * dot;
            if (dist < best) {
                best = dist;
                bj = j;
            }
        }
        idx[i] = (uint8_t)bj;
    }
}

/* Phases 1-3 (src/hxq_lloyd.c:100-260), one thread: centroid sums in
 * double in vector order; mean = sum * (1 / count) rounded to float;
 * every dead centroid -> the member of the largest cluster (first maximum
 * count) farthest from its updated centroid (largest fp32 squared
 * distance, first index on ties) times 1.001f.  Returns the dead count. */
int orc_lloyd_reassign(const float *w, float *cb, uint8_t *idx, size_t n, int k, int d)
{
    double sums[256 * 8];
    int counts[256];
    orc_lloyd_assign(w, cb, idx, n, k, d);
    for (int j = 0; j < k * d; j++) sums[j] = 0.0;
    for (int j = 0; j < k; j++) counts[j] = 0;
    for (size_t i = 0; i < n; i++) {
        const int j = idx[i];
        counts[j]++;
        for (int p = 0; p < d; p++) sums[j * d + p] += (double)w[i * (size_t)d + p];
    }
    for (int j = 0; j < k; j++)
        if (counts[j] > 0) {
            const double inv = 1.0 / (double)counts[j];
            for (int p = 0; p < d; p++) cb[j * d + p] = (float)(sums[j * d + p] * inv);
        }
    int dead = 0, largest = 0;
    for (int j = 0; j < k; j++) {
        if (counts[j] == 0) dead++;
        if (counts[j] > counts[largest]) largest = j;
    }
    if (dead == 0) return 0;
    const float *lc = cb + largest * d;
    float maxd = -1.0f;
    size_t far = 0;
    for (size_t i = 0; i < n; i++) {
        if (idx[i] != (uint8_t)largest) continue;
        float dist = 0.0f;
        for (int p = 0; p < d; p++) {
            const float diff = w[i * (size_t)d + p] - lc[p];
            dist += diff * diff;
        }
        if (dist > maxd) {
            maxd = dist;
            far = i;
        }
    }
    for (int j = 0; j < k; j++)
        if (counts[j] == 0)
            for (int p = 0; p < d; p++) cb[j * d + p] = w[far * (size_t)d + p] * 1.001f;
    return dead;
}

/* ---- PolarQuant rotation, src/polarquant.c:249-300 --------------------- */

/* In place: transpose != 0: head <- head Q^T (pq_rotate); else head <- head
 * Q (pq_unrotate).  fp32 sums in k order from 0. */
void orc_pq_apply(float *values, const float *Q, size_t nvec, uint32_t hd, int transpose, float *tmp)
{
    for (size_t v = 0; v < nvec; v++) {
        float *head = values + v * hd;
        for (uint32_t j = 0; j < hd; j++) {
            float sum = 0.0f;
            for (uint32_t k = 0; k < hd; k++)
                sum += head[k] * (transpose ? Q[(size_t)j * hd + k] : Q[(size_t)k * hd + j]);
            tmp[j] = sum;
        }
        for (uint32_t j = 0; j < hd; j++) head[j] = tmp[j];
    }
}
