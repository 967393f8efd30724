// vq_tc_gemv.cu -- fused 12-bit VQ dequant-matmul for 1..16 bf16 tokens on
// the tensor cores: y[n, o] = sum_i x[n, i] W[o, i], W never written.
//
// The weights are the bf16 codebook pairs of the image's matmul tables
// (the weights the tcgen05 VQ GEMM uses): each packed 12-bit index names a
// pair of consecutive weights, and its bf16x2 codebook entry is exactly one
// A-fragment register of an m16n8k16 product (two consecutive K values of
// one row).  So a lane's A fragment is one 4-byte gather per register from a
// shared codebook, no conversion; the activations are bf16 already.
//   * Codebook: the 4096 pairs twice (32 KB, static shared): copy 0 holds
//     entry c at word c, copy 1 at word 4096 + (c ^ ((c >> 5) & 31)), a bank
//     independent of c's.  A warp-wide gather of 32 random entries from one
//     copy needs about 3.5 shared-memory wavefronts (the fullest of 32 banks);
//     with each lane's copy chosen when the image is built, about 2.
//   * Index stream: the image's GEMV stream holds, per pair, the byte offset
//     of the entry in the copy its lane reads (16 bits), in the matrix's
//     row-major pair order.  A producer thread copies each 16-row block, 1024
//     weights of K per stage (1 KB per row), as eight TMA tensor copies of
//     128 bytes x 16 rows (128-byte swizzle: the 16-byte units of row r XOR
//     r & 7); bytes past a row and rows past the image read as zero.
//   * Fragments: a consumer warp owns a 128-weight window of K of every
//     stage (two 64-weight chunks), one TMA box.  Lane (g, t) takes the
//     window's pairs [16t, 16t + 16) of rows g and g + 8: in chunk u pairs
//     [16t + 8u, +8), one 128-bit load per row (units 2t + u; rows g and
//     g ^ 1 of a quarter-warp have swizzle phases of different parity, so the
//     loads are free of bank conflicts).  Word jj of the load holds pairs 2jj
//     (low half: the A register of MMA column pair t) and 2jj + 1 (high half:
//     column pair t + 4) -- the K permutation, shared with the activations;
//     each half is directly the gather's byte offset.
//   * Activations: raw bf16 staged once per matrix in fragment order (within
//     each 128-weight window: chunk, then lane t, then its 16 weights; rows
//     of in_f + 8 so that the 8 tokens' 16-byte loads fall in distinct
//     banks); a lane's B fragments of a chunk are two 128-bit loads.  4
//     products per chunk, fp32 accumulation in two chains.
//   * Sidecar: the positions where the decoded weight differs from the
//     codebook pair carry d = bf16(final weight) - bf16(codebook value)
//     (image table, one entry per position, rows in order).  After a row
//     block's products, consumer warp w sums d x[n, col] over the positions
//     of rows 2w and 2w + 1, one row per half-warp (16 lanes strided over
//     the row's positions, activations from the staged copy, a transposed
//     butterfly over the half) and the sum is added to the output it
//     stores.  The result equals the tcgen05 VQ
//     GEMM's weights: bf16 of each final weight (|error| <= 2^-9 sum |x w|
//     per output, fp32 accumulation).
//   * The 8 warps' sums of a row block are added in warp order
//     (deterministic) and stored into every output buffer.
// Every mbarrier wait is bounded (about one second of clock) and reports
// through a status word.  Launched with programmatic stream serialization.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "hxq_cuda.h"
#include "hxq_cuda_internal.h"
#include "tc_pipe.cuh"

namespace hxq {
namespace vqtc {

using namespace pipe;

constexpr uint32_t kConsumers = 8;
constexpr uint32_t kThreads = (kConsumers + 1u) * 32u;
constexpr uint32_t kChunk = 64;                       // weights of K per chunk
constexpr uint32_t kWarpK = 2u * kChunk;              // per warp per stage
constexpr uint32_t kKC = kWarpK * kConsumers;         // 1024 per stage
constexpr uint32_t kRows = 16;
constexpr uint32_t kRowStageBytes = kKC / 2u * 2u;    // 1 KB of pair offsets per row per stage
constexpr uint32_t kStageBytes = kRows * kRowStageBytes;   // 16 KB
constexpr uint32_t kMaxStages = 8;
constexpr uint32_t kCbBytes = 2u * 4096u * 4u;         // two copies of the bf16x2 codebook
constexpr uint32_t kXPad = 8;                          // activation row pitch: in_f + 8
constexpr uint32_t kCsStride = 16;                     // sidecar sums per row (tokens)

__device__ uint32_t g_vqtc_err;
__shared__ __align__(16) uint32_t s_cb[2u * 4096u];    // the matrix's bf16x2 codebook, two copies

struct Job {
    CUtensorMap map;            // pair offsets [rows][in_f bytes], boxes of 128 B x 16 rows
    const uint32_t *cbh;        // bf16x2 pairs [4096]
    const uint16_t *x;          // bf16 [N][in_f]
    const uint32_t *prow;       // sidecar: first entry of each row (null: none)
    const uint32_t *e4;         // sidecar entries: column in bits 0..15
    const float *ed;            // sidecar weight differences
    uint32_t n_patch;
    OutPtrs out;
    uint32_t ldy, rows, in_f;   // in_f: the K length this job covers
    uint32_t k0, ldx;           // its first K column in the matrix; x's row stride (the matrix's in_f)
    uint32_t rb_begin;
    uint64_t w_begin;
};

struct Jobs {
    Job job[kMaxVqTcJobs];
    uint32_t n, N, total_rb, in_max, stages;
    uint64_t total_w;
};
static_assert(sizeof(Jobs) <= 4096, "kernel parameters are limited to 4 KB");

struct Layout {
    uint32_t bars, abort, xh, red, cs, total;
};

constexpr uint32_t kAlignSlack = 1024;
__host__ __device__ inline Layout layout(uint32_t S, uint32_t N, uint32_t in_f)
{
    Layout L;
    uint32_t o = S * kStageBytes;                 // 16 KB stages: 1024-byte aligned
    L.bars = o;  o += 2u * kMaxStages * 8u;
    L.abort = o; o += 16u;
    o = (o + 127u) & ~127u;
    L.xh = o;    o += N * (in_f + kXPad) * 2u;
    o = (o + 15u) & ~15u;
    L.red = o;   o += 2u * kConsumers * kRows * 8u * (N > 8u ? 2u : 1u) * 4u;
    L.cs = o;    o += 2u * kRows * kCsStride * 4u;
    L.total = o + kAlignSlack;
    return L;
}

__device__ __forceinline__ uint32_t rb_at(const Jobs &J, uint64_t w)
{
    if (w >= J.total_w) return J.total_rb;
    uint32_t j = 0;
    while (j + 1u < J.n && w >= J.job[j + 1u].w_begin) ++j;
    const Job &b = J.job[j];
    const uint64_t per = (uint64_t)kRows * b.in_f;
    const uint64_t r = (w - b.w_begin + per - 1u) / per;
    const uint32_t nrb = (b.rows + kRows - 1u) / kRows;
    return b.rb_begin + (uint32_t)(r < nrb ? r : nrb);
}

// Shared-memory byte offset, within a stage, of byte o (a multiple of 8) of
// the stage slice of row r: box o / 128 (2 KB each), line r, 16-byte unit
// XOR r & 7.
__device__ __forceinline__ uint32_t stage_off(uint32_t r, uint32_t o)
{
    const uint32_t b = o & 127u;
    return (o >> 7) * 2048u + r * 128u + ((((b >> 4) ^ (r & 7u)) << 4) | (b & 15u));
}

// Codebook entry at byte offset o (a multiple of 4 below 32 KB).
__device__ __forceinline__ uint32_t cb_at(uint32_t o)
{
    return *reinterpret_cast<const uint32_t *>(reinterpret_cast<const uint8_t *>(s_cb) + o);
}

// One 64-weight chunk: w[0..3] / h[0..3] are the lane's 8 pair offsets of
// rows g / g + 8 (two per word), xb its 32 activation bytes per token tile
// (four 8-byte B fragments); two accumulation chains.
template <int NT>
__device__ __forceinline__ void chunk(const uint32_t *w, const uint32_t *h, const uint4 (&xb)[NT][2],
                                      float (&d)[NT][4], float (&e)[NT][4])
{
    uint32_t ag[8], ah[8];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        ag[2 * jj] = cb_at(w[jj] & 0xFFFFu);
        ag[2 * jj + 1] = cb_at(w[jj] >> 16);
        ah[2 * jj] = cb_at(h[jj] & 0xFFFFu);
        ah[2 * jj + 1] = cb_at(h[jj] >> 16);
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
            const uint4 &q = xb[tt][jj >> 1];
            const uint32_t b0 = (jj & 1) ? q.z : q.x, b1 = (jj & 1) ? q.w : q.y;
            if (jj & 1) mma16816_bf16(e[tt], ag[2 * jj], ah[2 * jj], ag[2 * jj + 1], ah[2 * jj + 1], b0, b1);
            else mma16816_bf16(d[tt], ag[2 * jj], ah[2 * jj], ag[2 * jj + 1], ah[2 * jj + 1], b0, b1);
        }
    }
}

// Fragment-order position of activation column k: within its 128-weight
// window, (chunk u, lane t, weight r) for k = 32t + 16u + r.
__device__ __forceinline__ uint32_t xpos(uint32_t k)
{
    return (k & ~127u) | (((k >> 4) & 1u) << 6) | (((k >> 5) & 3u) << 4) | (k & 15u);
}

// Sidecar ranges of rows 2w, 2w + 1 of row block rb: entries [pr[0], pr[1])
// and [pr[1], pr[2]) (rows past the image: empty; no sidecar: all zero).  A
// K part walks its rows' whole ranges and adds the entries of its columns.
__device__ __forceinline__ void side_rows(const Jobs &J, uint32_t rb, uint32_t warp, uint32_t (&pr)[3])
{
    uint32_t j = 0;
    while (j + 1u < J.n && rb >= J.job[j + 1u].rb_begin) ++j;
    const Job &b = J.job[j];
    pr[0] = pr[1] = pr[2] = 0u;
    if (!b.prow) return;
    const uint32_t r0 = (rb - b.rb_begin) * kRows + 2u * warp;
#pragma unroll
    for (int q = 0; q < 3; ++q) pr[q] = r0 + (uint32_t)q < b.rows ? ldg_pinned(b.prow + r0 + q) : b.n_patch;
}

// sn[n] += d x[n, col] for the tokens n < N <= NC (x: staged bf16 rows of
// ldx in fragment order).
template <int NC>
__device__ __forceinline__ void side_add(float (&sn)[NC], uint32_t e4, float dl, const uint16_t *xs, uint32_t ldx,
                                         uint32_t N, uint32_t k0, uint32_t klen)
{
    // only the entries of this job's K range [k0, k0 + klen), whose
    // activations are the ones staged
    const uint32_t kc = (e4 & 0xFFFFu) - k0;
    if (kc >= klen) return;
    const uint16_t *xc = xs + xpos(kc);
#pragma unroll
    for (int n = 0; n < NC; ++n)
        if (NC == 1 || (uint32_t)n < N)
            sn[n] = fmaf(dl, __uint_as_float((uint32_t)xc[(uint32_t)n * ldx] << 16), sn[n]);
}

// Sum over each half-warp (lanes 0-15, 16-31) of sn[n] for the tokens
// n < N <= NC, in a fixed order (deterministic): a transposed butterfly
// exchanges halves of the NC values over lane bits 3, 2, ... (log2 NC steps,
// NC - 1 shuffles), then a plain butterfly over the bits left; token n ends
// in lanes n * (16 / NC) .. of the half, the first of which stores it.
template <int NC>
__device__ __forceinline__ void side_reduce_half(float (&sn)[NC], uint32_t N, uint32_t lane, float *out)
{
    float v[NC];
#pragma unroll
    for (int n = 0; n < NC; ++n) v[n] = sn[n];
    uint32_t token = 0;
#pragma unroll
    for (int cnt = NC, bit = 8; cnt > 1; cnt >>= 1, bit >>= 1) {
        const bool up = lane & (uint32_t)bit;
#pragma unroll
        for (int i = 0; i < cnt / 2; ++i)
            v[i] = (up ? v[i + cnt / 2] : v[i]) + __shfl_xor_sync(0xffffffffu, up ? v[i] : v[i + cnt / 2], bit);
        token += up ? (uint32_t)(cnt / 2) : 0u;
    }
#pragma unroll
    for (int bit = 8 / NC; bit >= 1; bit >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], bit);
    if ((lane & (16u / NC - 1u)) == 0 && token < N) out[token] = v[0];
}

// NT token tiles of 8 (1: up to 8 tokens, two CTAs per SM; 2: up to 16,
// one); NC >= N bounds the sidecar's per-token loops.
template <int NT, int NC>
__global__ void __launch_bounds__(kThreads, NT == 1 ? 2 : 1)
vq_tc_gemv_kernel(const __grid_constant__ Jobs J)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t S = J.stages;
    const Layout L = layout(S, J.N, J.in_max);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *empty = full + kMaxStages;
    volatile uint32_t *abort_flag = reinterpret_cast<volatile uint32_t *>(smem + L.abort);

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kConsumers);
        }
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const uint32_t rb0 = rb_at(J, J.total_w * blockIdx.x / gridDim.x);
    const uint32_t rb1 = rb_at(J, J.total_w * (blockIdx.x + 1u) / gridDim.x);

    if (warp == kConsumers) {
        if (lane == 0) {
            uint32_t it = 0, slot = 0, ph = 0, j = 0;
            bool ok = true;
            for (uint32_t rb = rb0; rb < rb1 && ok; ++rb) {
                while (j + 1u < J.n && rb >= J.job[j + 1u].rb_begin) ++j;
                const Job &b = J.job[j];
                const uint32_t row0 = (rb - b.rb_begin) * kRows;
                const uint32_t nst = (b.in_f + kKC - 1u) / kKC;
                const uint32_t kx = b.k0;
                for (uint32_t st = 0; st < nst; ++st, ++it) {
                    if (it >= S && !mbar_wait(empty + slot, ph ^ 1u, abort_flag, &g_vqtc_err)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full + slot, kStageBytes);   // the full boxes, zero fill included
                    for (uint32_t c = 0; c < kRowStageBytes / 128u; ++c)
                        tma_load_2d(smem + slot * kStageBytes + c * 2048u, &b.map, full + slot,
                                    (int32_t)(kx + st * kRowStageBytes + c * 128u), (int32_t)row0);
                    if (++slot == S) { slot = 0; ph ^= 1u; }
                }
            }
            for (uint32_t kt = it > S ? it - S : 0u; kt < it; ++kt)
                mbar_drain(full + kt % S, (kt / S) & 1u, &g_vqtc_err);
        }
        // No griddepcontrol.wait in the producer warp: it reads only the
        // image, and a wait blocked on lanes 1-31 would hold lane 0's copies
        // back until the previous kernel had finished.
        __syncwarp();
        return;
    }

    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t ct = threadIdx.x;
    const uint32_t g = lane >> 2, t = lane & 3u;   // MMA rows g and g + 8 are block rows g and g + 8
    const uint32_t N = J.N;
    constexpr uint32_t NTOK = 8u * NT;
    const uint32_t stage_a = smem_u32(smem), xh_a = smem_u32(smem + L.xh);
    float *red = reinterpret_cast<float *>(smem + L.red);
    float *csum = reinterpret_cast<float *>(smem + L.cs);
    const uint16_t *xs = reinterpret_cast<const uint16_t *>(smem + L.xh);
    uint32_t slot = 0, ph = 0, j = 0, rbi = 0, cur = 0xFFFFFFFFu;
    bool ok = true;
    // Sidecar, software-pipelined over row blocks: the ranges of a block's
    // rows are loaded during the block before, its first 64 entries per row
    // at its start; both are used after its products.
    uint32_t pr[3] = {0u, 0u, 0u};
    if (rb0 < rb1) side_rows(J, rb0, warp, pr);
    for (uint32_t rb = rb0; rb < rb1; ++rb, ++rbi) {
        while (j + 1u < J.n && rb >= J.job[j + 1u].rb_begin) ++j;
        const Job &b = J.job[j];
        const uint32_t in_f = b.in_f, k0 = b.k0;
        if (j != cur) {
            // the matrix's codebook, both copies (four entries per 16-byte
            // load: copy 0 in place, copy 1 at its permuted words), and its
            // activations (raw bf16 in fragment order, rows of in_f + 8)
            const uint4 *cs = reinterpret_cast<const uint4 *>(b.cbh);
            uint4 *cd = reinterpret_cast<uint4 *>(s_cb);
            for (uint32_t i = ct; i < 4096u / 4u; i += kConsumers * 32u) {
                const uint4 v = __ldg(cs + i);
                cd[i] = v;
                const uint32_t c0 = 4u * i, r = (c0 >> 5) & 31u;   // the same r for the four entries
                s_cb[4096u + (c0 ^ r)] = v.x;
                s_cb[4096u + ((c0 + 1u) ^ r)] = v.y;
                s_cb[4096u + ((c0 + 2u) ^ r)] = v.z;
                s_cb[4096u + ((c0 + 3u) ^ r)] = v.w;
            }
            // (the job's fields read once: the stores below could alias
            // them as far as the compiler knows)
            const uint32_t per_tok = in_f / 8u, ldx = b.ldx;
            const uint16_t *xsrc = b.x + k0;
            uint16_t *xh = reinterpret_cast<uint16_t *>(smem + L.xh);
            for (uint32_t p = ct; p < N * per_tok; p += kConsumers * 32u) {
                const uint32_t n = p / per_tok, k8 = p - n * per_tok;
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(xsrc + (size_t)n * ldx) + k8);
                *reinterpret_cast<uint4 *>(xh + (size_t)n * (in_f + kXPad) + xpos(k8 * 8u)) = v;
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");
            cur = j;
        }
        const uint32_t row0 = (rb - b.rb_begin) * kRows;
        const uint32_t rv = min(kRows, b.rows - row0);
        const uint32_t nst = (in_f + kKC - 1u) / kKC;
        // sidecar: half h of the warp takes row 2w + h, its 16 lanes the
        // row's entries lo + s16 + 16m (the first 64 loaded here)
        const uint32_t sh = lane >> 4, s16 = lane & 15u;
        uint32_t plo = sh ? pr[1] : pr[0], phi = sh ? pr[2] : pr[1];
        uint32_t pe[4] = {0u, 0u, 0u, 0u};
        float pd[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (b.prow) {
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const uint32_t p = plo + s16 + 16u * (uint32_t)m;
                if (p < phi) {
                    pe[m] = ldg_pinned(b.e4 + p);
                    pd[m] = ldg_pinned(b.ed + p);
                }
            }
        }
        uint32_t pn[3] = {0u, 0u, 0u};
        if (rb + 1u < rb1) side_rows(J, rb + 1u, warp, pn);
        // this lane's pair offsets of chunk u: unit 2t + u of row g's line in
        // box `warp` (row g + 8: eight lines, 1 KB, on)
        uint32_t wo[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) wo[u] = stage_off(g, warp * 128u + t * 32u + (uint32_t)u * 16u);
        uint32_t xa0[NT];
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
            const uint32_t n = min((uint32_t)tt * 8u + g, N - 1u);   // columns past N are not stored
            xa0[tt] = xh_a + 2u * (n * (in_f + kXPad) + warp * kWarpK + t * 16u);
        }
        float d[NT][4], e[NT][4];
#pragma unroll
        for (int tt = 0; tt < NT; ++tt)
#pragma unroll
            for (int u = 0; u < 4; ++u) { d[tt][u] = 0.0f; e[tt][u] = 0.0f; }
        for (uint32_t st = 0; st < nst; ++st) {
            if (ok && !warp_wait(full + slot, ph, abort_flag, &g_vqtc_err)) ok = false;
            const uint32_t kb = st * kKC + warp * kWarpK;
            if (ok && kb < in_f) {
                // in_f is a multiple of 128: both chunks of the warp are inside K
                const uint32_t sa = stage_a + slot * kStageBytes;
                uint32_t wg[8], wh[8];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const uint4 a = lds128(sa + wo[u]), c = lds128(sa + wo[u] + 1024u);
                    wg[4 * u] = a.x; wg[4 * u + 1] = a.y; wg[4 * u + 2] = a.z; wg[4 * u + 3] = a.w;
                    wh[4 * u] = c.x; wh[4 * u + 1] = c.y; wh[4 * u + 2] = c.z; wh[4 * u + 3] = c.w;
                }
                warp_release(empty + slot, lane);   // the stage's offsets are in registers
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    uint4 xb[NT][2];
#pragma unroll
                    for (int tt = 0; tt < NT; ++tt) {
                        const uint32_t xa = xa0[tt] + 2u * st * kKC + (uint32_t)u * 128u;
                        xb[tt][0] = lds128(xa);
                        xb[tt][1] = lds128(xa + 16u);
                    }
                    chunk<NT>(wg + 4 * u, wh + 4 * u, xb, d, e);
                }
            } else {
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(empty + slot);
            }
            if (++slot == S) { slot = 0; ph ^= 1u; }
        }
        float *cw = csum + (size_t)(rbi & 1u) * kRows * kCsStride;
        if (b.prow) {
            float sn[NC];
#pragma unroll
            for (int n = 0; n < NC; ++n) sn[n] = 0.0f;
#pragma unroll
            for (int m = 0; m < 4; ++m)
                if (plo + s16 + 16u * (uint32_t)m < phi) side_add<NC>(sn, pe[m], pd[m], xs, in_f + kXPad, N, k0, in_f);
            for (uint32_t p = plo + 64u + s16; p < phi; p += 16u)
                side_add<NC>(sn, __ldg(b.e4 + p), __ldg(b.ed + p), xs, in_f + kXPad, N, k0, in_f);
            side_reduce_half<NC>(sn, N, lane, cw + (2u * warp + sh) * kCsStride);
        }
#pragma unroll
        for (int q = 0; q < 3; ++q) pr[q] = pn[q];
        float *rd = red + (size_t)(rbi & 1u) * kConsumers * kRows * NTOK;
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
            const uint32_t n0 = (uint32_t)tt * 8u + 2u * t;
            rd[(warp * kRows + g) * NTOK + n0] = d[tt][0] + e[tt][0];
            rd[(warp * kRows + g) * NTOK + n0 + 1u] = d[tt][1] + e[tt][1];
            rd[(warp * kRows + g + 8u) * NTOK + n0] = d[tt][2] + e[tt][2];
            rd[(warp * kRows + g + 8u) * NTOK + n0 + 1u] = d[tt][3] + e[tt][3];
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        for (uint32_t idx = ct; idx < kRows * NTOK; idx += kConsumers * 32u) {
            const uint32_t row = idx / NTOK, n = idx - row * NTOK;
            if (ok && row < rv && n < N) {
                float v = 0.0f;
#pragma unroll
                for (uint32_t w = 0; w < kConsumers; ++w) v += rd[(w * kRows + row) * NTOK + n];
                const uint32_t o = row0 + row;
                if (b.prow) v += cw[row * kCsStride + n];
                for (uint32_t k = 0; k < b.out.n; ++k) b.out.y[k][(size_t)n * b.ldy + o] = v;
            }
        }
    }
}

struct Plan {
    uint32_t stages, per_sm;
    Layout L;
};

Plan plan_for(uint32_t N, uint32_t in_f)
{
    // two 8-token tiles: one CTA per SM (the kernel is built for one)
    for (uint32_t s = kMaxStages; s >= 2u && N <= 8u; --s) {
        const Layout L = layout(s, N, in_f);
        if (2u * (L.total + kCbBytes + 1024u) <= 233472u) return Plan{s, 2u, L};
    }
    for (uint32_t s = kMaxStages; s >= 2u; --s) {
        const Layout L = layout(s, N, in_f);
        if (L.total + kCbBytes <= 227u * 1024u) return Plan{s, 1u, L};
    }
    return Plan{0u, 0u, {}};
}

// K parts of a matrix whose activations do not fit the staging whole: the
// fewest parts (at most kMaxParts, each `len` columns, a multiple of 128;
// the last one shorter) whose staging leaves room for two stages.  Each part
// is a job of its own that stores its partial products [N][rows] to a
// scratch buffer; part_sum_kernel adds them in part order.  The split
// depends only on N and in_f, so a matrix sums the same way alone and in a
// batch.  Two parts at most: where three would be needed (4096 x 11008 from
// 14 tokens) the tcgen05 GEMM is faster (28 us against 32 at 16 tokens).
constexpr uint32_t kMaxParts = 2;
struct Split {
    uint32_t parts, len;
};
Split split_for(uint32_t N, uint32_t in_f)
{
    const uint32_t w = in_f / 128u;
    for (uint32_t P = 1; P <= kMaxParts && P <= w; ++P) {
        const uint32_t len = (w + P - 1u) / P * 128u;
        if (plan_for(N, len).stages != 0) return Split{(in_f + len - 1u) / len, len};
    }
    return Split{0u, 0u};
}

// y[n, o] = sum over the K parts, in part order, of their partial products
// (part p's [N][rows] at part + p * N * rows), stored into every output.
__global__ void part_sum_kernel(const float *__restrict__ part, const __grid_constant__ OutPtrs out, uint32_t N,
                                uint32_t rows, uint32_t ldy, uint32_t parts)
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t total = N * rows;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        float v = 0.0f;
        for (uint32_t p = 0; p < parts; ++p) v += __ldg(part + (size_t)p * total + i);
        const uint32_t n = i / rows, o = i - n * rows;
        for (uint32_t k = 0; k < out.n; ++k) out.y[k][(size_t)n * ldy + o] = v;
    }
}

// Partial-product scratch, one per (device, stream) so that launches on
// different streams never share it; grown on demand (the first split call of
// a size on a stream allocates, later ones -- under graph capture too --
// reuse it).
float *part_buffer(size_t floats, cudaStream_t s)
{
    struct Buf {
        float *p = nullptr;
        size_t cap = 0;
    };
    static std::mutex mu;
    static std::map<std::pair<int, cudaStream_t>, Buf> bufs;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    std::lock_guard<std::mutex> lk(mu);
    Buf &b = bufs[{dev, s}];
    if (b.cap < floats) {
        if (b.p) { cudaStreamSynchronize(s); cudaFree(b.p); }
        b.p = nullptr;
        b.cap = 0;
        if (cudaMalloc(&b.p, floats * sizeof(float)) != cudaSuccess) { cudaGetLastError(); return nullptr; }
        b.cap = floats;
    }
    return b.p;
}

}  // namespace vqtc

bool vq_tc_fits(const uint16_t *x, uint32_t N, uint32_t in_f)
{
    if (N == 0 || N > 16u || in_f == 0 || in_f % 128u != 0 || in_f > 65536u || ((uintptr_t)x & 15u)) return false;
    return vqtc::split_for(N, in_f).parts != 0;
}

uint32_t vq_tc_group(uint32_t n, const VqTcMatrix *m, uint32_t N)
{
    if (n == 0) return 0;
    const vqtc::Split s0 = vqtc::split_for(N, m[0].in_f);
    uint32_t in_max = s0.len, jobs = s0.parts, k = 1;
    vqtc::Plan P = vqtc::plan_for(N, in_max);
    for (; k < n; ++k) {
        const vqtc::Split q = vqtc::split_for(N, m[k].in_f);
        if (q.parts == 0 || jobs + q.parts > kMaxVqTcJobs) break;
        const uint32_t in2 = q.len > in_max ? q.len : in_max;
        const vqtc::Plan Q = vqtc::plan_for(N, in2);
        if (Q.per_sm < P.per_sm) break;   // a second launch costs less than half the CTAs
        in_max = in2;
        P = Q;
        jobs += q.parts;
    }
    return k;
}

int launch_vq_tc_gemv(uint32_t n, const VqTcMatrix *m, uint32_t N, int sms, cudaStream_t s, uint32_t *launched)
{
    using namespace vqtc;
    if (launched) *launched = 0;
    if (n == 0 || N == 0) return 0;
    if (n > kMaxVqTcJobs) return 1;
    Split sp[kMaxVqTcJobs];
    uint32_t n_jobs = 0;
    size_t part_floats = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const VqTcMatrix &a = m[i];
        if (!vq_tc_fits(a.x, N, a.in_f) || a.out.n == 0 || a.out.n > HXQ_CUDA_MAX_PEERS || a.ldy < a.rows) return 1;
        if (!a.tx || (a.n_patch && (!a.rb || !a.e4 || !a.ed))) return 1;
        sp[i] = split_for(N, a.in_f);
        n_jobs += sp[i].parts;
        if (sp[i].parts > 1u) part_floats += (size_t)sp[i].parts * N * a.rows;
    }
    if (n_jobs > kMaxVqTcJobs) return 1;
    float *part = nullptr;
    if (part_floats && !(part = part_buffer(part_floats, s))) return -1;
    Jobs J{};
    uint32_t rb = 0, in_max = 0, jn = 0;
    uint64_t w = 0;
    size_t po = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const VqTcMatrix &a = m[i];
        const uint64_t row_bytes = (uint64_t)a.in_f;   // one 16-bit offset per pair
        CUtensorMap map;
        std::memset(&map, 0, sizeof(map));
        if (!pipe::encode_bytes_2d(&map, a.tx, row_bytes, a.rows, kRows)) return 1;
        const uint32_t nrb = (a.rows + kRows - 1u) / kRows;
        for (uint32_t q = 0; q < sp[i].parts; ++q) {
            // part q: K columns [q len, q len + in_f) of the matrix
            Job &b = J.job[jn++];
            b.map = map;
            b.cbh = a.cbh; b.x = a.x; b.rows = a.rows;
            b.k0 = q * sp[i].len;
            b.in_f = a.in_f - b.k0 < sp[i].len ? a.in_f - b.k0 : sp[i].len;
            b.ldx = a.in_f;
            if (sp[i].parts > 1u) {
                b.out = OutPtrs{};
                b.out.y[0] = part + po + (size_t)q * N * a.rows;
                b.out.n = 1;
                b.ldy = a.rows;
            } else {
                b.out = a.out;
                b.ldy = a.ldy;
            }
            if (a.n_patch) { b.prow = a.rb; b.e4 = a.e4; b.ed = a.ed; b.n_patch = a.n_patch; }
            b.rb_begin = rb;
            b.w_begin = w;
            rb += nrb;
            w += (uint64_t)nrb * kRows * b.in_f;
            in_max = b.in_f > in_max ? b.in_f : in_max;
        }
        if (sp[i].parts > 1u) po += (size_t)sp[i].parts * N * a.rows;
    }
    J.n = n_jobs;
    J.N = N;
    J.total_rb = rb;
    J.total_w = w;
    J.in_max = in_max;
    const Plan P = plan_for(N, in_max);
    if (P.stages == 0) return 1;
    J.stages = P.stages;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    using KernelFn = void (*)(Jobs);
    static const KernelFn kernels[5] = {vq_tc_gemv_kernel<1, 1>, vq_tc_gemv_kernel<1, 2>, vq_tc_gemv_kernel<1, 4>,
                                        vq_tc_gemv_kernel<1, 8>, vq_tc_gemv_kernel<2, 16>};
    const int kv = N <= 1u ? 0 : N <= 2u ? 1 : N <= 4u ? 2 : N <= 8u ? 3 : 4;
    static std::atomic<uint64_t> configured[5];   // one bit per device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) { cudaGetLastError(); return -1; }
    if (!(configured[kv].load(std::memory_order_acquire) & (1ull << dev))) {
        if (cudaFuncSetAttribute(kernels[kv], cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(227u * 1024u - kCbBytes)) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
        configured[kv].fetch_or(1ull << dev, std::memory_order_acq_rel);
    }
    uint32_t grid = (uint32_t)(sms > 0 ? sms : 148) * P.per_sm;
    if (grid > rb) grid = rb;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(vqtc::kThreads);
    cfg.dynamicSmemBytes = P.L.total;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kernels[kv], J) != cudaSuccess) { cudaGetLastError(); return -1; }
    uint32_t nl = 1;
    // the split matrices' part sums, each launched to overlap the tail of
    // the kernel before it (its threads wait for that kernel's stores)
    po = 0;
    for (uint32_t i = 0; i < n; ++i) {
        if (sp[i].parts < 2u) continue;
        const uint32_t total = N * m[i].rows;
        uint32_t blocks = (total + 255u) / 256u;
        const uint32_t cap = (uint32_t)(sms > 0 ? sms : 148) * 4u;
        if (blocks > cap) blocks = cap;
        cudaLaunchConfig_t rc = {};
        rc.gridDim = dim3(blocks);
        rc.blockDim = dim3(256);
        rc.stream = s;
        rc.attrs = attr;
        rc.numAttrs = 1;
        if (cudaLaunchKernelEx(&rc, part_sum_kernel, (const float *)(part + po), m[i].out, N, m[i].rows, m[i].ldy,
                               sp[i].parts) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
        po += (size_t)sp[i].parts * N * m[i].rows;
        ++nl;
    }
    if (launched) *launched = nl;
    return 0;
}

uint32_t vq_tc_status_take()
{
    uint32_t v = 0;
    if (cudaMemcpyFromSymbol(&v, vqtc::g_vqtc_err, sizeof(v)) != cudaSuccess) { cudaGetLastError(); return 0xFFFFFFFFu; }
    if (v) {
        const uint32_t z = 0;
        cudaMemcpyToSymbol(vqtc::g_vqtc_err, &z, sizeof(z));
    }
    return v;
}

}  // namespace hxq
