// affine_tc_gemv.cu -- affine group-quantized matmul for 1..16 bf16 tokens
// on the tensor cores, streaming the codes through shared memory.
//
//   Y[n,o] = sum_g ( s[o,g] * sum_{k in g} x[n,k]*q[o,k]
//                  + off[o,g] * sum_{k in g} x[n,k] ) + bias[o]
// (reference hxq-native src/hxq_affine.c:23-66).
//
// At a few tokens the matmul is a stream over the codes (one byte per
// weight); the work per code must stay well under the issue budget that
// HBM speed leaves (about 7 thread instructions per code on 148 SMs at
// 1.9 GHz).  Here the per-code work is one byte permute and one packed f16
// subtract per two codes, and m16n8k16 tensor-core products do the
// multiply-adds:
//   * codes: a producer thread copies each 16-row block of codes, 1024
//     codes of K per stage, with two TMA tensor copies per stage (a 3-D view
//     [rows][in_f / 128][128 B] of the matrix, box 16 rows x 4 x 128 B,
//     128-byte swizzle, so the 128-bit fragment loads are free of bank
//     conflicts; rows past the matrix read as zero) into a ring of
//     shared-memory stages; each row block's scales and offsets come in with
//     its first stage (cp.async.bulk) and are transposed once per row block
//     so that a warp reads a row pair's scale and offset with one 64-bit load;
//   * widening: [byte, 0x64] is the f16 1024 + byte, so a byte permute makes
//     two f16 values and one f16x2 subtract of 1024 leaves the code itself,
//     exactly, for every byte value;
//   * activations: each warp stages, once per matrix, the activations of
//     the K slices it owns (no cross-warp synchronisation), as f16: each
//     64-value chunk of a token scaled by a power of two 2^e that brings its
//     largest |x| into [2^14, 2^15), so every bf16 value converts exactly
//     (apart from ones 2^28 below the chunk's largest, which lose low bits as
//     f16 subnormals); 2^-e and the chunk's activation sum (fp32, unscaled)
//     are kept per (token, chunk);
//   * products: each consumer warp owns 128 codes of K of every stage (two
//     64-code chunks) and runs, per chunk and 8 tokens, four m16n8k16
//     products with fp32 accumulation in two independent chains, over a K
//     permutation shared by the code and activation fragments so that both
//     come from single 128-bit / 64-bit loads;
//   * groups: the group size is a power of two of at least 64, so a 64-code
//     chunk lies in one group; its fresh partial sums are scaled by 2^-e s[o,g] and it adds
//     off[o,g] times its activation sum;
//   * the 8 warps' partial sums of a row block are added in a fixed order,
//     bias fused into the store (into every output buffer).
// Products of f16 values are exact in fp32, so the only rounding is the
// fp32 accumulation.  Launched with programmatic stream serialization: the
// producer streams codes before the previous kernel has finished; the
// consumers wait (griddepcontrol.wait) before reading the activations.
// Every mbarrier wait is bounded (about one second of clock) and reports
// through a status word.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>

#include "hxq_cuda.h"
#include "hxq_cuda_internal.h"
#include "tc_pipe.cuh"

namespace hxq {
namespace tcg {

using namespace pipe;

constexpr uint32_t kConsumers = 8;                      // consumer warps
constexpr uint32_t kCThreads = kConsumers * 32u;        // consumer threads
constexpr uint32_t kThreads = kCThreads + 32u;          // + one producer warp
constexpr uint32_t kCtasPerSm = 2;                      // resident CTAs per SM
#define HXQ_TC_BAR_CONSUMERS "bar.sync 1, 256;"
constexpr uint32_t kChunk = 64;                         // codes of K per MMA chunk
constexpr uint32_t kWarpK = 2u * kChunk;                // codes of K per warp per stage
constexpr uint32_t kKC = kWarpK * kConsumers;           // 1024 codes of K per stage
constexpr uint32_t kRows = 16;                          // rows per block (MMA M)
constexpr uint32_t kHalfBytes = kRows * 512u;           // one box: [16 rows][4][128 B], swizzled
constexpr uint32_t kStageBytes = kRows * kKC;           // kKC / 512 boxes
constexpr uint32_t kMaxStages = 6;
constexpr uint32_t kSfStride = 2u * kRows + 2u;         // floats per group in the transposed scales

__device__ uint32_t g_tc_err;

struct Layout {
    uint32_t bars, abort, sbuf, sf, xh, xc, red, total;
};

// Shared memory (from a 1024-byte aligned base): stages [S][2 halves][16
// rows][4][128 B] | barriers full[S], empty[S], sdone | abort | scales and
// offsets as copied [2][16][ng] | transposed [ng][16 rows][s, off] (+2 pad) |
// f16 activations [N][in_f + 4] | per (token, 64-value chunk) {2^-e, sum} |
// reductions [2][8 warps][16][8 NT]
constexpr uint32_t kAlignSlack = 1024;
__host__ __device__ inline Layout layout(uint32_t S, uint32_t N, uint32_t nt, uint32_t ng, uint32_t in_f)
{
    Layout L;
    uint32_t o = S * kStageBytes;
    L.bars = o;   o += (2u * kMaxStages + 1u) * 8u;
    L.abort = o;  o += 8u;
    o = (o + 127u) & ~127u;
    L.sbuf = o;   o += 2u * kRows * ng * 4u;
    L.sf = o;     o += ng * kSfStride * 4u;
    o = (o + 127u) & ~127u;
    L.xh = o;     o += N * (in_f + 4u) * 2u;
    o = (o + 15u) & ~15u;
    L.xc = o;     o += N * (in_f / kChunk) * 8u;
    L.red = o;    o += 2u * kConsumers * kRows * 8u * nt * 4u;
    L.total = o + kAlignSlack;
    return L;
}

struct Job {
    CUtensorMap map;            // codes as [out_f][in_f / 128][128] bytes, box 16 x 4 x 128
    const uint16_t *x;          // bf16 activations [N][in_f]
    const uint8_t *codes;       // [out_f][in_f]
    const float *scales, *offsets, *bias;
    OutPtrs out;                // output o of token n at out.y[k][n * ldy + o]
    uint32_t in_f, out_f, gs, gs_shift, ng, ldy;
    uint32_t rb_begin;          // first row block of the job in the launch
    uint64_t w_begin;           // code weight (16 * in_f per row block) of the jobs before
};

struct Jobs {
    Job job[kMaxTcJobs];
    uint32_t n, N, total_rb, ng_max, in_max, stages;
    uint64_t total_w;
};

// Bytes 2i and 2i+1 of w as exact f16 values (f16 1024 + b, minus 1024).
template <int HI>
__device__ __forceinline__ uint32_t codes_f16x2(uint32_t w)
{
    const uint32_t h = __byte_perm(w, 0x64646464u, HI ? 0x4342u : 0x4140u);
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64006400u));
    return r;
}

__device__ __forceinline__ uint32_t f16x2_of(float lo, float hi)
{
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// First row block of the launch whose code weight starts at or after w.
__device__ __forceinline__ uint32_t rb_at(const Jobs &J, uint64_t w)
{
    if (w >= J.total_w) return J.total_rb;
    uint32_t j = 0;
    while (j + 1u < J.n && w >= J.job[j + 1u].w_begin) ++j;
    const Job &b = J.job[j];
    const uint64_t per = (uint64_t)kRows * b.in_f;
    const uint64_t r = (w - b.w_begin + per - 1u) / per;
    const uint32_t nrb = (b.out_f + kRows - 1u) / kRows;
    return b.rb_begin + (uint32_t)(r < nrb ? r : nrb);
}

__device__ __forceinline__ uint32_t group_of(uint32_t k, const Job &b)
{
    return b.gs_shift < 32u ? k >> b.gs_shift : k / b.gs;
}

// Stage, for one warp, the activations of the K slices it owns: chunks
// k0 = 1024 st + 128 warp + 64 u (u = 0, 1) of every token.  MERGE: the two
// chunks of a stage get one factor (the group size is a multiple of 128, so
// they also share the group).  A pass covers 4
// chunks of one token, 8 lanes per chunk, one 128-bit load (8 values) per
// lane; eight passes are in flight at a time (one round trip for a token of
// up to 16384 values).  Per chunk: the largest |x|
// and the sum over the 8 lanes (xor shuffles, a fixed tree), the power of
// two 2^e, the f16 values x 2^e into the activation rows, {2^-e, sum} into
// the chunk table.
template <bool MERGE>
__device__ void stage_x_warp(const Job &b, uint32_t N, uint8_t *smem, const Layout &L, uint32_t warp,
                             uint32_t lane)
{
    const uint32_t in_f = b.in_f, xs = in_f + 4u, nck = in_f / kChunk;
    const uint32_t nch = 2u * ((in_f + kKC - 1u) / kKC);     // chunk slots of this warp
    const uint32_t ncg = (nch + 3u) / 4u;                     // passes per token
    const uint32_t total = N * ncg;
    const uint32_t c8 = lane >> 3, j = lane & 7u;
    uint16_t *xh = reinterpret_cast<uint16_t *>(smem + L.xh);
    float2 *xc = reinterpret_cast<float2 *>(smem + L.xc);
    for (uint32_t q0 = 0; q0 < total; q0 += 4u) {
        uint4 v[4];
        uint32_t nn[4], kk[4];
        bool val[4];
#pragma unroll
        for (uint32_t r = 0; r < 4u; ++r) {
            const uint32_t qq = q0 + r;
            const uint32_t n = qq / ncg, c = 4u * (qq - n * ncg) + c8;
            const uint32_t k0 = (c >> 1) * kKC + warp * kWarpK + (c & 1u) * kChunk;
            nn[r] = n;
            kk[r] = k0;
            val[r] = qq < total && c < nch && k0 < in_f;
            v[r] = val[r] ? __ldg(reinterpret_cast<const uint4 *>(b.x + (size_t)n * in_f + k0) + j)
                          : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (uint32_t r = 0; r < 4u; ++r) {
            const uint32_t w[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
            float sum = 0.0f;
            uint32_t m = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                sum += __uint_as_float(w[e] << 16);
                sum += __uint_as_float(w[e] & 0xFFFF0000u);
                const uint32_t a = w[e] & 0x7FFF7FFFu;
                m = max(m, max(a & 0xFFFFu, a >> 16));
            }
#pragma unroll
            for (uint32_t o = 1; o < 8u; o <<= 1) {
                sum += __shfl_xor_sync(0xffffffffu, sum, o);
                m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
            }
            // merged: the warp's two chunks of a stage (lanes 16i..16i+7 and
            // 16i+8..16i+15) share one factor, from the larger of their maxima
            if (MERGE) m = max(m, __shfl_xor_sync(0xffffffffu, m, 8));
            if (!val[r]) continue;
            // 2^e brings the largest |x| (bf16 bits m, exponent field m >> 7) into [2^14, 2^15)
            const uint32_t ef = m >> 7;                  // 0: zero or subnormal; 255: inf or NaN
            int e = (ef == 0u || ef == 255u) ? (ef == 0u && m ? 126 : 0) : 14 - ((int)ef - 127);
            e = e > 126 ? 126 : e < -126 ? -126 : e;
            const float sc = __uint_as_float((uint32_t)(e + 127) << 23);
            uint32_t o4[4];
#pragma unroll
            for (int e2 = 0; e2 < 4; ++e2)
                o4[e2] = f16x2_of(__uint_as_float(w[e2] << 16) * sc, __uint_as_float(w[e2] & 0xFFFF0000u) * sc);
            // a token row is (in_f + 4) halves: 8-byte aligned, not 16
            uint2 *dst = reinterpret_cast<uint2 *>(xh + (size_t)nn[r] * xs + kk[r] + 8u * j);
            dst[0] = make_uint2(o4[0], o4[1]);
            dst[1] = make_uint2(o4[2], o4[3]);
            if (j == 0)
                xc[nn[r] * nck + kk[r] / kChunk] = make_float2(__uint_as_float((uint32_t)(127 - e) << 23), sum);
        }
    }
    __syncwarp();
}

// One 64-code chunk of a warp: rows g and g+8 of the row block (their 16
// codes at shared address ca and ca + 32 lines), the activation fragments of
// each token tile at xa[tt] (the lane's token, its 16 values of the chunk).
// Two independent accumulation chains, added at the end.
template <int NT>
__device__ __forceinline__ void chunk_mma(uint32_t ca, const uint32_t (&xa)[NT], float (&d)[NT][4])
{
    const uint4 q0 = lds128(ca);
    const uint4 q1 = lds128(ca + 32u * 128u);
    const uint32_t w0[4] = {q0.x, q0.y, q0.z, q0.w};
    const uint32_t w1[4] = {q1.x, q1.y, q1.z, q1.w};
    float e[NT][4];
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
#pragma unroll
        for (int u = 0; u < 4; ++u) { d[tt][u] = 0.0f; e[tt][u] = 0.0f; }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        const uint32_t a0 = codes_f16x2<0>(w0[jj]), a2 = codes_f16x2<1>(w0[jj]);
        const uint32_t a1 = codes_f16x2<0>(w1[jj]), a3 = codes_f16x2<1>(w1[jj]);
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
            const uint2 bb = lds64(xa[tt] + 8u * (uint32_t)jj);
            if (jj & 1) mma16816_f16(e[tt], a0, a1, a2, a3, bb.x, bb.y);
            else mma16816_f16(d[tt], a0, a1, a2, a3, bb.x, bb.y);
        }
    }
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
#pragma unroll
        for (int u = 0; u < 4; ++u) d[tt][u] += e[tt][u];
}

// A chunk's partial sums into the row pair's accumulators: times 2^-e and
// the group's scale, plus the group's offset times the chunk's activation
// sum.  sa: the {scale, offset} of row g for the chunk's group (row g + 8 is
// 64 bytes on); ca0 / ca1[tt]: the {2^-e, sum} of the lane's two tokens for
// the chunk.  Token columns past N read some valid token's values; those
// columns are never stored.
template <int NT>
__device__ __forceinline__ void chunk_apply(const float (&d)[NT][4], uint32_t sa, const uint32_t (&ca0)[NT],
                                           const uint32_t (&ca1)[NT], uint32_t kc, float (&as)[NT][4],
                                           float (&af)[NT][4])
{
    const uint2 s0 = lds64(sa), s1 = lds64(sa + 64u);
    const float sc0 = __uint_as_float(s0.x), of0 = __uint_as_float(s0.y);
    const float sc1 = __uint_as_float(s1.x), of1 = __uint_as_float(s1.y);
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) {
        const uint2 c0 = lds64(ca0[tt] + 8u * kc), c1 = lds64(ca1[tt] + 8u * kc);
        const float f0 = __uint_as_float(c0.x), x0 = __uint_as_float(c0.y);
        const float f1 = __uint_as_float(c1.x), x1 = __uint_as_float(c1.y);
        as[tt][0] = fmaf(sc0, d[tt][0] * f0, as[tt][0]);
        as[tt][1] = fmaf(sc0, d[tt][1] * f1, as[tt][1]);
        as[tt][2] = fmaf(sc1, d[tt][2] * f0, as[tt][2]);
        as[tt][3] = fmaf(sc1, d[tt][3] * f1, as[tt][3]);
        af[tt][0] = fmaf(of0, x0, af[tt][0]);
        af[tt][1] = fmaf(of0, x1, af[tt][1]);
        af[tt][2] = fmaf(of1, x0, af[tt][2]);
        af[tt][3] = fmaf(of1, x1, af[tt][3]);
    }
}

// Both 64-code chunks of a warp's stage into one set of accumulators (their
// activations share a factor): codes at ca0 and ca1, activations from xa[tt]
// (chunk 0) and xa[tt] + 128 bytes (chunk 1).
template <int NT>
__device__ __forceinline__ void pair_mma(uint32_t ca0, uint32_t ca1, const uint32_t (&xa)[NT], float (&d)[NT][4])
{
    float e[NT][4];
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
#pragma unroll
        for (int u = 0; u < 4; ++u) { d[tt][u] = 0.0f; e[tt][u] = 0.0f; }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t ca = h ? ca1 : ca0;
        const uint4 q0 = lds128(ca);
        const uint4 q1 = lds128(ca + 32u * 128u);
        const uint32_t w0[4] = {q0.x, q0.y, q0.z, q0.w};
        const uint32_t w1[4] = {q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const uint32_t a0 = codes_f16x2<0>(w0[jj]), a2 = codes_f16x2<1>(w0[jj]);
            const uint32_t a1 = codes_f16x2<0>(w1[jj]), a3 = codes_f16x2<1>(w1[jj]);
#pragma unroll
            for (int tt = 0; tt < NT; ++tt) {
                const uint2 bb = lds64(xa[tt] + 128u * (uint32_t)h + 8u * (uint32_t)jj);
                if (jj & 1) mma16816_f16(e[tt], a0, a1, a2, a3, bb.x, bb.y);
                else mma16816_f16(d[tt], a0, a1, a2, a3, bb.x, bb.y);
            }
        }
    }
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
#pragma unroll
        for (int u = 0; u < 4; ++u) d[tt][u] += e[tt][u];
}

// The stage's merged partial sums into the accumulators: one factor, one
// group scale, the offset times the two chunks' activation sums.
template <int NT>
__device__ __forceinline__ void pair_apply(const float (&d)[NT][4], uint32_t sa, const uint32_t (&ca0)[NT],
                                          const uint32_t (&ca1)[NT], uint32_t kc, float (&as)[NT][4],
                                          float (&af)[NT][4])
{
    const uint2 s0 = lds64(sa), s1 = lds64(sa + 64u);
    const float sc0 = __uint_as_float(s0.x), of0 = __uint_as_float(s0.y);
    const float sc1 = __uint_as_float(s1.x), of1 = __uint_as_float(s1.y);
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) {
        const uint4 c0 = lds128(ca0[tt] + 8u * kc), c1 = lds128(ca1[tt] + 8u * kc);
        const float f0 = __uint_as_float(c0.x), x0 = __uint_as_float(c0.y) + __uint_as_float(c0.w);
        const float f1 = __uint_as_float(c1.x), x1 = __uint_as_float(c1.y) + __uint_as_float(c1.w);
        as[tt][0] = fmaf(sc0, d[tt][0] * f0, as[tt][0]);
        as[tt][1] = fmaf(sc0, d[tt][1] * f1, as[tt][1]);
        as[tt][2] = fmaf(sc1, d[tt][2] * f0, as[tt][2]);
        as[tt][3] = fmaf(sc1, d[tt][3] * f1, as[tt][3]);
        af[tt][0] = fmaf(of0, x0, af[tt][0]);
        af[tt][1] = fmaf(of0, x1, af[tt][1]);
        af[tt][2] = fmaf(of1, x0, af[tt][2]);
        af[tt][3] = fmaf(of1, x1, af[tt][3]);
    }
}

template <int NT, bool MERGE>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
affine_tc_gemv_kernel(const __grid_constant__ Jobs J)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // stages on a 1024-byte boundary: the 128-byte swizzle pattern repeats every 1024 bytes
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t S = J.stages;
    const Layout L = layout(S, J.N, NT, J.ng_max, J.in_max);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *empty = full + kMaxStages;
    uint64_t *sdone = empty + kMaxStages;
    volatile uint32_t *abort_flag = reinterpret_cast<volatile uint32_t *>(smem + L.abort);
    float *sbuf = reinterpret_cast<float *>(smem + L.sbuf);
    const uint32_t sb_stride = kRows * J.ng_max;   // floats per array (scales, offsets)

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kConsumers);
        }
        mbar_init(sdone, kConsumers);
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const uint32_t rb0 = rb_at(J, J.total_w * blockIdx.x / gridDim.x);
    const uint32_t rb1 = rb_at(J, J.total_w * (blockIdx.x + 1u) / gridDim.x);

    if (warp == kConsumers) {
        // ---------------- producer ----------------
        if (lane == 0) {
            uint32_t it = 0, slot = 0, ph = 0, j = 0, rbi = 0;
            bool ok = true;
            for (uint32_t rb = rb0; rb < rb1 && ok; ++rb, ++rbi) {
                while (j + 1u < J.n && rb >= J.job[j + 1u].rb_begin) ++j;
                const Job &b = J.job[j];
                const uint32_t row0 = (rb - b.rb_begin) * kRows;
                const uint32_t rv = min(kRows, b.out_f - row0);
                const uint32_t nst = (b.in_f + kKC - 1u) / kKC;
                for (uint32_t st = 0; st < nst; ++st, ++it) {
                    if (it >= S && !mbar_wait(empty + slot, ph ^ 1u, abort_flag, &g_tc_err)) {
                        ok = false;
                        break;
                    }
                    uint32_t sbytes = 0;
                    if (st == 0) {
                        // the scales of the previous row block have been transposed
                        if (rbi >= 1u && !mbar_wait(sdone, (rbi - 1u) & 1u, abort_flag, &g_tc_err)) {
                            ok = false;
                            break;
                        }
                        sbytes = (rv * b.ng * 4u) & ~15u;
                    }
                    // the full boxes count, including the zero fill past the matrix
                    mbar_expect_tx(full + slot, kStageBytes + 2u * sbytes);
                    uint8_t *dst = smem + slot * kStageBytes;
#pragma unroll
                    for (uint32_t h = 0; h < kKC / 512u; ++h)
                        tma_load_3d(dst + h * kHalfBytes, &b.map, full + slot, 0,
                                    (int32_t)(st * (kKC / 128u) + 4u * h), (int32_t)row0);
                    if (sbytes) {
                        bulk_g2s(sbuf, b.scales + (size_t)row0 * b.ng, sbytes, full + slot);
                        bulk_g2s(sbuf + sb_stride, b.offsets + (size_t)row0 * b.ng, sbytes, full + slot);
                    }
                    if (++slot == S) { slot = 0; ph ^= 1u; }
                }
            }
            // every issued copy has landed before shared memory is released
            for (uint32_t kt = it > S ? it - S : 0u; kt < it; ++kt) mbar_drain(full + kt % S, (kt / S) & 1u, &g_tc_err);
        }
        // The producer reads only weights, so it never waits for the
        // previous kernel.  Lanes 1-31 must not execute griddepcontrol.wait
        // either: the warp is diverged around lane 0's loop, and a blocked
        // wait on the other path held lane 0's copies back until the
        // previous kernel had finished (measured: the codes were issued
        // after, not before, the consumers' wait).
        __syncwarp();
        return;
    }

    // ---------------- consumers ----------------
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t ct = threadIdx.x;        // 0..255
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t N = J.N;
    const uint32_t xh_a = smem_u32(smem + L.xh), xc_a = smem_u32(smem + L.xc), sf_a = smem_u32(smem + L.sf);
    const uint32_t stage_a = smem_u32(smem);
    float *sf = reinterpret_cast<float *>(smem + L.sf);
    float *red = reinterpret_cast<float *>(smem + L.red);
    constexpr uint32_t NTOK = 8u * NT;
    // this warp's 128 codes of a stage: line (warp & 3) of half stage (warp >> 2)
    const uint32_t half = warp >> 2, cl = warp & 3u;
    const uint32_t line = g * 4u + cl;
    const uint32_t unit0 = t ^ (line & 7u), unit1 = (4u + t) ^ (line & 7u);
    const uint32_t coff0 = half * kHalfBytes + line * 128u + unit0 * 16u;
    const uint32_t coff1 = half * kHalfBytes + line * 128u + unit1 * 16u;
    uint32_t slot = 0, ph = 0, j = 0, rbi = 0, cur = 0xFFFFFFFFu;
    bool ok = true;
    for (uint32_t rb = rb0; rb < rb1; ++rb, ++rbi) {
        while (j + 1u < J.n && rb >= J.job[j + 1u].rb_begin) ++j;
        const Job &b = J.job[j];
        if (j != cur) {
            stage_x_warp<MERGE>(b, N, smem, L, warp, lane);   // this warp's K slices only
            cur = j;
        }
        const uint32_t in_f = b.in_f, ng = b.ng;
        const uint32_t row0 = (rb - b.rb_begin) * kRows;
        const uint32_t rv = min(kRows, b.out_f - row0);
        const uint32_t nst = (in_f + kKC - 1u) / kKC;
        // 32-bit shared addresses of this lane's activation fragments and chunk
        // factors (tokens past N clamped to N - 1: their columns are not stored)
        const uint32_t nck = in_f / kChunk;
        uint32_t xa0[NT], ca0[NT], ca1[NT];
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
            const uint32_t n = min((uint32_t)tt * 8u + g, N - 1u);
            const uint32_t n0 = min((uint32_t)tt * 8u + 2u * t, N - 1u), n1 = min((uint32_t)tt * 8u + 2u * t + 1u, N - 1u);
            xa0[tt] = xh_a + 2u * (n * (in_f + 4u) + t * 16u);
            ca0[tt] = xc_a + 8u * n0 * nck;
            ca1[tt] = xc_a + 8u * n1 * nck;
        }
        const uint32_t gsh = b.gs_shift;
        float as[NT][4], af[NT][4];
#pragma unroll
        for (int tt = 0; tt < NT; ++tt)
#pragma unroll
            for (int u = 0; u < 4; ++u) { as[tt][u] = 0.0f; af[tt][u] = 0.0f; }
        for (uint32_t st = 0; st < nst; ++st) {
            if (ok && !warp_wait(full + slot, ph, abort_flag, &g_tc_err)) ok = false;
            if (st == 0) {
                // scales and offsets of the row block, transposed to [group][row][s, off];
                // rows past the copied bytes come from global memory, rows past the matrix are 0
                const uint32_t sbytes = (rv * ng * 4u) & ~15u;
                const float *gsc = b.scales + (size_t)row0 * ng, *gof = b.offsets + (size_t)row0 * ng;
                const uint32_t qs = kCThreads / ng, rs = kCThreads - qs * ng;
                uint32_t r = ct / ng, gg = ct - r * ng;
                for (uint32_t i = ct; i < kRows * ng; i += kCThreads) {
                    float sv = 0.0f, fv = 0.0f;
                    if (ok && r < rv) {
                        sv = i * 4u < sbytes ? sbuf[i] : __ldg(gsc + i);
                        fv = i * 4u < sbytes ? sbuf[sb_stride + i] : __ldg(gof + i);
                    }
                    sf[gg * kSfStride + 2u * r] = sv;
                    sf[gg * kSfStride + 2u * r + 1u] = fv;
                    gg += rs;
                    r += qs;
                    if (gg >= ng) { gg -= ng; ++r; }
                }
                async_proxy_fence();   // sbuf is refilled by the next row block's bulk copy
                asm volatile(HXQ_TC_BAR_CONSUMERS ::: "memory");
                if (ok && lane == 0) mbar_arrive(sdone);
            }
            const uint32_t kb = st * kKC + warp * kWarpK;
            if (ok && kb < in_f) {
                // in_f is a multiple of 128: both chunks of the warp are inside K
                const uint32_t sa = stage_a + slot * kStageBytes;
                uint32_t xa[NT];
                float d[NT][4];
#pragma unroll
                for (int tt = 0; tt < NT; ++tt) xa[tt] = xa0[tt] + 2u * kb;
                if constexpr (MERGE) {
                    pair_mma<NT>(sa + coff0, sa + coff1, xa, d);
                    warp_release(empty + slot, lane);   // the stage's codes are in registers
                    pair_apply<NT>(d, sf_a + (kb >> gsh) * (kSfStride * 4u) + 8u * g, ca0, ca1, kb >> 6, as, af);
                } else {
                    chunk_mma<NT>(sa + coff0, xa, d);
                    chunk_apply<NT>(d, sf_a + (kb >> gsh) * (kSfStride * 4u) + 8u * g, ca0, ca1, kb >> 6, as, af);
#pragma unroll
                    for (int tt = 0; tt < NT; ++tt) xa[tt] += 2u * kChunk;
                    chunk_mma<NT>(sa + coff1, xa, d);
                    warp_release(empty + slot, lane);   // the stage's codes are in registers
                    const uint32_t k1 = kb + kChunk;
                    chunk_apply<NT>(d, sf_a + (k1 >> gsh) * (kSfStride * 4u) + 8u * g, ca0, ca1, k1 >> 6, as, af);
                }
            } else {
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(empty + slot);
            }
            if (++slot == S) { slot = 0; ph ^= 1u; }
        }
        // the 8 warps' partial sums of this row block, added in warp order
        float *rd = red + (size_t)(rbi & 1u) * kConsumers * kRows * NTOK;
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
            const uint32_t n0 = (uint32_t)tt * 8u + 2u * t;
            rd[(warp * kRows + g) * NTOK + n0] = as[tt][0] + af[tt][0];
            rd[(warp * kRows + g) * NTOK + n0 + 1u] = as[tt][1] + af[tt][1];
            rd[(warp * kRows + g + 8u) * NTOK + n0] = as[tt][2] + af[tt][2];
            rd[(warp * kRows + g + 8u) * NTOK + n0 + 1u] = as[tt][3] + af[tt][3];
        }
        asm volatile(HXQ_TC_BAR_CONSUMERS ::: "memory");
        for (uint32_t idx = ct; idx < kRows * NTOK; idx += kCThreads) {
            const uint32_t row = idx / NTOK, n = idx - row * NTOK;
            if (ok && row < rv && n < N) {
                float v = 0.0f;
#pragma unroll
                for (uint32_t w = 0; w < kConsumers; ++w) v += rd[(w * kRows + row) * NTOK + n];
                const uint32_t o = row0 + row;
                if (b.bias) v += __ldg(b.bias + o);
                for (uint32_t k = 0; k < b.out.n; ++k) b.out.y[k][(size_t)n * b.ldy + o] = v;
            }
        }
    }
}

// Ring depth and CTAs per SM for a launch: the deepest ring (2..6 stages)
// that keeps two CTAs on an SM (228 KB, 1 KB reserved per CTA), else one
// CTA with the deepest ring that fits 227 KB.  0 stages: does not fit.
struct Plan {
    uint32_t stages, per_sm;
    Layout L;
};

Plan plan_for(uint32_t N, uint32_t ng, uint32_t in_f)
{
    const uint32_t nt = N > 8u ? 2u : 1u;
    Plan p{0u, 0u, {}};
    for (uint32_t s = kMaxStages; s >= 2u; --s) {
        const Layout L = layout(s, N, nt, ng, in_f);
        if (kCtasPerSm == 2u && 2u * (L.total + 1024u) <= 233472u) return Plan{s, 2u, L};
    }
    for (uint32_t s = kMaxStages; s >= 2u; --s) {
        const Layout L = layout(s, N, nt, ng, in_f);
        if (L.total <= 227u * 1024u) return Plan{s, 1u, L};
    }
    return p;
}

}  // namespace tcg

// Eligibility of one matrix for the tensor-core GEMV (host side).
bool tc_gemv_fits(const uint16_t *x, const uint8_t *codes, const float *scales, const float *offsets,
                  uint32_t N, uint32_t in_f, uint32_t out_f, uint32_t gs)
{
    auto al = [](const void *p) { return ((uintptr_t)p & 15u) == 0; };
    if (N == 0 || N > 16u || out_f == 0 || in_f == 0 || gs == 0) return false;
    if (in_f % 128u != 0 || gs < tcg::kChunk || (gs & (gs - 1u)) != 0 || in_f % gs != 0) return false;
    if (!x || !codes || !scales || !offsets || !al(x) || !al(codes) || !al(scales) || !al(offsets)) return false;
    return tcg::plan_for(N, in_f / gs, in_f).stages != 0;
}

// 0 launched, 1 a matrix does not fit this kernel, -1 CUDA error.
int launch_tc_gemv(uint32_t n, const TcMatrix *m, uint32_t N, int sms, cudaStream_t s)
{
    using namespace tcg;
    if (n == 0 || N == 0) return 0;
    if (n > kMaxTcJobs) return 1;
    tcg::Jobs J{};
    uint32_t rb = 0;
    uint64_t w = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const TcMatrix &a = m[i];
        if (!tc_gemv_fits(a.x, a.codes, a.scales, a.offsets, N, a.in_f, a.out_f, a.gs)) return 1;
        if (a.out.n == 0 || a.out.n > HXQ_CUDA_MAX_PEERS || a.ldy < a.out_f) return 1;
        Job &b = J.job[i];
        // the codes as [out_f][in_f / 128][128] bytes; a half stage is the box of 16 rows x 4 lines
        std::memset(&b.map, 0, sizeof(b.map));
        if (!pipe::encode_rows_map(&b.map, a.codes, a.in_f, a.out_f, 128u, 4u, kRows)) return 1;
        b.x = a.x; b.codes = a.codes; b.scales = a.scales; b.offsets = a.offsets; b.bias = a.bias;
        b.out = a.out; b.in_f = a.in_f; b.out_f = a.out_f; b.gs = a.gs; b.ng = a.in_f / a.gs; b.ldy = a.ldy;
        b.gs_shift = (a.gs & (a.gs - 1u)) == 0 ? (uint32_t)__builtin_ctz(a.gs) : 32u;
        b.rb_begin = rb;
        b.w_begin = w;
        const uint32_t nrb = (a.out_f + kRows - 1u) / kRows;
        rb += nrb;
        w += (uint64_t)nrb * kRows * a.in_f;
        J.ng_max = b.ng > J.ng_max ? b.ng : J.ng_max;
        J.in_max = a.in_f > J.in_max ? a.in_f : J.in_max;
    }
    J.n = n;
    J.N = N;
    J.total_rb = rb;
    J.total_w = w;
    const Plan P = plan_for(N, J.ng_max, J.in_max);
    if (P.stages == 0) return 1;
    J.stages = P.stages;
    const uint32_t nt = N > 8u ? 2u : 1u;
    // one factor and one scale per warp stage when every group size is a multiple of 128
    bool merge = true;
    for (uint32_t i = 0; i < n; ++i) merge = merge && m[i].gs % 128u == 0;
    const uint32_t variant = (nt - 1u) * 2u + (merge ? 1u : 0u);
    static std::atomic<uint64_t> configured[4];   // per instantiation: one bit per device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) { cudaGetLastError(); return -1; }
    void (*kerns[4])(Jobs) = {affine_tc_gemv_kernel<1, false>, affine_tc_gemv_kernel<1, true>,
                              affine_tc_gemv_kernel<2, false>, affine_tc_gemv_kernel<2, true>};
    auto kern = kerns[variant];
    if (!(configured[variant].load(std::memory_order_acquire) & (1ull << dev))) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
        configured[variant].fetch_or(1ull << dev, std::memory_order_acq_rel);
    }
    uint32_t grid = (uint32_t)(sms > 0 ? sms : 148) * P.per_sm;
    if (grid > rb) grid = rb;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(tcg::kThreads);
    cfg.dynamicSmemBytes = P.L.total;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, J) != cudaSuccess) { cudaGetLastError(); return -1; }
    return 0;
}

uint32_t tc_gemv_status_take()
{
    uint32_t v = 0;
    if (cudaMemcpyFromSymbol(&v, tcg::g_tc_err, sizeof(v)) != cudaSuccess) { cudaGetLastError(); return 0xFFFFFFFFu; }
    if (v) {
        const uint32_t z = 0;
        cudaMemcpyToSymbol(tcg::g_tc_err, &z, sizeof(z));
    }
    return v;
}

}  // namespace hxq
