// vq_tc_gemv.cu -- fused 12-bit VQ dequant-matmul for 1..8 bf16 tokens on
// the tensor cores: y[n, o] = sum_i x[n, i] W[o, i], W never written.
//
// The weights are the bf16 codebook pairs of the image's matmul tables
// (the weights the tcgen05 VQ GEMM uses): each packed 12-bit index names a
// pair of consecutive weights, and its bf16x2 codebook entry is exactly one
// A-fragment register of an m16n8k16 product (two consecutive K values of
// one row).  So a lane's A fragment is one 4-byte gather per register from a
// 16 KB shared codebook, no conversion; the activations are bf16 already.
//   * Index stream: a producer thread copies each 16-row block of packed
//     indices, 1024 weights of K per stage (768 B per row), with one TMA
//     tensor copy per stage: the rows as [rows][row_bytes / L][L] bytes with
//     L = 128, 64 or 32 (the largest dividing the row; swizzle of L bytes),
//     a box of 16 rows x 768 / L lines; rows past the image read as zero.
//   * Fragments: a consumer warp owns 128 weights of K of every stage (two
//     64-weight chunks); per chunk a lane reads its 8 pairs of rows g and
//     g + 8 (12 bytes each: three 4-byte loads through the swizzle), unpacks
//     the 8 indices and gathers their bf16x2 pairs; 4 products per chunk with
//     fp32 accumulation in two chains, over the K permutation of the affine
//     tensor-core GEMV (activation fragments: one 64-bit load of the
//     lane's token, raw bf16 staged once per matrix).
//   * Sidecar: the positions where the decoded weight differs from the
//     codebook pair carry d = bf16(final weight) - bf16(codebook value)
//     (image table, one entry per position, rows in order).  After a row
//     block's products, consumer warp w sums d x[n, col] over the positions
//     of rows 2w and 2w + 1 (lanes strided over the positions, activations
//     from the staged copy, a fixed butterfly across lanes) and the sum is
//     added to the output it stores.  The result equals the tcgen05 VQ
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
constexpr uint32_t kRowStageBytes = kKC / 4u * 3u;    // 768 B of indices per row per stage
constexpr uint32_t kStageBytes = kRows * kRowStageBytes;   // 12 KB
constexpr uint32_t kMaxStages = 8;
constexpr uint32_t kCbBytes = 4096u * 4u;              // bf16x2 codebook

__device__ uint32_t g_vqtc_err;

struct Job {
    CUtensorMap map;            // indices [rows][row_bytes / line][line]
    const uint32_t *cbh;        // bf16x2 pairs [4096]
    const uint16_t *x;          // bf16 [N][in_f]
    const uint32_t *prow;       // sidecar: first entry of each row (null: none)
    const uint32_t *e4;         // sidecar entries: column in bits 0..15
    const float *ed;            // sidecar weight differences
    uint32_t n_patch;
    OutPtrs out;
    uint32_t ldy, rows, in_f, line;
    uint32_t rb_begin;
    uint64_t w_begin;
};

struct Jobs {
    Job job[kMaxTcJobs];
    uint32_t n, N, total_rb, in_max, stages;
    uint64_t total_w;
};

struct Layout {
    uint32_t bars, abort, cb, xh, red, cs, total;
};

constexpr uint32_t kAlignSlack = 1024;
__host__ __device__ inline Layout layout(uint32_t S, uint32_t N, uint32_t in_f)
{
    Layout L;
    uint32_t o = S * kStageBytes;                 // 12 KB stages: 1024-byte aligned
    L.bars = o;  o += 2u * kMaxStages * 8u;
    L.abort = o; o += 16u;
    o = (o + 127u) & ~127u;
    L.cb = o;    o += kCbBytes;
    L.xh = o;    o += N * (in_f + 4u) * 2u;
    o = (o + 15u) & ~15u;
    L.red = o;   o += 2u * kConsumers * kRows * 8u * 4u;
    L.cs = o;    o += 2u * kRows * 8u * 4u;
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

// Shared-memory byte offset, within a stage, of byte o (a multiple of 4) of
// the stage slice of row r: line r * (768 / L) + o / L, its 16-byte unit
// XOR the swizzle bits 7.. of the line's address (128: line & 7; 64:
// (line >> 1) & 3; 32: (line >> 2) & 1).
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t o, uint32_t L)
{
    const uint32_t line = r * (kRowStageBytes / L) + o / L, b = o % L;
    const uint32_t x = L == 128u ? (line & 7u) : L == 64u ? ((line >> 1) & 3u) : ((line >> 2) & 1u);
    return line * L + ((((b >> 4) ^ x) << 4) | (b & 15u));
}

// The 8 indices of 12 packed bytes (four byte triples, each two 12-bit
// indices: a = b0 << 4 | b1 >> 4, b = (b1 & 15) << 8 | b2).
__device__ __forceinline__ void unpack8(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t (&id)[8])
{
    id[0] = ((w0 & 0xFFu) << 4) | ((w0 >> 12) & 0xFu);
    id[1] = (w0 & 0xF00u) | ((w0 >> 16) & 0xFFu);
    id[2] = ((w0 >> 24) << 4) | ((w1 >> 4) & 0xFu);
    id[3] = ((w1 & 0xFu) << 8) | ((w1 >> 8) & 0xFFu);
    id[4] = (((w1 >> 16) & 0xFFu) << 4) | (w1 >> 28);
    id[5] = (((w1 >> 24) & 0xFu) << 8) | (w2 & 0xFFu);
    id[6] = (((w2 >> 8) & 0xFFu) << 4) | ((w2 >> 20) & 0xFu);
    id[7] = (((w2 >> 16) & 0xFu) << 8) | (w2 >> 24);
}

// One 64-weight chunk: rows g and g+8 (index words at shared addresses
// a0 / a0 + 8 rows, +4, +8 through the swizzle), activation fragments from
// xa[tt]; two accumulation chains.
template <int NT>
__device__ __forceinline__ void chunk(uint32_t w_g[3], uint32_t w_h[3], uint32_t cb_a, const uint32_t (&xa)[NT],
                                      float (&d)[NT][4], float (&e)[NT][4])
{
    uint32_t ig[8], ih[8];
    unpack8(w_g[0], w_g[1], w_g[2], ig);
    unpack8(w_h[0], w_h[1], w_h[2], ih);
    uint32_t ag[8], ah[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        ag[m] = lds32(cb_a + 4u * ig[m]);
        ah[m] = lds32(cb_a + 4u * ih[m]);
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
            const uint2 bb = lds64(xa[tt] + 8u * (uint32_t)jj);
            if (jj & 1) mma16816_bf16(e[tt], ag[2 * jj], ah[2 * jj], ag[2 * jj + 1], ah[2 * jj + 1], bb.x, bb.y);
            else mma16816_bf16(d[tt], ag[2 * jj], ah[2 * jj], ag[2 * jj + 1], ah[2 * jj + 1], bb.x, bb.y);
        }
    }
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 2)
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
                const uint32_t lines = kRowStageBytes / b.line;
                for (uint32_t st = 0; st < nst; ++st, ++it) {
                    if (it >= S && !mbar_wait(empty + slot, ph ^ 1u, abort_flag, &g_vqtc_err)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full + slot, kStageBytes);   // the full box, zero fill included
                    tma_load_3d(smem + slot * kStageBytes, &b.map, full + slot, 0, (int32_t)(st * lines),
                                (int32_t)row0);
                    if (++slot == S) { slot = 0; ph ^= 1u; }
                }
            }
            for (uint32_t kt = it > S ? it - S : 0u; kt < it; ++kt)
                mbar_drain(full + kt % S, (kt / S) & 1u, &g_vqtc_err);
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
        return;
    }

    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t ct = threadIdx.x;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t N = J.N;
    constexpr uint32_t NTOK = 8u * NT;
    const uint32_t stage_a = smem_u32(smem), cb_a = smem_u32(smem + L.cb), xh_a = smem_u32(smem + L.xh);
    float *red = reinterpret_cast<float *>(smem + L.red);
    float *csum = reinterpret_cast<float *>(smem + L.cs);
    const uint16_t *xs = reinterpret_cast<const uint16_t *>(smem + L.xh);
    uint32_t slot = 0, ph = 0, j = 0, rbi = 0, cur = 0xFFFFFFFFu;
    bool ok = true;
    for (uint32_t rb = rb0; rb < rb1; ++rb, ++rbi) {
        while (j + 1u < J.n && rb >= J.job[j + 1u].rb_begin) ++j;
        const Job &b = J.job[j];
        const uint32_t in_f = b.in_f;
        if (j != cur) {
            // the matrix's codebook and activations (raw bf16, rows of in_f + 4)
            const uint4 *cs = reinterpret_cast<const uint4 *>(b.cbh);
            uint4 *cd = reinterpret_cast<uint4 *>(smem + L.cb);
            for (uint32_t i = ct; i < kCbBytes / 16u; i += kConsumers * 32u) cd[i] = __ldg(cs + i);
            const uint32_t per_tok = in_f / 8u;
            uint16_t *xh = reinterpret_cast<uint16_t *>(smem + L.xh);
            for (uint32_t p = ct; p < N * per_tok; p += kConsumers * 32u) {
                const uint32_t n = p / per_tok, k8 = p - n * per_tok;
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(b.x + (size_t)n * in_f) + k8);
                uint2 *dst = reinterpret_cast<uint2 *>(xh + (size_t)n * (in_f + 4u) + k8 * 8u);   // 8-byte aligned rows
                dst[0] = make_uint2(v.x, v.y);
                dst[1] = make_uint2(v.z, v.w);
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");
            cur = j;
        }
        const uint32_t row0 = (rb - b.rb_begin) * kRows;
        const uint32_t rv = min(kRows, b.rows - row0);
        const uint32_t nst = (in_f + kKC - 1u) / kKC;
        const uint32_t Lb = b.line;
        // sidecar ranges of this warp's two rows (consumed after the products)
        uint32_t pr[3] = {0u, 0u, 0u};
        if (b.prow) {
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                const uint32_t r = row0 + 2u * warp + (uint32_t)q;
                pr[q] = r < b.rows ? __ldg(b.prow + r) : b.n_patch;
            }
        }
        // this lane's index words: chunk u, word i of row g (row g + 8: 8 * 768 B on)
        uint32_t wo[2][3];
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int i = 0; i < 3; ++i)
                wo[u][i] = swz(g, warp * 96u + (uint32_t)u * 48u + t * 12u + (uint32_t)i * 4u, Lb);
        uint32_t xa0[NT];
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) {
            const uint32_t n = min((uint32_t)tt * 8u + g, N - 1u);   // columns past N are not stored
            xa0[tt] = xh_a + 2u * (n * (in_f + 4u) + t * 16u);
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
                uint32_t wg[2][3], wh[2][3];
#pragma unroll
                for (int u = 0; u < 2; ++u)
#pragma unroll
                    for (int i = 0; i < 3; ++i) {
                        wg[u][i] = lds32(sa + wo[u][i]);
                        wh[u][i] = lds32(sa + wo[u][i] + 8u * kRowStageBytes);
                    }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty + slot);   // the stage's indices are in registers
                uint32_t xa[NT];
#pragma unroll
                for (int tt = 0; tt < NT; ++tt) xa[tt] = xa0[tt] + 2u * kb;
                chunk<NT>(wg[0], wh[0], cb_a, xa, d, e);
#pragma unroll
                for (int tt = 0; tt < NT; ++tt) xa[tt] += 2u * kChunk;
                chunk<NT>(wg[1], wh[1], cb_a, xa, d, e);
            } else {
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(empty + slot);
            }
            if (++slot == S) { slot = 0; ph ^= 1u; }
        }
        float *cw = csum + (size_t)(rbi & 1u) * kRows * 8u;
        if (b.prow) {
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                float sn[8];
#pragma unroll
                for (int n = 0; n < 8; ++n) sn[n] = 0.0f;
                for (uint32_t p = pr[q] + lane; p < pr[q + 1]; p += 32u) {
                    const uint32_t col = __ldg(b.e4 + p) & 0xFFFFu;
                    const float dl = __ldg(b.ed + p);
#pragma unroll
                    for (int n = 0; n < 8; ++n)
                        if ((uint32_t)n < N)
                            sn[n] = fmaf(dl, __uint_as_float((uint32_t)xs[(size_t)n * (in_f + 4u) + col] << 16), sn[n]);
                }
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    if ((uint32_t)n < N) {
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) sn[n] += __shfl_xor_sync(0xffffffffu, sn[n], o);
                        if (lane == 0) cw[(2u * warp + (uint32_t)q) * 8u + (uint32_t)n] = sn[n];
                    }
                }
            }
        }
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
                if (b.prow) v += cw[row * 8u + n];
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
    for (uint32_t s = kMaxStages; s >= 2u; --s) {
        const Layout L = layout(s, N, in_f);
        if (2u * (L.total + 1024u) <= 233472u) return Plan{s, 2u, L};
    }
    for (uint32_t s = kMaxStages; s >= 2u; --s) {
        const Layout L = layout(s, N, in_f);
        if (L.total <= 227u * 1024u) return Plan{s, 1u, L};
    }
    return Plan{0u, 0u, {}};
}

}  // namespace vqtc

bool vq_tc_fits(const uint16_t *x, uint32_t N, uint32_t in_f)
{
    if (N == 0 || N > 8u || in_f == 0 || in_f % 128u != 0 || in_f > 65536u || ((uintptr_t)x & 15u)) return false;
    return vqtc::plan_for(N, in_f).stages != 0;
}

int launch_vq_tc_gemv(uint32_t n, const VqTcMatrix *m, uint32_t N, int sms, cudaStream_t s)
{
    using namespace vqtc;
    if (n == 0 || N == 0) return 0;
    if (n > kMaxTcJobs) return 1;
    Jobs J{};
    uint32_t rb = 0, in_max = 0;
    uint64_t w = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const VqTcMatrix &a = m[i];
        if (!vq_tc_fits(a.x, N, a.in_f) || a.out.n == 0 || a.out.n > HXQ_CUDA_MAX_PEERS || a.ldy < a.rows) return 1;
        const uint64_t row_bytes = (uint64_t)a.in_f / 4u * 3u;
        const uint32_t line = row_bytes % 128u == 0 ? 128u : row_bytes % 64u == 0 ? 64u : 32u;
        Job &b = J.job[i];
        std::memset(&b.map, 0, sizeof(b.map));
        if (!pipe::encode_rows_map(&b.map, a.idx, row_bytes, a.rows, line, kRowStageBytes / line, kRows)) return 1;
        b.cbh = a.cbh; b.x = a.x; b.out = a.out; b.ldy = a.ldy; b.rows = a.rows; b.in_f = a.in_f; b.line = line;
        if (a.n_patch) {
            if (!a.rb || !a.e4 || !a.ed) return 1;
            b.prow = a.rb; b.e4 = a.e4; b.ed = a.ed; b.n_patch = a.n_patch;
        }
        b.rb_begin = rb;
        b.w_begin = w;
        const uint32_t nrb = (a.rows + kRows - 1u) / kRows;
        rb += nrb;
        w += (uint64_t)nrb * kRows * a.in_f;
        in_max = a.in_f > in_max ? a.in_f : in_max;
    }
    J.n = n;
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
    static std::atomic<uint64_t> configured{0};   // one bit per device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) { cudaGetLastError(); return -1; }
    if (!(configured.load(std::memory_order_acquire) & (1ull << dev))) {
        if (cudaFuncSetAttribute(vq_tc_gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
            cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
        configured.fetch_or(1ull << dev, std::memory_order_acq_rel);
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
    if (cudaLaunchKernelEx(&cfg, vq_tc_gemv_kernel<1>, J) != cudaSuccess) { cudaGetLastError(); return -1; }
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
