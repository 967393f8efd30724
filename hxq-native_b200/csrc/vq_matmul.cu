// vq_matmul.cu -- fused VQ-dequant matmul for a few tokens (sm_100a).
//
//   y[n, o] = sum_k x[n, k] * W[o, k],  W = the image's decompressed weights
// (codebook[index] + in-range sidecar deltas, the reference's src/hxq.c:
// 239-350 decode), with W never written to memory.
//
// One warp per output row, 16 warps per CTA (two CTAs per SM), so one staged
// codebook serves many warps.  The CTA stages the fp32 codebook (32 KB) and
// the pass's activations (bf16) in shared memory once; each CTA serves one
// image of the batch (a contiguous range of its rows).  A row's packed
// 12-bit indices arrive in pieces of 2048 weights
// (1536 bytes) through a two-deep per-warp cp.async ring (coalesced 16-byte
// copies, L1 bypassed); each lane takes 4 consecutive byte triples per step
// (3 bank-conflict-free word reads, one PRMT per triple), gathers the 8 fp32
// pairs from the codebook and meets the activations in fp32 FMAs.  The row's
// sidecar entries are a sparse epilogue, y += delta * x[col]: their chunk
// range is read when the row starts and each lane's first two entries when
// its last piece starts, so the dependent loads overlap the streaming.
// Each warp keeps its next two rows of indices on their way to L2 by bulk
// prefetch, and the kernel is launched with programmatic stream
// serialization (the weights do not depend on the kernel before it; the
// activations do).
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "hxq_cuda_internal.h"

namespace hxq {
namespace {

constexpr uint32_t kGvWarps = 16;
constexpr uint32_t kGvThreads = kGvWarps * 32;
constexpr uint32_t kGvStages = 2;
constexpr uint32_t kPieceTrip = 512;                   // byte triples per piece
constexpr uint32_t kPieceVec = kPieceTrip * 3u / 16u;  // 96 16-byte copies
constexpr uint32_t kGvCbBytes = 4096u * 8u;
constexpr uint32_t kGvRingBytes = kGvWarps * kGvStages * kPieceVec * 16u;
constexpr uint32_t kGvXsBytesMax = 48u * 1024u;        // staged activations per pass

struct GemvArgs {
    const uint8_t *idx;          // packed rows, row_bytes apart, 16-B aligned
    const float *cb;             // fp32 codebook, 4096 pairs
    const uint32_t *chunk_ptr;   // first sidecar entry of each 2048-weight chunk
    const SideEntry *ent;        // sidecar entries, sorted by position
    const uint16_t *x;           // bf16 [ntok, in_f]
    OutPtrs out;                 // [ntok, ldy] each
    uint32_t rows, in_f, ntok, ldy, n_chunks;
    uint32_t cta_begin, n_ctas;  // the CTAs of the launch that serve this matrix
};

// A launch covers up to kMaxVqJobs matrices; each CTA serves one of them
// (a contiguous range of its rows), so it stages one codebook.
constexpr uint32_t kMaxVqJobs = 8;
struct GemvBatch {
    GemvArgs job[kMaxVqJobs];
    uint32_t n;
};

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ float lo_bf16(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// XS: activations staged in shared memory (else read through L1).
template <int NT, bool XS>
__global__ void __launch_bounds__(kGvThreads, 2)
vq_gemv_kernel(const __grid_constant__ GemvBatch B)
{
    extern __shared__ __align__(16) unsigned char smem[];
    uint32_t jb = 0;
    while (jb + 1u < B.n && blockIdx.x >= B.job[jb + 1u].cta_begin) ++jb;
    const GemvArgs &a = B.job[jb];
    float2 *cb = reinterpret_cast<float2 *>(smem);
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    uint4 *ring = reinterpret_cast<uint4 *>(smem + kGvCbBytes) + warp * kGvStages * kPieceVec;
    const uint16_t *xs = XS ? reinterpret_cast<const uint16_t *>(smem + kGvCbBytes + kGvRingBytes) : a.x;

    const uint32_t row_trip = a.in_f / 4u;             // in_f % 64 == 0: whole 16-B copies
    const size_t row_bytes = (size_t)row_trip * 3u;
    const uint32_t P = (row_trip + kPieceTrip - 1u) / kPieceTrip;
    // this CTA's rows of the matrix, taken by its warps in turn
    const uint32_t cb_i = blockIdx.x - a.cta_begin;
    const uint32_t r_lo = (uint32_t)((uint64_t)a.rows * cb_i / a.n_ctas);
    const uint32_t r_hi = (uint32_t)((uint64_t)a.rows * (cb_i + 1u) / a.n_ctas);
    const uint32_t stride = kGvWarps;
    const uint32_t first = r_lo + warp;
    const uint32_t my_rows = first < r_hi ? (r_hi - first + stride - 1u) / stride : 0u;
    const uint32_t total = my_rows * P;

    auto issue = [&](uint32_t s) {
        if (s < total) {
            const uint32_t o = first + (s / P) * stride, p0 = (s % P) * kPieceTrip;
            const uint32_t nvec = min(kPieceTrip, row_trip - p0) * 3u / 16u;
            const uint4 *src = reinterpret_cast<const uint4 *>(a.idx + (size_t)o * row_bytes + (size_t)p0 * 3u);
            uint4 *dst = ring + (s % kGvStages) * kPieceVec;
#pragma unroll
            for (uint32_t q = 0; q < 3u; ++q) {
                const uint32_t v = q * 32u + lane;
                if (v < nvec) cp_async16(dst + v, src + v);
            }
        }
        cp_commit();
    };
    // the next kernel on the stream may start now; this one waits for the
    // kernel before it (griddepcontrol.wait) only before it reads the
    // activations.  The warp's next two rows of indices go to L2 by bulk
    // prefetch (a window that stays far below L2 for any batch).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    auto prefetch_row = [&](uint32_t r) {
        if (lane == 0 && r < my_rows)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;"
                         ::"l"(a.idx + (size_t)(first + r * stride) * row_bytes), "r"((uint32_t)row_bytes) : "memory");
    };
    prefetch_row(0);
    prefetch_row(1);
    // the first piece is in flight while the codebook and activations are staged
    issue(0);
    for (uint32_t i = tid; i < kGvCbBytes / 16u; i += kGvThreads)
        reinterpret_cast<uint4 *>(smem)[i] = __ldg(reinterpret_cast<const uint4 *>(a.cb) + i);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if constexpr (XS) {
        const uint32_t nv = a.ntok * a.in_f / 8u;
        uint4 *xd = reinterpret_cast<uint4 *>(smem + kGvCbBytes + kGvRingBytes);
        for (uint32_t i = tid; i < nv; i += kGvThreads) xd[i] = __ldg(reinterpret_cast<const uint4 *>(a.x) + i);
    }
    __syncthreads();

    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
    // sidecar of the current row: chunks [ch0, ch0 + nc) hold its entries,
    // lane i keeps chunk_ptr[ch0 + i] (i <= nc), the entry range is
    // [e_lo, e_hi), and each lane prefetches the range's entries lane and
    // lane + 32
    uint32_t cpv = 0, nc = 0, e_lo = 0, e_hi = 0;
    uint2 en0 = make_uint2(0u, 0u), en1 = make_uint2(0u, 0u);
    for (uint32_t s = 0; s < total; ++s) {
        issue(s + 1u);
        const uint32_t o = first + (s / P) * stride, pc = s % P, p0 = pc * kPieceTrip;
        const uint64_t f0 = (uint64_t)o * a.in_f;
        const uint32_t ch0 = (uint32_t)(f0 / kChunkW);
        if (pc == 0) {
            prefetch_row(s / P + 2u);
            uint32_t ch1 = (uint32_t)((f0 + a.in_f - 1u) / kChunkW) + 1u;
            ch1 = ch1 < a.n_chunks ? ch1 : a.n_chunks;
            nc = ch1 - ch0;
            cpv = lane <= nc ? __ldg(a.chunk_ptr + ch0 + lane) : 0u;
        }
        if (pc + 1u == P) {
            e_lo = __shfl_sync(0xffffffffu, cpv, 0);
            e_hi = nc < 32u ? __shfl_sync(0xffffffffu, cpv, nc) : __ldg(a.chunk_ptr + ch0 + nc);
            en0 = e_lo + lane < e_hi ? __ldg(reinterpret_cast<const uint2 *>(a.ent + e_lo + lane)) : make_uint2(0u, 0u);
            en1 = e_lo + 32u + lane < e_hi ? __ldg(reinterpret_cast<const uint2 *>(a.ent + e_lo + 32u + lane))
                                           : make_uint2(0u, 0u);
        }
        cp_wait<kGvStages - 1>();
        __syncwarp();
        const uint32_t ngrp = min(kPieceTrip, row_trip - p0) / 4u;
        const uint32_t *sw = reinterpret_cast<const uint32_t *>(ring + (s % kGvStages) * kPieceVec);
#pragma unroll
        for (uint32_t m = 0; m < kPieceTrip / 128u; ++m) {
            const uint32_t g = m * 32u + lane;
            if (g < ngrp) {
                const uint32_t w0 = sw[3u * g], w1 = sw[3u * g + 1u], w2 = sw[3u * g + 2u];
                const uint32_t B0 = __byte_perm(w0, w1, 0x3012u), B1 = __byte_perm(w0, w1, 0x6345u);
                const uint32_t B2 = __byte_perm(w1, w2, 0x5234u), B3 = __byte_perm(w2, w2, 0x4123u);
                const float2 c0 = cb[(B0 >> 12) & 0xFFFu], c1 = cb[B0 & 0xFFFu];
                const float2 c2 = cb[(B1 >> 12) & 0xFFFu], c3 = cb[B1 & 0xFFFu];
                const float2 c4 = cb[(B2 >> 12) & 0xFFFu], c5 = cb[B2 & 0xFFFu];
                const float2 c6 = cb[(B3 >> 12) & 0xFFFu], c7 = cb[B3 & 0xFFFu];
                const size_t col = (size_t)p0 * 4u + 16u * g;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if ((uint32_t)t < a.ntok) {
                        const uint4 *xp = reinterpret_cast<const uint4 *>(xs + (size_t)t * a.in_f + col);
                        const uint4 xa = XS ? xp[0] : __ldg(xp), xb = XS ? xp[1] : __ldg(xp + 1);
                        float r = acc[t];
                        r = fmaf(c0.x, lo_bf16(xa.x), r); r = fmaf(c0.y, hi_bf16(xa.x), r);
                        r = fmaf(c1.x, lo_bf16(xa.y), r); r = fmaf(c1.y, hi_bf16(xa.y), r);
                        r = fmaf(c2.x, lo_bf16(xa.z), r); r = fmaf(c2.y, hi_bf16(xa.z), r);
                        r = fmaf(c3.x, lo_bf16(xa.w), r); r = fmaf(c3.y, hi_bf16(xa.w), r);
                        r = fmaf(c4.x, lo_bf16(xb.x), r); r = fmaf(c4.y, hi_bf16(xb.x), r);
                        r = fmaf(c5.x, lo_bf16(xb.y), r); r = fmaf(c5.y, hi_bf16(xb.y), r);
                        r = fmaf(c6.x, lo_bf16(xb.z), r); r = fmaf(c6.y, hi_bf16(xb.z), r);
                        r = fmaf(c7.x, lo_bf16(xb.w), r); r = fmaf(c7.y, hi_bf16(xb.w), r);
                        acc[t] = r;
                    }
                }
            }
        }
        if (pc + 1u == P) {
            // sparse epilogue: the row's sidecar deltas times the activations
            const uint32_t rounds = (e_hi - e_lo + 31u) / 32u;
            for (uint32_t k = 0; k < rounds; ++k) {
                const uint32_t e = e_lo + 32u * k + lane;
                const uint2 en = k == 0 ? en0 : k == 1 ? en1
                                 : (e < e_hi ? __ldg(reinterpret_cast<const uint2 *>(a.ent + e)) : make_uint2(0u, 0u));
                // the entry's chunk: ch0 + the number of later chunk starts <= e
                uint32_t c = ch0;
                if (nc < 32u) {
                    for (uint32_t i = 1; i < nc; ++i) c += __shfl_sync(0xffffffffu, cpv, i) <= e ? 1u : 0u;
                } else {
                    while (c + 1u < a.n_chunks && __ldg(a.chunk_ptr + c + 1u) <= e) ++c;
                }
                if (e >= e_hi) continue;
                const uint64_t pos = (uint64_t)c * kChunkW + (en.x & 0xFFFFu);
                if (pos < f0 || pos >= f0 + a.in_f) continue;
                const size_t col = (size_t)(pos - f0);
                const float v = __uint_as_float(en.y);
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    if ((uint32_t)t < a.ntok)
                        acc[t] = fmaf(v, lo_bf16(XS ? xs[(size_t)t * a.in_f + col] : __ldg(xs + (size_t)t * a.in_f + col)),
                                      acc[t]);
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                float v = acc[t];
#pragma unroll
                for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
                if (lane == 0 && (uint32_t)t < a.ntok)
                    for (uint32_t k = 0; k < a.out.n; ++k) a.out.y[k][(size_t)t * a.ldy + o] = v;
                acc[t] = 0.0f;
            }
        }
        __syncwarp();   // the slot just read is the next issue's target
    }
    cp_wait<0>();
}

template <int NT, bool XS>
cudaError_t configure_one(size_t smem)
{
    return cudaFuncSetAttribute(vq_gemv_kernel<NT, XS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

}  // namespace

// Fused VQ GEMV over a batch of 12-bit images (k = 4096, in_f % 64 == 0,
// 16-byte aligned x and index rows); up to 8 tokens per pass, fewer when
// their activations would not fit the staging budget.  Each image gets the
// CTAs a launch of it alone would have (one per 8 rows, at most a full
// grid), so a batch runs like back-to-back launches without their gaps.
cudaError_t launch_vq_gemv_batch(uint32_t n, const VqGemvJob *jobs, uint32_t ntok, int sms, cudaStream_t s)
{
    static std::atomic<uint64_t> configured{0};   // one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (n == 0 || ntok == 0) return cudaSuccess;
    if (n > kMaxVqJobs) return cudaErrorInvalidValue;
    const size_t base = kGvCbBytes + kGvRingBytes;
    if (!(configured.load(std::memory_order_acquire) & (1ull << dev))) {
        const size_t mx = base + kGvXsBytesMax;
        e = configure_one<1, true>(mx);
        if (e == cudaSuccess) e = configure_one<2, true>(mx);
        if (e == cudaSuccess) e = configure_one<4, true>(mx);
        if (e == cudaSuccess) e = configure_one<8, true>(mx);
        if (e == cudaSuccess) e = configure_one<1, false>(base);
        if (e == cudaSuccess) e = configure_one<2, false>(base);
        if (e == cudaSuccess) e = configure_one<4, false>(base);
        if (e == cudaSuccess) e = configure_one<8, false>(base);
        if (e != cudaSuccess) return e;
        configured.fetch_or(1ull << dev, std::memory_order_acq_rel);
    }
    uint32_t max_in = 0;
    for (uint32_t i = 0; i < n; ++i) max_in = jobs[i].in_f > max_in ? jobs[i].in_f : max_in;
    const size_t row_x = (size_t)max_in * 2u;
    const uint32_t fit = (uint32_t)(kGvXsBytesMax / row_x);      // tokens whose activations fit
    const bool xs = fit >= 1u;
    const uint32_t per_pass = xs ? (fit < 8u ? fit : 8u) : 8u;
    for (uint32_t n0 = 0; n0 < ntok; n0 += per_pass) {
        const uint32_t nt = ntok - n0 < per_pass ? ntok - n0 : per_pass;
        const size_t smem = base + (xs ? (size_t)nt * row_x : 0u);
        // resident CTAs per SM: shared memory (228 KB, 1 KB reserved per CTA), at most 2
        uint32_t per_sm = (uint32_t)(233472u / (smem + 1024u));
        per_sm = per_sm > 2u ? 2u : per_sm < 1u ? 1u : per_sm;
        const uint32_t G = (uint32_t)(sms > 0 ? sms : 148) * per_sm;
        GemvBatch B{};
        B.n = n;
        uint32_t cta = 0;
        for (uint32_t i = 0; i < n; ++i) {
            const VqGemvJob &j = jobs[i];
            GemvArgs &a = B.job[i];
            a.idx = j.idx; a.cb = j.cb; a.chunk_ptr = j.chunk_ptr; a.ent = j.ent;
            a.x = j.x + (size_t)n0 * j.in_f;
            a.out = j.out;
            for (uint32_t k = 0; k < j.out.n; ++k) a.out.y[k] = j.out.y[k] + (size_t)n0 * j.ldy;
            a.rows = j.rows; a.in_f = j.in_f; a.ntok = nt; a.ldy = j.ldy; a.n_chunks = j.n_chunks;
            // as many CTAs as a launch of this matrix alone would have: one
            // per 8 rows, at most a full grid
            const uint32_t cmax = (j.rows + kGvWarps - 1u) / kGvWarps;
            const uint32_t c = cmax < G ? cmax : G;
            a.cta_begin = cta;
            a.n_ctas = c;
            cta += c;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(cta);
        cfg.blockDim = dim3(kGvThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        void (*kern)(GemvBatch) = nullptr;
        if (nt == 1) kern = xs ? vq_gemv_kernel<1, true> : vq_gemv_kernel<1, false>;
        else if (nt == 2) kern = xs ? vq_gemv_kernel<2, true> : vq_gemv_kernel<2, false>;
        else if (nt <= 4) kern = xs ? vq_gemv_kernel<4, true> : vq_gemv_kernel<4, false>;
        else kern = xs ? vq_gemv_kernel<8, true> : vq_gemv_kernel<8, false>;
        e = cudaLaunchKernelEx(&cfg, kern, B);
        if (e != cudaSuccess) { cudaGetLastError(); return e; }
    }
    return cudaSuccess;
}

cudaError_t launch_vq_gemv(const uint8_t *idx, const float *cb, const uint32_t *chunk_ptr, const SideEntry *ent,
                           uint32_t n_chunks, uint32_t rows, uint32_t in_f, const uint16_t *x, uint32_t ntok,
                           const OutPtrs &out, uint32_t ldy, int sms, cudaStream_t s)
{
    VqGemvJob j{idx, cb, chunk_ptr, ent, n_chunks, rows, in_f, x, out, ldy};
    return launch_vq_gemv_batch(1, &j, ntok, sms, s);
}

}  // namespace hxq
