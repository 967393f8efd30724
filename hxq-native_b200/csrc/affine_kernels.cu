// affine_kernels.cu -- affine group-quantized fused matmul on sm_100a.
//
//   Y[n,o] = sum_g ( s[o,g] * sum_{k in g} x[n,k]*q[o,k]
//                  + off[o,g] * sum_{k in g} x[n,k] ) + bias[o]
// (reference hxq-native src/hxq_affine.c:23-66; GPU entry points replace
// src/hxq_affine_cuda.cu:184-294).
//
// Streaming dequant-GEMV for small token counts: one warp per output row
// (a one-token launch holds 32 warps per SM, so a 4096-row matrix runs in
// a single round), the warp's rows of codes first sent to L2 by bulk
// prefetch so the copy engine streams them from DRAM, then 16 codes per
// lane per 128-bit load, codes widened to fp32 exactly with a byte permute
// into the mantissa of 2^23, the pass's group scales and offsets loaded one
// per lane and handed out by shuffles, token activations read through L1,
// the group scale applied per 16-code slice and the offset term from the
// slice's activation sum, one warp reduction per row, bias fused into the
// store.  Launched with programmatic stream serialization: the codes do not
// depend on the kernel before it on the stream, so their loads start early
// and the kernel waits (griddepcontrol.wait) only before the activations.
// With bf16 activations, 1..8 tokens (up to 16 in a batch) go to the
// tensor-core GEMV (affine_tc_gemv.cu) and larger token counts to the
// tcgen05 GEMM (dequant_gemm.cu) when the shape allows it; this file's GEMVs take fp32
// activations and the shapes those kernels do not.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <vector>

#include "hxq_affine.h"
#include "hxq_cuda.h"
#include "hxq_cuda_internal.h"

namespace hxq {


namespace {

constexpr int kGemvTokens = 8;   // tokens per pass of the GEMV
// Up to this many bf16 tokens the tensor-core GEMV (exact products, fp32
// accumulation; it takes up to 16 when asked for by path); from there on the
// tcgen05 dequant-GEMM (split over K when the tiles alone would not fill the
// GPU), which is faster from about 9 tokens on a 4096 x 4096 matrix.
constexpr uint32_t kTcGemvMaxTokens = 8;
// In a batch the tensor-core GEMV shares one launch across the matrices and
// beats per-matrix GEMMs up to 16 tokens (7B layer at 16 tokens: 104.8 us
// against 136.4); a single matrix gains nothing from it past 8.
constexpr uint32_t kTcGemvBatchMaxTokens = 16;

__device__ __forceinline__ float code_to_float(uint32_t word, uint32_t i)
{
    // [byte_i, 0, 0, 0x4B] is the float 2^23 + byte_i; subtracting 2^23 is exact
    return __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7440u + i)) - 8388608.0f;
}

template <typename XT> struct XLoad;
template <> struct XLoad<float> {
    // 16 consecutive activations
    static __device__ __forceinline__ void load16(const float *p, float v[16])
    {
        const float4 *q = reinterpret_cast<const float4 *>(p);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 t = __ldg(q + i);
            v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
        }
    }
};
template <> struct XLoad<uint16_t> {
    static __device__ __forceinline__ void load16(const uint16_t *p, float v[16])
    {
        const uint4 *q = reinterpret_cast<const uint4 *>(p);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint4 t = __ldg(q + i);
            const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
                v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
            }
        }
    }
};

template <typename XT> __device__ __forceinline__ float xval(const XT *p);
template <> __device__ __forceinline__ float xval<float>(const float *p) { return *p; }
template <> __device__ __forceinline__ float xval<uint16_t>(const uint16_t *p)
{
    return __uint_as_float((uint32_t)*p << 16);
}

// Group of 16-code slice sl: (16 sl) / gs, a shift when gs is a power of two.
__device__ __forceinline__ uint32_t group_of(uint32_t sl, uint32_t gs, uint32_t gs_shift)
{
    return gs_shift < 32u ? (sl * 16u) >> gs_shift : (sl * 16u) / gs;
}

// Requirements: group_size % 16 == 0, in_f % 16 == 0, x and codes 16-B aligned.
// One warp per output row.  A lane owns 16-code slices sl = lane + 32*i; all
// SPL slices of a pass are loaded before any is used, so a warp keeps
// SPL*512 bytes of codes in flight.  Activations come from shared memory
// (staged once per block as fp32) when ntok*in_f floats fit in xs_floats,
// else through L1.
template <typename XT, int NT, int SPL>
__global__ void __launch_bounds__(256, NT == 1 ? 4 : 1)
affine_gemv_kernel(const XT *__restrict__ x, const uint8_t *__restrict__ codes,
                   const float *__restrict__ scales, const float *__restrict__ offsets,
                   const float *__restrict__ bias, const __grid_constant__ OutPtrs out, uint32_t ldy,
                   uint32_t n0, uint32_t ntok, uint32_t in_f, uint32_t out_f,
                   uint32_t gs, uint32_t gs_shift, uint32_t xs_floats)
{
    extern __shared__ float xs[];
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
    const uint32_t ng = in_f / gs;
    const uint32_t slices = in_f / 16u;
    const bool staged = (size_t)ntok * in_f <= xs_floats;
    // the next kernel on the stream may start loading its weights now; this
    // one reads activations and writes outputs only after the kernel before
    // it has finished (griddepcontrol.wait)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // this warp's rows of codes go to L2 by bulk prefetch (the copy engine
    // streams them from DRAM); the loads below then mostly hit L2
    if (lane == 0 && (in_f & 15u) == 0)
        for (uint32_t o = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; o < out_f; o += warps)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(codes + (size_t)o * in_f), "r"(in_f)
                         : "memory");
    __syncwarp();   // lane 0's prefetches are issued before any lane blocks in griddepcontrol.wait
    if (staged) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (uint32_t i = threadIdx.x; i < ntok * in_f; i += blockDim.x)
            xs[i] = xval<XT>(x + (size_t)n0 * in_f + i);
        __syncthreads();
    }
    for (uint32_t o = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; o < out_f; o += warps) {
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
        const uint4 *crow = reinterpret_cast<const uint4 *>(codes + (size_t)o * in_f);
        for (uint32_t base = 0; base < slices; base += 32u * SPL) {
            uint4 cw[SPL];
#pragma unroll
            for (int i = 0; i < SPL; ++i) {
                const uint32_t sl = base + (uint32_t)i * 32u + lane;
                if (sl < slices) cw[i] = __ldg(crow + sl);
            }
            // the pass's scales and offsets: one group per lane when the pass
            // spans at most 32 groups (then handed out by shuffles)
            const uint32_t g0 = group_of(base, gs, gs_shift);
            const uint32_t g1 = group_of(min(base + 32u * SPL, slices) - 1u, gs, gs_shift) + 1u;
            const bool by_lane = g1 - g0 <= 32u;
            float s_l = 0.0f, f_l = 0.0f;
            if (by_lane && g0 + lane < g1) {
                s_l = __ldg(scales + (size_t)o * ng + g0 + lane);
                f_l = __ldg(offsets + (size_t)o * ng + g0 + lane);
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
            for (int i = 0; i < SPL; ++i) {
                const uint32_t sl = base + (uint32_t)i * 32u + lane;
                const uint32_t g = group_of(sl < slices ? sl : slices - 1u, gs, gs_shift);
                float sv_i, fv_i;
                if (by_lane) {
                    sv_i = __shfl_sync(0xffffffffu, s_l, (g - g0) & 31u);
                    fv_i = __shfl_sync(0xffffffffu, f_l, (g - g0) & 31u);
                } else {
                    sv_i = __ldg(scales + (size_t)o * ng + g);
                    fv_i = __ldg(offsets + (size_t)o * ng + g);
                }
                if (sl >= slices) continue;
                float q[16];
                const uint32_t w[4] = {cw[i].x, cw[i].y, cw[i].z, cw[i].w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
#pragma unroll
                    for (int b = 0; b < 4; ++b) q[4 * j + b] = code_to_float(w[j], (uint32_t)b);
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if ((uint32_t)t < ntok) {
                        float xv[16];
                        if (staged) {
                            const float4 *p4 = reinterpret_cast<const float4 *>(xs + (size_t)t * in_f + sl * 16u);
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const float4 v4 = p4[u];
                                xv[4 * u] = v4.x; xv[4 * u + 1] = v4.y; xv[4 * u + 2] = v4.z; xv[4 * u + 3] = v4.w;
                            }
                        } else {
                            XLoad<XT>::load16(x + (size_t)(n0 + t) * in_f + sl * 16u, xv);
                        }
                        float dot = 0.0f, xsum = 0.0f;
#pragma unroll
                        for (int u = 0; u < 16; ++u) {
                            dot = fmaf(xv[u], q[u], dot);
                            xsum += xv[u];
                        }
                        acc[t] = fmaf(sv_i, dot, fmaf(fv_i, xsum, acc[t]));
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float v = acc[t];
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
            acc[t] = v;
        }
        if (lane == 0) {
            const float bo = bias ? __ldg(bias + o) : 0.0f;
#pragma unroll
            for (int t = 0; t < NT; ++t)
                if ((uint32_t)t < ntok)
                    for (uint32_t k = 0; k < out.n; ++k) out.y[k][(size_t)(n0 + t) * ldy + o] = acc[t] + bo;
        }
    }
}

// One-token GEMV over a batch of matrices (a layer's projections, or one
// matrix).  The rows of all jobs form one sequence; each CTA owns a
// contiguous range of it holding an equal share of the codes (so at most a
// few jobs), stages the job's
// activations once in shared memory as fp32 planes laid out for
// conflict-free 16-byte reads, with the sum of every 16-activation slice,
// and its warps take the range's rows in turn: 16 codes per lane per 128-bit
// load, a row's 4 KB pass in flight at once, the next two of the warp's rows
// sent to L2 by bulk prefetch.  Per slice: 16 byte-permute code widenings,
// 16 fp32 FMAs against the staged activations, the group scale times the
// dot and the group offset times the slice sum.  A launch carries every
// matrix of the batch, so launch, ramp-up and tail are paid once.
constexpr uint32_t kMaxGemvJobs = 8;
constexpr size_t kGemvStageMax = 200u * 1024u;   // staged activations + slice sums

struct GemvJob {
    const void *x;              // activations of this matrix, one token
    const uint8_t *codes;       // [out_f, in_f]
    const float *scales, *offsets, *bias;
    OutPtrs out;                // each output: o at out.y[k][o]
    uint32_t in_f, out_f, gs, gs_shift, ng;
    uint32_t row_begin;         // first row of the job in the batch's sequence
    uint64_t code_begin;        // codes of the jobs before this one
};

struct GemvJobs {
    GemvJob job[kMaxGemvJobs];
    uint32_t n, total_rows;
    uint64_t total_codes;
};

// First row of the batch sequence that starts at or after code position w.
__device__ __forceinline__ uint32_t row_at(const GemvJobs &J, uint64_t w)
{
    if (w >= J.total_codes) return J.total_rows;
    uint32_t j = 0;
    while (j + 1u < J.n && w >= J.job[j + 1u].code_begin) ++j;
    const GemvJob &b = J.job[j];
    const uint64_t rows_in = (w - b.code_begin + b.in_f - 1u) / b.in_f;
    return b.row_begin + (uint32_t)(rows_in < b.out_f ? rows_in : b.out_f);
}

template <typename XT>
__global__ void __launch_bounds__(256, 4)
affine_gemv_jobs_kernel(const __grid_constant__ GemvJobs J)
{
    constexpr int SPL = 8;
    extern __shared__ __align__(16) float xsm[];   // planes [4][slices] float4, then slice sums [slices]
    const uint32_t lane = threadIdx.x & 31u, wib = threadIdx.x >> 5;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // this CTA's rows: an equal share of the batch's codes, cut at whole rows
    const uint32_t r0 = row_at(J, J.total_codes * blockIdx.x / gridDim.x);
    const uint32_t r1 = row_at(J, J.total_codes * (blockIdx.x + 1u) / gridDim.x);
    uint32_t j = 0;
    while (j + 1u < J.n && r0 >= J.job[j + 1u].row_begin) ++j;
    bool waited = false;
    for (uint32_t seg = r0; seg < r1; ++j) {
        const GemvJob &b = J.job[j];
        const uint32_t seg_end = min(r1, b.row_begin + b.out_f);
        const uint32_t in_f = b.in_f, gs = b.gs, gs_shift = b.gs_shift, ng = b.ng;
        const uint32_t slices = in_f / 16u;
        const uint32_t first = seg + wib;
        // the warp's rows of this job: first, first + 8, ... < seg_end
        auto prefetch = [&](uint32_t r) {
            if (lane == 0 && r < seg_end)
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;"
                             ::"l"(b.codes + (size_t)(r - b.row_begin) * in_f), "r"(in_f) : "memory");
        };
        prefetch(first);
        prefetch(first + 8u);
        // stage this job's activations (the previous kernel's output)
        if (!waited) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            waited = true;
        }
        __syncthreads();    // the previous job's activations are no longer read
        float4 *planes = reinterpret_cast<float4 *>(xsm);   // 4 * slices float4 = in_f floats
        float *ssum = xsm + in_f;                            // slices floats
        for (uint32_t sl = threadIdx.x; sl < slices; sl += blockDim.x) {
            float v[16];
            XLoad<XT>::load16(static_cast<const XT *>(b.x) + (size_t)sl * 16u, v);
            float sum = 0.0f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                planes[(size_t)u * slices + sl] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
                sum += (v[4 * u] + v[4 * u + 1]) + (v[4 * u + 2] + v[4 * u + 3]);
            }
            ssum[sl] = sum;
        }
        __syncthreads();
        for (uint32_t r = first; r < seg_end; r += 8u) {
            prefetch(r + 16u);
            const uint32_t o = r - b.row_begin;
            const uint4 *crow = reinterpret_cast<const uint4 *>(b.codes + (size_t)o * in_f);
            float acc = 0.0f;
            for (uint32_t base = 0; base < slices; base += 32u * SPL) {
                uint4 cw[SPL];
#pragma unroll
                for (int i = 0; i < SPL; ++i) {
                    const uint32_t sl = base + (uint32_t)i * 32u + lane;
                    if (sl < slices) cw[i] = __ldg(crow + sl);
                }
                const uint32_t g0 = group_of(base, gs, gs_shift);
                const uint32_t g1 = group_of(min(base + 32u * SPL, slices) - 1u, gs, gs_shift) + 1u;
                const bool by_lane = g1 - g0 <= 32u;
                float s_l = 0.0f, f_l = 0.0f;
                if (by_lane && g0 + lane < g1) {
                    s_l = __ldg(b.scales + (size_t)o * ng + g0 + lane);
                    f_l = __ldg(b.offsets + (size_t)o * ng + g0 + lane);
                }
#pragma unroll
                for (int i = 0; i < SPL; ++i) {
                    const uint32_t sl = base + (uint32_t)i * 32u + lane;
                    const uint32_t slc = sl < slices ? sl : slices - 1u;
                    const uint32_t g = group_of(slc, gs, gs_shift);
                    float sv_i, fv_i;
                    if (by_lane) {
                        sv_i = __shfl_sync(0xffffffffu, s_l, (g - g0) & 31u);
                        fv_i = __shfl_sync(0xffffffffu, f_l, (g - g0) & 31u);
                    } else {
                        sv_i = __ldg(b.scales + (size_t)o * ng + g);
                        fv_i = __ldg(b.offsets + (size_t)o * ng + g);
                    }
                    if (sl >= slices) continue;
                    const uint32_t w[4] = {cw[i].x, cw[i].y, cw[i].z, cw[i].w};
                    float d[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float4 xv = planes[(size_t)u * slices + sl];
                        float t = xv.x * code_to_float(w[u], 0);
                        t = fmaf(xv.y, code_to_float(w[u], 1), t);
                        t = fmaf(xv.z, code_to_float(w[u], 2), t);
                        d[u] = fmaf(xv.w, code_to_float(w[u], 3), t);
                    }
                    acc = fmaf(sv_i, (d[0] + d[1]) + (d[2] + d[3]), fmaf(fv_i, ssum[sl], acc));
                }
            }
#pragma unroll
            for (int dd = 16; dd > 0; dd >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, dd);
            if (lane == 0) {
                const float bo = b.bias ? __ldg(b.bias + o) : 0.0f;
                for (uint32_t k = 0; k < b.out.n; ++k) b.out.y[k][o] = acc + bo;
            }
        }
        seg = seg_end;
    }
    if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <typename XT>
int launch_gemv_jobs(const GemvJobs &J, int sms, cudaStream_t s)
{
    if (J.n == 0 || J.total_rows == 0) return 0;
    uint32_t max_in = 0;
    for (uint32_t i = 0; i < J.n; ++i) max_in = J.job[i].in_f > max_in ? J.job[i].in_f : max_in;
    const size_t smem = (size_t)max_in * 4u + (size_t)(max_in / 16u) * 4u;   // fp32 planes + slice sums
    if (smem > kGemvStageMax) return 1;
    static std::atomic<uint64_t> configured{0};   // one bit per device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) { cudaGetLastError(); return -1; }
    if (!(configured.load(std::memory_order_acquire) & (1ull << dev))) {
        if (cudaFuncSetAttribute(affine_gemv_jobs_kernel<XT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kGemvStageMax) != cudaSuccess) { cudaGetLastError(); return -1; }
        configured.fetch_or(1ull << dev, std::memory_order_acq_rel);
    }
    // CTAs resident per SM: shared memory (228 KB, 1 KB reserved each) and 4 by registers
    uint32_t per_sm = (uint32_t)(233472u / (smem + 1024u));
    per_sm = per_sm > 4u ? 4u : per_sm < 1u ? 1u : per_sm;
    uint32_t blocks = (J.total_rows + 7u) / 8u;
    const uint32_t cap = (uint32_t)(sms > 0 ? sms : 148) * per_sm;
    if (blocks > cap) blocks = cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, affine_gemv_jobs_kernel<XT>, J) != cudaSuccess) { cudaGetLastError(); return -1; }
    return 0;
}

// Any shape: one thread per output, the reference's loop order.
template <typename XT>
__global__ void affine_generic_kernel(const XT *__restrict__ x, const uint8_t *__restrict__ codes,
                                      const float *__restrict__ scales,
                                      const float *__restrict__ offsets,
                                      const float *__restrict__ bias, float *__restrict__ y,
                                      uint32_t N, uint32_t in_f, uint32_t out_f, uint32_t gs)
{
    const uint32_t ng = in_f / gs;
    const uint64_t total = (uint64_t)N * out_f;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t n = (uint32_t)(i / out_f), o = (uint32_t)(i - (uint64_t)n * out_f);
        const XT *xr = x + (size_t)n * in_f;
        const uint8_t *qr = codes + (size_t)o * in_f;
        float acc = 0.0f;
        for (uint32_t g = 0; g < ng; ++g) {
            float dot = 0.0f, xs = 0.0f;
            for (uint32_t k = g * gs; k < (g + 1u) * gs; ++k) {
                const float xv = xval<XT>(xr + k);
                dot = __fadd_rn(dot, __fmul_rn(xv, (float)qr[k]));
                xs = __fadd_rn(xs, xv);
            }
            acc = __fadd_rn(acc, __fadd_rn(__fmul_rn(scales[(size_t)o * ng + g], dot),
                                           __fmul_rn(offsets[(size_t)o * ng + g], xs)));
        }
        if (bias) acc = __fadd_rn(acc, bias[o]);
        y[i] = acc;
    }
}

bool aligned(const void *p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

// out: the outputs, each [N, ldy] (a single [N, out_f] buffer for the
// reference entry points).  Several outputs or ldy != out_f need the GEMV or
// GEMM paths (group size and in_f multiples of 16, 16-B aligned x and codes).
int sm_count()
{
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

// path: HXQ_AFFINE_PATH_* (auto, CUDA-core GEMV, tensor-core GEMV, tcgen05
// GEMM); a forced path that cannot take the shape returns -1.
template <typename XT>
int run_affine(const XT *x, const uint8_t *codes, const float *scales, const float *offsets,
               const float *bias, const OutPtrs &out, uint32_t ldy, uint32_t N, uint32_t in_f, uint32_t out_f,
               uint32_t gs, cudaStream_t s, int path = HXQ_AFFINE_PATH_AUTO)
{
    if (!x || !codes || !scales || !offsets || out.n == 0 || out.n > HXQ_CUDA_MAX_PEERS) return -1;
    for (uint32_t k = 0; k < out.n; ++k)
        if (!out.y[k]) return -1;
    if (gs == 0 || in_f % gs != 0 || ldy < out_f) return -1;
    if (N == 0 || out_f == 0) return 0;
    const bool plain = out.n == 1 && ldy == out_f;
    float *y = out.y[0];
    if (in_f == 0) {  // empty reduction: bias only
        if (!plain) return -1;
        gemm_chain_break();
        affine_generic_kernel<XT><<<1, 256, 0, s>>>(x, codes, scales, offsets, bias, y, N, in_f, out_f, gs);
        return cudaGetLastError() == cudaSuccess ? 0 : -1;
    }
    if (path < HXQ_AFFINE_PATH_AUTO || path > HXQ_AFFINE_PATH_GEMM) return -1;
    if constexpr (sizeof(XT) == 2) {
        const uint16_t *xb = reinterpret_cast<const uint16_t *>(x);
        if ((path == HXQ_AFFINE_PATH_AUTO && N <= kTcGemvMaxTokens) || path == HXQ_AFFINE_PATH_TC_GEMV) {
            const TcMatrix m{xb, codes, scales, offsets, bias, out, ldy, in_f, out_f, gs};
            gemm_chain_break();
            const int r = launch_tc_gemv(1, &m, N, sm_count(), s);
            if (r <= 0) return r;  // launched (0) or failed (-1); 1 = shape not taken
            if (path == HXQ_AFFINE_PATH_TC_GEMV) return -1;
        }
        if ((path == HXQ_AFFINE_PATH_AUTO && N >= 2u) || path == HXQ_AFFINE_PATH_GEMM) {
            const int r = affine_gemm_bf16(xb, codes, scales, offsets, bias, out, ldy, N, in_f, out_f, gs, s);
            if (r <= 0) return r;
            if (path == HXQ_AFFINE_PATH_GEMM) return -1;
        }
    } else {
        if (path == HXQ_AFFINE_PATH_TC_GEMV || path == HXQ_AFFINE_PATH_GEMM) return -1;
    }
    gemm_chain_break();   // a GEMV follows
    const bool fast = gs % 16u == 0 && in_f % 16u == 0 && aligned(x, 16) && aligned(codes, 16);
    if (fast) {
        const int sms = sm_count();
        uint32_t blocks = (out_f + 7u) / 8u;
        const uint32_t cap = (uint32_t)sms * 8u;
        if (blocks > cap) blocks = cap;
        constexpr uint32_t kXsFloats = 12288;  // 48 KB of staged activations
        const uint32_t gs_shift = (gs & (gs - 1u)) == 0 ? (uint32_t)__builtin_ctz(gs) : 32u;
        if (N == 1) {
            GemvJobs J{};
            J.job[0] = GemvJob{x, codes, scales, offsets, bias, out, in_f, out_f, gs, gs_shift, in_f / gs, 0u, 0u};
            J.n = 1;
            J.total_rows = out_f;
            J.total_codes = (uint64_t)out_f * in_f;
            const int r = launch_gemv_jobs<XT>(J, sms, s);
            if (r <= 0) return r;   // 1: activations too long to stage; the kernel below takes it
        }
        for (uint32_t n0 = 0; n0 < N; n0 += kGemvTokens) {
            const uint32_t nt = N - n0 < (uint32_t)kGemvTokens ? N - n0 : (uint32_t)kGemvTokens;
            // one token: activations through L1 (staging would cost more than it saves)
            const size_t smem = (nt > 1 && (size_t)nt * in_f <= kXsFloats) ? (size_t)nt * in_f * sizeof(float) : 0;
            const uint32_t xs = smem ? kXsFloats : 0u;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(blocks);
            cfg.blockDim = dim3(256);
            cfg.dynamicSmemBytes = smem;
            cfg.stream = s;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            cudaError_t e;
            if (nt == 1)
                e = cudaLaunchKernelEx(&cfg, affine_gemv_kernel<XT, 1, 8>, x, codes, scales, offsets, bias, out, ldy, n0, nt, in_f, out_f, gs, gs_shift, xs);
            else if (nt <= 4)
                e = cudaLaunchKernelEx(&cfg, affine_gemv_kernel<XT, 4, 4>, x, codes, scales, offsets, bias, out, ldy, n0, nt, in_f, out_f, gs, gs_shift, xs);
            else
                e = cudaLaunchKernelEx(&cfg, affine_gemv_kernel<XT, kGemvTokens, 2>, x, codes, scales, offsets, bias, out, ldy, n0, nt, in_f, out_f, gs, gs_shift, xs);
            if (e != cudaSuccess) { cudaGetLastError(); return -1; }
        }
    } else {
        if (!plain || path != HXQ_AFFINE_PATH_AUTO) return -1;
        uint64_t blocks = ((uint64_t)N * out_f + 255u) / 256u;
        if (blocks > 148u * 32u) blocks = 148u * 32u;
        affine_generic_kernel<XT><<<(uint32_t)blocks, 256, 0, s>>>(x, codes, scales, offsets, bias, y, N, in_f, out_f, gs);
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace
}  // namespace hxq

namespace {
hxq::OutPtrs one_out(float *y)
{
    hxq::OutPtrs o{};
    o.y[0] = y;
    o.n = y ? 1u : 0u;
    return o;
}
}  // namespace

extern "C" {

int hxq_affine_group_matmul(const float *d_x, const hxq_affine_tensor_t *t, float *d_output,
                            uint32_t N)
{
    if (!t) return -1;
    return hxq::run_affine<float>(d_x, t->indices, t->scales, t->offsets, t->bias, one_out(d_output),
                                  t->out_features, N, t->in_features, t->out_features, t->group_size,
                                  (cudaStream_t)0);
}

int hxq_affine_matmul_flat(const float *d_x, const uint8_t *d_indices, const float *d_scales,
                           const float *d_offsets, const float *d_bias, float *d_output,
                           uint32_t N, uint32_t in_f, uint32_t out_f, uint32_t group_size)
{
    return hxq::run_affine<float>(d_x, d_indices, d_scales, d_offsets, d_bias, one_out(d_output), out_f, N,
                                  in_f, out_f, group_size, (cudaStream_t)0);
}

int hxq_affine_group_matmul_bf16(const uint16_t *d_x_bf16, const hxq_affine_tensor_t *t,
                                 float *d_output, uint32_t N, void *stream)
{
    if (!t) return -1;
    return hxq::run_affine<uint16_t>(d_x_bf16, t->indices, t->scales, t->offsets, t->bias, one_out(d_output),
                                     t->out_features, N, t->in_features, t->out_features, t->group_size,
                                     static_cast<cudaStream_t>(stream));
}

int hxq_affine_group_matmul_bf16_path(const uint16_t *d_x_bf16, const hxq_affine_tensor_t *t,
                                      float *d_output, uint32_t N, int path, void *stream)
{
    if (!t) return -1;
    return hxq::run_affine<uint16_t>(d_x_bf16, t->indices, t->scales, t->offsets, t->bias, one_out(d_output),
                                     t->out_features, N, t->in_features, t->out_features, t->group_size,
                                     static_cast<cudaStream_t>(stream), path);
}

int hxq_affine_group_matmul_bf16_auto_path(const uint16_t *d_x_bf16, const hxq_affine_tensor_t *t, uint32_t N)
{
    if (!t || N == 0) return -1;
    if (N <= hxq::kTcGemvMaxTokens &&
        hxq::tc_gemv_fits(d_x_bf16, t->indices, t->scales, t->offsets, N, t->in_features, t->out_features,
                          t->group_size))
        return HXQ_AFFINE_PATH_TC_GEMV;
    if (N >= 2u && hxq::affine_gemm_fits(d_x_bf16, t->indices, N, t->in_features, t->out_features, t->group_size))
        return HXQ_AFFINE_PATH_GEMM;
    return HXQ_AFFINE_PATH_GEMV;
}

int hxq_affine_group_matmul_bf16_multi(const uint16_t *d_x_bf16, const hxq_affine_tensor_t *t,
                                       float *const *d_ys, uint32_t n_out, uint32_t ldy, uint32_t N,
                                       void *stream)
{
    if (!t || !d_ys || n_out == 0 || n_out > HXQ_CUDA_MAX_PEERS) return -1;
    hxq::OutPtrs o{};
    for (uint32_t k = 0; k < n_out; ++k) o.y[k] = d_ys[k];
    o.n = n_out;
    return hxq::run_affine<uint16_t>(d_x_bf16, t->indices, t->scales, t->offsets, t->bias, o, ldy, N,
                                     t->in_features, t->out_features, t->group_size,
                                     static_cast<cudaStream_t>(stream));
}

int hxq_affine_group_matmul_bf16_batch(uint32_t n, const hxq_affine_tensor_t *tensors,
                                       const uint16_t *const *d_xs, float *const *d_ys, uint32_t n_out,
                                       const uint32_t *ldys, uint32_t N, void *stream)
{
    if (n == 0 || N == 0) return 0;
    if (!tensors || !d_xs || !d_ys || !ldys || n_out == 0 || n_out > HXQ_CUDA_MAX_PEERS) return -1;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto outs_of = [&](uint32_t i, hxq::OutPtrs &o) {
        o = hxq::OutPtrs{};
        for (uint32_t k = 0; k < n_out; ++k) {
            o.y[k] = d_ys[(size_t)i * n_out + k];
            if (!o.y[k]) return false;
        }
        o.n = n_out;
        return true;
    };
    // The batch in three parts, each matrix in the first that takes it:
    // up to 16 tokens, matrices that suit the tensor-core GEMV share
    // launches of up to 8; at one token, the rest that suit the streaming
    // GEMV share launches of up to 8; anything left runs one call per matrix.
    std::vector<uint8_t> done(n, 0);
    const int sms = hxq::sm_count();
    if (N <= hxq::kTcGemvBatchMaxTokens) {
        hxq::TcMatrix m[hxq::kMaxTcJobs];
        uint32_t k = 0;
        for (uint32_t i = 0; i <= n; ++i) {
            if (i < n) {
                const hxq_affine_tensor_t &t = tensors[i];
                if (ldys[i] < t.out_features ||
                    !hxq::tc_gemv_fits(d_xs[i], t.indices, t.scales, t.offsets, N, t.in_features, t.out_features,
                                       t.group_size))
                    continue;
                hxq::OutPtrs o;
                if (!outs_of(i, o)) return -1;
                m[k++] = hxq::TcMatrix{d_xs[i], t.indices, t.scales, t.offsets, t.bias, o, ldys[i], t.in_features,
                                       t.out_features, t.group_size};
                done[i] = 1;
            }
            if (k == hxq::kMaxTcJobs || (i == n && k > 0)) {
                if (hxq::launch_tc_gemv(k, m, N, sms, s) != 0) return -1;
                k = 0;
            }
        }
    }
    if (N == 1) {
        hxq::GemvJobs J{};
        uint32_t rows = 0;
        uint64_t ncodes = 0;
        for (uint32_t i = 0; i <= n; ++i) {
            if (i < n && !done[i]) {
                const hxq_affine_tensor_t &t = tensors[i];
                const bool fits = t.indices && t.scales && t.offsets && d_xs[i] && t.group_size && t.in_features &&
                                  t.group_size % 16u == 0 && t.in_features % t.group_size == 0 &&
                                  t.in_features % 16u == 0 && ldys[i] >= t.out_features &&
                                  hxq::aligned(d_xs[i], 16) && hxq::aligned(t.indices, 16) &&
                                  (size_t)t.in_features * 4u + (size_t)(t.in_features / 16u) * 4u <=
                                      hxq::kGemvStageMax;
                if (fits) {
                    hxq::OutPtrs o;
                    if (!outs_of(i, o)) return -1;
                    const uint32_t gs = t.group_size;
                    const uint32_t gs_shift = (gs & (gs - 1u)) == 0 ? (uint32_t)__builtin_ctz(gs) : 32u;
                    J.job[J.n++] = hxq::GemvJob{d_xs[i], t.indices, t.scales, t.offsets, t.bias, o, t.in_features,
                                                t.out_features, gs, gs_shift, t.in_features / gs, rows, ncodes};
                    rows += t.out_features;
                    ncodes += (uint64_t)t.out_features * t.in_features;
                    done[i] = 1;
                }
            }
            if (J.n == hxq::kMaxGemvJobs || (i == n && J.n > 0)) {
                J.total_rows = rows;
                J.total_codes = ncodes;
                if (hxq::launch_gemv_jobs<uint16_t>(J, sms, s) != 0) return -1;
                J = hxq::GemvJobs{};
                rows = 0;
                ncodes = 0;
            }
        }
    }
    // one call per matrix; consecutive GEMMs overlap their wave tails
    hxq::GemmChainScope chain(s);
    for (uint32_t i = 0; i < n; ++i) {
        if (done[i]) continue;
        const hxq_affine_tensor_t &t = tensors[i];
        hxq::OutPtrs o;
        if (!outs_of(i, o)) return -1;
        const int r = hxq::run_affine<uint16_t>(d_xs[i], t.indices, t.scales, t.offsets, t.bias, o, ldys[i], N,
                                                t.in_features, t.out_features, t.group_size, s);
        if (r != 0) return r;
    }
    return 0;
}

int hxq_affine_group_matmul_async(const float *d_x, const hxq_affine_tensor_t *t,
                                  float *d_output, uint32_t N, void *stream)
{
    if (!t) return -1;
    return hxq::run_affine<float>(d_x, t->indices, t->scales, t->offsets, t->bias, one_out(d_output),
                                  t->out_features, N, t->in_features, t->out_features, t->group_size,
                                  static_cast<cudaStream_t>(stream));
}

}  // extern "C"
