// vq_kernels.cu -- sm_100a kernels of the HXQ VQ decompress path.
//
// Fast kernel (scalar k=256 and 12-bit k=4096 x dim 2 with in_features % 4
// == 0).  Semantics follow the reference CPU decoder (hxq-native
// src/hxq.c:218-235 scalar, :239-298 12-bit, :330-350 sidecar):
//   W = codebook[index], then in-range sidecar deltas added in array order;
//   the sum of squared in-range deltas is reduced exactly (fp64), and the
//   confidence output receives the reference's own value (sqrtf of its fp32
//   running sum in array order), which the host fixes when the image is
//   built: that sum is sequential by definition, so no parallel reduction
//   can reproduce its rounding.
// Design (not a port of src/hxq_cuda.cu):
//   * the tensor is a flat stream of 2048-weight chunks; one warp owns one
//     chunk at a time and needs no CTA-wide barrier inside a chunk;
//   * index bytes arrive as coalesced 128-bit non-allocating loads
//     (3 x 512 B per warp for 12-bit, 4 x 512 B for scalar), are staged in a
//     per-warp shared buffer and unpacked with one PRMT per byte triple;
//   * the codebook sits in shared memory once per CTA and job: 4096 float2
//     (fp32 out), 4096 packed bf16x2 (bf16 out), or for k=256 a 32-way
//     lane-replicated copy that makes the scalar gather bank-conflict free;
//   * every warp store is a fully coalesced 512 B (fp32) / 256 B (bf16) row;
//   * the sidecar is a fused epilogue: the chunk's entries (pre-sorted by
//     position at upload, equal positions adjacent and in array order) are
//     applied by the same warp, the base value re-derived from the staged
//     index so no global read-modify-write is needed; squared deltas are
//     accumulated in fp64, reduced with warp shuffles, per CTA into a fixed
//     slot, and the last CTA of a job adds the slots in order (deterministic,
//     no host round trip) and stores the job's sum and confidence;
//   * one launch covers up to 64 jobs (e.g. a whole transformer layer) over
//     a grid of 4 CTAs per SM with contiguous chunk ranges per CTA.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "hxq_cuda_internal.h"

namespace hxq {
namespace {

constexpr uint32_t kCbBytes = 32768;

__device__ __forceinline__ uint4 ld_stream_v4(const uint4 *p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ SideEntry ld_entry(const SideEntry *p)
{
    uint2 v = __ldg(reinterpret_cast<const uint2 *>(p));
    return SideEntry{v.x, v.y};
}

__device__ __forceinline__ double warp_sum(double v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Byte triple j of a staged chunk as a big-endian 24-bit number
// B = b0 << 16 | b1 << 8 | b2, so index a = B >> 12 and b = B & 0xFFF
// (the pair layout of hxq.h:245-252).  Reads words q and q+1, q = 3j/4.
__device__ __forceinline__ uint32_t triple_be(const uint32_t *sw, uint32_t j)
{
    const uint32_t byte = 3u * j;
    const uint32_t q = byte >> 2, s = byte & 3u;
    const uint32_t w0 = sw[q], w1 = sw[q + 1];
    // selector nibbles: result byte0 = src byte s+2, byte1 = s+1, byte2 = s
    return __byte_perm(w0, w1, 0x3012u + s * 0x1111u);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi)
{
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

template <uint32_t KIND, bool BF16>
__device__ __forceinline__ void load_codebook(unsigned char *cb_area,
                                              const VqJob &J, uint32_t tid)
{
    // Every load of the table is in flight before a CTA waits for it, so it
    // costs one memory round trip per codebook, not one per loop trip: the
    // fp32 table is copied with asynchronous 16-byte copies (no registers;
    // the caller's barrier follows the wait), the bf16 table is converted in
    // batches small enough not to spill (the next chunk's index registers
    // are live meanwhile).
    if (KIND == kKindVq12) {
        // k is 256 or 4096 entries (even): two float2 entries per 16 bytes
        const uint32_t n2 = (J.k < 4096u ? J.k : 4096u) / 2u;
        const uint4 *src = reinterpret_cast<const uint4 *>(J.cb);
        if (!BF16) {
            const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(cb_area));
            for (uint32_t i = tid; i < n2; i += kThreads)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst + 16u * i), "l"(src + i)
                             : "memory");
            asm volatile("cp.async.wait_all;" ::: "memory");
        } else {
#pragma unroll 1
            for (uint32_t i0 = tid; i0 < n2; i0 += 2u * kThreads) {
                uint4 v[2];
#pragma unroll
                for (uint32_t m = 0; m < 2u; ++m)
                    if (i0 + m * kThreads < n2) v[m] = __ldg(src + i0 + m * kThreads);
#pragma unroll
                for (uint32_t m = 0; m < 2u; ++m) {
                    const uint32_t i = i0 + m * kThreads;
                    if (i < n2)
                        reinterpret_cast<uint2 *>(cb_area)[i] =
                            make_uint2(pack_bf16x2(__uint_as_float(v[m].x), __uint_as_float(v[m].y)),
                                       pack_bf16x2(__uint_as_float(v[m].z), __uint_as_float(v[m].w)));
                }
            }
        }
    } else {
        // lane-replicated scalar table: entry e for lane l at e*32 + l
        float *dst = reinterpret_cast<float *>(cb_area);
#pragma unroll 1
        for (uint32_t i0 = tid; i0 < 256u * 32u; i0 += 8u * kThreads) {
            float v[8];
#pragma unroll
            for (uint32_t m = 0; m < 8u; ++m) v[m] = __ldg(J.cb + ((i0 + m * kThreads) >> 5));
#pragma unroll
            for (uint32_t m = 0; m < 8u; ++m) dst[i0 + m * kThreads] = v[m];
        }
    }
}

// Inputs of one chunk, loaded one chunk ahead of their use.
template <uint32_t VPL>
struct ChunkIn {
    uint4     r[VPL];      // this lane's 16-byte pieces of the index bytes
    uint32_t  e0, e1;      // sidecar entries [e0, e1) of the chunk
    SideEntry ent;         // entry e0 + lane (if any)
    uint32_t  c;           // chunk index within its job
};

template <uint32_t VPL>
__device__ __forceinline__ void prefetch_chunk(const VqJob &J, uint32_t c, uint32_t lane,
                                               ChunkIn<VPL> &in)
{
    const uint4 *src = J.idx + (size_t)c * (VPL * 32u);
#pragma unroll
    for (uint32_t q = 0; q < VPL; ++q) in.r[q] = ld_stream_v4(src + q * 32u + lane);
    in.e0 = __ldg(J.chunk_ptr + c);
    in.e1 = __ldg(J.chunk_ptr + c + 1);
    in.c = c;
}

template <uint32_t VPL>
__device__ __forceinline__ void prefetch_entry(const VqJob &J, uint32_t lane, ChunkIn<VPL> &in)
{
    in.ent = SideEntry{0u, 0u};
    if (in.e0 + lane < in.e1) in.ent = ld_entry(J.ent + in.e0 + lane);
}

template <uint32_t VPL>
__device__ __forceinline__ void stage_chunk(const ChunkIn<VPL> &in, uint4 *stage, uint32_t lane)
{
    __syncwarp();  // previous chunk's readers of `stage` are done
#pragma unroll
    for (uint32_t q = 0; q < VPL; ++q) stage[q * 32u + lane] = in.r[q];
    __syncwarp();
}

// One 12-bit chunk (512 triples, 2048 weights) whose index bytes are already
// staged in `stage` (stage_chunk).
template <bool BF16, bool CHECK_K>
__device__ __forceinline__ void chunk_vq12(const VqJob &J, uint32_t c, const ChunkIn<3> &in,
                                           const unsigned char *cb_area, uint4 *stage,
                                           uint32_t lane, double &acc, uint32_t &errflag)
{
    const uint32_t e0 = in.e0, e1 = in.e1;
    const uint64_t w0 = (uint64_t)c * kChunkW;
    const uint64_t left = J.numel - w0;
    const uint32_t ntrip = (left >= kChunkW ? kChunkW : (uint32_t)left) >> 2;
    const uint32_t *sw = reinterpret_cast<const uint32_t *>(stage);

#pragma unroll 2
    for (uint32_t m = 0; m < 16u; ++m) {
        const uint32_t jt = m * 32u + lane;
        if (jt < ntrip) {
            const uint32_t B = triple_be(sw, jt);
            const uint32_t a = (B >> 12) & 0xFFFu, b = B & 0xFFFu;
            if (CHECK_K && (a >= J.k || b >= J.k)) errflag |= kErrIndexOOB;
            if (!BF16) {
                const float2 *cb = reinterpret_cast<const float2 *>(cb_area);
                const float2 va = cb[a], vb = cb[b];
                float4 *dst = reinterpret_cast<float4 *>(J.out) + (w0 >> 2) + jt;
                *dst = make_float4(va.x, va.y, vb.x, vb.y);
            } else {
                const uint32_t *cb = reinterpret_cast<const uint32_t *>(cb_area);
                uint2 *dst = reinterpret_cast<uint2 *>(J.out) + (w0 >> 2) + jt;
                *dst = make_uint2(cb[a], cb[b]);
            }
        }
    }

    if (e1 == e0) return;  // warp-uniform
    __syncwarp();          // base stores of the chunk precede the corrections
    for (uint32_t base = e0; base < e1; base += 32u) {
        const uint32_t e = base + lane;
        if (e >= e1) continue;
        const SideEntry en = (base == e0) ? in.ent : ld_entry(J.ent + e);
        const float v = __uint_as_float(en.y);
        acc += (double)v * (double)v;
        const uint32_t run = en.x >> 16;
        if (run == 0u) continue;
        const uint32_t off = en.x & 0xFFFFu;
        const uint32_t B = triple_be(sw, off >> 2);
        const uint32_t id = ((off >> 1) & 1u) ? (B & 0xFFFu) : ((B >> 12) & 0xFFFu);
        if (CHECK_K && id >= J.k) continue;  // already flagged by the gather
        float val;
        if (!BF16)
            val = reinterpret_cast<const float *>(cb_area)[2u * id + (off & 1u)];
        else
            val = __ldg(J.cb + 2u * id + (off & 1u));
        val = __fadd_rn(val, v);
        for (uint32_t r = 1; r < run; ++r)
            val = __fadd_rn(val, __uint_as_float(ld_entry(J.ent + e + r).y));
        if (!BF16)
            reinterpret_cast<float *>(J.out)[w0 + off] = val;
        else
            reinterpret_cast<__nv_bfloat16 *>(J.out)[w0 + off] = __float2bfloat16_rn(val);
    }
}

// One scalar chunk (2048 uint8 indices, 2048 weights), index bytes staged.
template <bool BF16>
__device__ __forceinline__ void chunk_scalar(const VqJob &J, uint32_t c, const ChunkIn<4> &in,
                                             const unsigned char *cb_area, uint4 *stage,
                                             uint32_t lane, double &acc)
{
    const uint32_t e0 = in.e0, e1 = in.e1;
    const SideEntry ent = in.ent;
    const uint64_t w0 = (uint64_t)c * kChunkW;
    const uint64_t left = J.numel - w0;
    const uint32_t nw = left >= kChunkW ? kChunkW : (uint32_t)left;
    const uint32_t *sw = reinterpret_cast<const uint32_t *>(stage);
    const float *cbr = reinterpret_cast<const float *>(cb_area);

#pragma unroll 2
    for (uint32_t p = 0; p < 16u; ++p) {
        const uint32_t w = p * 32u + lane;
        const uint32_t first = 4u * w;
        if (first >= nw) continue;
        const uint32_t word = sw[w];
        const float f0 = cbr[((word      ) & 0xFFu) * 32u + lane];
        const float f1 = cbr[((word >>  8) & 0xFFu) * 32u + lane];
        const float f2 = cbr[((word >> 16) & 0xFFu) * 32u + lane];
        const float f3 = cbr[((word >> 24)        ) * 32u + lane];
        if (first + 4u <= nw) {
            if (!BF16) {
                reinterpret_cast<float4 *>(J.out)[(w0 >> 2) + w] = make_float4(f0, f1, f2, f3);
            } else {
                reinterpret_cast<uint2 *>(J.out)[(w0 >> 2) + w] =
                    make_uint2(pack_bf16x2(f0, f1), pack_bf16x2(f2, f3));
            }
        } else {  // ragged tail of the last chunk
            const float f[4] = {f0, f1, f2, f3};
            for (uint32_t i = 0; first + i < nw; ++i) {
                if (!BF16) reinterpret_cast<float *>(J.out)[w0 + first + i] = f[i];
                else reinterpret_cast<__nv_bfloat16 *>(J.out)[w0 + first + i] = __float2bfloat16_rn(f[i]);
            }
        }
    }

    if (e1 == e0) return;
    __syncwarp();
    const uint8_t *sb = reinterpret_cast<const uint8_t *>(stage);
    for (uint32_t base = e0; base < e1; base += 32u) {
        const uint32_t e = base + lane;
        if (e >= e1) continue;
        const SideEntry en = (base == e0) ? ent : ld_entry(J.ent + e);
        const float v = __uint_as_float(en.y);
        acc += (double)v * (double)v;
        const uint32_t run = en.x >> 16;
        if (run == 0u) continue;
        const uint32_t off = en.x & 0xFFFFu;
        float val = cbr[(uint32_t)sb[off] * 32u];
        val = __fadd_rn(val, v);
        for (uint32_t r = 1; r < run; ++r)
            val = __fadd_rn(val, __uint_as_float(ld_entry(J.ent + e + r).y));
        if (!BF16)
            reinterpret_cast<float *>(J.out)[w0 + off] = val;
        else
            reinterpret_cast<__nv_bfloat16 *>(J.out)[w0 + off] = __float2bfloat16_rn(val);
    }
}

template <uint32_t KIND>
__host__ __device__ constexpr uint32_t stage_bytes()
{
    return (KIND == kKindVq12 ? kChunkBytes12 : kChunkBytes8) + kIdxPad;
}

template <uint32_t KIND>
__host__ __device__ constexpr uint32_t fast_smem_bytes()
{
    return kCbBytes + kWarps * stage_bytes<KIND>();
}

// First job whose unit range contains u, scanning forward from j (the units
// a CTA receives only increase).
__device__ __forceinline__ uint32_t job_of_unit(const VqLaunch &p, uint32_t j, uint32_t u)
{
    while (j + 1u < p.n_jobs && u >= p.job[j].unit_begin + p.job[j].n_units) ++j;
    return j;
}

// A unit's warp partials are added in order into the unit's slot (lane 0
// of warp 0, after the CTA barrier that completed the unit).  The slots are
// added per job by sumsq_reduce_kernel, launched after this kernel on the
// same stream: no fences or counters here, whose round trips stalled the
// CTA at its next barrier and, for the last job, sat on the launch's tail
// (7B layer: 173.3 us with them, 162.7 without).  Without a requested
// exact sum the job's first unit stores the confidence (the image's own
// value).
__device__ __forceinline__ void finish_unit(const VqLaunch &p, uint32_t j, uint32_t u,
                                            const double *red, uint32_t lane)
{
    const VqJob &J = p.job[j];
    if (lane != 0) return;
    if (!J.sumsq) {
        if (u == J.unit_begin && J.conf) *J.conf = J.ref_conf;
        return;
    }
    double s = 0.0;
#pragma unroll
    for (uint32_t w = 0; w < kWarps; ++w) s += red[w];
    p.slots[u] = s;
}

template <uint32_t KIND, bool BF16, bool CHECK_K>
__global__ void __launch_bounds__(kThreads, ctas_per_sm(KIND))
vq_fast_kernel(const __grid_constant__ VqLaunch p)
{
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ uint32_t s_unit[3];
    __shared__ double s_red[2][kWarps];
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    unsigned char *cb_area = smem;
    uint4 *stage = reinterpret_cast<uint4 *>(smem + kCbBytes + warp * stage_bytes<KIND>());
    constexpr uint32_t VPL = (KIND == kKindVq12) ? 3u : 4u;
    const uint32_t total = p.total_units;
    const uint32_t cpw = p.cpw, unit_chunks = cpw * kWarps;   // chunk c*kWarps + w of a unit -> warp w

    // Units are handed out by an atomic counter, two ahead of use, so a
    // warp knows its next chunk (and prefetches it) while it works on the
    // current one, and faster SMs simply take more units.  A launch with one
    // CTA per unit (small tensors) takes unit blockIdx.x without the counter,
    // whose round trips would sit on its critical path.
    const bool one_each = total <= gridDim.x;
    if (tid == 0) {
        if (one_each) {
            s_unit[0] = blockIdx.x;
            s_unit[1] = total;
        } else {
            s_unit[0] = atomicAdd(p.work, 1u);
            s_unit[1] = s_unit[0] < total ? atomicAdd(p.work, 1u) : total;
        }
    }
    __syncthreads();

    uint32_t u = s_unit[0];
    uint32_t j = 0, cb_job = 0xFFFFFFFFu;
    uint32_t errflag = 0;
    ChunkIn<VPL> cur, nxt;
    bool have_cur = false;
    if (u < total) {
        j = job_of_unit(p, 0, u);
        const uint32_t c = (u - p.job[j].unit_begin) * unit_chunks + warp;
        if (c < p.job[j].n_chunks) {
            prefetch_chunk<VPL>(p.job[j], c, lane, cur);
            prefetch_entry<VPL>(p.job[j], lane, cur);
            have_cur = true;
        }
    }
    for (uint32_t it = 0; u < total; ++it) {
        if (j != cb_job) {  // every thread is past the previous unit (barrier below)
            load_codebook<KIND, BF16>(cb_area, p.job[j], tid);
            __syncthreads();
            cb_job = j;
        }
        const uint32_t un = s_unit[(it + 1u) % 3u];
        if (tid == 0) s_unit[(it + 2u) % 3u] = (un < total && !one_each) ? atomicAdd(p.work, 1u) : total;
        const uint32_t jn = un < total ? job_of_unit(p, j, un) : j;
        const uint32_t ubase = (u - p.job[j].unit_begin) * unit_chunks + warp;
        double acc = 0.0;
#pragma unroll 1
        for (uint32_t k = 0; k < cpw; ++k) {
            // stage this chunk first: its index registers are then free for the next one
            if (have_cur) stage_chunk<VPL>(cur, stage, lane);
            // this warp's next chunk: the unit's next one, else the first of unit un
            bool have_nxt = false;
            uint32_t jx = j;
            if (k + 1u < cpw) {
                const uint32_t c = ubase + (k + 1u) * kWarps;
                if (c < p.job[j].n_chunks) {
                    prefetch_chunk<VPL>(p.job[j], c, lane, nxt);
                    have_nxt = true;
                }
            } else if (un < total) {
                jx = jn;
                const uint32_t c = (un - p.job[jn].unit_begin) * unit_chunks + warp;
                if (c < p.job[jn].n_chunks) {
                    prefetch_chunk<VPL>(p.job[jn], c, lane, nxt);
                    have_nxt = true;
                }
            }
            if (have_cur) {
                if constexpr (KIND == kKindVq12)
                    chunk_vq12<BF16, CHECK_K>(p.job[j], cur.c, cur, cb_area, stage, lane, acc, errflag);
                else
                    chunk_scalar<BF16>(p.job[j], cur.c, cur, cb_area, stage, lane, acc);
            }
            if (have_nxt) {
                prefetch_entry<VPL>(p.job[jx], lane, nxt);
                cur = nxt;
            }
            have_cur = have_nxt;
        }
        acc = warp_sum(acc);
        if (lane == 0) s_red[it & 1u][warp] = acc;
        __syncthreads();  // s_red and s_unit[(it+2)%3] published; codebook free
        if (warp == 0) finish_unit(p, j, u, s_red[it & 1u], lane);
        u = un;
        j = jn;
    }
    if (CHECK_K && errflag) atomicOr(p.err, errflag);
    if (tid == 0 && !one_each) {  // the last CTA out leaves the work counters at zero
        __threadfence();
        if (atomicAdd(p.work + 1, 1u) + 1u == gridDim.x) {
            p.work[0] = 0u;
            p.work[1] = 0u;
        }
    }
}

// The exact sum of squared sidecar deltas of job blockIdx.x (when
// requested): its unit slots added in a fixed order -- thread i sums slots
// i, i + 256, ... in order, eight loads in flight, then warp 0 adds eight
// per lane in order and the lanes by a fixed butterfly -- so the result does
// not depend on which SM ran which unit.  Stores the sum and the confidence.
__global__ void __launch_bounds__(kThreads) sumsq_reduce_kernel(const __grid_constant__ VqLaunch p)
{
    __shared__ double red[kThreads];
    const VqJob &J = p.job[blockIdx.x];
    if (!J.sumsq) return;
    const uint32_t tid = threadIdx.x;
    const double *sl = p.slots + J.unit_begin;
    double v[8];
#pragma unroll
    for (uint32_t q = 0; q < 8u; ++q) {
        const uint32_t i = tid + q * kThreads;
        v[q] = i < J.n_units ? sl[i] : 0.0;
    }
    double t = 0.0;
#pragma unroll
    for (uint32_t q = 0; q < 8u; ++q) t += v[q];
    for (uint32_t i = tid + 8u * kThreads; i < J.n_units; i += kThreads) t += sl[i];
    red[tid] = t;
    __syncthreads();
    if (tid < 32u) {
        double w = 0.0;
#pragma unroll
        for (uint32_t q = 0; q < kThreads / 32u; ++q) w += red[tid * (kThreads / 32u) + q];
        w = warp_sum(w);
        if (tid == 0) {
            *J.sumsq = w;
            if (J.conf) *J.conf = J.ref_conf;
        }
    }
}

template <uint32_t KIND, bool BF16, bool CHECK_K>
cudaError_t launch_one(const VqLaunch &p, cudaStream_t s)
{
    constexpr uint32_t smem = fast_smem_bytes<KIND>();
    vq_fast_kernel<KIND, BF16, CHECK_K><<<p.grid, kThreads, smem, s>>>(p);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Generic kernels: any shape and output alignment, one image per launch.

__device__ __forceinline__ void store_out(void *out, uint64_t i, float v, int bf16)
{
    if (bf16) reinterpret_cast<__nv_bfloat16 *>(out)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float *>(out)[i] = v;
}

__global__ void generic_decompress_kernel(const __grid_constant__ GenericJob j,
                                          uint32_t *err)
{
    uint32_t errflag = 0;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j.kind == kKindVq12 || j.kind == kKindVq12Any) {
        const uint64_t units = (uint64_t)j.rows * j.triples_per_row;
        for (uint64_t u = tid; u < units; u += stride) {
            const uint32_t r = (uint32_t)(u / j.triples_per_row);
            const uint32_t t = (uint32_t)(u - (uint64_t)r * j.triples_per_row);
            const uint8_t *pb = j.idx + u * 3u;
            const uint32_t b0 = pb[0], b1 = pb[1], b2 = pb[2];
            const uint32_t a = (b0 << 4) | (b1 >> 4);
            const uint32_t b = ((b1 & 0xFu) << 8) | b2;
            if (a >= j.k || b >= j.k) { errflag = kErrIndexOOB; continue; }
            const uint64_t rowbase = (uint64_t)r * j.in_f;
            const uint32_t ca = 4u * t, cbc = ca + 2u;
            if (ca + 1u < j.in_f) {
                store_out(j.out, rowbase + ca, j.cb[2u * a], j.bf16);
                store_out(j.out, rowbase + ca + 1u, j.cb[2u * a + 1u], j.bf16);
            }
            if (cbc + 1u < j.in_f) {
                store_out(j.out, rowbase + cbc, j.cb[2u * b], j.bf16);
                store_out(j.out, rowbase + cbc + 1u, j.cb[2u * b + 1u], j.bf16);
            }
        }
    } else if (j.kind == kKindRaw) {
        // nothing to reconstruct
    } else if (j.kind == kKindScalar) {
        const uint64_t n = (uint64_t)j.rows * j.in_f;
        for (uint64_t i = tid; i < n; i += stride) store_out(j.out, i, j.cb[j.idx[i]], j.bf16);
    } else {  // affine: rounded product, then rounded add (src/hxq.c:320)
        const uint64_t n = (uint64_t)j.rows * j.in_f;
        const uint32_t ng = j.in_f / j.gs;
        for (uint64_t i = tid; i < n; i += stride) {
            const uint32_t o = (uint32_t)(i / j.in_f);
            const uint32_t c = (uint32_t)(i - (uint64_t)o * j.in_f);
            const uint64_t g = (uint64_t)o * ng + c / j.gs;
            const float w = __fadd_rn(__fmul_rn((float)j.idx[i], j.scales[g]), j.offsets[g]);
            store_out(j.out, i, w, j.bf16);
        }
    }
    if (errflag) atomicOr(err, errflag);
}

// Value a position holds before its sidecar corrections.  For 12-bit rows
// whose last pair is incomplete the reference never writes that column, so
// the correction lands on whatever the buffer held: read it back.
__device__ __forceinline__ bool base_value(const GenericJob &j, uint32_t pos, float &v)
{
    if (j.kind == kKindScalar) {
        v = j.cb[j.idx[pos]];
        return true;
    }
    if (j.kind == kKindRaw) {
        v = reinterpret_cast<const float *>(j.out)[pos];
        return true;
    }
    const uint32_t r = pos / j.in_f, c = pos - r * j.in_f;
    if (j.kind == kKindAffine) {
        const uint32_t ng = j.in_f / j.gs;
        const uint64_t g = (uint64_t)r * ng + c / j.gs;
        v = __fadd_rn(__fmul_rn((float)j.idx[pos], j.scales[g]), j.offsets[g]);
        return true;
    }
    if ((c | 1u) < j.in_f) {
        const uint8_t *pb = j.idx + ((uint64_t)r * j.triples_per_row + (c >> 2)) * 3u;
        const uint32_t b0 = pb[0], b1 = pb[1], b2 = pb[2];
        const uint32_t id = ((c >> 1) & 1u) ? (((b1 & 0xFu) << 8) | b2) : ((b0 << 4) | (b1 >> 4));
        if (id >= j.k) return false;
        v = j.cb[2u * id + (c & 1u)];
        return true;
    }
    if (j.bf16)
        v = __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(j.out)[pos]);
    else
        v = reinterpret_cast<const float *>(j.out)[pos];
    return true;
}

// Chunk of entry e in the chunk-relative encoding: the last c with
// chunk_ptr[c] <= e.
__device__ __forceinline__ uint32_t chunk_of_entry(const uint32_t *cp, uint32_t n_chunks, uint32_t e)
{
    uint32_t lo = 0, hi = n_chunks - 1u;
    while (lo < hi) {
        const uint32_t mid = lo + (hi - lo + 1u) / 2u;
        if (__ldg(cp + mid) <= e) lo = mid; else hi = mid - 1u;
    }
    return lo;
}

__global__ void generic_sidecar_kernel(const __grid_constant__ GenericJob j,
                                       double *slots, uint32_t *counter)
{
    __shared__ double red[32];
    double acc = 0.0;
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < j.n_ent; e += stride) {
        const SideEntry en = ld_entry(j.ent + e);
        const float v = __uint_as_float(en.y);
        acc += (double)v * (double)v;
        uint32_t pos, run;
        if (j.chunk_ptr) {  // fast-image encoding: run length marks the head
            run = en.x >> 16;
            if (run == 0u) continue;
            pos = chunk_of_entry(j.chunk_ptr, j.n_chunks, e) * kChunkW + (en.x & 0xFFFFu);
        } else {
            if (e > 0 && ld_entry(j.ent + e - 1).x == en.x) continue;  // not a run head
            pos = en.x;
            run = 1u;
            while (e + run < j.n_ent && ld_entry(j.ent + e + run).x == pos) ++run;
        }
        float val;
        if (!base_value(j, pos, val)) continue;
        val = __fadd_rn(val, v);
        for (uint32_t r = 1; r < run; ++r) val = __fadd_rn(val, __uint_as_float(ld_entry(j.ent + e + r).y));
        store_out(j.out, pos, val, j.bf16);
    }
    acc = warp_sum(acc);
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (uint32_t w = 0; w < blockDim.x / 32u; ++w) s += red[w];
        slots[blockIdx.x] = s;
        __threadfence();
        const uint32_t prev = atomicAdd(counter, 1u);
        if (prev + 1u == gridDim.x) {
            __threadfence();
            double tot = 0.0;
            for (uint32_t i = 0; i < gridDim.x; ++i) tot += __ldcg(slots + i);
            if (j.sumsq) *j.sumsq = tot;
            if (j.conf) *j.conf = j.conf_exact ? (float)sqrt(tot) : j.ref_conf;
            *counter = 0u;
        }
    }
}

template <uint32_t KIND, bool BF16, bool CHECK_K>
cudaError_t configure_one()
{
    return cudaFuncSetAttribute(vq_fast_kernel<KIND, BF16, CHECK_K>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                fast_smem_bytes<KIND>());
}

}  // namespace

// Opt every fast-kernel instantiation into its dynamic shared memory size;
// called once per device before the first launch.
cudaError_t configure_vq_kernels()
{
    cudaError_t e;
    if ((e = configure_one<kKindVq12, false, false>()) != cudaSuccess) return e;
    if ((e = configure_one<kKindVq12, false, true>()) != cudaSuccess) return e;
    if ((e = configure_one<kKindVq12, true, false>()) != cudaSuccess) return e;
    if ((e = configure_one<kKindVq12, true, true>()) != cudaSuccess) return e;
    if ((e = configure_one<kKindScalar, false, false>()) != cudaSuccess) return e;
    return configure_one<kKindScalar, true, false>();
}

uint32_t fast_cpw(uint64_t chunks, int sms, uint32_t kind)
{
    const uint64_t resident = (uint64_t)(sms > 0 ? sms : 148) * ctas_per_sm(kind);
    return chunks >= 4u * resident * unit_chunks(kChunksPerWarp) ? kChunksPerWarp : 1u;
}

uint32_t fast_grid(uint64_t total_units, int sms, uint32_t kind)
{
    uint64_t g = (uint64_t)(sms > 0 ? sms : 148) * ctas_per_sm(kind);
    if (g > total_units) g = total_units;
    return (uint32_t)(g == 0 ? 1 : g);
}

cudaError_t launch_vq_fast(const VqLaunch &p, uint32_t kind, int bf16,
                           int check_k, cudaStream_t s)
{
    cudaError_t e;
    if (kind == kKindVq12) {
        if (bf16) e = check_k ? launch_one<kKindVq12, true, true>(p, s)
                              : launch_one<kKindVq12, true, false>(p, s);
        else e = check_k ? launch_one<kKindVq12, false, true>(p, s)
                         : launch_one<kKindVq12, false, false>(p, s);
    } else {
        e = bf16 ? launch_one<kKindScalar, true, false>(p, s)
                 : launch_one<kKindScalar, false, false>(p, s);
    }
    if (e != cudaSuccess) return e;
    bool sums = false;
    for (uint32_t j = 0; j < p.n_jobs; ++j) sums |= p.job[j].sumsq != nullptr;
    if (!sums) return cudaSuccess;
    sumsq_reduce_kernel<<<p.n_jobs, kThreads, 0, s>>>(p);
    return cudaGetLastError();
}

uint32_t vq_fast_launches(const VqLaunch &p)
{
    for (uint32_t j = 0; j < p.n_jobs; ++j)
        if (p.job[j].sumsq) return 2u;
    return 1u;
}

cudaError_t launch_generic(const GenericJob &j, const Scratch &sc, cudaStream_t s)
{
    uint64_t units;
    if (j.kind == kKindVq12 || j.kind == kKindVq12Any)
        units = (uint64_t)j.rows * j.triples_per_row;
    else if (j.kind == kKindRaw)
        units = 0;
    else
        units = (uint64_t)j.rows * j.in_f;
    if (units > 0) {
        uint64_t blocks = (units + 255u) / 256u;
        if (blocks > 148u * 16u) blocks = 148u * 16u;
        generic_decompress_kernel<<<(uint32_t)blocks, 256, 0, s>>>(j, sc.err);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (j.n_ent > 0) {
        uint32_t blocks = (j.n_ent + 255u) / 256u;
        if (blocks > sc.n_slots) blocks = sc.n_slots;
        // the kernel applies runs in order only within one launch, and its
        // base_value for unwritten 12-bit columns reads the output, so it
        // must run after the decompress kernel (same stream).
        generic_sidecar_kernel<<<blocks, 256, 0, s>>>(j, sc.slots, sc.counters);
        return cudaGetLastError();
    }
    cudaError_t e = cudaSuccess;
    if (j.sumsq) e = cudaMemsetAsync(j.sumsq, 0, sizeof(double), s);
    if (e == cudaSuccess && j.conf) e = cudaMemsetAsync(j.conf, 0, sizeof(float), s);
    return e;
}

}  // namespace hxq
