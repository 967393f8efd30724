// polarquant.cu -- PolarQuant rotation of KV-cache vectors on the GPU
// (reference hxq-native src/polarquant.c:249-300).
//
//   rotate:    out[v][j] = sum_k x[v][k] * Q[j][k]   (x Q^T)
//   unrotate:  out[v][j] = sum_k x[v][k] * Q[k][j]   (x Q)
// Each output is the reference's fp32 sum in k order, one product then one
// add per term (no fused multiply-add), starting from 0: bit-identical.
//
// head_dim 32, 64, 128: a CTA stages M[k][j] (Q^T or Q) once in shared
// memory (64 KB at 128) and loops over tiles of 4096 / head_dim vectors
// (16 KB), loaded whole before any is overwritten (in place); each thread
// owns 4 vectors x 4 consecutive outputs and per k reads one 128-bit row
// segment of M (consecutive threads, consecutive columns: no bank
// conflicts) and four broadcast activations, 16 products and 16 adds.
// The work is 2 head_dim^2 floating-point operations per vector against
// 8 head_dim bytes, so the kernel is bound by the fp32 pipe, not by HBM
// (the no-contraction rule doubles the instruction count of an FMA form).
// Other head_dim: one thread per output, M from L1/L2.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "hxq_cuda.h"
#include "polarquant.h"

namespace hxq {
namespace pq {

constexpr int kThreads = 256;

template <int HD>
__global__ void __launch_bounds__(kThreads)
apply_kernel(float *__restrict__ x, const float *__restrict__ Q, uint64_t nvec, bool transpose)
{
    constexpr int JG = HD / 4;                 // column groups of 4
    constexpr int VG = kThreads / JG;          // vector groups of 4
    constexpr int TV = VG * 4;                 // vectors per tile
    extern __shared__ __align__(16) float sm[];
    float *M = sm;                             // [HD][HD]: M[k][j]
    float *xs = sm + HD * HD;                  // [TV][HD]
    for (int i = threadIdx.x; i < HD * HD; i += kThreads) {
        const int k = i / HD, j = i - k * HD;
        M[i] = transpose ? Q[j * HD + k] : Q[k * HD + j];
    }
    const int jg = threadIdx.x % JG, vg = threadIdx.x / JG;
    for (uint64_t v0 = (uint64_t)blockIdx.x * TV; v0 < nvec; v0 += (uint64_t)gridDim.x * TV) {
        const int tv = (nvec - v0 < (uint64_t)TV) ? (int)(nvec - v0) : TV;
        __syncthreads();   // the previous tile's reads are done (and M is written)
        for (int i = threadIdx.x; i < tv * HD; i += kThreads) xs[i] = x[v0 * HD + i];
        __syncthreads();
        float acc[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) acc[a][b] = 0.0f;
        const float *xr = xs + (vg * 4) * HD;
#pragma unroll 4
        for (int k = 0; k < HD; ++k) {
            const float4 m = *reinterpret_cast<const float4 *>(M + k * HD + jg * 4);
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                const float xv = xr[a * HD + k];
                acc[a][0] = __fadd_rn(acc[a][0], __fmul_rn(xv, m.x));
                acc[a][1] = __fadd_rn(acc[a][1], __fmul_rn(xv, m.y));
                acc[a][2] = __fadd_rn(acc[a][2], __fmul_rn(xv, m.z));
                acc[a][3] = __fadd_rn(acc[a][3], __fmul_rn(xv, m.w));
            }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int v = vg * 4 + a;
            if (v < tv)
                *reinterpret_cast<float4 *>(x + (v0 + v) * HD + jg * 4) =
                    make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
        }
    }
}

// Any head_dim: a CTA per vector, its thread j computes output j (the
// vector is read whole into shared memory before it is overwritten).
__global__ void apply_generic_kernel(float *__restrict__ x, const float *__restrict__ Q, uint64_t nvec, uint32_t hd,
                                     bool transpose)
{
    extern __shared__ __align__(16) float xv[];
    for (uint64_t v = blockIdx.x; v < nvec; v += gridDim.x) {
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) xv[i] = x[v * hd + i];
        __syncthreads();
        for (uint32_t j = threadIdx.x; j < hd; j += blockDim.x) {
            float s = 0.0f;
            for (uint32_t k = 0; k < hd; ++k)
                s = __fadd_rn(s, __fmul_rn(xv[k], transpose ? __ldg(Q + (size_t)j * hd + k) : __ldg(Q + (size_t)k * hd + j)));
            x[v * hd + j] = s;
        }
    }
}

int sm_count()
{
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

template <int HD>
cudaError_t launch_fast(float *x, const float *Q, uint64_t nvec, bool transpose, cudaStream_t s)
{
    constexpr int TV = (kThreads / (HD / 4)) * 4;
    const size_t smem = (size_t)(HD * HD + TV * HD) * sizeof(float);
    static std::atomic<uint64_t> configured{0};   // one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!(configured.load(std::memory_order_acquire) & (1ull << dev))) {
        e = cudaFuncSetAttribute(apply_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured.fetch_or(1ull << dev, std::memory_order_acq_rel);
    }
    const uint64_t tiles = (nvec + TV - 1) / TV;
    const uint64_t cap = (uint64_t)sm_count() * (HD == 128 ? 2u : 4u);
    const unsigned grid = (unsigned)(tiles < cap ? tiles : cap);
    apply_kernel<HD><<<grid, kThreads, smem, s>>>(x, Q, nvec, transpose);
    return cudaGetLastError();
}

hxq_error_t apply(float *x, const float *Q, uint64_t nvec, uint32_t hd, bool transpose, cudaStream_t s)
{
    if (!x || !Q) return HXQ_ERR_NULL_PTR;
    if (hd == 0) return HXQ_ERR_INVALID_ARG;
    if (nvec == 0) return HXQ_OK;
    cudaError_t e;
    const bool aligned = ((uintptr_t)x & 15u) == 0;
    if (aligned && hd == 128) e = launch_fast<128>(x, Q, nvec, transpose, s);
    else if (aligned && hd == 64) e = launch_fast<64>(x, Q, nvec, transpose, s);
    else if (aligned && hd == 32) e = launch_fast<32>(x, Q, nvec, transpose, s);
    else {
        if ((size_t)hd * sizeof(float) > 48u * 1024u) return HXQ_ERR_INVALID_ARG;
        const uint64_t cap = (uint64_t)sm_count() * 16u;
        const unsigned grid = (unsigned)(nvec < cap ? nvec : cap);
        apply_generic_kernel<<<grid, 256, hd * sizeof(float), s>>>(x, Q, nvec, hd, transpose);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return HXQ_ERR_CUDA;
    }
    return HXQ_OK;
}

// Host-pointer form: copy in, apply on a private stream, copy back.
pq_error_t host_apply(float *values, const float *Q, uint32_t n_heads, uint32_t head_dim, bool transpose)
{
    if (!values || !Q) return PQ_ERR_NULL_PTR;
    if (head_dim == 0 || n_heads == 0) return PQ_ERR_INVALID_DIM;
    const size_t vb = (size_t)n_heads * head_dim * sizeof(float), qb = (size_t)head_dim * head_dim * sizeof(float);
    cudaStream_t s = nullptr;
    float *dv = nullptr, *dq = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        return PQ_ERR_ALLOC_FAILED;
    }
    pq_error_t rc = PQ_OK;
    if (cudaMalloc(&dv, vb) != cudaSuccess || cudaMalloc(&dq, qb) != cudaSuccess) rc = PQ_ERR_ALLOC_FAILED;
    if (rc == PQ_OK && (cudaMemcpyAsync(dv, values, vb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
                        cudaMemcpyAsync(dq, Q, qb, cudaMemcpyHostToDevice, s) != cudaSuccess))
        rc = PQ_ERR_ALLOC_FAILED;
    if (rc == PQ_OK && apply(dv, dq, n_heads, head_dim, transpose, s) != HXQ_OK) rc = PQ_ERR_ALLOC_FAILED;
    if (rc == PQ_OK && cudaMemcpyAsync(values, dv, vb, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        rc = PQ_ERR_ALLOC_FAILED;
    if (cudaStreamSynchronize(s) != cudaSuccess) rc = PQ_ERR_ALLOC_FAILED;
    cudaGetLastError();
    cudaFree(dv);
    cudaFree(dq);
    cudaStreamDestroy(s);
    return rc;
}

}  // namespace pq
}  // namespace hxq

extern "C" {

hxq_error_t hxq_cuda_pq_rotate(float *d_values, const float *d_Q, uint64_t n_vectors, uint32_t head_dim, void *stream)
{
    return hxq::pq::apply(d_values, d_Q, n_vectors, head_dim, true, static_cast<cudaStream_t>(stream));
}

hxq_error_t hxq_cuda_pq_unrotate(float *d_values, const float *d_Q, uint64_t n_vectors, uint32_t head_dim,
                                 void *stream)
{
    return hxq::pq::apply(d_values, d_Q, n_vectors, head_dim, false, static_cast<cudaStream_t>(stream));
}

pq_error_t pq_rotate(float *values, const float *Q, uint32_t n_heads, uint32_t head_dim)
{
    return hxq::pq::host_apply(values, Q, n_heads, head_dim, true);
}

pq_error_t pq_unrotate(float *values, const float *Q, uint32_t n_heads, uint32_t head_dim)
{
    return hxq::pq::host_apply(values, Q, n_heads, head_dim, false);
}

}  // extern "C"
