// lloyd.cu -- one iteration of Lloyd's algorithm on grouped VQ codebooks
// (reference hxq-native src/hxq_lloyd.c:41-308), on the GPU.
//
//   assign   one thread per vector; the codebook and its squared norms in
//            shared memory; dist = (||w||^2 + ||c||^2) - 2 (w . c) in fp32
//            with every sum in component order and no fused multiply-add,
//            strict < so the first minimum wins: the reference's indices,
//            bit for bit.
//   update   each vector's components are added, as 64-bit fixed-point
//            integers (w x 2^s, s a power of two from the largest |w| so the
//            sum of n of them cannot overflow), into per-CTA shared
//            accumulators and then into global ones.  Integer addition
//            does not depend on order, so the sums are reproducible run to
//            run; the mean is (sum x 2^-s) x (1 / count) in double, rounded
//            to fp32 like the reference's (sum / count).
//   reinit   the largest cluster (first maximum count); its member farthest
//            from the updated centroid (fp32 sum of squared differences in
//            component order; the largest distance, then the lowest index)
//            by a 64-bit atomic max of (distance bits, ~index); every dead
//            centroid becomes that member x 1.001f.
// All steps are stream-ordered; the dead count is written to device memory.
#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>
#include <cstdint>
#include <map>
#include <mutex>

#include "hxq_cuda.h"
#include "hxq_lloyd.h"

namespace hxq {
namespace lloyd {

constexpr int kThreads = 256;
constexpr int kMaxK = 256;
constexpr int kMaxD = 8;

// Device scratch of one call: fixed-point sums, counts, the largest |w|,
// the packed farthest member, and {dead count, largest cluster, non-finite}.
struct Scratch {
    unsigned long long sums[kMaxK * kMaxD];
    int counts[kMaxK];
    unsigned int wmax;
    unsigned int pad_;
    unsigned long long far;
    int info[4];
};

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }

// Largest |w| over all components (bits of a non-negative float order like
// the values; a NaN or inf sets the non-finite flag).
__global__ void maxabs_kernel(const float *__restrict__ w, uint64_t count, Scratch *sc)
{
    __shared__ unsigned int red[kThreads / 32];
    unsigned int m = 0, bad = 0;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const unsigned int b = __float_as_uint(w[i]) & 0x7FFFFFFFu;
        if (b >= 0x7F800000u) bad = 1u;
        else m = max(m, b);
    }
    for (int o = 16; o > 0; o >>= 1) {
        m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = m;
    if (bad && (threadIdx.x & 31u) == 0) atomicOr(&sc->info[2], 1);
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned int r = 0;
        for (int i = 0; i < kThreads / 32; ++i) r = max(r, red[i]);
        atomicMax(&sc->wmax, r);
    }
}

// Fixed-point exponent: |w| x 2^s < 2^62 / n for every component.
__device__ __forceinline__ int fixed_shift(unsigned int wmax_bits, uint64_t n)
{
    if (wmax_bits == 0u) return 0;
    const int e = (int)(wmax_bits >> 23) - 127 + 1;   // |w| < 2^e (subnormals: e = -126)
    int ln = 0;
    while (ln < 63 && (1ull << ln) < n) ++ln;         // n <= 2^ln
    int s = 62 - ln - e;
    return s > 1000 ? 1000 : s < -1000 ? -1000 : s;
}

template <int D, bool ACC>
__global__ void __launch_bounds__(kThreads)
assign_kernel(const float *__restrict__ w, const float *__restrict__ cb, uint8_t *__restrict__ idx, uint64_t n,
              int k, Scratch *sc)
{
    __shared__ float scb[kMaxK * D];
    __shared__ float csq[kMaxK];
    __shared__ unsigned long long bsum[ACC ? kMaxK * D : 1];
    __shared__ int bcnt[ACC ? kMaxK : 1];
    for (int i = threadIdx.x; i < k * D; i += kThreads) scb[i] = cb[i];
    if (ACC) {
        for (int i = threadIdx.x; i < k * D; i += kThreads) bsum[i] = 0ull;
        for (int i = threadIdx.x; i < k; i += kThreads) bcnt[i] = 0;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < k; j += kThreads) {
        float s = 0.0f;
#pragma unroll
        for (int p = 0; p < D; ++p) s = fadd(s, fmul(scb[j * D + p], scb[j * D + p]));
        csq[j] = s;
    }
    double scale = 0.0;
    if (ACC) scale = ldexp(1.0, fixed_shift(sc->wmax, n));
    __syncthreads();
    for (uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (uint64_t)gridDim.x * kThreads) {
        float wv[D];
#pragma unroll
        for (int p = 0; p < D; ++p) wv[p] = w[i * D + p];
        float wsq = 0.0f;
#pragma unroll
        for (int p = 0; p < D; ++p) wsq = fadd(wsq, fmul(wv[p], wv[p]));
        float best = FLT_MAX;
        int bj = 0;
        for (int j = 0; j < k; ++j) {
            float dot = 0.0f;
#pragma unroll
            for (int p = 0; p < D; ++p) dot = fadd(dot, fmul(wv[p], scb[j * D + p]));
            const float dist = __fsub_rn(fadd(wsq, csq[j]), fmul(2.0f, dot));
            if (dist < best) {
                best = dist;
                bj = j;
            }
        }
        idx[i] = (uint8_t)bj;
        if (ACC) {
            atomicAdd(&bcnt[bj], 1);
#pragma unroll
            for (int p = 0; p < D; ++p) {
                const long long q = __double2ll_rn((double)wv[p] * scale);
                atomicAdd(&bsum[bj * D + p], (unsigned long long)q);
            }
        }
    }
    if (ACC) {
        __syncthreads();
        for (int i = threadIdx.x; i < k * D; i += kThreads)
            if (bsum[i]) atomicAdd(&sc->sums[i], bsum[i]);
        for (int i = threadIdx.x; i < k; i += kThreads)
            if (bcnt[i]) atomicAdd(&sc->counts[i], bcnt[i]);
    }
}

// New centroids for clusters with vectors; the dead count and the largest
// cluster (first maximum count).
template <int D>
__global__ void finalize_kernel(float *__restrict__ cb, int k, uint64_t n, Scratch *sc)
{
    const double inv_scale = ldexp(1.0, -fixed_shift(sc->wmax, n));
    const bool bad = sc->info[2] != 0;
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        const int c = sc->counts[j];
        if (c == 0) continue;
        const double inv = 1.0 / (double)c;
#pragma unroll
        for (int p = 0; p < D; ++p) {
            const double sum = (double)(long long)sc->sums[j * D + p] * inv_scale;
            cb[j * D + p] = bad ? __int_as_float(0x7FC00000) : (float)(sum * inv);
        }
    }
    if (threadIdx.x == 0) {
        int dead = 0, largest = 0;
        for (int j = 0; j < k; ++j) {
            if (sc->counts[j] == 0) ++dead;
            if (sc->counts[j] > sc->counts[largest]) largest = j;
        }
        sc->info[0] = dead;
        sc->info[1] = largest;
    }
}

template <int D>
__global__ void farthest_kernel(const float *__restrict__ w, const uint8_t *__restrict__ idx,
                                const float *__restrict__ cb, uint64_t n, Scratch *sc)
{
    if (sc->info[0] == 0) return;
    const int largest = sc->info[1];
    float lc[D];
#pragma unroll
    for (int p = 0; p < D; ++p) lc[p] = cb[largest * D + p];
    unsigned long long best = 0ull;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        if (idx[i] != (uint8_t)largest) continue;
        float dist = 0.0f;
#pragma unroll
        for (int p = 0; p < D; ++p) {
            const float diff = __fsub_rn(w[i * D + p], lc[p]);
            dist = fadd(dist, fmul(diff, diff));
        }
        if (!(dist > -1.0f)) continue;   // NaN never wins (the reference's dist > max_dist)
        const unsigned long long key =
            ((unsigned long long)__float_as_uint(dist) << 32) | (unsigned long long)(~(uint32_t)i);
        best = best > key ? best : key;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = best > other ? best : other;
    }
    if ((threadIdx.x & 31u) == 0 && best) atomicMax(&sc->far, best);
}

template <int D>
__global__ void reinit_kernel(const float *__restrict__ w, float *__restrict__ cb, int k, Scratch *sc,
                              int *n_dead)
{
    const int dead = sc->info[0];
    if (n_dead && threadIdx.x == 0) *n_dead = dead;
    if (dead == 0) return;
    // no candidate (every distance NaN): the reference keeps vector 0
    const uint64_t f = sc->far ? (uint64_t)(~(uint32_t)(sc->far & 0xFFFFFFFFull)) : 0ull;
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        if (sc->counts[j] != 0) continue;
#pragma unroll
        for (int p = 0; p < D; ++p) cb[j * D + p] = fmul(w[f * D + p], 1.001f);
    }
}

// One scratch block per (device, stream): calls on different streams never
// share it; calls on one stream are ordered.
Scratch *scratch_for(cudaStream_t s)
{
    static std::mutex mu;
    static std::map<std::pair<int, cudaStream_t>, Scratch *> bufs;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    std::lock_guard<std::mutex> lk(mu);
    Scratch *&p = bufs[{dev, s}];
    if (!p && cudaMalloc(&p, sizeof(Scratch)) != cudaSuccess) {
        cudaGetLastError();
        p = nullptr;
    }
    return p;
}

int grid_for(uint64_t n)
{
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t blocks = (n + kThreads - 1) / kThreads;
    const uint64_t cap = (uint64_t)sms * 8u;
    return (int)(blocks < cap ? (blocks ? blocks : 1) : cap);
}

int check_args(const void *w, const void *cb, const void *idx, size_t n, int k, int d)
{
    if (!w || !cb || !idx) return HXQ_LLOYD_ERR_NULL;
    if (k < 1 || k > kMaxK) return HXQ_LLOYD_ERR_K;
    if (d != 1 && d != 2 && d != 4 && d != 8) return HXQ_LLOYD_ERR_DIM;
    if ((uint64_t)n >= (1ull << 32)) return HXQ_LLOYD_ERR_DIM;
    return HXQ_LLOYD_OK;
}

template <int D>
int run(const float *w, float *cb, uint8_t *idx, uint64_t n, int k, int *n_dead, bool update, cudaStream_t s)
{
    const int g = grid_for(n);
    if (!update) {
        assign_kernel<D, false><<<g, kThreads, 0, s>>>(w, cb, idx, n, k, nullptr);
        return cudaGetLastError() == cudaSuccess ? HXQ_LLOYD_OK : HXQ_LLOYD_ERR_CUDA;
    }
    Scratch *sc = scratch_for(s);
    if (!sc) return HXQ_LLOYD_ERR_ALLOC;
    if (cudaMemsetAsync(sc, 0, sizeof(Scratch), s) != cudaSuccess) { cudaGetLastError(); return HXQ_LLOYD_ERR_CUDA; }
    maxabs_kernel<<<grid_for(n * D), kThreads, 0, s>>>(w, n * D, sc);
    assign_kernel<D, true><<<g, kThreads, 0, s>>>(w, cb, idx, n, k, sc);
    finalize_kernel<D><<<1, kThreads, 0, s>>>(cb, k, n, sc);
    farthest_kernel<D><<<g, kThreads, 0, s>>>(w, idx, cb, n, sc);
    reinit_kernel<D><<<1, kThreads, 0, s>>>(w, cb, k, sc, n_dead);
    return cudaGetLastError() == cudaSuccess ? HXQ_LLOYD_OK : HXQ_LLOYD_ERR_CUDA;
}

int dispatch(const float *w, float *cb, uint8_t *idx, uint64_t n, int k, int d, int *n_dead, bool update,
             cudaStream_t s)
{
    switch (d) {
    case 1: return run<1>(w, cb, idx, n, k, n_dead, update, s);
    case 2: return run<2>(w, cb, idx, n, k, n_dead, update, s);
    case 4: return run<4>(w, cb, idx, n, k, n_dead, update, s);
    default: return run<8>(w, cb, idx, n, k, n_dead, update, s);
    }
}

// Host-pointer form: copy in, run on a private stream, copy out.
int host_call(const float *w, float *cb, uint8_t *idx, size_t n, int k, int d, int *n_dead, bool update)
{
    const int a = check_args(w, cb, idx, n, k, d);
    if (a != HXQ_LLOYD_OK) return a;
    if (n == 0) {
        if (n_dead) *n_dead = 0;
        return HXQ_LLOYD_OK;
    }
    cudaStream_t s = nullptr;
    float *dw = nullptr, *dcb = nullptr;
    uint8_t *didx = nullptr;
    int *dnd = nullptr;
    int rc = HXQ_LLOYD_OK;
    const size_t wb = n * (size_t)d * sizeof(float), cbb = (size_t)k * d * sizeof(float);
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) { cudaGetLastError(); return HXQ_LLOYD_ERR_CUDA; }
    if (cudaMalloc(&dw, wb) != cudaSuccess || cudaMalloc(&dcb, cbb) != cudaSuccess || cudaMalloc(&didx, n) != cudaSuccess ||
        cudaMalloc(&dnd, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        rc = HXQ_LLOYD_ERR_ALLOC;
    }
    if (rc == HXQ_LLOYD_OK && (cudaMemcpyAsync(dw, w, wb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
                               cudaMemcpyAsync(dcb, cb, cbb, cudaMemcpyHostToDevice, s) != cudaSuccess))
        rc = HXQ_LLOYD_ERR_CUDA;
    if (rc == HXQ_LLOYD_OK) rc = dispatch(dw, dcb, didx, n, k, d, dnd, update, s);
    int nd = 0;
    if (rc == HXQ_LLOYD_OK && (cudaMemcpyAsync(idx, didx, n, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
                               (update && cudaMemcpyAsync(cb, dcb, cbb, cudaMemcpyDeviceToHost, s) != cudaSuccess) ||
                               (update && cudaMemcpyAsync(&nd, dnd, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess)))
        rc = HXQ_LLOYD_ERR_CUDA;
    if (cudaStreamSynchronize(s) != cudaSuccess && rc == HXQ_LLOYD_OK) rc = HXQ_LLOYD_ERR_CUDA;
    cudaGetLastError();
    if (rc == HXQ_LLOYD_OK && update && n_dead) *n_dead = nd;
    cudaFree(dw);
    cudaFree(dcb);
    cudaFree(didx);
    cudaFree(dnd);
    cudaStreamDestroy(s);
    return rc;
}

}  // namespace lloyd
}  // namespace hxq

extern "C" {

int hxq_cuda_lloyd_assign(const float *d_weights, const float *d_codebook, uint8_t *d_indices, size_t n, int k,
                          int d, void *stream)
{
    const int a = hxq::lloyd::check_args(d_weights, d_codebook, d_indices, n, k, d);
    if (a != HXQ_LLOYD_OK || n == 0) return a;
    return hxq::lloyd::dispatch(d_weights, const_cast<float *>(d_codebook), d_indices, n, k, d, nullptr, false,
                                static_cast<cudaStream_t>(stream));
}

int hxq_cuda_lloyd_reassign(const float *d_weights, float *d_codebook, uint8_t *d_indices, size_t n, int k, int d,
                            int *d_n_dead, void *stream)
{
    const int a = hxq::lloyd::check_args(d_weights, d_codebook, d_indices, n, k, d);
    if (a != HXQ_LLOYD_OK) return a;
    if (n == 0) {
        if (d_n_dead && cudaMemsetAsync(d_n_dead, 0, sizeof(int), static_cast<cudaStream_t>(stream)) != cudaSuccess) {
            cudaGetLastError();
            return HXQ_LLOYD_ERR_CUDA;
        }
        return HXQ_LLOYD_OK;
    }
    return hxq::lloyd::dispatch(d_weights, d_codebook, d_indices, n, k, d, d_n_dead, true,
                                static_cast<cudaStream_t>(stream));
}

int hxq_lloyd_reassign(const float *weights, float *codebook, uint8_t *indices, size_t n_vectors, int k, int d,
                       int *n_dead)
{
    return hxq::lloyd::host_call(weights, codebook, indices, n_vectors, k, d, n_dead, true);
}

int hxq_lloyd_assign_only(const float *weights, const float *codebook, uint8_t *indices, size_t n_vectors, int k,
                          int d)
{
    return hxq::lloyd::host_call(weights, const_cast<float *>(codebook), indices, n_vectors, k, d, nullptr, false);
}

}  // extern "C"
