// peer.cu -- output buffers shared by the GPUs of one node (CUDA IPC) and
// the step flags that tell a rank every peer's output shards have landed.
//
// A fused matmul that splits output features across ranks stores each
// output element straight into every rank's [tokens, out_features] buffer
// (peer pointers over NVLink), so no separate gather runs.  After a step's
// matmuls, hxq_cuda_peer_signal bumps this rank's step counter and, after a
// system-scope fence, writes it into every peer's flag slot for this rank;
// hxq_cuda_peer_wait polls the local flags until every rank has reached
// this rank's counter.  Counters live on the device, so a CUDA graph that
// holds these kernels advances them on every replay.  The wait is bounded
// (about two seconds of clock); when it runs out it sets a status word and
// returns, leaving the context usable.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "hxq_cuda.h"

namespace {

constexpr uint64_t kPeerWaitCycles = 4000000000ull;   // ~2 s at 1.9 GHz

struct PeerFlags {
    uint32_t *peer[HXQ_CUDA_MAX_PEERS];   // rank p's flag array (one slot per rank)
};

__global__ void peer_signal_kernel(const __grid_constant__ PeerFlags f, uint32_t world, uint32_t rank,
                                   uint32_t *counter)
{
    __shared__ uint32_t e;
    if (threadIdx.x == 0) {
        e = *counter + 1u;
        *counter = e;
        // the step's stores to peer memory are complete (earlier kernels on
        // this stream); order them before the flags at system scope
        __threadfence_system();
    }
    __syncthreads();
    if (threadIdx.x < world) {
        uint32_t *slot = f.peer[threadIdx.x] + rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(slot), "r"(e) : "memory");
    }
}

__global__ void peer_wait_kernel(const uint32_t *flags, uint32_t world, const uint32_t *counter, uint32_t *status)
{
    const uint32_t e = *counter;
    if (threadIdx.x < world) {
        const uint64_t t0 = clock64();
        while (true) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + threadIdx.x) : "memory");
            if ((int32_t)(v - e) >= 0) break;
            if (clock64() - t0 > kPeerWaitCycles) {
                atomicOr(status, 1u);
                break;
            }
            __nanosleep(100);
        }
    }
    __syncthreads();
}

}  // namespace

extern "C" {

hxq_error_t hxq_cuda_ipc_alloc(size_t bytes, void **d_ptr, void *handle)
{
    if (!d_ptr || !handle) return HXQ_ERR_NULL_PTR;
    *d_ptr = nullptr;
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes ? bytes : 16);
    if (e != cudaSuccess) { cudaGetLastError(); return HXQ_ERR_ALLOC_FAILED; }
    e = cudaMemset(p, 0, bytes ? bytes : 16);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        return HXQ_ERR_CUDA;
    }
    std::memcpy(handle, &h, sizeof(h));
    *d_ptr = p;
    return HXQ_OK;
}

hxq_error_t hxq_cuda_ipc_open(const void *handle, void **d_peer)
{
    if (!handle || !d_peer) return HXQ_ERR_NULL_PTR;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(d_peer, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) { cudaGetLastError(); *d_peer = nullptr; return HXQ_ERR_CUDA; }
    return HXQ_OK;
}

hxq_error_t hxq_cuda_ipc_close(void *d_peer)
{
    if (!d_peer) return HXQ_OK;
    if (cudaIpcCloseMemHandle(d_peer) != cudaSuccess) { cudaGetLastError(); return HXQ_ERR_CUDA; }
    return HXQ_OK;
}

hxq_error_t hxq_cuda_ipc_free(void *d_ptr)
{
    if (!d_ptr) return HXQ_OK;
    if (cudaFree(d_ptr) != cudaSuccess) { cudaGetLastError(); return HXQ_ERR_CUDA; }
    return HXQ_OK;
}

hxq_error_t hxq_cuda_peer_signal(uint32_t *const *peer_flags, uint32_t world, uint32_t rank,
                                 uint32_t *d_counter, void *stream)
{
    if (!peer_flags || !d_counter) return HXQ_ERR_NULL_PTR;
    if (world == 0 || world > HXQ_CUDA_MAX_PEERS || rank >= world) return HXQ_ERR_INVALID_ARG;
    PeerFlags f;
    std::memset(&f, 0, sizeof(f));
    for (uint32_t p = 0; p < world; ++p) {
        if (!peer_flags[p]) return HXQ_ERR_NULL_PTR;
        f.peer[p] = peer_flags[p];
    }
    peer_signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(f, world, rank, d_counter);
    return cudaGetLastError() == cudaSuccess ? HXQ_OK : HXQ_ERR_CUDA;
}

hxq_error_t hxq_cuda_peer_wait(const uint32_t *d_flags, uint32_t world, const uint32_t *d_counter,
                               uint32_t *d_status, void *stream)
{
    if (!d_flags || !d_counter || !d_status) return HXQ_ERR_NULL_PTR;
    if (world == 0 || world > HXQ_CUDA_MAX_PEERS) return HXQ_ERR_INVALID_ARG;
    peer_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(d_flags, world, d_counter, d_status);
    return cudaGetLastError() == cudaSuccess ? HXQ_OK : HXQ_ERR_CUDA;
}

}  // extern "C"
