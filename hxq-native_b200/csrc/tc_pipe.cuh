// tc_pipe.cuh -- shared-memory pipeline pieces of the tensor-core GEMVs
// (affine_tc_gemv.cu, vq_tc_gemv.cu): bounded mbarrier waits, TMA tensor
// and bulk copies, 32-bit shared loads, m16n8k16 products, the
// cuTensorMapEncodeTiled entry point.  Internal header.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

namespace hxq {
namespace pipe {

constexpr uint64_t kWaitCycles = 2000000000ull;   // ~1 s at 1.9 GHz
constexpr uint32_t kErrTimeout = 4u;

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Order this thread's reads of a shared-memory buffer (generic proxy)
// before a TMA or bulk copy that will overwrite it (async proxy).  Without
// it the copy can land before reads still in flight and they see the new
// data (measured: nondeterministic results in a two-stage TMA ring).
__device__ __forceinline__ void async_proxy_fence()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Hand back a buffer this warp has read to the copy that refills it: every
// lane's proxy fence, then one arrival per warp.
__device__ __forceinline__ void warp_release(uint64_t *bar, uint32_t lane)
{
    async_proxy_fence();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait; false if it ran out (then *err |= kErrTimeout and *abort
// is set) or another thread already gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *abort, uint32_t *err)
{
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = clock64();
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > kWaitCycles) {
            *abort = 1u;
            atomicOr(err, kErrTimeout);
            return false;
        }
    }
}

// Warp-uniform bounded wait: every lane waits, the warp goes on only if all did.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *abort, uint32_t *err)
{
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, err)) != 0;
}

// Teardown wait: bounded, not cut short by the abort flag.
__device__ __forceinline__ void mbar_drain(uint64_t *bar, uint32_t parity, uint32_t *err)
{
    const uint64_t t0 = clock64();
    while (!mbar_try(bar, parity)) {
        if (clock64() - t0 > kWaitCycles) {
            atomicOr(err, kErrTimeout);
            return;
        }
    }
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int32_t c0,
                                            int32_t c1, int32_t c2)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int32_t c0, int32_t c1)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// Read-only global loads that stay where they are written (issued early,
// consumed much later).
__device__ __forceinline__ uint32_t ldg_pinned(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ float ldg_pinned(const float *p)
{
    float v;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t a)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t a)
{
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}

__device__ __forceinline__ uint32_t lds32(uint32_t a)
{
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}

// d += A (16 x 16, row) * B (16 x 8, col), fp32 accumulation; f16 or bf16
// operands (A and B of the same type).
__device__ __forceinline__ void mma16816_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma16816_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static std::atomic<bool> tried{false};
    if (!tried.load(std::memory_order_acquire)) {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
        else
            cudaGetLastError();
        tried.store(true, std::memory_order_release);
    }
    return fn;
}

// A byte matrix [rows][row_bytes] as [rows][row_bytes / line][line] with a
// box of `lines` x rows_box lines of `line` bytes and the swizzle of that
// span (line 128, 64 or 32 bytes); rows past the matrix read as 0.
inline bool encode_rows_map(CUtensorMap *map, const void *base, uint64_t row_bytes, uint32_t rows, uint32_t line,
                            uint32_t lines, uint32_t rows_box)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc || (line != 128u && line != 64u && line != 32u) || row_bytes % line != 0) return false;
    const CUtensorMapSwizzle sw = line == 128u ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : line == 64u ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
    const cuuint64_t dims[3] = {line, row_bytes / line, rows};
    const cuuint64_t strides[2] = {line, row_bytes};
    const cuuint32_t box[3] = {line, lines, rows_box};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A byte matrix [rows][row_bytes] (row_bytes a multiple of 16) as a 2D
// tensor with a box of 128 bytes x rows_box rows, 128-byte swizzle; bytes
// past a row and rows past the matrix read as 0.
inline bool encode_bytes_2d(CUtensorMap *map, const void *base, uint64_t row_bytes, uint32_t rows, uint32_t rows_box)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc || row_bytes % 16u != 0 || ((uintptr_t)base & 15u) != 0) return false;
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {128u, rows_box};
    const cuuint32_t estr[2] = {1u, 1u};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace pipe
}  // namespace hxq
