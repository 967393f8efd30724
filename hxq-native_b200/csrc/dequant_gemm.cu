// dequant_gemm.cu -- tcgen05 dequant-GEMM for the quantized matmuls at
// batch sizes where they are dense contractions (sm_100a).
//
//   Y[n, o] = sum_k x[n, k] * W[o, k] (+ bias[o])
// with W decoded on the fly from either
//   - affine group-quantized codes, W = code * scale + offset (the
//     reference's src/hxq_affine.c:23-66 algebra, evaluated as a GEMM), or
//   - a 12-bit 2D-VQ image, W = codebook[index] + sidecar deltas (the
//     reference's src/hxq.c:239-350 decode), with no dense W in memory.
//
// CTA tile: 128 output features (M, TMEM lanes) x BN tokens (N), K in steps
// of 128.  Warp roles (320 threads):
//   warps 0-7  converters: thread (warp w, lane l) owns output row
//              32*(w%4) + l and half (w/4) of each 128-wide K step.
//              Affine: 64 codes (4 x 128-bit loads), W = fma(code, s, off)
//              in fp32, rounded to bf16.  VQ: 48 index bytes (3 x 128-bit
//              loads), one PRMT per byte triple, each 12-bit index gathers
//              one bf16 pair from a shared-memory copy of the codebook;
//              sidecar positions are recomputed in fp32 (codebook value +
//              deltas in array order) and rounded once.  The packed pairs go
//              straight into tensor memory (tcgen05.st) as the MMA's A
//              operand -- no shared-memory staging or swizzle for weights.
//              VQ with 256-token tiles instead takes the tensor-core
//              GEMV's lane layout (lane (g, t) of warp w: rows 16w + g and
//              16w + g + 8, pairs 16t .. 16t + 15 of the step), reads the
//              image's GEMV offset stream (16-bit offsets into a two-copy
//              codebook, bank-balanced per gather instruction when the image
//              was built) from its own TMA ring, writes the A tile to shared
//              memory (the MMA's K-major 128-byte-swizzled layout, two 32 KB
//              buffers) and patches the sidecar positions there by warp from
//              a table grouped per 32 rows and half step (a patch is one
//              2-byte store, where a register fragment needs a select over
//              its 32 words).  At the end the converters drain the
//              accumulator (tcgen05.ld), add the bias and store coalesced
//              rows of Y;
//   warp 8     TMA producer: activation tiles [BN tokens x 64 K] bf16 with
//              128-byte swizzle into a 2-4 stage shared-memory ring (the VQ
//              tile of 256 tokens: three half steps, a box each);
//   warp 9     allocates tensor memory and issues tcgen05.mma
//              (kind::f16, bf16 x bf16 -> fp32, M=128, N=BN, K=16) from one
//              thread; tcgen05.commit frees A buffers and ring stages.
// Tensor memory: accumulator [128 x BN] fp32 from column 0, two A buffers of
// 64 columns (128 bf16 of K) after it; 256 columns for BN <= 128 (two CTAs
// per SM), else 512.
// In a batch, a GEMM that follows an unsplit GEMM of the same batch is
// launched with programmatic stream serialization: it may start while the
// previous GEMM's last wave runs (the previous GEMM signals its dependents
// only after it has waited for its own predecessor, so the activations are
// ready), and waits for the previous GEMM at its end instead of its start,
// so that the batch still completes in order.  Other GEMMs are launched in
// plain stream order.  A GEMM outside a batch whose 256-token tiles leave a
// last wave filling at most half of the SMs splits those last tiles along K
// into two ranges (one CTA each): both store partial sums to a scratch
// buffer and count themselves, and the second adds the other's sums to its
// own (4096 x 4096 VQ at 4096 tokens: 200.9 -> 184.4 us).  Every mbarrier
// wait is bounded (about one second of clock); a wait that runs out records
// an error word and the CTA unwinds, releasing its tensor memory.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "hxq_cuda.h"
#include "hxq_cuda_internal.h"

namespace hxq {
namespace gemm {

constexpr uint32_t kBM = 128;
constexpr uint32_t kBK = 128;            // K per pipeline step
constexpr uint32_t kConvWarps = 8;
constexpr uint32_t kThreads = (kConvWarps + 2) * 32;
constexpr uint32_t kProducerWarp = 8;
constexpr uint32_t kMmaWarp = 9;
// VQ with 256-token tiles keeps its A tiles in shared memory.
__host__ __device__ constexpr bool smem_a(uint32_t bn, bool vq) { return vq && bn == 256u; }
constexpr uint32_t kABytes = kBM * kBK * 2u;   // one A tile: [2 halves of K][128 rows][128 B]
// Tensor memory: the accumulator takes BN columns from 0, the two A buffers
// (when in tensor memory) 64 columns each right after it (rounded to 128); a
// tile of BN <= 128 fits in 256 columns, so two CTAs can share an SM.
__host__ __device__ constexpr uint32_t tmem_a_col(uint32_t bn) { return bn <= 128 ? 128u : 256u; }
__host__ __device__ constexpr uint32_t tmem_cols(uint32_t bn, bool vq)
{
    return smem_a(bn, vq) ? bn : bn <= 128 ? 256u : 512u;
}
constexpr uint64_t kWaitCycles = 2000000000ull;  // ~1 s at 1.9 GHz
constexpr uint32_t kErrTimeout = 2u;

__device__ uint32_t g_gemm_err;          // device status word of this kernel

// The VQ tile of 256 tokens moves its activations in half steps (64 of K,
// one TMA box each) through a ring of three, 96 KB where two whole steps
// took 128 KB: the room goes to a two-copy codebook and a ring for the
// GEMV's offset stream (below).
__host__ __device__ constexpr bool half_steps(uint32_t bn, bool vq) { return vq && bn == 256u; }
// Activation ring depth: 3 stages for the affine tile of 256 tokens, 4 for
// the small tiles; the tiles of 128 tokens keep 2 so that two CTAs share an
// SM; the VQ tile of 256 keeps 3 half steps.
__host__ __device__ constexpr uint32_t stages_for(uint32_t bn, bool vq)
{
    return (void)vq, bn >= 256 ? 3u : bn == 128 ? 2u : 4u;
}
__host__ __device__ constexpr uint32_t stage_bytes(uint32_t bn, bool vq)
{
    return bn * (half_steps(bn, vq) ? kBK / 2u : kBK) * 2u;
}
// VQ: the 4096 bf16 pairs once, or (the tile of 256 tokens) twice: copy 0
// at word c, copy 1 at word 4096 + (c ^ ((c >> 5) & 31)), the copies the
// image's offset stream was balanced for
__host__ __device__ constexpr uint32_t codebook_bytes(uint32_t bn) { return bn >= 256 ? 32768u : 16384u; }
// Weight ring: each K step's weight bytes of the CTA's 128 rows arrive by
// TMA -- affine codes 128 x 128 B (128-byte swizzle), VQ index bytes
// 128 x 96 B, or for the VQ tile of 256 tokens the GEMV offset stream,
// 128 x 128 B (64 pairs x 16 bits, 128-byte swizzle) -- instead of one
// 16-byte load per thread from 32 rows' lines per warp instruction.  Two
// stages.
__host__ __device__ constexpr uint32_t wstage_bytes(uint32_t bn, bool vq)
{
    return kBM * ((vq && bn < 256) ? 96u : 128u);
}
__host__ __device__ constexpr uint32_t wstages_for(uint32_t bn, bool vq) { return (void)bn, (void)vq, 2u; }
// ring | (A tiles in shared memory) A[2] | weight ring | barriers (full[S],
// empty[S], a_full[2], a_empty[2], d_full, w_full[W], w_empty[W]) | tmem
// addr | abort | (VQ) codebook
__host__ __device__ constexpr uint32_t smem_bytes(uint32_t bn, bool vq)
{
    return 1024u /* alignment slack */ + stages_for(bn, vq) * stage_bytes(bn, vq) +
           (smem_a(bn, vq) ? 2u * kABytes : 0u) + wstages_for(bn, vq) * wstage_bytes(bn, vq) + 256u +
           (vq ? codebook_bytes(bn) : 0u);
}
static_assert(smem_bytes(256, true) <= 232448u, "VQ tile of 256 tokens: shared memory");
static_assert(smem_bytes(256, false) <= 232448u, "affine tile of 256 tokens: shared memory");

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
// before the TMA copy that will overwrite it (async proxy); without it the
// copy can land before reads still in flight (measured: nondeterministic
// GEMM results with the two-stage weight ring).
__device__ __forceinline__ void async_proxy_fence()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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

// Bounded wait; false if it ran out or another thread already gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *abort)
{
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = clock64();
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > kWaitCycles) {
            *abort = 1u;
            atomicOr(&g_gemm_err, kErrTimeout);
            return false;
        }
    }
}

// Teardown wait: bounded, but not cut short by the abort flag.
__device__ __forceinline__ void mbar_drain(uint64_t *bar, uint32_t parity)
{
    const uint64_t t0 = clock64();
    while (!mbar_try(bar, parity)) {
        if (clock64() - t0 > kWaitCycles) {
            atomicOr(&g_gemm_err, kErrTimeout);
            return;
        }
    }
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int32_t c0,
                                            int32_t c1)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1 (sm100), base offset 0 (1024-B aligned).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr)
{
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both
// K-major, N = bn, M = 128.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t bn)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((bn >> 3) << 17) | ((kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
        "%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
        "[%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
          "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
          "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15])
        : "r"(taddr));
}

template <uint32_t EW>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&v)[EW])
{
    if constexpr (EW == 32u) tmem_ld32(taddr, v);
    else tmem_ld16(taddr, v);
}

__device__ __forceinline__ float code_f32(uint32_t word, uint32_t i)
{
    return __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7440u + i)) - 8388608.0f;
}

__device__ __forceinline__ uint32_t bf16x2(float lo, float hi)
{
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ uint64_t f32x2_splat(float f)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(f));
    return r;
}

// Codes i and i + 1 (bytes of `word`) as bf16 weights RN(fma(code, s, off))
// packed into one word (code i in the low half), two fp32 lanes at a time:
// a byte permute puts each code into the float 2^23 + code, a packed
// subtraction of 2^23 makes it exact, a packed fma rounds each weight once,
// as two scalar fmaf would.  Half the fp32 instructions of the scalar form.
__device__ __forceinline__ uint32_t code_pair_bf16(uint32_t word, uint32_t i, uint64_t s2, uint64_t o2)
{
    const uint32_t m0 = __byte_perm(word, 0x4B000000u, 0x7440u + i);
    const uint32_t m1 = __byte_perm(word, 0x4B000000u, 0x7441u + i);
    uint32_t out;
    asm("{\n\t.reg .b64 c, m;\n\t.reg .f32 lo, hi;\n\t"
        "mov.b64 c, {%1, %2};\n\t"
        "mov.b64 m, {%5, %5};\n\t"
        "sub.rn.f32x2 c, c, m;\n\t"
        "fma.rn.f32x2 c, c, %3, %4;\n\t"
        "mov.b64 {lo, hi}, c;\n\t"
        "cvt.rn.bf16x2.f32 %0, hi, lo;\n\t}"
        : "=r"(out)
        : "r"(m0), "r"(m1), "l"(s2), "l"(o2), "r"(0x4B000000u));
    return out;
}

struct Params {
    // affine weights
    const uint8_t *codes;     // [O, I]
    const float *scales;      // [O, I/gs]
    const float *offsets;     // [O, I/gs]
    const float *bias;        // [O] or null
    // 12-bit VQ weights (an image with its matmul tables): rows of I*3/4
    // packed bytes; bf16 codebook pairs; sidecar patches (col | bf16 << 16)
    // of row o from rb[o], those of half step hs (64 columns) from offset
    // kq[o*(I/64)+hs] & 0xFFFF, kq[...] >> 16 of them
    const uint8_t *vidx;
    const uint32_t *cbh;
    const uint32_t *rb;
    const uint32_t *kq;
    const uint32_t *e4;
    // (tiles of 256 tokens) the same patches grouped per 32 rows and half
    // step: group g = (row / 32) * (I / 64) + col / 64 is g4[gp[g] ..
    // gp[g + 1]), each (row % 32) << 22 | (col % 64) << 16 | bf16
    const uint32_t *g4;
    const uint32_t *gp;
    const uint16_t *tx;       // (tiles of 256 tokens) the GEMV offset stream [O][I / 2]
    OutPtrs out;              // the [T, ldy] outputs (all get the same values)
    float *part;              // [splits][T, O] partial sums when splits > 1
    uint32_t T, I, O, gs, ldy;
    uint32_t splits;          // K ranges (gridDim.z); >1 writes partials, no bias
    uint32_t chain;           // 1: follows an unsplit GEMM of the same batch
    // Last-wave split (tail_s > 0; a one-dimensional grid): CTAs below n_full
    // take tiles 0 .. n_full-1 whole (tile t: row tile t % tiles_m, token
    // tile t / tiles_m); the others take the remaining tiles' K steps in
    // tail_s ranges each, write partial sums to ws ([tail tile][range][BN
    // columns][128 rows]) and count themselves in cnt[tail tile]; the last
    // to arrive adds the ranges in order and stores the tile.
    uint32_t tiles_m, n_full, tail_s;
    float *ws;
    uint32_t *cnt;
};

// Replace the bf16 at position `local` (0..63) of a thread's 32 packed
// pairs.  The register array is indexed statically: a switch on the word
// (a branch to the one update that applies) instead of a compare and
// select on all 32 registers per patch.
__device__ __forceinline__ void patch_pair(uint32_t (&v)[32], uint32_t local, uint32_t nb)
{
    const uint32_t keep = (local & 1u) ? 0xFFFFu : 0xFFFF0000u;
    const uint32_t put = (local & 1u) ? (nb << 16) : nb;
    switch (local >> 1) {
#define HXQ_PATCH_WORD(i) \
    case i: v[i] = (v[i] & keep) | put; break;
        HXQ_PATCH_WORD(0) HXQ_PATCH_WORD(1) HXQ_PATCH_WORD(2) HXQ_PATCH_WORD(3)
        HXQ_PATCH_WORD(4) HXQ_PATCH_WORD(5) HXQ_PATCH_WORD(6) HXQ_PATCH_WORD(7)
        HXQ_PATCH_WORD(8) HXQ_PATCH_WORD(9) HXQ_PATCH_WORD(10) HXQ_PATCH_WORD(11)
        HXQ_PATCH_WORD(12) HXQ_PATCH_WORD(13) HXQ_PATCH_WORD(14) HXQ_PATCH_WORD(15)
        HXQ_PATCH_WORD(16) HXQ_PATCH_WORD(17) HXQ_PATCH_WORD(18) HXQ_PATCH_WORD(19)
        HXQ_PATCH_WORD(20) HXQ_PATCH_WORD(21) HXQ_PATCH_WORD(22) HXQ_PATCH_WORD(23)
        HXQ_PATCH_WORD(24) HXQ_PATCH_WORD(25) HXQ_PATCH_WORD(26) HXQ_PATCH_WORD(27)
        HXQ_PATCH_WORD(28) HXQ_PATCH_WORD(29) HXQ_PATCH_WORD(30) HXQ_PATCH_WORD(31)
#undef HXQ_PATCH_WORD
        default: break;
    }
}

template <uint32_t BN, bool VQ>
__global__ void __launch_bounds__(kThreads, BN <= 128 ? 2 : 1)
dequant_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                    const __grid_constant__ Params p)
{
    constexpr uint32_t S = stages_for(BN, VQ);
    constexpr uint32_t SB = stage_bytes(BN, VQ);
    constexpr bool HS = half_steps(BN, VQ);
    constexpr bool SA = smem_a(BN, VQ);
    constexpr uint32_t kTmemA = tmem_a_col(BN);
    constexpr uint32_t kTmemCols = tmem_cols(BN, VQ);
    constexpr uint32_t kAOff = SA ? 2u * kABytes : 0u;   // A tiles after the ring
    constexpr uint32_t W = wstages_for(BN, VQ);
    constexpr uint32_t WB = wstage_bytes(BN, VQ);
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *ring = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~(uintptr_t)1023u);
    unsigned char *abuf = ring + S * SB;                  // SA: A[2], 1024-byte aligned
    unsigned char *wring = ring + S * SB + kAOff;         // weight ring, 1024-byte aligned
    uint64_t *full = reinterpret_cast<uint64_t *>(wring + W * WB);
    uint64_t *empty = full + S;
    uint64_t *a_full = empty + S;
    uint64_t *a_empty = a_full + 2;
    uint64_t *d_full = a_empty + 2;
    uint64_t *w_full = d_full + 1;
    uint64_t *w_empty = w_full + W;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(w_empty + W);
    volatile uint32_t *abort_flag = tmem_slot + 1;
    volatile uint32_t *last_flag = tmem_slot + 2;     // last-wave tile: this CTA adds the ranges
    uint32_t *cbh = reinterpret_cast<uint32_t *>(wring + W * WB + 256u);   // VQ: bf16 pairs

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t KT_all = p.I / kBK;                          // K steps of the matrix
    uint32_t o0, n0, kt_lo, KT;
    uint32_t tail = 0xFFFFFFFFu, trange = 0;   // last-wave tile and K range
    if (BN < 256u || p.tail_s == 0u) {
        o0 = blockIdx.x * kBM;
        n0 = blockIdx.y * BN;
        kt_lo = (uint32_t)((uint64_t)KT_all * blockIdx.z / p.splits);
        KT = (uint32_t)((uint64_t)KT_all * (blockIdx.z + 1u) / p.splits) - kt_lo;
    } else {
        uint32_t t = blockIdx.x;
        kt_lo = 0;
        KT = KT_all;
        if (t >= p.n_full) {
            const uint32_t j = t - p.n_full;
            tail = j / p.tail_s;
            trange = j % p.tail_s;
            t = p.n_full + tail;
            kt_lo = (uint32_t)((uint64_t)KT_all * trange / p.tail_s);
            KT = (uint32_t)((uint64_t)KT_all * (trange + 1u) / p.tail_s) - kt_lo;
        }
        o0 = (t % p.tiles_m) * kBM;
        n0 = (t / p.tiles_m) * BN;
    }

    if (!p.chain) asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(a_full + b, kConvWarps * 32);
            mbar_init(a_empty + b, 1);
        }
        mbar_init(d_full, 1);
        for (uint32_t s = 0; s < W; ++s) {
            mbar_init(w_full + s, 1);
            mbar_init(w_empty + s, kConvWarps);
        }
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

    uint32_t issued = 0, w_issued = 0;  // producer: activation and weight loads issued
    if (warp == kProducerWarp) {
        if (lane == 0) {
            // a step's weight tile goes first (the converters need it before
            // the MMA needs the step's activations); the weight ring runs up
            // to W steps ahead of the converters, the activation ring S ahead
            // of the MMA
            uint32_t kw = 0;
            bool ok = true;
            auto issue_w = [&](uint32_t k) {
                const uint32_t sw = k % W;
                if (k >= W && !mbar_wait(w_empty + sw, ((k / W) - 1u) & 1u, abort_flag)) return false;
                mbar_expect_tx(w_full + sw, WB);
                const uint32_t xw = (kt_lo + k) * ((VQ && !HS) ? 96u : kBK);
                tma_load_2d(wring + sw * WB, &wmap, w_full + sw, (int32_t)xw, (int32_t)o0);
                w_issued = k + 1u;
                return true;
            };
            for (uint32_t kt = 0; kt < KT && ok; ++kt) {
                for (; kw < KT && kw <= kt + W - 1u && ok; ++kw) ok = issue_w(kw);
                if (!ok) break;
                const uint32_t kg = (kt_lo + kt) * kBK;
                if constexpr (HS) {
                    // two half steps, a ring slot each (issued counts half steps)
                    for (uint32_t hh = 0; hh < 2u && ok; ++hh) {
                        const uint32_t u = 2u * kt + hh, s = u % S;
                        if (u >= S && !mbar_wait(empty + s, ((u / S) - 1u) & 1u, abort_flag)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(full + s, SB);
                        tma_load_2d(ring + s * SB, &xmap, full + s, (int32_t)(kg + 64u * hh), (int32_t)n0);
                        issued = u + 1u;
                    }
                } else {
                    const uint32_t s = kt % S;
                    if (kt >= S && !mbar_wait(empty + s, ((kt / S) - 1u) & 1u, abort_flag)) break;
                    mbar_expect_tx(full + s, SB);
                    unsigned char *dst = ring + s * SB;
                    tma_load_2d(dst, &xmap, full + s, (int32_t)kg, (int32_t)n0);
                    tma_load_2d(dst + BN * 128u, &xmap, full + s, (int32_t)(kg + 64u), (int32_t)n0);
                    issued = kt + 1u;
                }
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(BN);
            for (uint32_t kt = 0; kt < KT; ++kt) {
                const uint32_t s = kt % S, b = kt & 1u;
                if (!mbar_wait(a_full + b, (kt >> 1) & 1u, abort_flag)) break;
                if constexpr (HS) {
                    // both operands from shared memory; each half step's
                    // activations free their slot as soon as its four MMAs end
                    const uint32_t abase = smem_u32(abuf + b * kABytes);
                    bool good = true;
                    for (uint32_t hh = 0; hh < 2u; ++hh) {
                        const uint32_t u = 2u * kt + hh, su = u % S;
                        if (!mbar_wait(full + su, (u / S) & 1u, abort_flag)) {
                            good = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;");
                        const uint32_t bbase = smem_u32(ring + su * SB);
#pragma unroll
                        for (uint32_t k4 = 0; k4 < 4u; ++k4) {
                            const uint32_t kk = 4u * hh + k4;
                            mma_ss(tmem, smem_desc(abase + hh * (kBM * 128u) + k4 * 32u), smem_desc(bbase + k4 * 32u),
                                   idesc, (kt | kk) != 0u ? 1u : 0u);
                        }
                        mma_commit(empty + su);
                    }
                    if (!good) break;
                    mma_commit(a_empty + b);
                    continue;
                }
                if (!mbar_wait(full + s, (kt / S) & 1u, abort_flag)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t bbase = smem_u32(ring + s * SB);
                const uint32_t abase = smem_u32(abuf + b * kABytes);
#pragma unroll
                for (uint32_t kk = 0; kk < kBK / 16u; ++kk) {
                    const uint64_t bd = smem_desc(bbase + (kk >> 2) * (BN * 128u) + (kk & 3u) * 32u);
                    if constexpr (SA) {
                        const uint64_t ad = smem_desc(abase + (kk >> 2) * (kBM * 128u) + (kk & 3u) * 32u);
                        mma_ss(tmem, ad, bd, idesc, (kt | kk) != 0u ? 1u : 0u);
                    } else {
                        mma_ts(tmem, tmem + kTmemA + b * 64u + kk * 8u, bd, idesc, (kt | kk) != 0u ? 1u : 0u);
                    }
                }
                mma_commit(a_empty + b);
                mma_commit(empty + s);
            }
            mma_commit(d_full);
        }
    } else {
        // converters, then the epilogue
        const uint32_t q = warp & 3u, h = warp >> 2;
        const uint32_t row = q * 32u + lane;
        const uint32_t o = o0 + row;
        const bool valid = o < p.O;
        const uint32_t lane_base = (q * 32u) << 16;
        bool ok = true;
        if constexpr (!VQ) {
            const uint32_t ng = p.I / p.gs;
            // scales and offsets are loaded four K steps ahead, into one
            // register pair per step modulo 4: the loop is unrolled by four so
            // that no register holding a load in flight is ever copied (a
            // copy waits for the load, which would shrink the distance to
            // one step).  The codes come from the weight ring (row `row` of
            // the stage: 128 B, its 16-byte units swizzled by row & 7, so a
            // warp's loads are free of bank conflicts).
            float sq0 = 0.0f, sq1 = 0.0f, sq2 = 0.0f, sq3 = 0.0f;
            float oq0 = 0.0f, oq1 = 0.0f, oq2 = 0.0f, oq3 = 0.0f;
            auto fetch = [&](uint32_t kt, float &sv, float &fv) {
                if (valid && kt < KT) {
                    const uint32_t g = ((kt_lo + kt) * kBK + h * 64u) / p.gs;
                    sv = __ldg(p.scales + (size_t)o * ng + g);
                    fv = __ldg(p.offsets + (size_t)o * ng + g);
                }
            };
            fetch(0, sq0, oq0);
            fetch(1, sq1, oq1);
            fetch(2, sq2, oq2);
            fetch(3, sq3, oq3);
            // one K step: the codes into bf16 weights, into A buffer kt & 1;
            // false if a wait ran out
            auto step = [&](uint32_t kt, float &sq, float &oq) -> bool {
                const uint32_t b = kt & 1u, sw = kt % W;
                if (!mbar_wait(w_full + sw, (kt / W) & 1u, abort_flag)) return false;
                uint4 c[4];
                const unsigned char *wr = wring + sw * WB + row * 128u;
#pragma unroll
                for (uint32_t i = 0; i < 4u; ++i)
                    c[i] = *reinterpret_cast<const uint4 *>(wr + (((4u * h + i) ^ (row & 7u)) << 4));
                async_proxy_fence();
                __syncwarp();
                if (lane == 0) mbar_arrive(w_empty + sw);
                const float sc = sq, of = oq;
                const uint64_t s2 = BN >= 256 ? f32x2_splat(sc) : 0ull, o2 = BN >= 256 ? f32x2_splat(of) : 0ull;
                fetch(kt + 4u, sq, oq);
                uint32_t v[32];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t w4[4] = {c[i].x, c[i].y, c[i].z, c[i].w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if constexpr (BN >= 256) {
                            v[8 * i + 2 * j] = code_pair_bf16(w4[j], 0u, s2, o2);
                            v[8 * i + 2 * j + 1] = code_pair_bf16(w4[j], 2u, s2, o2);
                        } else {
                            // (the two-CTA tiles have no registers to spare
                            // for the packed operands)
                            const float f0 = fmaf(code_f32(w4[j], 0), sc, of);
                            const float f1 = fmaf(code_f32(w4[j], 1), sc, of);
                            const float f2 = fmaf(code_f32(w4[j], 2), sc, of);
                            const float f3 = fmaf(code_f32(w4[j], 3), sc, of);
                            v[8 * i + 2 * j] = bf16x2(f0, f1);
                            v[8 * i + 2 * j + 1] = bf16x2(f2, f3);
                        }
                    }
                }
                if (kt >= 2 && !mbar_wait(a_empty + b, ((kt >> 1) - 1u) & 1u, abort_flag)) return false;
                tmem_st32(tmem + lane_base + kTmemA + b * 64u + h * 32u, v);
                asm volatile("tcgen05.wait::st.sync.aligned;");
                asm volatile("tcgen05.fence::before_thread_sync;");
                mbar_arrive(a_full + b);
                return true;
            };
            for (uint32_t kt = 0; kt < KT && ok; kt += 4u) {
                ok = step(kt, sq0, oq0);
                if (ok && kt + 1u < KT) ok = step(kt + 1u, sq1, oq1);
                if (ok && kt + 2u < KT) ok = step(kt + 2u, sq2, oq2);
                if (ok && kt + 3u < KT) ok = step(kt + 3u, sq3, oq3);
            }
        } else if constexpr (SA) {
            // VQ, tiles of 256 tokens: A tiles in shared memory.  The image's
            // bf16 codebook twice (copy 0 at word c, copy 1 at word 4096 +
            // (c ^ ((c >> 5) & 31))): a pair's offset names one packed pair.
            for (uint32_t i = tid; i < 4096u; i += kConvWarps * 32u) {
                const uint32_t e = __ldg(p.cbh + i);
                cbh[i] = e;
                cbh[4096u + (i ^ ((i >> 5) & 31u))] = e;
            }
            // The weights come from the image's GEMV offset stream -- per
            // pair the 16-bit byte offset of its entry in the two-copy
            // codebook, in natural pair order, the copy chosen when the image
            // was built so that each gather instruction of the GEMV's lane
            // layout (8 rows x 4 pair slots of a 64-pair window) spreads over
            // the banks: about 2 shared-memory wavefronts per warp-wide
            // gather against 3.5 from one copy.  A K step is one such window
            // and the converters take the GEMV's lanes: lane (g, t) of warp w
            // converts tile rows 16w + g and 16w + g + 8, pairs [16t, 16t +
            // 16) of the step, so each of its 32 gathers per step is one of
            // the builder's instructions.  The stream comes through the
            // weight ring (128 rows x 128 B per step, 128-byte swizzle).
            const unsigned char *cbb = reinterpret_cast<const unsigned char *>(cbh);
            const uint32_t g = lane >> 2, t = lane & 3u;
            const uint32_t ra = 16u * warp + g;              // tile rows ra and ra + 8 (both = g mod 8)
            // Sidecar patches by warp from the table grouped per 32 rows and
            // half K step: warp w's rows are half of group o0 / 32 + w / 2,
            // and a K step is two consecutive groups (both halves, adjacent
            // in the table); lane i takes the step's entry i (past 32,
            // again) and applies it when its row is one of the warp's 16.
            // The group offsets sit in four slots, each refilled four steps
            // ahead; a step's first 32 entries (one per lane) in one of two
            // registers, loaded two steps ahead.  The loop is unrolled by four
            // so that the slots are fixed registers: a register holding a load
            // in flight is never copied (a copy would wait for the load).
            const uint32_t NH = p.I / 64u;
            const uint32_t grp = o0 / 32u + (warp >> 1), rsel = warp & 1u;
            const bool gvalid = grp * 32u < p.O;
            const uint32_t *gpp = p.gp + (size_t)(gvalid ? grp : 0u) * NH + 2u * kt_lo;
            auto gload = [&](uint32_t k) -> uint3 {
                return (gvalid && k < KT)
                           ? make_uint3(__ldg(gpp + 2u * k), __ldg(gpp + 2u * k + 1u), __ldg(gpp + 2u * k + 2u))
                           : make_uint3(0u, 0u, 0u);
            };
            auto eload = [&](uint3 r) -> uint32_t { return lane < r.z - r.x ? __ldg(p.g4 + r.x + lane) : 0u; };
            uint3 gq0 = gload(0), gq1 = gload(1), gq2 = gload(2), gq3 = gload(3);
            uint32_t ea = KT > 0 ? eload(gq0) : 0u, ez = KT > 1 ? eload(gq1) : 0u;
            asm volatile("bar.sync 1, %0;" ::"n"(kConvWarps * 32) : "memory");
            // 16 packed pairs of one row from its two 16-byte units of offsets
            auto gather = [&](const uint4 &q0, const uint4 &q1, uint32_t (&v)[16]) {
                const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (uint32_t i = 0; i < 8u; ++i) {
                    v[2u * i] = *reinterpret_cast<const uint32_t *>(cbb + (w[i] & 0xFFFFu));
                    v[2u * i + 1u] = *reinterpret_cast<const uint32_t *>(cbb + (w[i] >> 16));
                }
            };
            // one row's 64 bytes of the A tile: K half t / 2, 16-byte units
            // 4 (t & 1) .. +3, unit u at (u ^ g) << 4
            auto put = [&](unsigned char *arow, const uint32_t (&v)[16]) {
                const uint32_t ub = (t & 1u) * 4u;
#pragma unroll
                for (uint32_t u = 0; u < 4u; ++u)
                    *reinterpret_cast<uint4 *>(arow + (((ub + u) ^ g) << 4)) =
                        make_uint4(v[4u * u], v[4u * u + 1u], v[4u * u + 2u], v[4u * u + 3u]);
            };
            // one K step: g_cur the group offsets of step kt (its slot,
            // refilled with step kt + 4's), g_2 those of step kt + 2, E this
            // lane's first entry of step kt (refilled with step kt + 2's);
            // false if a wait ran out
            auto step = [&](uint32_t kt, uint3 &g_cur, uint3 g_2, uint32_t &E) -> bool {
                const uint32_t b = kt & 1u, sw = kt % W;
                if (!mbar_wait(w_full + sw, (kt / W) & 1u, abort_flag)) return false;
                // units 2t and 2t + 1 of lines ra and ra + 8 (unit u of line r
                // at (u ^ (r & 7)) << 4): a quarter-warp's eight loads cover
                // all 32 banks
                const unsigned char *ws = wring + sw * WB;
                const uint4 q0 = *reinterpret_cast<const uint4 *>(ws + ra * 128u + (((2u * t) ^ g) << 4));
                const uint4 q1 = *reinterpret_cast<const uint4 *>(ws + ra * 128u + (((2u * t + 1u) ^ g) << 4));
                const uint4 q2 = *reinterpret_cast<const uint4 *>(ws + (ra + 8u) * 128u + (((2u * t) ^ g) << 4));
                const uint4 q3 = *reinterpret_cast<const uint4 *>(ws + (ra + 8u) * 128u + (((2u * t + 1u) ^ g) << 4));
                async_proxy_fence();
                __syncwarp();
                if (lane == 0) mbar_arrive(w_empty + sw);
                uint32_t v0[16], v1[16];
                gather(q0, q1, v0);
                gather(q2, q3, v1);
                __syncwarp();
                if (kt >= 2 && !mbar_wait(a_empty + b, ((kt >> 1) - 1u) & 1u, abort_flag)) return false;
                unsigned char *ab = abuf + b * kABytes;
                put(ab + (t >> 1) * (kBM * 128u) + ra * 128u, v0);
                put(ab + (t >> 1) * (kBM * 128u) + (ra + 8u) * 128u, v1);
                // the warp's patches: the reference's fp32 value rounded once
                // to bf16, over the codebook pair's half, once all the warp's
                // rows are stored
                __syncwarp();
                const uint32_t n = g_cur.z - g_cur.x;
                unsigned char *ag = ab + (32u * (warp >> 1)) * 128u;
                auto apply = [&](uint32_t i, uint32_t e) {
                    const uint32_t r = (e >> 22) & 31u, lc = (e >> 16) & 63u;
                    if ((r >> 4) != rsel) return;
                    const uint32_t half = g_cur.x + i >= g_cur.y ? 1u : 0u;
                    *reinterpret_cast<uint16_t *>(ag + half * (kBM * 128u) + r * 128u +
                                                  ((((lc >> 3) ^ (r & 7u)) << 4) | ((lc & 7u) << 1))) = (uint16_t)e;
                };
                if (lane < n) apply(lane, E);
#pragma unroll 1
                for (uint32_t base = 32u; base < n; base += 32u)
                    if (base + lane < n) apply(base + lane, __ldg(p.g4 + g_cur.x + base + lane));
                // the generic-proxy stores, visible to the tensor cores' reads
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(a_full + b);
                if (kt + 2u < KT) E = eload(g_2);
                g_cur = gload(kt + 4u);
                return true;
            };
            for (uint32_t kt = 0; kt < KT && ok; kt += 4u) {
                ok = step(kt, gq0, gq2, ea);
                if (ok && kt + 1u < KT) ok = step(kt + 1u, gq1, gq3, ez);
                if (ok && kt + 2u < KT) ok = step(kt + 2u, gq2, gq0, ea);
                if (ok && kt + 3u < KT) ok = step(kt + 3u, gq3, gq1, ez);
            }
        } else {
            // VQ, tiles of up to 128 tokens: A into tensor memory.  The
            // image's bf16 codebook, one 32-bit pair per entry: an index
            // gathers exactly one TMEM column (low half = even k)
            for (uint32_t i = tid; i < codebook_bytes(BN) / 16u; i += kConvWarps * 32u)
                reinterpret_cast<uint4 *>(cbh)[i] = __ldg(reinterpret_cast<const uint4 *>(p.cbh) + i);
            // patches: those of this thread's half of step kt are n entries
            // from pb + lo, kq[2 kt + h] = lo | n << 16 (kq of this row,
            // from this CTA's first step), so a warp walks only its own
            // 64 columns' patches.  The entries sit in four slots, each
            // refilled four steps ahead; the first four patches of a step in
            // one of two sets, loaded two steps ahead.  The loop is unrolled
            // by four so that the slots and sets are fixed registers: a
            // register holding a load in flight is never copied (a copy
            // would wait for the load).
            const uint32_t *kqr = p.kq + (size_t)(valid ? o : 0u) * (2u * KT_all) + 2u * kt_lo + h;
            const uint32_t pb = valid ? __ldg(p.rb + o) : 0u;
            auto kload = [&](uint32_t j) -> uint32_t { return valid && j < KT ? __ldg(kqr + 2u * j) : 0u; };
            auto load4 = [&](uint32_t k, uint32_t (&q)[4]) {
                const uint32_t *src = p.e4 + pb + (k & 0xFFFFu);
                const uint32_t n = k >> 16;
                q[0] = n > 0u ? __ldg(src) : 0u;
                q[1] = n > 1u ? __ldg(src + 1) : 0u;
                q[2] = n > 2u ? __ldg(src + 2) : 0u;
                q[3] = n > 3u ? __ldg(src + 3) : 0u;
            };
            uint32_t kq0 = kload(0), kq1 = kload(1), kq2 = kload(2), kq3 = kload(3);
            uint32_t pa[4] = {0u, 0u, 0u, 0u}, pz[4] = {0u, 0u, 0u, 0u};
            if (KT > 0) load4(kq0, pa);
            if (KT > 1) load4(kq1, pz);
            asm volatile("bar.sync 1, %0;" ::"n"(kConvWarps * 32) : "memory");
            // one K step: k_lo = kq entry of step kt (its slot, refilled with
            // step kt + 4's), k_2 step kt + 2's; P the step's first four
            // patches (refilled with those of step kt + 2); false if a wait ran out
            auto step = [&](uint32_t kt, uint32_t &k_lo, uint32_t k_2, uint32_t (&P)[4]) -> bool {
                const uint32_t b = kt & 1u, sw = kt % W;
                // 64 weights = 16 byte triples = 3 x 16 bytes of this thread's
                // row of the weight ring stage (96 B per row)
                if (!mbar_wait(w_full + sw, (kt / W) & 1u, abort_flag)) return false;
                uint4 cn[3];
                const unsigned char *wr = wring + sw * WB + row * 96u + h * 48u;
#pragma unroll
                for (uint32_t i = 0; i < 3u; ++i) cn[i] = *reinterpret_cast<const uint4 *>(wr + 16u * i);
                async_proxy_fence();
                __syncwarp();
                if (lane == 0) mbar_arrive(w_empty + sw);
                const uint32_t w[12] = {cn[0].x, cn[0].y, cn[0].z, cn[0].w, cn[1].x, cn[1].y,
                                        cn[1].z, cn[1].w, cn[2].x, cn[2].y, cn[2].z, cn[2].w};
                const uint32_t n_cur = k_lo >> 16, lo_cur = k_lo & 0xFFFFu;
                uint32_t v[32];
#pragma unroll
                for (uint32_t t = 0; t < 16u; ++t) {
                    const uint32_t byte = 3u * t, wq = byte >> 2;
                    const uint32_t B = __byte_perm(w[wq], w[wq + 1u < 12u ? wq + 1u : 11u], 0x3012u + (byte & 3u) * 0x1111u);
                    v[2u * t] = cbh[(B >> 12) & 0xFFFu];
                    v[2u * t + 1u] = cbh[B & 0xFFFu];
                }
                // sidecar: the patches of this half-step replace their weights
                // with the reference's fp32 value rounded once to bf16
                const uint32_t k0 = (kt_lo + kt) * kBK + h * 64u;
                uint32_t r0 = P[0], r1 = P[1], r2 = P[2], r3 = P[3];
                {
#pragma unroll 1
                    for (uint32_t i = 0; i < n_cur; ++i) {
                        const uint32_t q = i < 4u ? r0 : __ldg(p.e4 + pb + lo_cur + i);
                        r0 = r1; r1 = r2; r2 = r3;
                        const uint32_t local = (q & 0xFFFFu) - k0;
                        if (local < 64u) patch_pair(v, local, q >> 16);
                    }
                    __syncwarp();
                    if (kt >= 2 && !mbar_wait(a_empty + b, ((kt >> 1) - 1u) & 1u, abort_flag)) return false;
                    tmem_st32(tmem + lane_base + kTmemA + b * 64u + h * 32u, v);
                    asm volatile("tcgen05.wait::st.sync.aligned;");
                    asm volatile("tcgen05.fence::before_thread_sync;");
                    mbar_arrive(a_full + b);
                }
                if (kt + 2u < KT) load4(k_2, P);
                k_lo = kload(kt + 4u);
                return true;
            };
            for (uint32_t kt = 0; kt < KT && ok; kt += 4u) {
                ok = step(kt, kq0, kq2, pa);
                if (ok && kt + 1u < KT) ok = step(kt + 1u, kq1, kq3, pz);
                if (ok && kt + 2u < KT) ok = step(kt + 2u, kq2, kq0, pa);
                if (ok && kt + 3u < KT) ok = step(kt + 3u, kq3, kq1, pz);
            }
        }
        // this half's accumulator columns; a 32-column load may read past
        // them (inside the allocation) when BN < 64: those are not stored.
        // 32 columns per load for the wide tiles, 16 for BN <= 64 (whose
        // converters hold fewer registers free)
        const uint32_t cbeg = h * (BN / 2u), cend = cbeg + BN / 2u;
        constexpr uint32_t EW = BN >= 128 ? 32u : 16u;
        const bool done = ok && mbar_wait(d_full, 0u, abort_flag);
        if (done) asm volatile("tcgen05.fence::after_thread_sync;");
        if (BN < 256u || tail == 0xFFFFFFFFu) {
            if (done) {
                const bool partial = p.splits > 1u;
                const float bo = (valid && p.bias && !partial) ? __ldg(p.bias + o) : 0.0f;
                const uint32_t nout = partial ? 1u : p.out.n;
                const uint32_t ld = partial ? p.O : p.ldy;
#pragma unroll 1
                for (uint32_t c0 = cbeg; c0 < cend; c0 += EW) {
                    uint32_t v[EW];
                    tmem_ld<EW>(tmem + lane_base + c0, v);
                    asm volatile("tcgen05.wait::ld.sync.aligned;");
                    if (valid) {
                        for (uint32_t k = 0; k < nout; ++k) {
                            float *yo = partial ? p.part + (size_t)blockIdx.z * p.T * p.O : p.out.y[k];
#pragma unroll
                            for (uint32_t j = 0; j < EW; ++j) {
                                const uint32_t n = n0 + c0 + j;
                                if (c0 + j < cend && n < p.T) yo[(size_t)n * ld + o] = __uint_as_float(v[j]) + bo;
                            }
                        }
                    }
                }
            }
        } else if constexpr (BN == 256u) {
            // a last-wave tile in two K ranges: both write their partial
            // sums (column-major, so that a warp's stores of one column are
            // 128 contiguous bytes) and count themselves; the second to
            // arrive adds the other's partial sums to its own, still in
            // tensor memory.  x0 + x1 == x1 + x0 in IEEE arithmetic, so the
            // result does not depend on which range arrives last.
            float *tile_ws = p.ws + (size_t)tail * 2u * (BN * kBM);
            if (done) {
                float *wp = tile_ws + (size_t)trange * (BN * kBM);
#pragma unroll 1
                for (uint32_t c0 = cbeg; c0 < cend; c0 += EW) {
                    uint32_t v[EW];
                    tmem_ld<EW>(tmem + lane_base + c0, v);
                    asm volatile("tcgen05.wait::ld.sync.aligned;");
#pragma unroll
                    for (uint32_t j = 0; j < EW; ++j)
                        if (c0 + j < cend) wp[(c0 + j) * kBM + row] = __uint_as_float(v[j]);
                }
            }
            __threadfence();
            // every converter thread reaches both barriers, also after a wait
            // gave up (it set the abort flag first); then nothing is counted
            asm volatile("bar.sync 1, %0;" ::"n"(kConvWarps * 32) : "memory");
            if (tid == 0) {
                uint32_t last = 0;
                if (!*abort_flag) {
                    last = atomicAdd(p.cnt + tail, 1u) == 1u ? 1u : 0u;
                    if (last) p.cnt[tail] = 0u;   // both ranges counted: ready for the next launch
                }
                *last_flag = last;
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kConvWarps * 32) : "memory");
            if (*last_flag) {
                __threadfence();
                const float *other = tile_ws + (size_t)(1u - trange) * (BN * kBM);
                const float bo = (valid && p.bias) ? __ldg(p.bias + o) : 0.0f;
#pragma unroll 1
                for (uint32_t c0 = cbeg; c0 < cend; c0 += EW) {
                    uint32_t v[EW];
                    float ot[EW];
#pragma unroll
                    for (uint32_t j = 0; j < EW; ++j)
                        ot[j] = c0 + j < cend ? __ldcg(other + (c0 + j) * kBM + row) : 0.0f;
                    tmem_ld<EW>(tmem + lane_base + c0, v);
                    asm volatile("tcgen05.wait::ld.sync.aligned;");
                    if (valid) {
                        for (uint32_t k = 0; k < p.out.n; ++k) {
#pragma unroll
                            for (uint32_t j = 0; j < EW; ++j) {
                                const uint32_t n = n0 + c0 + j;
                                if (c0 + j < cend && n < p.T)
                                    p.out.y[k][(size_t)n * p.ldy + o] = (__uint_as_float(v[j]) + ot[j]) + bo;
                            }
                        }
                    }
                }
            }
        }
    }
    // Teardown: every issued MMA (the d_full commit follows the last one)
    // and every issued activation load has landed before tensor memory and
    // shared memory are released, also when a wait above gave up.
    if (warp == kMmaWarp && lane == 0) mbar_drain(d_full, 0u);
    if (warp == kProducerWarp && lane == 0) {
        for (uint32_t kt = issued > S ? issued - S : 0u; kt < issued; ++kt) mbar_drain(full + kt % S, (kt / S) & 1u);
        for (uint32_t kt = w_issued > W ? w_issued - W : 0u; kt < w_issued; ++kt)
            mbar_drain(w_full + kt % W, (kt / W) & 1u);
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
    // a chained GEMM completes only after the one before it
    if (p.chain) asm volatile("griddepcontrol.wait;" ::: "memory");
}

// y[n, o] = sum over the K ranges, in order, of the partial sums + bias,
// stored into every output.
__global__ void splitk_reduce_kernel(const float *__restrict__ part, const float *__restrict__ bias,
                                     const __grid_constant__ OutPtrs out, uint32_t T, uint32_t O, uint32_t ldy,
                                     uint32_t splits)
{
    const uint64_t total = (uint64_t)T * O;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (uint64_t)gridDim.x * blockDim.x) {
        float acc = 0.0f;
        for (uint32_t k = 0; k < splits; ++k) acc += part[(size_t)k * total + i];
        const uint32_t o = (uint32_t)(i % O);
        if (bias) acc += __ldg(bias + o);
        for (uint32_t k = 0; k < out.n; ++k) out.y[k][(i / O) * ldy + o] = acc;
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
        else
            cudaGetLastError();
    }
    return fn;
}

template <uint32_t BN, bool VQ>
int launch(const uint16_t *x, const Params &p, cudaStream_t s)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc) return -1;
    CUtensorMap map;
    std::memset(&map, 0, sizeof(map));
    const cuuint64_t dims[2] = {p.I, p.T};
    const cuuint64_t strides[1] = {(cuuint64_t)p.I * 2u};
    const cuuint32_t box[2] = {64u, BN};
    const cuuint32_t estr[2] = {1u, 1u};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return -1;
    // the weights: affine codes [O][I] in boxes of 128 B x 128 rows with
    // 128-byte swizzle, VQ index bytes [O][I * 3 / 4] in boxes of 96 B x
    // 128 rows (no swizzle), or for the VQ tile of 256 tokens the GEMV
    // offset stream [O][I bytes] in boxes of 128 B x 128 rows with 128-byte
    // swizzle; rows past O read as zero
    constexpr bool HSL = half_steps(BN, VQ);
    CUtensorMap wmap;
    std::memset(&wmap, 0, sizeof(wmap));
    const cuuint64_t wrow = (VQ && !HSL) ? (cuuint64_t)(p.I / 4u) * 3u : (cuuint64_t)p.I;
    const cuuint64_t wdims[2] = {wrow, p.O};
    const cuuint64_t wstrides[1] = {wrow};
    const cuuint32_t wbox[2] = {(VQ && !HSL) ? 96u : 128u, kBM};
    const void *wbase = HSL ? static_cast<const void *>(p.tx) : VQ ? static_cast<const void *>(p.vidx)
                                                                    : static_cast<const void *>(p.codes);
    if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(wbase), wdims, wstrides, wbox, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, (VQ && !HSL) ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return -1;
    auto kern = dequant_gemm_kernel<BN, VQ>;
    const uint32_t smem = smem_bytes(BN, VQ);
    // the shared-memory opt-in is made once per device and instantiation
    static std::atomic<uint64_t> configured{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) { cudaGetLastError(); return -1; }
    const uint64_t bit = 1ull << dev;
    if (!(configured.load(std::memory_order_acquire) & bit)) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
        configured.fetch_or(bit, std::memory_order_acq_rel);
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    const uint32_t tiles = ((p.O + kBM - 1) / kBM) * ((p.T + BN - 1) / BN);
    cfg.gridDim = p.tail_s ? dim3(p.n_full + (tiles - p.n_full) * p.tail_s, 1, 1)
                           : dim3((p.O + kBM - 1) / kBM, (p.T + BN - 1) / BN, p.splits);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    // only a chained GEMM is launched ahead of its predecessor's end: an
    // early launch behind other kernels (the GEMVs signal at their start)
    // measured slower
    cfg.numAttrs = p.chain ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, map, wmap, p) != cudaSuccess) { cudaGetLastError(); return -1; }
    return 0;
}

// Partial-sum buffer for split-K, one per (device, stream) so calls on
// different streams never share it; grown on demand (the first call of a
// shape on a stream allocates; later calls, e.g. under graph capture, reuse).
float *splitk_buffer(size_t floats, cudaStream_t s)
{
    struct Buf { float *p = nullptr; size_t cap = 0; };
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

// Last-wave split state, one per (device, stream) like the split-K buffer:
// partial sums of the last wave's tiles and their arrival counters.  The
// counters start at zero when allocated and every completed tile returns its
// counter to zero; a launch that gave up (device status set) can leave one
// counted, so gemm_reset_tail_counters() clears them when that status is
// taken.
struct TailBuf {
    float *ws = nullptr;
    size_t cap = 0;
    uint32_t *cnt = nullptr;
};
constexpr uint32_t kMaxTailTiles = 1024;
std::mutex g_tail_mu;
std::map<std::pair<int, cudaStream_t>, TailBuf> g_tail;

bool tail_buffer(size_t floats, cudaStream_t s, float **ws, uint32_t **cnt)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return false; }
    std::lock_guard<std::mutex> lk(g_tail_mu);
    TailBuf &b = g_tail[{dev, s}];
    if (!b.cnt) {
        if (cudaMalloc(&b.cnt, kMaxTailTiles * sizeof(uint32_t)) != cudaSuccess) {
            cudaGetLastError();
            b.cnt = nullptr;
            return false;
        }
        if (cudaMemsetAsync(b.cnt, 0, kMaxTailTiles * sizeof(uint32_t), s) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(b.cnt);
            b.cnt = nullptr;
            return false;
        }
    }
    if (b.cap < floats) {
        if (b.ws) { cudaStreamSynchronize(s); cudaFree(b.ws); }
        b.ws = nullptr;
        b.cap = 0;
        if (cudaMalloc(&b.ws, floats * sizeof(float)) != cudaSuccess) { cudaGetLastError(); return false; }
        b.cap = floats;
    }
    *ws = b.ws;
    *cnt = b.cnt;
    return true;
}

// Chain state of the batch being launched on this host thread: whether the
// last kernel it put on `s` was an unsplit GEMM.
struct Chain {
    bool active = false, prev_gemm = false;
    cudaStream_t s = nullptr;
};
thread_local Chain g_chain;

}  // namespace gemm

void gemm_chain_begin(cudaStream_t s) { gemm::g_chain = gemm::Chain{true, false, s}; }

void gemm_reset_tail_counters()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return; }
    std::lock_guard<std::mutex> lk(gemm::g_tail_mu);
    for (auto &kv : gemm::g_tail)
        if (kv.first.first == dev && kv.second.cnt)
            if (cudaMemset(kv.second.cnt, 0, gemm::kMaxTailTiles * sizeof(uint32_t)) != cudaSuccess) cudaGetLastError();
}
void gemm_chain_end() { gemm::g_chain = gemm::Chain{}; }
void gemm_chain_break() { gemm::g_chain.prev_gemm = false; }

namespace {

// Token tile, K split and launch for one matmul; p.splits, p.out and p.part are set
// here.  0 on launch, -1 on error.
template <bool VQ>
int run(const uint16_t *x, gemm::Params p, const OutPtrs &out, cudaStream_t s)
{
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t T = p.T, O = p.O;
    const uint32_t bn = T <= 16 ? 16u : T <= 32 ? 32u : T <= 64 ? 64u : T <= 128 ? 128u : 256u;
    // Split K when the (rows x token) tiles alone would leave SMs idle.
    const uint32_t tiles = ((O + gemm::kBM - 1) / gemm::kBM) * ((T + bn - 1) / bn);
    const uint32_t KT = p.I / gemm::kBK;
    const uint32_t resident = (uint32_t)sms * (bn <= 128 ? 2u : 1u);  // CTAs the GPU holds at once
    uint32_t splits = 1;
    if (tiles < resident) {
        splits = resident / tiles;                 // one wave: tiles * splits <= resident
        // at least two K steps per CTA; eight for the affine converters,
        // which reach the split's one-wave time with fewer, longer ranges
        // (4096 x 4096 at 64 / 128 tokens: 4 ranges 15.7 / 19.4 us, 9 ranges
        // 16.5 / 21.3), where the VQ converters want every resident CTA
        const uint32_t min_steps = VQ ? 2u : 8u;
        if (splits > KT / min_steps) splits = KT / min_steps;
        if (splits > 16u) splits = 16u;
        if (splits < 1u) splits = 1u;
    }
    float *part = nullptr;
    if (splits > 1) {
        part = gemm::splitk_buffer((size_t)splits * T * O, s);
        if (!part) return -1;
    }
    p.splits = splits;
    p.out = out;
    p.part = part;
    gemm::Chain &ch = gemm::g_chain;
    const bool in_batch = ch.active && ch.s == s;
    // Last-wave split: when whole waves of tiles leave a last wave that
    // fills at most half of the GPU, its tiles are split along K into two
    // ranges: 512 tiles of 128 x 256 on 148 SMs run as 3 waves and one of
    // half-length tiles instead of 4 waves.  Not inside a batch, whose GEMMs
    // already overlap one another's last waves; only for the 256-token tiles
    // (the smaller ones are split along K whenever they leave SMs idle).
    p.tiles_m = (O + gemm::kBM - 1) / gemm::kBM;
    p.n_full = tiles;
    p.tail_s = 0;
    if (bn == 256u && splits == 1 && !in_batch && tiles > resident && KT >= 8u) {
        const uint32_t rem = tiles % resident;
        if (rem != 0 && rem * 2u <= resident && rem <= gemm::kMaxTailTiles) {
            float *ws = nullptr;
            uint32_t *cnt = nullptr;
            if (!gemm::tail_buffer((size_t)rem * 2u * gemm::kBM * bn, s, &ws, &cnt)) return -1;
            p.n_full = tiles - rem;
            p.tail_s = 2;
            p.ws = ws;
            p.cnt = cnt;
        }
    }
    p.chain = in_batch && ch.prev_gemm && splits == 1 ? 1u : 0u;
    if (in_batch) ch.prev_gemm = false;   // set again below on an unsplit launch
    int r;
    switch (bn) {
    case 16: r = gemm::launch<16, VQ>(x, p, s); break;
    case 32: r = gemm::launch<32, VQ>(x, p, s); break;
    case 64: r = gemm::launch<64, VQ>(x, p, s); break;
    case 128: r = gemm::launch<128, VQ>(x, p, s); break;
    default: r = gemm::launch<256, VQ>(x, p, s); break;
    }
    if (r == 0 && splits == 1 && in_batch) ch.prev_gemm = true;
    if (r != 0 || splits == 1) return r;
    const uint64_t total = (uint64_t)T * O;
    uint64_t blocks = (total + 255u) / 256u;
    if (blocks > (uint64_t)sms * 8u) blocks = (uint64_t)sms * 8u;
    gemm::splitk_reduce_kernel<<<(uint32_t)blocks, 256, 0, s>>>(part, p.bias, out, T, O, p.ldy, splits);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace

bool affine_gemm_fits(const uint16_t *x, const uint8_t *codes, uint32_t T, uint32_t I, uint32_t O, uint32_t gs)
{
    if (T == 0 || O == 0) return false;
    if (I == 0 || I % gemm::kBK != 0 || gs == 0 || gs % 64u != 0 || I % gs != 0) return false;
    if (((uintptr_t)x & 15u) || ((uintptr_t)codes & 15u)) return false;
    return (uint64_t)T * I < (1ull << 40);
}

// Tensor-core path for bf16 activations.  Returns 1 when the shape is not
// one it takes (the caller uses the GEMV), 0 on launch, -1 on error.
int affine_gemm_bf16(const uint16_t *x, const uint8_t *codes, const float *scales, const float *offsets,
                     const float *bias, const OutPtrs &out, uint32_t ldy, uint32_t T, uint32_t I, uint32_t O,
                     uint32_t gs, cudaStream_t s)
{
    if (!affine_gemm_fits(x, codes, T, I, O, gs)) return 1;
    gemm::Params p{};
    p.codes = codes; p.scales = scales; p.offsets = offsets; p.bias = bias;
    if (ldy < O || out.n == 0 || out.n > HXQ_CUDA_MAX_PEERS) return 1;
    p.T = T; p.I = I; p.O = O; p.gs = gs; p.ldy = ldy;
    return run<false>(x, p, out, s);
}

// Fused VQ-dequant GEMM on a 12-bit image with its matmul tables: x bf16
// [T, I], y fp32 [T, ldy].  Returns 1 when the shape is not one it takes, 0
// on launch, -1 on error.
int vq_gemm_bf16(const uint16_t *x, const uint8_t *idx, const uint32_t *cbh, const uint32_t *rb,
                 const uint32_t *kq, const uint32_t *e4, const uint32_t *g4, const uint32_t *gp,
                 const uint16_t *tx, const OutPtrs &out, uint32_t T, uint32_t I, uint32_t O, uint32_t ldy,
                 cudaStream_t s)
{
    if (T == 0 || O == 0) return 1;
    if (I == 0 || I % gemm::kBK != 0 || ldy < O) return 1;
    if (((uintptr_t)x & 15u) || ((uintptr_t)idx & 15u) || ((uintptr_t)cbh & 15u)) return 1;
    if ((uint64_t)T * I >= (1ull << 40)) return 1;
    gemm::Params p{};
    if (!g4 || !gp || !tx || ((uintptr_t)tx & 15u)) return 1;
    p.vidx = idx; p.cbh = cbh; p.rb = rb; p.kq = kq; p.e4 = e4; p.g4 = g4; p.gp = gp; p.tx = tx;
    if (out.n == 0 || out.n > HXQ_CUDA_MAX_PEERS) return 1;
    p.T = T; p.I = I; p.O = O; p.gs = 0; p.ldy = ldy;
    return run<true>(x, p, out, s);
}

}  // namespace hxq

extern "C" int hxq_cuda_affine_device_status(void)
{
    uint32_t v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) { cudaGetLastError(); return -1; }
    if (cudaMemcpyFromSymbol(&v, hxq::gemm::g_gemm_err, sizeof(v)) != cudaSuccess) { cudaGetLastError(); return -1; }
    if (v) {
        const uint32_t z = 0;
        cudaMemcpyToSymbol(hxq::gemm::g_gemm_err, &z, sizeof(z));
        hxq::gemm_reset_tail_counters();
    }
    const uint32_t tc = hxq::tc_gemv_status_take(), vq = hxq::vq_tc_status_take();
    if (tc == 0xFFFFFFFFu || vq == 0xFFFFFFFFu) return -1;
    return (int)(v | tc | vq);
}
