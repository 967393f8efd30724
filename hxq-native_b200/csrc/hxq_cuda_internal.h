// hxq_cuda_internal.h -- structures shared by the CUDA runtime layer and the
// sm_100a kernels of the HXQ decompress path.  Internal; not installed.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "hxq_cuda.h"

namespace hxq {

// A chunk is the unit of work of one warp: 2048 consecutive weights of one
// job.  12-bit indices: 512 byte triples = 1536 B.  Scalar: 2048 B.
constexpr uint32_t kChunkW        = 2048;
constexpr uint32_t kChunkBytes12  = 1536;
constexpr uint32_t kChunkBytes8   = 2048;
constexpr uint32_t kWarps         = 8;      // warps per CTA of the fast kernel
constexpr uint32_t kThreads       = kWarps * 32;
constexpr uint32_t kMaxJobs       = HXQ_CUDA_MAX_BATCH;
// Device index buffers are padded by this much past the last whole chunk so
// the unpack may read one word beyond a chunk without leaving the buffer.
constexpr uint32_t kIdxPad        = 16;

enum ImageKind : uint32_t {
    kKindScalar   = 0,   // uint8 indices, fast kernel
    kKindVq12     = 1,   // 12-bit, in_features % 4 == 0, fast kernel
    kKindVq12Any  = 2,   // 12-bit, any in_features, generic kernel
    kKindAffine   = 3,   // affine codes, generic kernel
    kKindRaw      = 4,   // corrections on an existing buffer (read-modify-write)
};

// Sidecar entry as stored on the device.  Entries are stably sorted by
// position, so equal coordinates are adjacent and keep array order.
//   fast kinds:    x = (offset in chunk) | (run length << 16); run length is
//                  0 on all but the first entry of a run of equal positions.
//   generic kinds: x = flat position in the image; y = value bits.
struct SideEntry { uint32_t x; uint32_t y; };

// Work of the fast kernel is handed out dynamically in units of
// cpw * kWarps chunks (chunk k*kWarps + w of a unit goes to warp w), cpw =
// chunks per warp of the launch: 2, or 1 when a launch has too few units to
// give every CTA several (single tensors); units never span two jobs.
constexpr uint32_t kChunksPerWarp = 2;
constexpr uint32_t kUnitChunks = kChunksPerWarp * kWarps;   // the largest unit
__host__ __device__ constexpr uint32_t unit_chunks(uint32_t cpw) { return cpw * kWarps; }

// One job of a launch of the fast kernel.
struct VqJob {
    const uint4     *idx;        // chunk-padded index bytes
    const float     *cb;         // fp32 codebook, k * vdim floats
    const uint32_t  *chunk_ptr;  // [n_chunks + 1] first entry of each chunk
    const SideEntry *ent;        // sidecar entries
    void            *out;        // fp32 or bf16 output, 16-B aligned
    uint64_t         numel;      // weights in the job
    uint32_t         n_chunks;
    uint32_t         k;          // codebook entries (index bound)
    uint32_t         unit_begin; // first global unit of the job (also its first slot)
    uint32_t         n_units;
    double          *sumsq;      // optional device output: exact sum of squares
    float           *conf;       // optional device output: receives ref_conf
    float            ref_conf;   // the reference's confidence for the job
    uint32_t         pad_;
};

struct VqLaunch {
    VqJob     job[kMaxJobs];
    uint32_t  n_jobs;
    uint32_t  grid;
    uint32_t  total_units;
    uint32_t  cpw;               // chunks per warp and unit (1 or 2)
    double   *slots;             // one partial sum per unit (scratch)
    uint32_t *counters;          // per job: units finished (scratch, zero)
    uint32_t *work;              // [0] next unit to hand out, [1] CTAs done (zero)
    uint32_t *err;               // device error word (scratch)
};

// Device scratch owned by the runtime, one per (device, stream).  The
// decompress kernels leave `counters` at zero when they finish.
struct Scratch {
    void     *base      = nullptr;   // the allocation holding all of the below
    double   *slots     = nullptr;
    uint32_t  n_slots   = 0;
    uint32_t *counters  = nullptr;   // kMaxJobs
    uint32_t *work      = nullptr;   // 2 words, zero between launches
    uint32_t *err       = nullptr;   // 1 word
    double   *sumsq     = nullptr;   // kMaxJobs results for internal calls
    float    *conf      = nullptr;   // kMaxJobs
};

// Resident CTAs per SM of the fast kernel: the scalar variant holds four
// 16-byte index pieces per lane in flight and needs more registers.
#ifndef HXQ_VQ12_CTAS_PER_SM
#define HXQ_VQ12_CTAS_PER_SM 3
#endif
__host__ __device__ constexpr uint32_t ctas_per_sm(uint32_t kind)
{
    return kind == kKindVq12 ? HXQ_VQ12_CTAS_PER_SM : 3u;
}

// Error bits written to the device error word.
constexpr uint32_t kErrIndexOOB = 1u;

// Launch helpers implemented in vq_kernels.cu.  All return cudaError_t of
// the launch.  `sms` is the device's SM count.
cudaError_t configure_vq_kernels();
cudaError_t launch_vq_fast(const VqLaunch &p, uint32_t kind, int bf16,
                           int check_k, cudaStream_t s);
// Kernels launch_vq_fast puts on the stream: 1, or 2 when a job requests the
// exact sum of squares (the ordered reduction runs as a second kernel).
uint32_t vq_fast_launches(const VqLaunch &p);
uint32_t    fast_grid(uint64_t total_chunks, int sms, uint32_t kind);
// Chunks per warp for a launch of `chunks` chunks in total: 2, or 1 when
// units of two would not give every resident CTA about four of them.
uint32_t    fast_cpw(uint64_t chunks, int sms, uint32_t kind);

// Generic kernels (any shape/alignment; one image per launch).
struct GenericJob {
    uint32_t          kind;       // kKindScalar / kKindVq12Any / kKindAffine / kKindVq12
    const uint8_t    *idx;        // raw index bytes of the image rows
    const float      *cb;
    const float      *scales;     // affine
    const float      *offsets;    // affine
    uint32_t          rows, in_f, k, gs;
    uint32_t          triples_per_row; // 12-bit
    const SideEntry  *ent;        // sidecar entries
    uint32_t          n_ent;
    // non-null when `ent` uses the chunk-relative encoding of fast images
    const uint32_t   *chunk_ptr;
    uint32_t          n_chunks;
    void             *out;
    int               bf16;
    double           *sumsq;
    float            *conf;
    // value stored into *conf: ref_conf, or sqrt of the kernel's exact sum
    // of squares when conf_exact is set
    float             ref_conf;
    int               conf_exact;
};
cudaError_t launch_generic(const GenericJob &j, const Scratch &sc,
                           cudaStream_t s);

// Output buffers of a matmul: the same [tokens, ldy] result stored into each
// (local or peer-mapped).
struct OutPtrs {
    float *y[HXQ_CUDA_MAX_PEERS];
    uint32_t n;
};

// Fused VQ-dequant matmul on 12-bit images with k = 4096 (vq_matmul.cu,
// dequant_gemm.cu).  x bf16 [ntok, in_f]; outputs fp32 [ntok, ldy].
struct VqGemvJob {
    const uint8_t *idx;
    const float *cb;
    const uint32_t *chunk_ptr;
    const SideEntry *ent;
    uint32_t n_chunks, rows, in_f;
    const uint16_t *x;
    OutPtrs out;
    uint32_t ldy;
};
cudaError_t launch_vq_gemv_batch(uint32_t n, const VqGemvJob *jobs, uint32_t ntok, int sms, cudaStream_t s);
cudaError_t launch_vq_gemv(const uint8_t *idx, const float *cb, const uint32_t *chunk_ptr, const SideEntry *ent,
                           uint32_t n_chunks, uint32_t rows, uint32_t in_f, const uint16_t *x, uint32_t ntok,
                           const OutPtrs &out, uint32_t ldy, int sms, cudaStream_t s);
// A batch's GEMMs on one stream, launched by this host thread between
// begin and end, overlap each unsplit GEMM's tail with the next one's start;
// a batch that launches any other kernel in between calls break after it.
void gemm_chain_begin(cudaStream_t s);
void gemm_chain_end();
void gemm_chain_break();
// Zero the tcgen05 GEMMs' last-wave counters of the current device (after a
// launch gave up; the device must be idle).
void gemm_reset_tail_counters();
struct GemmChainScope {
    explicit GemmChainScope(cudaStream_t s) { gemm_chain_begin(s); }
    ~GemmChainScope() { gemm_chain_end(); }
    GemmChainScope(const GemmChainScope &) = delete;
    GemmChainScope &operator=(const GemmChainScope &) = delete;
};
int vq_gemm_bf16(const uint16_t *x, const uint8_t *idx, const uint32_t *cbh, const uint32_t *rb,
                 const uint32_t *kq, const uint32_t *e4, const uint32_t *g4, const uint32_t *gp,
                 const uint16_t *tx, const OutPtrs &out, uint32_t T, uint32_t I, uint32_t O, uint32_t ldy,
                 cudaStream_t s);
bool affine_gemm_fits(const uint16_t *x, const uint8_t *codes, uint32_t T, uint32_t I, uint32_t O, uint32_t gs);
int affine_gemm_bf16(const uint16_t *x, const uint8_t *codes, const float *scales, const float *offsets,
                     const float *bias, const OutPtrs &out, uint32_t ldy, uint32_t T, uint32_t I, uint32_t O,
                     uint32_t gs, cudaStream_t s);

// One matrix of a tensor-core affine GEMV launch (affine_tc_gemv.cu).
constexpr uint32_t kMaxTcJobs = 8;
struct TcMatrix {
    const uint16_t *x;                    // bf16 activations [N][in_f]
    const uint8_t *codes;                 // [out_f][in_f]
    const float *scales, *offsets, *bias;
    OutPtrs out;
    uint32_t ldy, in_f, out_f, gs;
};
// Shape, alignment and shared-memory test for the tensor-core GEMV:
// 1 <= N <= 16, in_f and gs multiples of 64, 16-byte aligned operands.
bool tc_gemv_fits(const uint16_t *x, const uint8_t *codes, const float *scales, const float *offsets,
                  uint32_t N, uint32_t in_f, uint32_t out_f, uint32_t gs);
// Up to kMaxTcJobs matrices in one launch: 0 launched, 1 not taken, -1 error.
int launch_tc_gemv(uint32_t n, const TcMatrix *m, uint32_t N, int sms, cudaStream_t s);
// Reads and clears the kernel's status word (nonzero: a wait ran out).
uint32_t tc_gemv_status_take();

// One image of a tensor-core VQ GEMV launch (vq_tc_gemv.cu): the image's
// GEMV index stream [rows][in_f / 2] (per pair the byte offset of its entry
// in the two-copy shared codebook), the image's matmul tables (bf16x2
// codebook, first patch per row, patch columns, patch weight differences),
// bf16 activations [N][in_f].
struct VqTcMatrix {
    const uint16_t *tx;
    const uint32_t *cbh, *rb, *e4;
    const float *ed;
    uint32_t n_patch;
    const uint16_t *x;
    OutPtrs out;
    uint32_t ldy, rows, in_f;
};
// 1 <= N <= 16, in_f a multiple of 128 (at most 65536), x 16-byte aligned,
// and the activations fit in shared memory whole or in two K parts.
bool vq_tc_fits(const uint16_t *x, uint32_t N, uint32_t in_f);
// Jobs of one VQ GEMV launch (a matrix split along K: one per part).
constexpr uint32_t kMaxVqTcJobs = 8;
// How many of m[0..n) share one launch (at most kMaxVqTcJobs jobs, a matrix
// split along K counting one per part) without costing the first ones
// residency (CTAs per SM).
uint32_t vq_tc_group(uint32_t n, const VqTcMatrix *m, uint32_t N);
// Up to kMaxVqTcJobs jobs in one launch, plus one part-sum launch per matrix
// split along K: 0 launched (*launched: how many kernels), 1 not taken,
// -1 error.
int launch_vq_tc_gemv(uint32_t n, const VqTcMatrix *m, uint32_t N, int sms, cudaStream_t s,
                      uint32_t *launched = nullptr);
uint32_t vq_tc_status_take();

}  // namespace hxq
