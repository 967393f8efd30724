// hxq_cuda_rt.cu -- host runtime of the CUDA backend (C-ABI layer).
//
// Owns everything the kernels need that the reference API does not carry:
//   * a side table from hxq_tensor_t* to the tensor's device image (the
//     struct layout is frozen by the reference ABI, so device state cannot
//     live in it);
//   * the registry of device arenas (hxq_shared_buffer_t with HBM data);
//   * per (device, stream) scratch for the kernels' reductions and errors;
//   * image construction: index bytes padded to whole chunks, codebook,
//     sidecar entries filtered to the reference's in-range rule, stably
//     sorted by position and indexed per chunk;
//   * launch planning for batched decompress.
// Every CUDA error is mapped to an hxq status; nothing falls back to the CPU.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <numeric>
#include <thread>
#include <unordered_map>
#include <vector>

#include <cuda.h>
#include <cuda_runtime.h>

#include "hxq_cuda_internal.h"
#include "hxq_internal.h"

using namespace hxq;

struct hxq_cuda_image {
    int       device = -1;
    uint32_t  kind = 0;
    uint32_t  rows = 0, in_f = 0, k = 0, vdim = 0, gs = 0;
    uint32_t  triples_per_row = 0;
    uint64_t  numel = 0;
    bool      check_k = false;
    // one block holding every array below, laid out at the offsets o_*;
    // resident images own d_block, streamed images keep h_block (pinned)
    // and point d_block at wherever hxq_cuda_image_upload copied it
    void     *d_block = nullptr;
    void     *h_block = nullptr;
    bool      owns_device = false;
    size_t    block_bytes = 0;
    size_t    o_idx = 0, o_cb = 0, o_sc = 0, o_of = 0, o_cp = 0, o_en = 0;
    bool      has_cb = false, has_aff = false, has_cp = false;
    uint8_t  *d_idx = nullptr;
    float    *d_cb = nullptr;
    float    *d_scales = nullptr, *d_offsets = nullptr;
    uint32_t *d_chunk_ptr = nullptr;
    SideEntry *d_ent = nullptr;
    uint32_t  n_chunks = 0;
    uint32_t  n_ent = 0;
    double    sumsq = 0.0;     // exact sum of squared in-range deltas
    float     ref_l2 = 0.0f;   // sqrtf of the fp32 running sum in array order
    float     ref_l2_tensor = 0.0f;  // the same over every row of the tensor
    // fused-matmul extras (12-bit, k = 4096, in_features % 128 == 0): bf16
    // codebook pairs; per row the first patch; per (row, 64-wide half K
    // step) the 16-bit offset of its first patch from the row's | its patch
    // count << 16; patches
    // col | bf16(final weight) << 16, one per distinct sidecar position
    // and per patch bf16(final weight) - bf16(codebook value) in fp32
    bool      has_mm = false;
    // and the tensor-core GEMV's own index stream (build_tc_stream)
    // and the same patches grouped per 32 rows and 64-wide half step for
    // the tcgen05 GEMM's 256-token tiles (build_patches)
    size_t    o_cbh = 0, o_rb = 0, o_kq = 0, o_e4 = 0, o_ed = 0, o_tx = 0, o_g4 = 0, o_gp = 0;
    uint32_t *d_cbh = nullptr, *d_rb = nullptr, *d_kq = nullptr, *d_e4 = nullptr, *d_g4 = nullptr, *d_gp = nullptr;
    uint16_t *d_tx = nullptr;
    float    *d_ed = nullptr;
    uint32_t  n_patch = 0;
};

namespace {

std::mutex g_mu;
std::atomic<unsigned long long> g_launches{0};

struct Snapshot {
    const float *codebook; uint32_t k, vdim;
    const uint8_t *idx; size_t idx_len;
    const uint32_t *sr, *sc; const float *sv; uint32_t nnz;
    uint32_t out_f, in_f; int mode;
    const float *as, *ao; uint32_t gs;
    int device;
    bool operator==(const Snapshot &o) const { return std::memcmp(this, &o, sizeof(*this)) == 0; }
};

Snapshot snap(const hxq_tensor_t *t, int device)
{
    Snapshot s;
    std::memset(&s, 0, sizeof(s));
    s.codebook = t->codebook; s.k = t->k; s.vdim = t->vector_dim;
    s.idx = t->indices_raw; s.idx_len = t->indices_len;
    s.sr = t->sidecar_rows; s.sc = t->sidecar_cols; s.sv = t->sidecar_vals; s.nnz = t->sidecar_nnz;
    s.out_f = t->out_features; s.in_f = t->in_features; s.mode = (int)t->mode;
    s.as = t->affine_scales; s.ao = t->affine_offsets; s.gs = t->affine_group_size;
    s.device = device;
    return s;
}

struct Cached { Snapshot snap; hxq_cuda_image *img; };
std::unordered_map<const hxq_tensor_t *, Cached> g_images;
std::unordered_map<const hxq_shared_buffer_t *, int> g_arenas;   // buf -> device

struct DevCtx {
    bool      ready = false;
    int       sms = 0;
    std::map<cudaStream_t, Scratch> scratch;
    void     *readback = nullptr;     // pinned host, 4 KB
    float    *stage = nullptr;        // internal device buffer for host-buffer dequant
    size_t    stage_floats = 0;
};
constexpr int kMaxDev = 64;
DevCtx g_dev[kMaxDev];
int g_cuda_present = -1;

hxq_error_t map_cuda(cudaError_t e)
{
    if (e == cudaSuccess) return HXQ_OK;
    if (e == cudaErrorMemoryAllocation) return HXQ_ERR_ALLOC_FAILED;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return HXQ_ERR_BACKEND_UNAVAILABLE;
    return HXQ_ERR_CUDA;
}

bool cuda_present()
{
    if (g_cuda_present < 0) {
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e != cudaSuccess) cudaGetLastError();
        g_cuda_present = (e == cudaSuccess && n > 0) ? 1 : 0;
    }
    return g_cuda_present == 1;
}

// Driver entry point, resolved without linking libcuda.
typedef CUresult (*PrimaryCtxGetStateFn)(CUdevice, unsigned int *, int *);
PrimaryCtxGetStateFn primary_state_fn()
{
    static PrimaryCtxGetStateFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuDevicePrimaryCtxGetState", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PrimaryCtxGetStateFn>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

// True when some device already has an active primary context, i.e. device
// memory may exist in this process.  Never creates a context itself.
bool any_context_active()
{
    PrimaryCtxGetStateFn fn = primary_state_fn();
    if (!fn) return true;  // cannot tell: let the pointer query decide
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return false; }
    for (int d = 0; d < n; ++d) {
        unsigned int flags = 0; int active = 0;
        if (fn((CUdevice)d, &flags, &active) == CUDA_SUCCESS && active) return true;
    }
    return false;
}

hxq_error_t current_device(int *dev)
{
    if (!cuda_present()) return HXQ_ERR_BACKEND_UNAVAILABLE;
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess || *dev < 0 || *dev >= kMaxDev) { cudaGetLastError(); return HXQ_ERR_CUDA; }
    return HXQ_OK;
}

// Per-device setup; caller holds g_mu.
hxq_error_t dev_ready(int dev)
{
    DevCtx &d = g_dev[dev];
    if (d.ready) return HXQ_OK;
    int sms = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = configure_vq_kernels();
    if (e == cudaSuccess) e = cudaMallocHost(&d.readback, 4096);
    if (e != cudaSuccess) { cudaGetLastError(); return map_cuda(e); }
    d.sms = sms;
    d.ready = true;
    return HXQ_OK;
}

// Scratch layout: [err u32 x 4][conf f32 x kMaxJobs][sumsq f64 x kMaxJobs]
// [counters u32 x kMaxJobs][work u32 x 4][slots f64 x n_slots].  Zeroed at
// allocation; kernels leave counters and work at zero.  A stream's scratch
// grows (reallocated, zeroed) when a launch needs more slots than it has,
// which the first, uncaptured call of a workload on that stream does.
// Caller holds g_mu.
hxq_error_t get_scratch(int dev, cudaStream_t s, Scratch **out, uint32_t min_slots = 0)
{
    DevCtx &d = g_dev[dev];
    const uint32_t floor_slots = (uint32_t)(kMaxJobs + 8u * (uint32_t)std::max(d.sms, 148) + 1024u);
    auto it = d.scratch.find(s);
    if (it != d.scratch.end() && it->second.n_slots >= min_slots) { *out = &it->second; return HXQ_OK; }
    const uint32_t n_slots = std::max(floor_slots, min_slots + min_slots / 4u);
    const size_t head = 16 + kMaxJobs * 4 + kMaxJobs * 8 + kMaxJobs * 4 + 16;
    const size_t bytes = head + (size_t)n_slots * 8;
    unsigned char *base = nullptr;
    cudaError_t e = cudaMalloc(&base, bytes);
    if (e == cudaSuccess) e = cudaMemset(base, 0, bytes);
    if (e != cudaSuccess) { cudaGetLastError(); if (base) cudaFree(base); return map_cuda(e); }
    if (it != d.scratch.end()) {  // replace a smaller one once its work is done
        cudaStreamSynchronize(s);
        cudaFree(it->second.base);
        d.scratch.erase(it);
    }
    Scratch sc;
    sc.base = base;
    sc.err = reinterpret_cast<uint32_t *>(base);
    sc.conf = reinterpret_cast<float *>(base + 16);
    sc.sumsq = reinterpret_cast<double *>(base + 16 + kMaxJobs * 4);
    sc.counters = reinterpret_cast<uint32_t *>(base + 16 + kMaxJobs * 12);
    sc.work = reinterpret_cast<uint32_t *>(base + 16 + kMaxJobs * 16);
    sc.slots = reinterpret_cast<double *>(base + head);
    sc.n_slots = n_slots;
    auto res = d.scratch.emplace(s, sc);
    *out = &res.first->second;
    return HXQ_OK;
}

size_t align256(size_t x) { return (x + 255u) & ~(size_t)255u; }

// ---------------------------------------------------------------------------
// Image construction

struct HostEntry { uint64_t pos; float val; };

// Sidecar entries of rows [r0, r1) that the reference would apply (r < out_f
// and c < in_f, src/hxq.c:343), in array order, positions relative to r0.
// Also returns, in *seq, the confidence exactly as the reference computes
// it: a float running sum of v*v in array order (src/hxq.c:335-349).  That
// order is inherently sequential, and over 1e5 terms its rounding drifts a
// few 1e-5 from the true value, beyond reach of any parallel reduction; it
// depends only on the loaded sidecar, so it is computed here once.
// *seq_tensor is the same value over every row of the tensor, which a row
// slice carries so that a matrix split over GPUs can still report it.
void collect_sidecar(const hxq_tensor_t *t, uint32_t r0, uint32_t r1,
                     std::vector<HostEntry> &ents, double &sumsq, float *seq,
                     float *seq_tensor)
{
    sumsq = 0.0;
    volatile float run = 0.0f;   // one rounded product, one rounded add per term
    volatile float run_all = 0.0f;
    *seq = 0.0f;
    *seq_tensor = 0.0f;
    ents.clear();
    if (t->sidecar_nnz == 0 || !t->sidecar_rows || !t->sidecar_cols || !t->sidecar_vals) return;
    const uint32_t in_f = t->in_features, out_f = t->out_features;
    for (uint32_t i = 0; i < t->sidecar_nnz; ++i) {
        const uint32_t r = t->sidecar_rows[i], c = t->sidecar_cols[i];
        if (r >= out_f || c >= in_f) continue;
        const float v = t->sidecar_vals[i];
        volatile float sq = v * v;
        run_all = run_all + sq;
        if (r < r0 || r >= r1) continue;
        ents.push_back({(uint64_t)(r - r0) * in_f + c, v});
        sumsq += (double)v * (double)v;
        run = run + sq;
    }
    *seq = sqrtf(run);
    *seq_tensor = sqrtf(run_all);
    bool sorted = true;
    for (size_t i = 1; i < ents.size() && sorted; ++i) sorted = ents[i - 1].pos <= ents[i].pos;
    if (!sorted)
        std::stable_sort(ents.begin(), ents.end(),
                         [](const HostEntry &a, const HostEntry &b) { return a.pos < b.pos; });
}

// Error the reference decoder reports for a 12-bit stream that is too
// short: INDEX_OOB if an index before the shortfall is >= k, else
// PACK_FORMAT (src/hxq.c:262,271 -- length is checked before the indices
// of each triple).
hxq_error_t short_stream_error(const hxq_tensor_t *t, size_t start, size_t avail_bytes)
{
    const size_t n_trip = avail_bytes / 3u;
    for (size_t i = 0; i < n_trip; ++i) {
        uint16_t a, b;
        hxq_unpack_12bit_pair(t->indices_raw + start + 3u * i, &a, &b);
        if (a >= t->k || b >= t->k) return HXQ_ERR_INDEX_OOB;
    }
    return HXQ_ERR_PACK_FORMAT;
}

// Point the image's device arrays into a block at `base` (layout o_*).
void bind_image(hxq_cuda_image *img, void *base)
{
    unsigned char *b = static_cast<unsigned char *>(base);
    img->d_block = base;
    img->d_idx = b + img->o_idx;
    img->d_cb = img->has_cb ? reinterpret_cast<float *>(b + img->o_cb) : nullptr;
    img->d_scales = img->has_aff ? reinterpret_cast<float *>(b + img->o_sc) : nullptr;
    img->d_offsets = img->has_aff ? reinterpret_cast<float *>(b + img->o_of) : nullptr;
    img->d_chunk_ptr = img->has_cp ? reinterpret_cast<uint32_t *>(b + img->o_cp) : nullptr;
    img->d_ent = reinterpret_cast<SideEntry *>(b + img->o_en);
    if (img->has_mm) {
        img->d_cbh = reinterpret_cast<uint32_t *>(b + img->o_cbh);
        img->d_rb = reinterpret_cast<uint32_t *>(b + img->o_rb);
        img->d_kq = reinterpret_cast<uint32_t *>(b + img->o_kq);
        img->d_e4 = reinterpret_cast<uint32_t *>(b + img->o_e4);
        img->d_ed = reinterpret_cast<float *>(b + img->o_ed);
        img->d_tx = reinterpret_cast<uint16_t *>(b + img->o_tx);
        img->d_g4 = reinterpret_cast<uint32_t *>(b + img->o_g4);
        img->d_gp = reinterpret_cast<uint32_t *>(b + img->o_gp);
    }
}

uint16_t bf16_rne(float f)
{
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// Fused-matmul patch tables of a 12-bit image (see hxq_cuda_image).  Each
// distinct sidecar position gets the weight the reference decoder produces
// there -- codebook value, then the deltas added in array order in fp32
// (src/hxq.c:343-346) -- rounded once to bf16.  False if a row has more
// than 65535 patches (16-bit offsets); the image then has no tables.
float bf16_to_float(uint32_t h)
{
    const uint32_t u = (h & 0xFFFFu) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// The fused matmuls' patch tables (see hxq_cuda_image): per distinct
// sidecar position of rows [0, rows) col | bf16(final weight) << 16 (e4, rows
// in order) and bf16(final) - bf16(codebook value) (ed); per row its first
// entry (rb); per (row, 64-wide half K step) the offset of the half step's
// first entry from the row's | its entry count << 16 (kq); and the same
// entries grouped per 32 rows and
// 64-wide half step for the tcgen05 GEMM's 256-token tiles (a converter
// warp's rows and half of a K step): group g = (row / 32) * (in_f / 64) +
// col / 64 holds g4[gp[g] .. gp[g + 1]), each (row % 32) << 22 | (col % 64)
// << 16 | bf16(final).
bool build_patches(const hxq_tensor_t *t, const uint8_t *idx_rows, uint32_t rows, uint32_t in_f,
                   const std::vector<HostEntry> &ents, std::vector<uint32_t> &cbh,
                   std::vector<uint32_t> &rb, std::vector<uint32_t> &kq, std::vector<uint32_t> &e4,
                   std::vector<float> &ed, std::vector<uint32_t> &g4, std::vector<uint32_t> &gp)
{
    const uint32_t KT = in_f / 128u;
    const size_t row_bytes = (size_t)(in_f / 4u) * 3u;
    cbh.resize(4096);
    for (uint32_t j = 0; j < 4096u; ++j)
        cbh[j] = (uint32_t)bf16_rne(t->codebook[2u * j]) | ((uint32_t)bf16_rne(t->codebook[2u * j + 1u]) << 16);
    std::vector<uint32_t> erow;
    e4.clear();
    ed.clear();
    for (size_t i = 0; i < ents.size();) {
        const uint64_t pos = ents[i].pos;
        const uint32_t r = (uint32_t)(pos / in_f), c = (uint32_t)(pos % in_f);
        const uint8_t *b = idx_rows + (size_t)r * row_bytes + (size_t)(c / 4u) * 3u;
        const uint32_t id = ((c / 2u) & 1u) ? (((uint32_t)(b[1] & 15u) << 8) | b[2])
                                            : (((uint32_t)b[0] << 4) | (b[1] >> 4));
        volatile float w = t->codebook[2u * id + (c & 1u)];
        for (; i < ents.size() && ents[i].pos == pos; ++i) w = w + ents[i].val;
        const uint16_t fw = bf16_rne(w);
        e4.push_back(c | ((uint32_t)fw << 16));
        ed.push_back(bf16_to_float(fw) - bf16_to_float(cbh[id] >> (16u * (c & 1u))));
        erow.push_back(r);
    }
    rb.assign(rows, 0u);
    kq.assign((size_t)rows * 2u * KT, 0u);
    size_t e = 0;
    for (uint32_t r = 0; r < rows; ++r) {
        while (e < e4.size() && erow[e] < r) ++e;
        rb[r] = (uint32_t)e;
        size_t f = e;
        for (uint32_t hs = 0; hs < 2u * KT; ++hs) {
            const size_t f0 = f;
            while (f < e4.size() && erow[f] == r && (e4[f] & 0xFFFFu) < (hs + 1u) * 64u) ++f;
            if (f0 - e > 0xFFFFu) return false;
            kq[(size_t)r * 2u * KT + hs] = (uint32_t)(f0 - e) | ((uint32_t)(f - f0) << 16);
        }
    }
    const uint32_t NH = in_f / 64u;
    const size_t n_groups = (size_t)((rows + 31u) / 32u) * NH;
    gp.assign(n_groups + 1u, 0u);
    for (size_t i = 0; i < e4.size(); ++i) ++gp[(size_t)(erow[i] / 32u) * NH + (e4[i] & 0xFFFFu) / 64u + 1u];
    for (size_t g = 0; g < n_groups; ++g) gp[g + 1u] += gp[g];
    g4.assign(e4.size(), 0u);
    std::vector<uint32_t> fill(gp.begin(), gp.end() - 1);
    for (size_t i = 0; i < e4.size(); ++i) {
        const uint32_t c = e4[i] & 0xFFFFu;
        g4[fill[(size_t)(erow[i] / 32u) * NH + c / 64u]++] = ((erow[i] & 31u) << 22) | ((c & 63u) << 16) | (e4[i] >> 16);
    }
    return true;
}

// Index stream of the tensor-core GEMV (vq_tc_gemv.cu).  Its shared
// codebook holds the 4096 bf16 pairs twice: copy 0 has entry c at word c
// (bank c & 31), copy 1 at word 4096 + (c ^ ((c >> 5) & 31)), whose bank
// is independent of c's.  Every pair of the matrix is stored as the 16-bit
// byte offset of the copy its lane reads: 4c, or 16384 + 4 * perm(c).  A
// gather instruction of the GEMV is one of a lane's sixteen per 64-weight
// chunk, and the lanes that make it up are known from the kernel's layout
// (lane (g, t) of warp w, chunk u, word jj, half h, row set s reads pair
// 512 st + 64 w + 16 t + 8 u + 2 jj + h of row 16 rb + g + 8 s); per
// instruction the copies are chosen here so that the fullest bank holds as
// few distinct words as possible (the instruction's shared-memory
// wavefronts): about 2 for 32 random entries, against 3.5 with one copy.
uint32_t tc_perm(uint32_t c) { return c ^ ((c >> 5) & 31u); }

uint32_t idx12_at(const uint8_t *row, uint32_t pair)
{
    const uint8_t *b = row + (size_t)(pair >> 1) * 3u;
    return (pair & 1u) ? (((uint32_t)(b[1] & 15u) << 8) | b[2]) : (((uint32_t)b[0] << 4) | (b[1] >> 4));
}

// Copies for the 32 lanes of one gather instruction (c[l] entry of lane l;
// live[l] false for a lane past the matrix, which reads word 0 of copy 0).
void choose_copies(const uint32_t (&c)[32], const bool (&live)[32], uint8_t (&copy)[32])
{
    uint16_t words[32][32];   // distinct words per bank
    uint8_t refs[32][32] = {};   // lanes per (bank, word)
    uint8_t load[32] = {0};
    auto find = [&](uint32_t b, uint16_t w) -> int {
        for (uint32_t i = 0; i < load[b]; ++i)
            if (words[b][i] == w) return (int)i;
        return -1;
    };
    auto add = [&](uint32_t b, uint16_t w) {
        const int i = find(b, w);
        if (i >= 0) { ++refs[b][i]; return; }
        words[b][load[b]] = w;
        refs[b][load[b]] = 1;
        ++load[b];
    };
    auto remove = [&](uint32_t b, uint16_t w) {
        const int i = find(b, w);
        if (--refs[b][i] == 0) {
            --load[b];
            words[b][i] = words[b][load[b]];
            refs[b][i] = refs[b][load[b]];
        }
    };
    auto opt = [&](uint32_t l, uint32_t k, uint32_t &b, uint16_t &w) {
        if (k == 0) { w = (uint16_t)c[l]; b = c[l] & 31u; }
        else { const uint32_t q = tc_perm(c[l]); w = (uint16_t)(4096u + q); b = q & 31u; }
    };
    auto cost = [&](uint32_t b, uint16_t w) { return find(b, w) >= 0 ? load[b] : load[b] + 1u; };
    for (uint32_t l = 0; l < 32; ++l) {
        copy[l] = 0;
        if (!live[l]) { add(0, 0); continue; }
        uint32_t b0, b1;
        uint16_t w0, w1;
        opt(l, 0, b0, w0);
        opt(l, 1, b1, w1);
        copy[l] = cost(b1, w1) < cost(b0, w0) ? 1 : 0;
        if (copy[l]) add(b1, w1); else add(b0, w0);
    }
    // move lanes out of the fullest banks while that lowers them
    for (int pass = 0; pass < 4; ++pass) {
        uint32_t L = 0;
        for (uint32_t b = 0; b < 32; ++b) L = load[b] > L ? load[b] : L;
        bool moved = false;
        for (uint32_t l = 0; l < 32; ++l) {
            if (!live[l]) continue;
            uint32_t bc, ba;
            uint16_t wc, wa;
            opt(l, copy[l], bc, wc);
            opt(l, copy[l] ^ 1u, ba, wa);
            if (load[bc] != L || refs[bc][find(bc, wc)] != 1) continue;
            if (cost(ba, wa) < L) {
                remove(bc, wc);
                add(ba, wa);
                copy[l] ^= 1u;
                moved = true;
            }
        }
        if (!moved) break;
    }
}

// The stream for rows [0, rows) of a 12-bit image (in_f % 128 == 0): one
// uint16 per pair, rows of in_f / 2 pairs.
void build_tc_stream(const uint8_t *idx_rows, uint32_t rows, uint32_t in_f, std::vector<uint16_t> &tx)
{
    const uint32_t pairs = in_f / 2u, n_rb = (rows + 15u) / 16u, n_st = (in_f + 1023u) / 1024u;
    const size_t row_bytes = (size_t)(in_f / 4u) * 3u;
    tx.assign((size_t)rows * pairs, 0u);
    auto work = [&](uint32_t rb_lo, uint32_t rb_hi) {
        uint32_t c[32];
        bool live[32];
        uint8_t copy[32];
        for (uint32_t rb = rb_lo; rb < rb_hi; ++rb)
            for (uint32_t st = 0; st < n_st; ++st)
                for (uint32_t w = 0; w < 8u; ++w) {
                    const uint32_t p0 = st * 512u + w * 64u;
                    if (p0 >= pairs) continue;   // the warp's window is past the row (kernel skips it)
                    for (uint32_t u = 0; u < 2u; ++u)
                        for (uint32_t jj = 0; jj < 4u; ++jj)
                            for (uint32_t h = 0; h < 2u; ++h)
                                for (uint32_t s = 0; s < 2u; ++s) {
                                    for (uint32_t l = 0; l < 32u; ++l) {
                                        const uint32_t g = l >> 2, t = l & 3u;
                                        const uint32_t row = rb * 16u + g + 8u * s;
                                        const uint32_t pr = p0 + 16u * t + 8u * u + 2u * jj + h;
                                        live[l] = row < rows;
                                        c[l] = live[l] ? idx12_at(idx_rows + (size_t)row * row_bytes, pr) : 0u;
                                    }
                                    choose_copies(c, live, copy);
                                    for (uint32_t l = 0; l < 32u; ++l) {
                                        if (!live[l]) continue;
                                        const uint32_t g = l >> 2, t = l & 3u;
                                        const uint32_t row = rb * 16u + g + 8u * s;
                                        const uint32_t pr = p0 + 16u * t + 8u * u + 2u * jj + h;
                                        tx[(size_t)row * pairs + pr] =
                                            (uint16_t)(copy[l] ? 16384u + 4u * tc_perm(c[l]) : 4u * c[l]);
                                    }
                                }
                }
    };
    unsigned nt = std::thread::hardware_concurrency();
    nt = nt == 0 ? 1u : std::min(nt, 16u);
    if ((uint64_t)rows * in_f < (1u << 22) || nt == 1) { work(0, n_rb); return; }
    std::vector<std::thread> th;
    for (unsigned i = 0; i < nt; ++i)
        th.emplace_back(work, (uint32_t)((uint64_t)n_rb * i / nt), (uint32_t)((uint64_t)n_rb * (i + 1) / nt));
    for (auto &x : th) x.join();
}

hxq_error_t build_image(const hxq_tensor_t *t, uint32_t r0, uint32_t r1, int dev,
                        bool streamed, bool matmul, hxq_cuda_image **out)
{
    if (!t || !out) return HXQ_ERR_NULL_PTR;
    if (!t->indices_raw) return HXQ_ERR_NULL_PTR;
    if (t->mode != HXQ_AFFINE_G128 && !t->codebook) return HXQ_ERR_NULL_PTR;
    if (r0 > r1 || r1 > t->out_features) return HXQ_ERR_INVALID_ARG;

    hxq_cuda_image *img = new (std::nothrow) hxq_cuda_image();
    if (!img) return HXQ_ERR_ALLOC_FAILED;
    img->device = dev;
    img->rows = r1 - r0;
    img->in_f = t->in_features;
    img->k = t->k;
    img->vdim = t->vector_dim;
    img->numel = (uint64_t)img->rows * img->in_f;

    size_t idx_off = 0, idx_len = 0;   // byte range of the rows in indices_raw
    switch (t->mode) {
    case HXQ_SCALAR_VQ: {
        img->kind = kKindScalar;
        idx_off = (size_t)r0 * img->in_f;
        idx_len = (size_t)img->numel;
        if (idx_off + idx_len > t->indices_len) { delete img; return HXQ_ERR_PACK_FORMAT; }
        break;
    }
    case HXQ_VQ2D_12BIT: {
        // The reference reads cb[2*idx+1] whatever vector_dim is; with
        // vector_dim 1 that leaves the codebook, so it is refused here.
        if (t->vector_dim != 2) { delete img; return HXQ_ERR_INVALID_DIM; }
        const uint32_t ppr = img->in_f / 2u;
        img->triples_per_row = (ppr + 1u) / 2u;
        idx_off = (size_t)r0 * img->triples_per_row * 3u;
        idx_len = (size_t)img->rows * img->triples_per_row * 3u;
        if (idx_off + idx_len > t->indices_len) {
            const size_t avail = t->indices_len > idx_off ? t->indices_len - idx_off : 0;
            hxq_error_t e = short_stream_error(t, idx_off, avail);
            delete img;
            return e;
        }
        img->kind = (img->in_f % 4u == 0u) ? kKindVq12 : kKindVq12Any;
        img->check_k = t->k < 4096u;
        break;
    }
    case HXQ_AFFINE_G128: {
        if (!t->affine_scales || !t->affine_offsets || t->affine_group_size == 0 ||
            img->in_f % t->affine_group_size != 0) { delete img; return HXQ_ERR_NULL_PTR; }
        img->kind = kKindAffine;
        img->gs = t->affine_group_size;
        idx_off = (size_t)r0 * img->in_f;
        idx_len = (size_t)img->numel;
        if (idx_off + idx_len > t->indices_len) { delete img; return HXQ_ERR_PACK_FORMAT; }
        break;
    }
    default:
        delete img;
        return HXQ_ERR_INVALID_DIM;
    }

    std::vector<HostEntry> ents;
    collect_sidecar(t, r0, r1, ents, img->sumsq, &img->ref_l2, &img->ref_l2_tensor);
    const bool fast = img->kind == kKindScalar || img->kind == kKindVq12;
    if (!fast && img->numel > 0xFFFFFFFFull) { delete img; return HXQ_ERR_INVALID_ARG; }

    // device-side sidecar encoding
    std::vector<SideEntry> dev_ents(ents.size());
    std::vector<uint32_t> chunk_ptr;
    if (fast) {
        img->n_chunks = (uint32_t)((img->numel + kChunkW - 1) / kChunkW);
        chunk_ptr.assign((size_t)img->n_chunks + 1u, 0u);
        size_t i = 0;
        while (i < ents.size()) {
            size_t jx = i;
            while (jx < ents.size() && ents[jx].pos == ents[i].pos) ++jx;
            const size_t run = jx - i;
            if (run > 0xFFFFu) { delete img; return HXQ_ERR_INVALID_ARG; }
            const uint32_t off = (uint32_t)(ents[i].pos % kChunkW);
            for (size_t m = i; m < jx; ++m) {
                uint32_t bits;
                std::memcpy(&bits, &ents[m].val, 4);
                dev_ents[m].x = off | (m == i ? (uint32_t)run << 16 : 0u);
                dev_ents[m].y = bits;
            }
            i = jx;
        }
        // chunk_ptr[c] = first entry whose chunk >= c
        size_t e = 0;
        for (uint32_t c = 0; c <= img->n_chunks; ++c) {
            while (e < ents.size() && ents[e].pos / kChunkW < c) ++e;
            chunk_ptr[c] = (uint32_t)e;
        }
    } else {
        for (size_t m = 0; m < ents.size(); ++m) {
            uint32_t bits;
            std::memcpy(&bits, &ents[m].val, 4);
            dev_ents[m].x = (uint32_t)ents[m].pos;
            dev_ents[m].y = bits;
        }
    }
    img->n_ent = (uint32_t)dev_ents.size();

    std::vector<uint32_t> mm_cbh, mm_rb, mm_kq, mm_e4, mm_g4, mm_gp;
    std::vector<uint16_t> mm_tx;
    std::vector<float> mm_ed;
    if (matmul && img->kind == kKindVq12 && !img->check_k && img->k == 4096u && img->in_f % 128u == 0u &&
        img->in_f <= 65536u)
        img->has_mm = build_patches(t, t->indices_raw + idx_off, img->rows, img->in_f, ents, mm_cbh, mm_rb,
                                    mm_kq, mm_e4, mm_ed, mm_g4, mm_gp);
    if (img->has_mm) build_tc_stream(t->indices_raw + idx_off, img->rows, img->in_f, mm_tx);
    img->n_patch = (uint32_t)mm_e4.size();

    // one block: idx | cb | scales | offsets | chunk_ptr | entries
    const size_t chunk_bytes = img->kind == kKindVq12 ? kChunkBytes12 : kChunkBytes8;
    const size_t idx_alloc = fast ? (size_t)img->n_chunks * chunk_bytes + kIdxPad
                                  : std::max<size_t>(idx_len, 16);
    const size_t cb_floats = img->kind == kKindAffine ? 0 : (size_t)t->k * t->vector_dim;
    const size_t ng = img->gs ? img->in_f / img->gs : 0;
    const size_t aff_floats = img->kind == kKindAffine ? (size_t)img->rows * ng : 0;
    size_t off = 0;
    img->o_idx = off;  off = align256(off + idx_alloc);
    img->o_cb = off;   off = align256(off + cb_floats * 4);
    img->o_sc = off;   off = align256(off + aff_floats * 4);
    img->o_of = off;   off = align256(off + aff_floats * 4);
    img->o_cp = off;   off = align256(off + chunk_ptr.size() * 4);
    img->o_en = off;   off = align256(off + std::max<size_t>(dev_ents.size(), 1) * sizeof(SideEntry));
    if (img->has_mm) {
        img->o_cbh = off;  off = align256(off + mm_cbh.size() * 4);
        img->o_rb = off;   off = align256(off + std::max<size_t>(mm_rb.size(), 1) * 4);
        img->o_kq = off;   off = align256(off + std::max<size_t>(mm_kq.size(), 1) * 4);
        img->o_e4 = off;   off = align256(off + (mm_e4.size() + 4) * 4);   // + speculative-read slack
        img->o_ed = off;   off = align256(off + std::max<size_t>(mm_ed.size(), 1) * 4);
        img->o_tx = off;   off = align256(off + std::max<size_t>(mm_tx.size(), 8) * 2);
        img->o_g4 = off;   off = align256(off + std::max<size_t>(mm_g4.size(), 1) * 4);
        img->o_gp = off;   off = align256(off + mm_gp.size() * 4);
    }
    img->block_bytes = off;
    img->has_cb = cb_floats > 0;
    img->has_aff = aff_floats > 0;
    img->has_cp = !chunk_ptr.empty();

    unsigned char *hb = nullptr;
    cudaError_t ce;
    if (streamed) {
        ce = cudaHostAlloc(reinterpret_cast<void **>(&hb), img->block_bytes, cudaHostAllocDefault);
        if (ce != cudaSuccess) { cudaGetLastError(); delete img; return map_cuda(ce); }
    } else {
        hb = static_cast<unsigned char *>(std::malloc(img->block_bytes));
        if (!hb) { delete img; return HXQ_ERR_ALLOC_FAILED; }
    }
    std::memset(hb, 0, img->block_bytes);
    if (idx_len) std::memcpy(hb + img->o_idx, t->indices_raw + idx_off, idx_len);
    if (cb_floats) std::memcpy(hb + img->o_cb, t->codebook, cb_floats * 4);
    if (aff_floats) {
        std::memcpy(hb + img->o_sc, t->affine_scales + (size_t)r0 * ng, aff_floats * 4);
        std::memcpy(hb + img->o_of, t->affine_offsets + (size_t)r0 * ng, aff_floats * 4);
    }
    if (!chunk_ptr.empty()) std::memcpy(hb + img->o_cp, chunk_ptr.data(), chunk_ptr.size() * 4);
    if (!dev_ents.empty()) std::memcpy(hb + img->o_en, dev_ents.data(), dev_ents.size() * sizeof(SideEntry));
    if (img->has_mm) {
        std::memcpy(hb + img->o_cbh, mm_cbh.data(), mm_cbh.size() * 4);
        if (!mm_rb.empty()) std::memcpy(hb + img->o_rb, mm_rb.data(), mm_rb.size() * 4);
        if (!mm_kq.empty()) std::memcpy(hb + img->o_kq, mm_kq.data(), mm_kq.size() * 4);
        if (!mm_e4.empty()) std::memcpy(hb + img->o_e4, mm_e4.data(), mm_e4.size() * 4);
        if (!mm_ed.empty()) std::memcpy(hb + img->o_ed, mm_ed.data(), mm_ed.size() * 4);
        if (!mm_tx.empty()) std::memcpy(hb + img->o_tx, mm_tx.data(), mm_tx.size() * 2);
        if (!mm_g4.empty()) std::memcpy(hb + img->o_g4, mm_g4.data(), mm_g4.size() * 4);
        std::memcpy(hb + img->o_gp, mm_gp.data(), mm_gp.size() * 4);
    }

    if (streamed) {
        img->h_block = hb;
    } else {
        unsigned char *blk = nullptr;
        ce = cudaMalloc(&blk, img->block_bytes);
        if (ce == cudaSuccess) ce = cudaMemcpy(blk, hb, img->block_bytes, cudaMemcpyHostToDevice);
        std::free(hb);
        if (ce != cudaSuccess) {
            cudaGetLastError();
            if (blk) cudaFree(blk);
            delete img;
            return map_cuda(ce);
        }
        img->owns_device = true;
        bind_image(img, blk);
    }
    *out = img;
    return HXQ_OK;
}

void destroy_image(hxq_cuda_image *img)
{
    if (!img) return;
    if (img->h_block) cudaFreeHost(img->h_block);
    if (img->d_block && img->owns_device) {
        int cur = -1;
        cudaGetDevice(&cur);
        if (cur != img->device) cudaSetDevice(img->device);
        cudaFree(img->d_block);
        if (cur >= 0 && cur != img->device) cudaSetDevice(cur);
        cudaGetLastError();
    }
    delete img;
}

// ---------------------------------------------------------------------------
// Launch planning

bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// Work units of an image at `cpw` chunks per warp (the default: the largest
// units, which the no-alloc limit counts).
uint32_t units_of(const hxq_cuda_image *im, uint32_t cpw = kChunksPerWarp)
{
    return (im->n_chunks + unit_chunks(cpw) - 1) / unit_chunks(cpw);
}

hxq_error_t launch_fast_group(const std::vector<uint32_t> &which,
                              hxq_cuda_image *const *imgs, char *out_base,
                              const size_t *offs, size_t elem, int bf16,
                              double *d_sumsq, float *d_conf, const Scratch &sc,
                              int sms, cudaStream_t s)
{
    if (which.empty()) return HXQ_OK;
    VqLaunch p;
    std::memset(&p, 0, sizeof(p));
    uint64_t chunks = 0;
    for (uint32_t i : which) chunks += imgs[i]->n_chunks;
    const uint32_t cpw = fast_cpw(chunks, sms, imgs[which[0]]->kind);
    uint32_t units = 0;
    for (uint32_t n = 0; n < which.size(); ++n) {
        const uint32_t i = which[n];
        const hxq_cuda_image *im = imgs[i];
        VqJob &J = p.job[n];
        J.idx = reinterpret_cast<const uint4 *>(im->d_idx);
        J.cb = im->d_cb;
        J.chunk_ptr = im->d_chunk_ptr;
        J.ent = im->d_ent;
        J.out = out_base + offs[i] * elem;
        J.numel = im->numel;
        J.n_chunks = im->n_chunks;
        J.k = im->k;
        J.unit_begin = units;
        J.n_units = units_of(im, cpw);
        J.sumsq = d_sumsq ? d_sumsq + i : nullptr;
        J.conf = d_conf ? d_conf + i : nullptr;
        J.ref_conf = im->ref_l2;
        units += J.n_units;
    }
    if (units > sc.n_slots) return HXQ_ERR_INVALID_ARG;
    p.n_jobs = (uint32_t)which.size();
    p.total_units = units;
    p.cpw = cpw;
    p.grid = fast_grid(units, sms, imgs[which[0]]->kind);
    p.slots = sc.slots;
    p.counters = sc.counters;
    p.work = sc.work;
    p.err = sc.err;
    const hxq_cuda_image *first = imgs[which[0]];
    const cudaError_t e = launch_vq_fast(p, first->kind, bf16, first->check_k ? 1 : 0, s);
    if (e == cudaSuccess) g_launches.fetch_add(vq_fast_launches(p), std::memory_order_relaxed);
    return map_cuda(e);
}

hxq_error_t launch_images(hxq_cuda_image *const *imgs, uint32_t n, void *d_out,
                          const size_t *offs, int bf16, double *d_sumsq,
                          float *d_conf, int dev, cudaStream_t s)
{
    Scratch *sc = nullptr;
    hxq_error_t err;
    uint32_t need = 0;
    for (uint32_t i = 0; i < n; ++i)
        if (imgs[i] && (imgs[i]->kind == kKindScalar || imgs[i]->kind == kKindVq12)) need += units_of(imgs[i], 1u);
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if ((err = dev_ready(dev)) != HXQ_OK) return err;
        if ((err = get_scratch(dev, s, &sc, need)) != HXQ_OK) return err;
    }
    const int sms = g_dev[dev].sms;
    const size_t elem = bf16 ? 2u : 4u;
    char *base = static_cast<char *>(d_out);
    // group: fast scalar, fast 12-bit (k checked or not); the rest generic
    std::vector<uint32_t> g_scalar, g_vq12, g_vq12k, generic;
    for (uint32_t i = 0; i < n; ++i) {
        const hxq_cuda_image *im = imgs[i];
        if (im->device != dev) return HXQ_ERR_INVALID_ARG;
        if (!im->d_block) return HXQ_ERR_INVALID_ARG;  // streamed image never uploaded
        if (im->numel == 0) {
            cudaError_t ce = cudaSuccess;
            if (d_sumsq) ce = cudaMemsetAsync(d_sumsq + i, 0, sizeof(double), s);
            if (ce == cudaSuccess && d_conf) ce = cudaMemsetAsync(d_conf + i, 0, sizeof(float), s);
            if (ce != cudaSuccess) return map_cuda(ce);
            continue;
        }
        const bool ok_align = aligned16(base + offs[i] * elem);
        if (im->kind == kKindScalar && ok_align) g_scalar.push_back(i);
        else if (im->kind == kKindVq12 && ok_align) (im->check_k ? g_vq12k : g_vq12).push_back(i);
        else generic.push_back(i);
    }
    if ((err = launch_fast_group(g_vq12, imgs, base, offs, elem, bf16, d_sumsq, d_conf, *sc, sms, s)) != HXQ_OK) return err;
    if ((err = launch_fast_group(g_vq12k, imgs, base, offs, elem, bf16, d_sumsq, d_conf, *sc, sms, s)) != HXQ_OK) return err;
    if ((err = launch_fast_group(g_scalar, imgs, base, offs, elem, bf16, d_sumsq, d_conf, *sc, sms, s)) != HXQ_OK) return err;
    for (uint32_t i : generic) {
        const hxq_cuda_image *im = imgs[i];
        GenericJob j;
        std::memset(&j, 0, sizeof(j));
        j.kind = im->kind;
        j.idx = im->d_idx;
        j.cb = im->d_cb;
        j.scales = im->d_scales;
        j.offsets = im->d_offsets;
        j.rows = im->rows;
        j.in_f = im->in_f;
        j.k = im->k;
        j.gs = im->gs;
        j.triples_per_row = im->kind == kKindVq12 ? im->in_f / 4u : im->triples_per_row;
        j.out = base + offs[i] * elem;
        j.bf16 = bf16;
        j.sumsq = d_sumsq ? d_sumsq + i : nullptr;
        j.conf = d_conf ? d_conf + i : nullptr;
        j.ref_conf = im->ref_l2;
        j.conf_exact = 0;
        j.ent = im->d_ent;
        j.n_ent = im->n_ent;
        if (im->kind == kKindScalar || im->kind == kKindVq12) {
            if (im->numel > 0xFFFFFFFFull) return HXQ_ERR_INVALID_ARG;
            j.chunk_ptr = im->d_chunk_ptr;
            j.n_chunks = im->n_chunks;
        }
        const cudaError_t ce = launch_generic(j, *sc, s);
        if (ce != cudaSuccess) return map_cuda(ce);
        g_launches.fetch_add((im->numel ? 1u : 0u) + (im->n_ent ? 1u : 0u), std::memory_order_relaxed);
    }
    return HXQ_OK;
}

// Wait for `s`, then read and clear the device error word.
hxq_error_t sync_and_check(int dev, cudaStream_t s, float *conf_out)
{
    Scratch *sc = nullptr;
    void *rb = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        hxq_error_t err = get_scratch(dev, s, &sc);
        if (err != HXQ_OK) return err;
        rb = g_dev[dev].readback;
    }
    // err word and conf[0] are adjacent at the start of the scratch block
    cudaError_t ce = cudaMemcpyAsync(rb, sc->err, 16 + 4, cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) { cudaGetLastError(); return map_cuda(ce); }
    const uint32_t word = *static_cast<uint32_t *>(rb);
    if (conf_out) std::memcpy(conf_out, static_cast<char *>(rb) + 16, 4);
    if (word) {
        ce = cudaMemsetAsync(sc->err, 0, 4, s);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
        if (ce != cudaSuccess) { cudaGetLastError(); return map_cuda(ce); }
        if (word & kErrIndexOOB) return HXQ_ERR_INDEX_OOB;
    }
    return HXQ_OK;
}

// Cached full-tensor image of t on the current device (caller holds no lock).
hxq_error_t tensor_image(const hxq_tensor_t *t, int dev, hxq_cuda_image **out)
{
    const Snapshot now = snap(t, dev);
    hxq_cuda_image *stale = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_images.find(t);
        if (it != g_images.end()) {
            if (it->second.snap == now) { *out = it->second.img; return HXQ_OK; }
            stale = it->second.img;
            g_images.erase(it);
        }
    }
    destroy_image(stale);
    hxq_cuda_image *img = nullptr;
    hxq_error_t err = build_image(t, 0, t->out_features, dev, false, false, &img);
    if (err != HXQ_OK) return err;
    std::lock_guard<std::mutex> lk(g_mu);
    g_images[t] = Cached{now, img};
    *out = img;
    return HXQ_OK;
}

hxq_error_t decompress_sync(hxq_tensor_t *t, void *d_out, int bf16, float *l2)
{
    int dev = 0;
    hxq_error_t err = current_device(&dev);
    if (err != HXQ_OK) return err;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if ((err = dev_ready(dev)) != HXQ_OK) return err;
    }
    hxq_cuda_image *img = nullptr;
    if ((err = tensor_image(t, dev, &img)) != HXQ_OK) return err;
    Scratch *sc = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if ((err = get_scratch(dev, (cudaStream_t)0, &sc)) != HXQ_OK) return err;
    }
    const size_t off0 = 0;
    // The drop-in API reports the reference's own value (see
    // collect_sidecar), which the image carries; the exact sum of squares is
    // not asked for, so the kernel skips its cross-CTA reduction.
    err = launch_images(&img, 1, d_out, &off0, bf16, nullptr, sc->conf, dev, (cudaStream_t)0);
    if (err != HXQ_OK) return err;
    float gpu_conf = 0.0f;
    if ((err = sync_and_check(dev, (cudaStream_t)0, &gpu_conf)) != HXQ_OK) return err;
    *l2 = img->ref_l2;
    return HXQ_OK;
}

}  // namespace

// ===========================================================================
// Internal interface used by the C host library (hxq_internal.h)

extern "C" {

int hxqi_cuda_available(void) { return cuda_present() ? 1 : 0; }

int hxqi_cuda_ptr_is_device(const void *p)
{
    if (!p) return 0;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        for (const auto &kv : g_arenas)
            if (kv.first->data == p) return 1;
    }
    if (!cuda_present() || !any_context_active()) return 0;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) { cudaGetLastError(); return 0; }
    return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) ? 1 : 0;
}

void hxqi_cuda_forget_tensor(const hxq_tensor_t *t)
{
    hxq_cuda_image *img = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_images.find(t);
        if (it == g_images.end()) return;
        img = it->second.img;
        g_images.erase(it);
    }
    destroy_image(img);
}

int hxqi_cuda_is_arena(const hxq_shared_buffer_t *buf)
{
    std::lock_guard<std::mutex> lk(g_mu);
    return g_arenas.count(buf) ? 1 : 0;
}

void hxqi_cuda_arena_forget(const hxq_shared_buffer_t *buf)
{
    std::lock_guard<std::mutex> lk(g_mu);
    g_arenas.erase(buf);
}

void hxqi_cuda_arena_release(hxq_shared_buffer_t *buf)
{
    int dev = -1;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_arenas.find(buf);
        if (it == g_arenas.end()) return;
        dev = it->second;
        g_arenas.erase(it);
    }
    if (buf->data) {
        int cur = -1;
        cudaGetDevice(&cur);
        if (cur != dev) cudaSetDevice(dev);
        cudaFree(buf->data);
        if (cur >= 0 && cur != dev) cudaSetDevice(cur);
        cudaGetLastError();
    }
    buf->data = nullptr;
    buf->capacity = 0;
    buf->high_water = 0;
}

// Grow a device arena to at least `floats` floats, keeping its contents.
hxq_error_t hxqi_cuda_arena_reserve(hxq_shared_buffer_t *buf, size_t floats)
{
    if (floats <= buf->capacity) return HXQ_OK;
    int dev = 0;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_arenas.find(buf);
        if (it == g_arenas.end()) return HXQ_ERR_INVALID_ARG;
        dev = it->second;
    }
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != dev) cudaSetDevice(dev);
    float *nd = nullptr;
    cudaError_t ce = cudaMalloc(&nd, floats * sizeof(float));
    if (ce == cudaSuccess && buf->data && buf->capacity)
        ce = cudaMemcpy(nd, buf->data, buf->capacity * sizeof(float), cudaMemcpyDeviceToDevice);
    if (ce == cudaSuccess) {
        if (buf->data) cudaFree(buf->data);
        buf->data = nd;
        buf->capacity = floats;
    } else {
        cudaGetLastError();
        if (nd) cudaFree(nd);
    }
    if (cur >= 0 && cur != dev) cudaSetDevice(cur);
    return map_cuda(ce);
}

hxq_error_t hxqi_cuda_decompress(hxq_tensor_t *t, void *d_out, int bf16, float *l2)
{
    return decompress_sync(t, d_out, bf16, l2);
}

// GPU decompress into an internal device buffer, then copy to host memory.
hxq_error_t hxqi_cuda_decompress_to_host(hxq_tensor_t *t, float *h_out, float *l2)
{
    int dev = 0;
    hxq_error_t err = current_device(&dev);
    if (err != HXQ_OK) return err;
    const size_t n = (size_t)t->out_features * t->in_features;
    float *stage = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if ((err = dev_ready(dev)) != HXQ_OK) return err;
        DevCtx &d = g_dev[dev];
        if (d.stage_floats < n) {
            if (d.stage) cudaFree(d.stage);
            d.stage = nullptr;
            d.stage_floats = 0;
            cudaError_t ce = cudaMalloc(&d.stage, std::max<size_t>(n, 4) * sizeof(float));
            if (ce != cudaSuccess) { cudaGetLastError(); return map_cuda(ce); }
            d.stage_floats = std::max<size_t>(n, 4);
        }
        stage = d.stage;
    }
    // Columns the 12-bit decoder leaves untouched (an odd pair count per
    // row, hxq.c:290-294) must keep the caller's data, so only those images
    // copy the buffer in first; every other kind writes each element.
    hxq_cuda_image *img = nullptr;
    if ((err = tensor_image(t, dev, &img)) != HXQ_OK) return err;
    cudaError_t ce = cudaSuccess;
    if (n && img->kind == kKindVq12Any) ce = cudaMemcpy(stage, h_out, n * sizeof(float), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) { cudaGetLastError(); return map_cuda(ce); }
    float conf = 0.0f;
    if ((err = decompress_sync(t, stage, 0, &conf)) != HXQ_OK) return err;
    if (n) ce = cudaMemcpy(h_out, stage, n * sizeof(float), cudaMemcpyDeviceToHost);
    if (ce != cudaSuccess) { cudaGetLastError(); return map_cuda(ce); }
    *l2 = conf;
    return HXQ_OK;
}

// ===========================================================================
// Public additive API (hxq_cuda.h)

const char *hxq_error_string(hxq_error_t err)
{
    switch ((int)err) {
    case HXQ_OK: return "ok";
    case HXQ_ERR_NULL_PTR: return "null pointer";
    case HXQ_ERR_INVALID_K: return "codebook size must be 256 or 4096";
    case HXQ_ERR_INVALID_DIM: return "invalid vector dimension or mode";
    case HXQ_ERR_ALLOC_FAILED: return "allocation failed";
    case HXQ_ERR_INDEX_OOB: return "index >= codebook size";
    case HXQ_ERR_PACK_FORMAT: return "packed index data too short";
    case HXQ_ERR_SIDECAR_OOB: return "sidecar coordinate out of range";
    case 32: return "CUDA runtime error";
    case 33: return "backend unavailable";
    case 34: return "invalid argument";
    case 35: return "NCCL error";
    default: return "unknown error";
    }
}

const char *hxq_b200_version(void) { return "hxq-b200 0.1.0 (sm_100a)"; }

int hxq_cuda_device_count(void)
{
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n;
}

hxq_error_t hxq_cuda_arena_init(hxq_shared_buffer_t *buf, size_t capacity_floats)
{
    if (!buf) return HXQ_ERR_NULL_PTR;
    int dev = 0;
    hxq_error_t err = current_device(&dev);
    if (err != HXQ_OK) return err;
    float *d = nullptr;
    if (capacity_floats) {
        cudaError_t ce = cudaMalloc(&d, capacity_floats * sizeof(float));
        if (ce == cudaSuccess) ce = cudaMemset(d, 0, capacity_floats * sizeof(float));
        if (ce != cudaSuccess) { cudaGetLastError(); if (d) cudaFree(d); return map_cuda(ce); }
    }
    buf->data = d;
    buf->capacity = capacity_floats;
    buf->high_water = 0;
    std::lock_guard<std::mutex> lk(g_mu);
    g_arenas[buf] = dev;
    return HXQ_OK;
}

int hxq_cuda_buffer_is_device(const hxq_shared_buffer_t *buf)
{
    return buf ? hxqi_cuda_is_arena(buf) : 0;
}

hxq_error_t hxq_cuda_decompress(hxq_tensor_t *t, void *d_out, hxq_out_dtype_t dtype)
{
    if (!t || !d_out) return HXQ_ERR_NULL_PTR;
    if (dtype != HXQ_OUT_F32 && dtype != HXQ_OUT_BF16) return HXQ_ERR_INVALID_ARG;
    if (!t->indices_raw) return HXQ_ERR_NULL_PTR;
    if (t->mode != HXQ_AFFINE_G128 && !t->codebook) return HXQ_ERR_NULL_PTR;
    float l2 = 0.0f;
    hxq_error_t err = decompress_sync(t, d_out, dtype == HXQ_OUT_BF16, &l2);
    if (err != HXQ_OK) return err;
    t->sidecar_l2_norm = l2;
    return HXQ_OK;
}

hxq_error_t hxq_dequant_bf16(hxq_tensor_t *t, hxq_shared_buffer_t *arena, hxq_result_t *result)
{
    if (!t || !arena || !result) return HXQ_ERR_NULL_PTR;
    if (!hxqi_cuda_is_arena(arena)) return HXQ_ERR_INVALID_ARG;
    const size_t n = (size_t)t->out_features * t->in_features;
    const size_t floats = (n + 1) / 2;
    hxq_error_t err = hxqi_cuda_arena_reserve(arena, floats);
    if (err != HXQ_OK) return err;
    if (floats > arena->high_water) arena->high_water = floats;
    if ((err = hxq_cuda_decompress(t, arena->data, HXQ_OUT_BF16)) != HXQ_OK) return err;
    result->weights = arena->data;
    result->confidence = t->sidecar_l2_norm;
    result->out_features = t->out_features;
    result->in_features = t->in_features;
    return HXQ_OK;
}

void hxq_cuda_tensor_invalidate(const hxq_tensor_t *t) { hxqi_cuda_forget_tensor(t); }

hxq_error_t hxq_cuda_image_create_ex(const hxq_tensor_t *t, uint32_t row_begin, uint32_t row_end,
                                     uint32_t flags, hxq_cuda_image_t **img)
{
    if (!t || !img) return HXQ_ERR_NULL_PTR;
    if (flags & ~(uint32_t)(HXQ_IMAGE_STREAMED | HXQ_IMAGE_MATMUL)) return HXQ_ERR_INVALID_ARG;
    int dev = 0;
    hxq_error_t err = current_device(&dev);
    if (err != HXQ_OK) return err;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if ((err = dev_ready(dev)) != HXQ_OK) return err;
    }
    return build_image(t, row_begin, row_end, dev, (flags & HXQ_IMAGE_STREAMED) != 0,
                       (flags & HXQ_IMAGE_MATMUL) != 0, img);
}

hxq_error_t hxq_cuda_image_create(const hxq_tensor_t *t, uint32_t row_begin,
                                  uint32_t row_end, hxq_cuda_image_t **img)
{
    return hxq_cuda_image_create_ex(t, row_begin, row_end, 0u, img);
}

hxq_error_t hxq_cuda_image_create_streamed(const hxq_tensor_t *t, uint32_t row_begin,
                                           uint32_t row_end, hxq_cuda_image_t **img)
{
    return hxq_cuda_image_create_ex(t, row_begin, row_end, HXQ_IMAGE_STREAMED, img);
}

int hxq_cuda_image_has_matmul_tables(const hxq_cuda_image_t *img) { return img && img->has_mm ? 1 : 0; }

size_t hxq_cuda_image_block_bytes(const hxq_cuda_image_t *img) { return img ? img->block_bytes : 0; }

hxq_error_t hxq_cuda_image_upload(hxq_cuda_image_t *img, void *d_dst, void *stream)
{
    if (!img || !d_dst) return HXQ_ERR_NULL_PTR;
    if (!img->h_block || ((uintptr_t)d_dst & 255u)) return HXQ_ERR_INVALID_ARG;
    const cudaError_t ce = cudaMemcpyAsync(d_dst, img->h_block, img->block_bytes,
                                           cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
    if (ce != cudaSuccess) { cudaGetLastError(); return map_cuda(ce); }
    bind_image(img, d_dst);
    return HXQ_OK;
}

unsigned long long hxq_cuda_launch_count(void) { return g_launches.load(); }

void hxq_cuda_image_destroy(hxq_cuda_image_t *img) { destroy_image(img); }

size_t hxq_cuda_image_numel(const hxq_cuda_image_t *img) { return img ? (size_t)img->numel : 0; }

size_t hxq_cuda_image_device_bytes(const hxq_cuda_image_t *img) { return img ? img->block_bytes : 0; }

double hxq_cuda_image_sidecar_sumsq(const hxq_cuda_image_t *img) { return img ? img->sumsq : 0.0; }

float hxq_cuda_image_reference_confidence(const hxq_cuda_image_t *img) { return img ? img->ref_l2 : 0.0f; }

float hxq_cuda_image_tensor_confidence(const hxq_cuda_image_t *img) { return img ? img->ref_l2_tensor : 0.0f; }

hxq_error_t hxq_cuda_decompress_images(hxq_cuda_image_t *const *imgs, uint32_t n,
                                       void *d_out, const size_t *out_offsets,
                                       hxq_out_dtype_t dtype, double *d_sumsq,
                                       float *d_conf, void *stream)
{
    if (n == 0) return HXQ_OK;
    if (!imgs || !d_out || !out_offsets) return HXQ_ERR_NULL_PTR;
    if (n > kMaxJobs) return HXQ_ERR_INVALID_ARG;
    if (dtype != HXQ_OUT_F32 && dtype != HXQ_OUT_BF16) return HXQ_ERR_INVALID_ARG;
    for (uint32_t i = 0; i < n; ++i)
        if (!imgs[i]) return HXQ_ERR_NULL_PTR;
    int dev = 0;
    hxq_error_t err = current_device(&dev);
    if (err != HXQ_OK) return err;
    return launch_images(imgs, n, d_out, out_offsets, dtype == HXQ_OUT_BF16, d_sumsq, d_conf,
                         dev, static_cast<cudaStream_t>(stream));
}

namespace {

// path: 0 the exact fp32 GEMV, 1 the tcgen05 GEMM, 2 the tensor-core GEMV
// (1 and 2 need the image's matmul tables).
hxq::VqTcMatrix tc_matrix(const hxq_cuda_image_t *img, const uint16_t *x, const hxq::OutPtrs &out, uint32_t ldy)
{
    return hxq::VqTcMatrix{img->d_tx, img->d_cbh, img->d_rb, img->d_e4, img->d_ed, img->n_patch, x, out, ldy,
                           img->rows, img->in_f};
}

int default_path(const hxq_cuda_image_t *img, const uint16_t *x, uint32_t N)
{
    if (!img || !img->has_mm) return 0;
    return N <= HXQ_VQ_MATMUL_TC_MAX && hxq::vq_tc_fits(x, N, img->in_f) ? 2 : 1;
}

hxq_error_t vq_matmul(const hxq_cuda_image_t *img, const uint16_t *d_x_bf16, uint32_t N, const hxq::OutPtrs &out,
                      uint32_t ldy, int path, void *stream)
{
    if (!img || !d_x_bf16) return HXQ_ERR_NULL_PTR;
    if (out.n == 0 || out.n > HXQ_CUDA_MAX_PEERS) return HXQ_ERR_INVALID_ARG;
    for (uint32_t k = 0; k < out.n; ++k)
        if (!out.y[k]) return HXQ_ERR_NULL_PTR;
    if (img->kind != kKindVq12 || img->check_k || img->k != 4096u || img->in_f % 64u != 0u)
        return HXQ_ERR_INVALID_ARG;
    if (path < 0 || path > 2 || (path != 0 && !img->has_mm)) return HXQ_ERR_INVALID_ARG;
    if (!img->d_block) return HXQ_ERR_INVALID_ARG;   // streamed image never uploaded
    if (ldy < img->rows || !aligned16(d_x_bf16)) return HXQ_ERR_INVALID_ARG;
    if (N == 0 || img->rows == 0) return HXQ_OK;
    int dev = 0;
    hxq_error_t err = current_device(&dev);
    if (err != HXQ_OK) return err;
    if (img->device != dev) return HXQ_ERR_INVALID_ARG;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if ((err = dev_ready(dev)) != HXQ_OK) return err;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (path != 1) hxq::gemm_chain_break();   // a GEMV follows
    if (path == 2) {
        const hxq::VqTcMatrix m = tc_matrix(img, d_x_bf16, out, ldy);
        uint32_t nl = 0;
        const int r = hxq::launch_vq_tc_gemv(1, &m, N, g_dev[dev].sms, s, &nl);
        if (r != 0) { cudaGetLastError(); return r > 0 ? HXQ_ERR_INVALID_ARG : HXQ_ERR_CUDA; }
        g_launches.fetch_add(nl - 1u, std::memory_order_relaxed);   // the part sums, if any
    } else if (path == 1) {
        const int r = hxq::vq_gemm_bf16(d_x_bf16, img->d_idx, img->d_cbh, img->d_rb, img->d_kq, img->d_e4,
                                        img->d_g4, img->d_gp, img->d_tx, out, N, img->in_f, img->rows, ldy, s);
        if (r != 0) { cudaGetLastError(); return r > 0 ? HXQ_ERR_INVALID_ARG : HXQ_ERR_CUDA; }
    } else {
        const cudaError_t e = hxq::launch_vq_gemv(img->d_idx, img->d_cb, img->d_chunk_ptr, img->d_ent,
                                                  img->n_chunks, img->rows, img->in_f, d_x_bf16, N, out, ldy,
                                                  g_dev[dev].sms, s);
        if (e != cudaSuccess) return map_cuda(e);
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return HXQ_OK;
}

}  // namespace

hxq_error_t hxq_cuda_vq_matmul_path(const hxq_cuda_image_t *img, const uint16_t *d_x_bf16,
                                    uint32_t N, float *d_y, uint32_t ldy, int path, void *stream)
{
    if (!d_y) return HXQ_ERR_NULL_PTR;
    hxq::OutPtrs o{};
    o.y[0] = d_y;
    o.n = 1;
    return vq_matmul(img, d_x_bf16, N, o, ldy, path, stream);
}

hxq_error_t hxq_cuda_vq_matmul(const hxq_cuda_image_t *img, const uint16_t *d_x_bf16,
                               uint32_t N, float *d_y, uint32_t ldy, void *stream)
{
    return hxq_cuda_vq_matmul_path(img, d_x_bf16, N, d_y, ldy, default_path(img, d_x_bf16, N), stream);
}

hxq_error_t hxq_cuda_vq_matmul_multi(const hxq_cuda_image_t *img, const uint16_t *d_x_bf16,
                                     uint32_t N, float *const *d_ys, uint32_t n_out,
                                     uint32_t ldy, void *stream)
{
    if (!d_ys) return HXQ_ERR_NULL_PTR;
    if (n_out == 0 || n_out > HXQ_CUDA_MAX_PEERS) return HXQ_ERR_INVALID_ARG;
    hxq::OutPtrs o{};
    for (uint32_t k = 0; k < n_out; ++k) o.y[k] = d_ys[k];
    o.n = n_out;
    return vq_matmul(img, d_x_bf16, N, o, ldy, default_path(img, d_x_bf16, N), stream);
}

hxq_error_t hxq_cuda_vq_matmul_batch(uint32_t n, hxq_cuda_image_t *const *imgs, const uint16_t *const *d_xs,
                                     float *const *d_ys, uint32_t n_out, const uint32_t *ldys, uint32_t N,
                                     void *stream)
{
    if (n == 0 || N == 0) return HXQ_OK;
    if (!imgs || !d_xs || !d_ys || !ldys) return HXQ_ERR_NULL_PTR;
    if (n_out == 0 || n_out > HXQ_CUDA_MAX_PEERS) return HXQ_ERR_INVALID_ARG;
    auto outs_of = [&](uint32_t i, hxq::OutPtrs &o) -> hxq_error_t {
        o = hxq::OutPtrs{};
        for (uint32_t k = 0; k < n_out; ++k) {
            o.y[k] = d_ys[(size_t)i * n_out + k];
            if (!o.y[k]) return HXQ_ERR_NULL_PTR;
        }
        o.n = n_out;
        return HXQ_OK;
    };
    int dev = 0;
    hxq_error_t err = current_device(&dev);
    if (err != HXQ_OK) return err;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if ((err = dev_ready(dev)) != HXQ_OK) return err;
    }
    for (uint32_t i = 0; i < n; ++i) {
        const hxq_cuda_image_t *img = imgs[i];
        if (!img || !d_xs[i]) return HXQ_ERR_NULL_PTR;
        if (img->kind != kKindVq12 || img->check_k || img->k != 4096u || img->in_f % 64u != 0u || !img->d_block ||
            img->device != dev || ldys[i] < img->rows || !aligned16(d_xs[i]))
            return HXQ_ERR_INVALID_ARG;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The batch in three parts, each image in the first that takes it: up to
    // HXQ_VQ_MATMUL_TC_MAX tokens, images with matmul tables that suit the
    // tensor-core GEMV share its launches (up to 8 jobs, a matrix split
    // along K counting one per part); up to
    // HXQ_VQ_MATMUL_GEMV_MAX tokens the rest share exact-GEMV launches;
    // anything left runs one call per image.
    std::vector<uint8_t> done(n, 0);
    std::vector<hxq::VqTcMatrix> tcs;
    for (uint32_t i = 0; i < n; ++i) {
        hxq::OutPtrs o;
        if ((err = outs_of(i, o)) != HXQ_OK) return err;
        if (imgs[i]->rows == 0) { done[i] = 1; continue; }
        if (default_path(imgs[i], d_xs[i], N) == 2) {
            tcs.push_back(tc_matrix(imgs[i], d_xs[i], o, ldys[i]));
            done[i] = 1;
        }
    }
    // narrow matrices first, so that a wide one's activations do not cost
    // the narrow ones stages or residency
    std::stable_sort(tcs.begin(), tcs.end(),
                     [](const hxq::VqTcMatrix &a, const hxq::VqTcMatrix &b) { return a.in_f < b.in_f; });
    for (size_t j0 = 0; j0 < tcs.size();) {
        const uint32_t cnt = hxq::vq_tc_group((uint32_t)(tcs.size() - j0), tcs.data() + j0, N);
        uint32_t nl = 0;
        const int r = hxq::launch_vq_tc_gemv(cnt, tcs.data() + j0, N, g_dev[dev].sms, s, &nl);
        j0 += cnt;
        if (r != 0) { cudaGetLastError(); return r > 0 ? HXQ_ERR_INVALID_ARG : HXQ_ERR_CUDA; }
        g_launches.fetch_add(nl, std::memory_order_relaxed);
    }
    if (N > HXQ_VQ_MATMUL_GEMV_MAX) {
        // one call per image; consecutive GEMMs overlap their wave tails
        hxq::GemmChainScope chain(s);
        for (uint32_t i = 0; i < n; ++i) {
            if (done[i]) continue;
            hxq::OutPtrs o;
            if ((err = outs_of(i, o)) != HXQ_OK) return err;
            err = vq_matmul(imgs[i], d_xs[i], N, o, ldys[i], default_path(imgs[i], d_xs[i], N), stream);
            if (err != HXQ_OK) return err;
        }
        return HXQ_OK;
    }
    std::vector<hxq::VqGemvJob> jobs;
    jobs.reserve(n);
    for (uint32_t i = 0; i < n; ++i) {
        if (done[i]) continue;
        const hxq_cuda_image_t *img = imgs[i];
        hxq::OutPtrs o;
        if ((err = outs_of(i, o)) != HXQ_OK) return err;
        jobs.push_back(hxq::VqGemvJob{img->d_idx, img->d_cb, img->d_chunk_ptr, img->d_ent, img->n_chunks, img->rows,
                                      img->in_f, d_xs[i], o, ldys[i]});
    }
    for (size_t j0 = 0; j0 < jobs.size(); j0 += 8) {
        const uint32_t cnt = (uint32_t)std::min<size_t>(8, jobs.size() - j0);
        const cudaError_t e = hxq::launch_vq_gemv_batch(cnt, jobs.data() + j0, N, g_dev[dev].sms, s);
        if (e != cudaSuccess) return map_cuda(e);
        g_launches.fetch_add(1, std::memory_order_relaxed);
    }
    return HXQ_OK;
}

hxq_error_t hxq_cuda_stream_synchronize(void *stream)
{
    int dev = 0;
    hxq_error_t err = current_device(&dev);
    if (err != HXQ_OK) return err;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if ((err = dev_ready(dev)) != HXQ_OK) return err;
    }
    return sync_and_check(dev, static_cast<cudaStream_t>(stream), nullptr);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// The reference's undeclared GPU launchers (src/hxq_cuda.cu:209-288), on the
// generic kernels.  Index layout is the one hxq.c decodes (each row holds
// ceil((in_f/2)/2) triples), which equals the launcher's flat pair stream
// whenever in_f/2 is even.

namespace {

int raw_launch(uint32_t kind, const float *cb, const uint8_t *idx, float *out,
               uint32_t out_f, uint32_t in_f)
{
    int dev = 0;
    if (current_device(&dev) != HXQ_OK || !cb || !idx || !out) return -1;
    Scratch *sc = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (dev_ready(dev) != HXQ_OK || get_scratch(dev, (cudaStream_t)0, &sc) != HXQ_OK) return -1;
    }
    GenericJob j;
    std::memset(&j, 0, sizeof(j));
    j.kind = kind;
    j.idx = idx;
    j.cb = cb;
    j.rows = out_f;
    j.in_f = in_f;
    j.k = kind == kKindScalar ? 256u : 4096u;
    j.triples_per_row = (in_f / 2u + 1u) / 2u;
    j.out = out;
    if (launch_generic(j, *sc, (cudaStream_t)0) != cudaSuccess) { cudaGetLastError(); return -1; }
    return 0;
}

typedef CUresult (*AddrRangeFn)(CUdeviceptr *, size_t *, CUdeviceptr);

// Bytes from p to the end of the device allocation holding it (0 if unknown).
size_t bytes_to_alloc_end(const void *p)
{
    static AddrRangeFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<AddrRangeFn>(f);
        else
            cudaGetLastError();
    }
    if (!fn) return 0;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, (CUdeviceptr)(uintptr_t)p) != CUDA_SUCCESS) return 0;
    const uintptr_t end = (uintptr_t)base + size;
    return end > (uintptr_t)p ? end - (uintptr_t)p : 0;
}

}  // namespace

extern "C" {

int hxq_cuda_decompress_scalar(const float *d_codebook, const uint8_t *d_indices,
                               float *d_output, uint32_t out_f, uint32_t in_f)
{
    return raw_launch(kKindScalar, d_codebook, d_indices, d_output, out_f, in_f);
}

int hxq_cuda_decompress_vq2d_12bit(const float *d_codebook, const uint8_t *d_packed,
                                   float *d_output, uint32_t out_f, uint32_t in_f)
{
    // With an odd pair count per row the reference launcher's flat pair
    // stream is shorter than hxq.c's per-row layout; refuse rather than read
    // past a buffer sized for the former.
    if ((in_f / 2u) % 2u != 0u) return -1;
    return raw_launch(kKindVq12Any, d_codebook, d_packed, d_output, out_f, in_f);
}

// The reference launcher applies every entry with no bound at all; here an
// entry is applied when its element lies inside the allocation holding
// d_output (so a bad coordinate cannot write outside it), equal coordinates
// in array order.  Returns sqrt of the applied squares, or -1 on error.
float hxq_cuda_apply_sidecar(const uint32_t *d_rows, const uint32_t *d_cols,
                             const float *d_vals, float *d_output, uint32_t in_f,
                             uint32_t nnz)
{
    if (nnz == 0) return 0.0f;
    int dev = 0;
    if (!d_rows || !d_cols || !d_vals || !d_output || current_device(&dev) != HXQ_OK) return -1.0f;
    const size_t limit = bytes_to_alloc_end(d_output) / sizeof(float);
    if (limit == 0) return -1.0f;
    std::vector<uint32_t> r(nnz), c(nnz);
    std::vector<float> v(nnz);
    if (cudaMemcpy(r.data(), d_rows, nnz * 4u, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(c.data(), d_cols, nnz * 4u, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(v.data(), d_vals, nnz * 4u, cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return -1.0f;
    }
    std::vector<HostEntry> ents;
    ents.reserve(nnz);
    for (uint32_t i = 0; i < nnz; ++i) {
        const uint64_t pos = (uint64_t)r[i] * in_f + c[i];
        if (pos < limit && pos <= 0xFFFFFFFFull) ents.push_back({pos, v[i]});
    }
    std::stable_sort(ents.begin(), ents.end(),
                     [](const HostEntry &a, const HostEntry &b) { return a.pos < b.pos; });
    std::vector<SideEntry> de(ents.size());
    for (size_t i = 0; i < ents.size(); ++i) {
        de[i].x = (uint32_t)ents[i].pos;
        std::memcpy(&de[i].y, &ents[i].val, 4);
    }
    if (de.empty()) return 0.0f;
    Scratch *sc = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (dev_ready(dev) != HXQ_OK || get_scratch(dev, (cudaStream_t)0, &sc) != HXQ_OK) return -1.0f;
    }
    SideEntry *d_ent = nullptr;
    if (cudaMalloc(&d_ent, de.size() * sizeof(SideEntry)) != cudaSuccess) { cudaGetLastError(); return -1.0f; }
    float conf = -1.0f;
    GenericJob j;
    std::memset(&j, 0, sizeof(j));
    j.kind = kKindRaw;
    j.in_f = in_f;
    j.ent = d_ent;
    j.n_ent = (uint32_t)de.size();
    j.out = d_output;
    j.conf = sc->conf;
    j.conf_exact = 1;  // this launcher's L2 is a parallel sum, not hxq.c's order
    if (cudaMemcpy(d_ent, de.data(), de.size() * sizeof(SideEntry), cudaMemcpyHostToDevice) == cudaSuccess &&
        launch_generic(j, *sc, (cudaStream_t)0) == cudaSuccess &&
        sync_and_check(dev, (cudaStream_t)0, &conf) == HXQ_OK) {
        cudaFree(d_ent);
        return conf;
    }
    cudaGetLastError();
    cudaFree(d_ent);
    return -1.0f;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decompress without allocating.
//
// Some callers cannot let a library call cudaMalloc: inference engines that
// reserve nearly all of HBM for weights and KV cache at start-up and hand
// plugins pre-planned buffers (a cudaMalloc there can fail or fragment the
// pool), and latency-critical serving loops, where cudaMalloc/cudaFree may
// synchronise the device.  The regular batched entry point allocates its
// reduction scratch per stream on first use (cudaMalloc) and a pinned
// read-back buffer per device (cudaMallocHost).  This variant of the same
// fused decompress launch instead takes its scratch from a fixed array in
// the module's global memory, which every GPU that loads the library holds
// until the process exits.

namespace {

constexpr uint32_t kNoAllocUnits = 8192;          // one fp64 slot per unit
constexpr size_t   kNoAllocHead = 512;            // err | counters | work
constexpr size_t   kNoAllocOffCounters = 16;
constexpr size_t   kNoAllocOffWork = 16 + 4 * kMaxJobs;
constexpr size_t   kNoAllocBytes = kNoAllocHead + (size_t)kNoAllocUnits * sizeof(double);

// In host code this name is only a host-side stand-in for the array, not a
// device address; the address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

struct NoAllocDev {
    bool ready = false;
    unsigned char *ptr = nullptr;   // device address of g_noalloc_scratch
    int sms = 0;
};
NoAllocDev g_noalloc[kMaxDev];

// Once per device, with that device current: look up the array's device
// address and prepare the kernels (no allocation).  Caller holds g_mu.
hxq_error_t noalloc_setup(int dev, NoAllocDev **out)
{
    NoAllocDev &d = g_noalloc[dev];
    if (!d.ready) {
        void *ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        int sms = 0;
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e == cudaSuccess) e = configure_vq_kernels();
        if (e != cudaSuccess) { cudaGetLastError(); return map_cuda(e); }
        d.ptr = static_cast<unsigned char *>(ptr);
        d.sms = sms;
        d.ready = true;
    }
    *out = &d;
    return HXQ_OK;
}

}  // namespace

extern "C" hxq_error_t hxq_cuda_decompress_images_noalloc(hxq_cuda_image_t *const *imgs, uint32_t n,
                                                          void *d_out, const size_t *out_offsets,
                                                          hxq_out_dtype_t dtype, double *d_sumsq,
                                                          float *d_conf, void *stream)
{
    if (n == 0) return HXQ_OK;
    if (!imgs || !d_out || !out_offsets) return HXQ_ERR_NULL_PTR;
    if (n > kMaxJobs) return HXQ_ERR_INVALID_ARG;
    if (dtype != HXQ_OUT_F32 && dtype != HXQ_OUT_BF16) return HXQ_ERR_INVALID_ARG;
    int dev = 0;
    hxq_error_t err = current_device(&dev);
    if (err != HXQ_OK) return err;
    NoAllocDev *na = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if ((err = noalloc_setup(dev, &na)) != HXQ_OK) return err;
    }
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int bf16 = dtype == HXQ_OUT_BF16;
    const size_t elem = bf16 ? 2u : 4u;
    char *base = static_cast<char *>(d_out);

    // Only images the fused kernel takes (12-bit with in_f % 4 == 0, or
    // scalar; output slot 16-byte aligned) and at most kNoAllocUnits units
    // per launch group; everything is checked before anything is enqueued.
    std::vector<uint32_t> g_scalar, g_vq12, g_vq12k, empty;
    uint32_t u_scalar = 0, u_vq12 = 0, u_vq12k = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const hxq_cuda_image *im = imgs[i];
        if (!im) return HXQ_ERR_NULL_PTR;
        if (im->device != dev || !im->d_block) return HXQ_ERR_INVALID_ARG;
        if (im->numel == 0) { empty.push_back(i); continue; }
        if (!aligned16(base + out_offsets[i] * elem)) return HXQ_ERR_INVALID_ARG;
        if (im->kind == kKindScalar) { g_scalar.push_back(i); u_scalar += units_of(im); }
        else if (im->kind == kKindVq12 && im->check_k) { g_vq12k.push_back(i); u_vq12k += units_of(im); }
        else if (im->kind == kKindVq12) { g_vq12.push_back(i); u_vq12 += units_of(im); }
        else return HXQ_ERR_INVALID_ARG;
    }
    if (u_scalar > kNoAllocUnits || u_vq12 > kNoAllocUnits || u_vq12k > kNoAllocUnits)
        return HXQ_ERR_INVALID_ARG;

    Scratch sc;
    sc.base = na->ptr;
    sc.err = reinterpret_cast<uint32_t *>(na->ptr);
    sc.counters = reinterpret_cast<uint32_t *>(na->ptr + kNoAllocOffCounters);
    sc.work = reinterpret_cast<uint32_t *>(na->ptr + kNoAllocOffWork);
    sc.slots = reinterpret_cast<double *>(na->ptr + kNoAllocHead);
    sc.n_slots = kNoAllocUnits;

    // The array keeps whatever the last call left: clear the error word and
    // the counters the kernel expects at zero.  (Unit slots are written
    // before they are read.)
    // Once anything is enqueued, an error return first waits for the stream
    // (ignoring what that reports), so the shared array is idle when the
    // call returns, as the synchronous contract says.
    auto drain_and = [s](hxq_error_t e) {
        cudaStreamSynchronize(s);
        cudaGetLastError();
        return e;
    };
    cudaError_t ce = cudaMemsetAsync(na->ptr, 0, kNoAllocHead, s);
    for (uint32_t i : empty) {
        if (ce == cudaSuccess && d_sumsq) ce = cudaMemsetAsync(d_sumsq + i, 0, sizeof(double), s);
        if (ce == cudaSuccess && d_conf) ce = cudaMemsetAsync(d_conf + i, 0, sizeof(float), s);
    }
    if (ce != cudaSuccess) return drain_and(map_cuda(ce));
    const std::vector<uint32_t> *groups[3] = {&g_vq12, &g_vq12k, &g_scalar};
    for (const std::vector<uint32_t> *g : groups) {
        if (g->empty()) continue;
        ce = cudaMemsetAsync(na->ptr + kNoAllocOffCounters, 0, kNoAllocHead - kNoAllocOffCounters, s);
        if (ce != cudaSuccess) return drain_and(map_cuda(ce));
        if ((err = launch_fast_group(*g, imgs, base, out_offsets, elem, bf16, d_sumsq, d_conf, sc,
                                     na->sms, s)) != HXQ_OK)
            return drain_and(err);
    }
    // Synchronous: wait for the work, then read the device error word.
    uint32_t word = 0;
    ce = cudaMemcpyAsync(&word, na->ptr, sizeof(word), cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) { cudaGetLastError(); return map_cuda(ce); }
    return (word & kErrIndexOOB) ? HXQ_ERR_INDEX_OOB : HXQ_OK;
}
