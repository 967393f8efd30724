/*
 * hxq_cuda.h -- additive B200 (sm_100a) API of the HXQ codec.
 *
 * Nothing here replaces a reference symbol; these are the extra entry
 * points that make the CUDA backend usable at model scale:
 *   - a device arena (a hxq_shared_buffer_t whose data lives in HBM),
 *   - stream-ordered and bf16-output decompress,
 *   - "images": device copies of whole tensors or of row slices, which a
 *     multi-GPU driver uses to shard weight matrices by out_features,
 *   - batched decompress of many images in one kernel launch,
 *   - the reference's undeclared GPU launchers (src/hxq_cuda.cu:209-288)
 *     re-implemented on the new kernels,
 *   - bf16-activation and stream variants of the affine matmul.
 * Streams are passed as `void *` (a cudaStream_t; NULL = the legacy
 * default stream, which orders with every blocking stream of the device,
 * e.g. PyTorch's default stream) so the header needs no CUDA include.
 */
#ifndef HXQ_CUDA_H
#define HXQ_CUDA_H

#include "hxq.h"
#include "hxq_affine.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes beyond the reference enum (values the reference never
 * returns, so existing switch statements fall to their default). */
#define HXQ_ERR_CUDA                 ((hxq_error_t)32) /* CUDA runtime failure   */
#define HXQ_ERR_BACKEND_UNAVAILABLE  ((hxq_error_t)33) /* no device / backend    */
#define HXQ_ERR_INVALID_ARG          ((hxq_error_t)34) /* bad size, range, dtype */
#define HXQ_ERR_NCCL                 ((hxq_error_t)35) /* collective failed      */

/* Human-readable name of any status code above or in hxq.h. */
const char *hxq_error_string(hxq_error_t err);

/* Version of this implementation (the API level is HXQ_VERSION_STRING). */
const char *hxq_b200_version(void);

/* Number of visible CUDA devices (0 when there is none or no driver). */
int hxq_cuda_device_count(void);

/* -- Device arena -------------------------------------------------------
 * A shared buffer whose `data` is device memory on the current device.
 * hxq_dequant / hxq_tensor_decompress_shared grow it as the reference's
 * realloc does (new allocation, old contents copied over) and
 * hxq_shared_buffer_free releases it. */
hxq_error_t hxq_cuda_arena_init(hxq_shared_buffer_t *buf,
                                size_t capacity_floats);
/* 1 if `buf` is a device arena, 0 if it is a host buffer. */
int hxq_cuda_buffer_is_device(const hxq_shared_buffer_t *buf);

/* -- Output element type ------------------------------------------------ */
typedef enum {
    HXQ_OUT_F32  = 0,    /* fp32, bit-exact with the reference            */
    HXQ_OUT_BF16 = 1,    /* bf16 = round-to-nearest-even of the fp32 value */
} hxq_out_dtype_t;

/* Decompress into device memory in the given dtype; same semantics as
 * hxq_tensor_decompress (which is the fp32 case).  Synchronous. */
hxq_error_t hxq_cuda_decompress(hxq_tensor_t *t, void *d_out,
                                hxq_out_dtype_t dtype);

/* bf16 meta-kernel into a device arena: result->weights points at bf16
 * data (cast it to uint16_t / __nv_bfloat16).  The arena's capacity is
 * counted in floats, so a bf16 tensor needs half of out_f*in_f. */
hxq_error_t hxq_dequant_bf16(hxq_tensor_t *t, hxq_shared_buffer_t *arena,
                             hxq_result_t *result);

/* Drop the device copy of `t` (the next CUDA decompress rebuilds it).
 * Loaders and hxq_tensor_free already do this; call it after changing a
 * loaded host array in place. */
void hxq_cuda_tensor_invalidate(const hxq_tensor_t *t);

/* -- Images and batched decompress -------------------------------------- */

/* A device copy of rows [row_begin, row_end) of a loaded VQ tensor
 * (scalar or 12-bit), on the device current at creation.  The image does
 * not reference `t` afterwards. */
typedef struct hxq_cuda_image hxq_cuda_image_t;

hxq_error_t hxq_cuda_image_create(const hxq_tensor_t *t, uint32_t row_begin,
                                  uint32_t row_end, hxq_cuda_image_t **img);
void        hxq_cuda_image_destroy(hxq_cuda_image_t *img);
/* rows * in_features of the image. */
size_t      hxq_cuda_image_numel(const hxq_cuda_image_t *img);
/* Device bytes held by the image (index bytes, codebook, sidecar). */
size_t      hxq_cuda_image_device_bytes(const hxq_cuda_image_t *img);
/* Sum of squared in-range sidecar deltas of the image, computed on the
 * host at creation (double); the shards of one tensor add up to the
 * tensor's, and sqrt of the total is its confidence. */
double      hxq_cuda_image_sidecar_sumsq(const hxq_cuda_image_t *img);
/* The confidence as the reference library reports it for these rows:
 * sqrtf of a float running sum of squares in the sidecar's array order
 * (src/hxq.c:335-349).  hxq_dequant, hxq_tensor_decompress and the d_conf
 * output of hxq_cuda_decompress_images return this value, bit-identical to
 * the reference.  Over ~1e5 entries it differs from the exact value (sqrt
 * of hxq_cuda_image_sidecar_sumsq, and of the d_sumsq output) by the
 * reference's own fp32 rounding, a few 1e-5 relative. */
float       hxq_cuda_image_reference_confidence(const hxq_cuda_image_t *img);
/* The reference's confidence for the whole tensor the image was cut from
 * (every row, not only the image's): what hxq_dequant reports for that
 * tensor.  Lets a matrix split by rows over several GPUs report the
 * reference's value without gathering its sidecar; equal to
 * hxq_cuda_image_reference_confidence for an image of all rows. */
float       hxq_cuda_image_tensor_confidence(const hxq_cuda_image_t *img);

/* Streamed image: the same preprocessed block, kept in pinned host memory
 * instead of HBM, for weights that live on the host and cross PCIe each
 * time they are used.  hxq_cuda_image_upload copies the block
 * (hxq_cuda_image_block_bytes of it) to d_dst (256-B aligned device
 * memory) on `stream` and makes the image decompress from there; order the
 * decompress after the copy (same stream or an event), and do not reuse
 * d_dst while a decompress of the image may still read it. */
hxq_error_t hxq_cuda_image_create_streamed(const hxq_tensor_t *t, uint32_t row_begin,
                                           uint32_t row_end, hxq_cuda_image_t **img);
size_t      hxq_cuda_image_block_bytes(const hxq_cuda_image_t *img);
hxq_error_t hxq_cuda_image_upload(hxq_cuda_image_t *img, void *d_dst, void *stream);

/* Image with options: HXQ_IMAGE_STREAMED (as hxq_cuda_image_create_streamed)
 * and HXQ_IMAGE_MATMUL, which adds the tables the tensor-core path of
 * hxq_cuda_vq_matmul reads (a bf16 codebook copy and per-row sidecar
 * patches, about 5% of the index bytes) to 12-bit images with k = 4096 and
 * in_features % 128 == 0; other images are built without them. */
#define HXQ_IMAGE_STREAMED 1u
#define HXQ_IMAGE_MATMUL   2u
hxq_error_t hxq_cuda_image_create_ex(const hxq_tensor_t *t, uint32_t row_begin,
                                     uint32_t row_end, uint32_t flags,
                                     hxq_cuda_image_t **img);
/* 1 if the image carries the fused-matmul tables. */
int         hxq_cuda_image_has_matmul_tables(const hxq_cuda_image_t *img);

/* Kernels this library has launched in this process (all devices). */
unsigned long long hxq_cuda_launch_count(void);

/* Decompress n images in one stream-ordered launch.  Image i is written
 * at element offset out_offsets[i] of d_out (elements of `dtype`).
 * d_sumsq (n doubles) and d_conf (n floats) are optional device outputs:
 * each image's exact sum of squared sidecar deltas, reduced on the GPU in
 * fp64 in a fixed order, and its confidence as the reference reports it
 * (hxq_cuda_image_reference_confidence, bit-identical to hxq.c).
 * Device-side errors (an index >= k) are reported by
 * hxq_cuda_stream_synchronize.  n <= HXQ_CUDA_MAX_BATCH. */
#define HXQ_CUDA_MAX_BATCH 64
hxq_error_t hxq_cuda_decompress_images(hxq_cuda_image_t *const *imgs,
                                       uint32_t n, void *d_out,
                                       const size_t *out_offsets,
                                       hxq_out_dtype_t dtype, double *d_sumsq,
                                       float *d_conf, void *stream);

/* Wait for `stream` and report (and clear) errors its decompress kernels
 * recorded on the device. */
hxq_error_t hxq_cuda_stream_synchronize(void *stream);

/* The same batched decompress, for callers that must not have the library
 * allocate memory: engines that reserve HBM up front and give plugins
 * pre-planned buffers (a cudaMalloc can fail or fragment the pool there),
 * or serving loops where cudaMalloc/cudaFree would stall the device.  No
 * counterpart in the reference library.
 *   - Allocates nothing: no cudaMalloc, cudaFree or cudaMallocHost.  The
 *     caller passes the images (created and, if streamed, uploaded
 *     beforehand) and the output buffers, as for
 *     hxq_cuda_decompress_images.  The kernels' scratch is a fixed
 *     66,048-byte array in the library's global memory, which every GPU
 *     that loads the library holds until the process exits.
 *   - Limit: at most 8,192 work units (16 chunks of 2048 weights each, i.e.
 *     268,435,456 weights) per kind of image (12-bit, 12-bit with k = 256,
 *     scalar) in one call, and only images the fused kernel takes (12-bit
 *     with in_features % 4 == 0, or scalar) with 16-byte aligned output
 *     slots; otherwise HXQ_ERR_INVALID_ARG before anything is enqueued.
 *   - Synchronous: returns once the work on `stream` is done, with
 *     HXQ_ERR_INDEX_OOB if an index was >= k.
 *   - The first call on a device looks up the array's address and prepares
 *     the kernels; make that first call before any stream capture.
 *   - All calls share the one array: calls that overlap on the GPU (other
 *     streams, other threads) race and must be serialised by the caller. */
hxq_error_t hxq_cuda_decompress_images_noalloc(hxq_cuda_image_t *const *imgs,
                                               uint32_t n, void *d_out,
                                               const size_t *out_offsets,
                                               hxq_out_dtype_t dtype, double *d_sumsq,
                                               float *d_conf, void *stream);

/* -- The reference's GPU launchers (src/hxq_cuda.cu:209-288) -------------
 * Exported, undeclared in the reference; device pointers throughout.
 * Return 0 on success and -1 on error (the reference's convention). */
int   hxq_cuda_decompress_scalar(const float *d_codebook,
                                 const uint8_t *d_indices, float *d_output,
                                 uint32_t out_f, uint32_t in_f);
int   hxq_cuda_decompress_vq2d_12bit(const float *d_codebook,
                                     const uint8_t *d_packed, float *d_output,
                                     uint32_t out_f, uint32_t in_f);
/* Adds the in-range entries to d_output (in array order per coordinate)
 * and returns sqrt(sum v^2); negative on error. */
float hxq_cuda_apply_sidecar(const uint32_t *d_rows, const uint32_t *d_cols,
                             const float *d_vals, float *d_output,
                             uint32_t in_f, uint32_t nnz);

/* -- Affine matmul variants --------------------------------------------- */

/* bf16 activations (uint16_t bit patterns, [N, in_f]); fp32 output.
 * Up to 8 tokens, when in_f is a multiple of 128, the group size a multiple
 * of 64 and the operands 16-byte aligned: the tensor-core GEMV (codes and
 * activations exact in f16, exact products, fp32 accumulation).  From 9
 * tokens, when
 * in_f % 128 == 0 and the group size is a multiple of 64: the tcgen05
 * dequant-GEMM, which rounds W = code*scale + offset to bf16 before the
 * tensor-core product (fp32 accumulation): per output the error is at most
 * 2^-9 of sum |x_i w_i|.  Other shapes: the CUDA-core streaming GEMV (exact
 * products, fp32 accumulation). */
int hxq_affine_group_matmul_bf16(const uint16_t *d_x_bf16,
                                 const hxq_affine_tensor_t *tensor,
                                 float *d_output, uint32_t N, void *stream);
/* The same with the kernel chosen by the caller; -1 if that kernel cannot
 * take the shape or alignment (the tensor-core GEMV: more than 16 tokens,
 * in_f not a multiple of 128 or group size of 64, activations too long to
 * stage;
 * the GEMM: in_f not a multiple of 128, group size not a multiple of 64). */
#define HXQ_AFFINE_PATH_AUTO     0
#define HXQ_AFFINE_PATH_GEMV     1   /* CUDA-core streaming GEMV */
#define HXQ_AFFINE_PATH_TC_GEMV  2   /* tensor-core GEMV, 1..16 tokens (auto: up to 8) */
#define HXQ_AFFINE_PATH_GEMM     3   /* tcgen05 dequant-GEMM */
int hxq_affine_group_matmul_bf16_path(const uint16_t *d_x_bf16,
                                      const hxq_affine_tensor_t *tensor,
                                      float *d_output, uint32_t N, int path, void *stream);
/* The kernel hxq_affine_group_matmul_bf16 takes for these operands
 * (HXQ_AFFINE_PATH_GEMV, _TC_GEMV or _GEMM), which fixes its error bound;
 * -1 on a NULL tensor or N == 0. */
int hxq_affine_group_matmul_bf16_auto_path(const uint16_t *d_x_bf16,
                                           const hxq_affine_tensor_t *tensor, uint32_t N);
/* Waits for the device, then returns (and clears) the status words of the
 * tcgen05 dequant-GEMMs and the tensor-core GEMVs (affine and VQ): 0 when
 * every pipeline wait
 * completed, nonzero if one ran out of time (the kernel then unwinds
 * without writing results); -1 on a CUDA error. */
int hxq_cuda_affine_device_status(void);

/* -- Fused VQ-dequant matmul -------------------------------------------
 * No counterpart function in the reference library (its fused matmul is
 * affine only); the result is that of decompressing the image with
 * hxq_tensor_decompress and multiplying:
 *     d_y[n * ldy + o] = sum_i x[n, i] * W[o, i],  n < N, o < image rows,
 * W = codebook[index] + in-range sidecar deltas.  W is never written to
 * memory.  Images: 12-bit 2D-VQ with k = 4096 and in_features % 64 == 0
 * (HXQ_ERR_INVALID_ARG otherwise), resident or uploaded.  d_x: bf16 bit
 * patterns [N, in_features], 16-byte aligned; d_y: fp32, ldy >= rows.
 *   - Images with the matmul tables (HXQ_IMAGE_MATMUL), up to
 *     HXQ_VQ_MATMUL_TC_MAX tokens: the tensor-core GEMV, where the
 *     activations fit its shared memory whole or in two K parts
 *     (in_features 11008: up to 13 tokens); otherwise, and for more tokens:
 *     the tcgen05 dequant-GEMM.  Both use each weight rounded to bf16 (the bf16
 *     codebook pair, or bf16 of the sidecar-corrected weight):
 *     |error| <= 2^-9 sum_i |x_i w_i| per output, fp32 accumulation.
 *   - Images without the tables: the fused GEMV with exact fp32 weights
 *     and fp32 accumulation.
 * Stream-ordered on `stream` (0: the legacy default stream); no sync. */
#define HXQ_VQ_MATMUL_GEMV_MAX 4
#define HXQ_VQ_MATMUL_TC_MAX 16
hxq_error_t hxq_cuda_vq_matmul(const hxq_cuda_image_t *img, const uint16_t *d_x_bf16,
                               uint32_t N, float *d_y, uint32_t ldy, void *stream);
/* The same with the kernel chosen by the caller: path 0 the exact fp32
 * GEMV, 1 the tcgen05 GEMM, 2 the tensor-core GEMV (1..16 tokens); 1 and 2
 * need the image's matmul tables (HXQ_ERR_INVALID_ARG otherwise). */
hxq_error_t hxq_cuda_vq_matmul_path(const hxq_cuda_image_t *img, const uint16_t *d_x_bf16,
                                    uint32_t N, float *d_y, uint32_t ldy, int path, void *stream);

/* -- Outputs shared across the GPUs of one node ---------------------------
 * For a matmul whose output features are split over the ranks of one node:
 * every rank's output buffer is mapped into every other rank (CUDA IPC), the
 * matmul stores each output element into all of them (the *_multi entry
 * points), and a step's flags tell each rank when all peers' shards have
 * landed.  No reference counterpart (the reference has no multi-GPU code).
 *   hxq_cuda_ipc_alloc: cudaMalloc + zero fill + IPC handle (64 bytes);
 *   hxq_cuda_ipc_open / _close: map / unmap a peer's allocation;
 *   hxq_cuda_peer_signal: after this step's matmuls on `stream`, add one to
 *     *d_counter (this rank's step count, device memory) and store it, after
 *     a system-scope fence, into slot `rank` of every rank's flag array
 *     (peer_flags[p] = rank p's flags, mapped here; host array of world
 *     device pointers);
 *   hxq_cuda_peer_wait: on `stream`, wait until every slot of this rank's
 *     flags has reached *d_counter; bounded (about two seconds), then sets
 *     *d_status nonzero and returns.
 * Use two output buffers alternately (by step parity) so a rank never
 * overwrites outputs a peer may still be reading. */
#define HXQ_CUDA_MAX_PEERS 8
hxq_error_t hxq_cuda_ipc_alloc(size_t bytes, void **d_ptr, void *handle);
hxq_error_t hxq_cuda_ipc_open(const void *handle, void **d_peer);
hxq_error_t hxq_cuda_ipc_close(void *d_peer);
hxq_error_t hxq_cuda_ipc_free(void *d_ptr);
hxq_error_t hxq_cuda_peer_signal(uint32_t *const *peer_flags, uint32_t world, uint32_t rank,
                                 uint32_t *d_counter, void *stream);
hxq_error_t hxq_cuda_peer_wait(const uint32_t *d_flags, uint32_t world, const uint32_t *d_counter,
                               uint32_t *d_status, void *stream);

/* The fused matmuls with the same result stored into n_out buffers
 * (n_out <= HXQ_CUDA_MAX_PEERS; d_ys is a host array of device pointers,
 * local or peer-mapped), each [N, ldy]: output o of token n at
 * d_ys[k][n * ldy + o]. */
hxq_error_t hxq_cuda_vq_matmul_multi(const hxq_cuda_image_t *img, const uint16_t *d_x_bf16,
                                     uint32_t N, float *const *d_ys, uint32_t n_out,
                                     uint32_t ldy, void *stream);
int hxq_affine_group_matmul_bf16_multi(const uint16_t *d_x_bf16,
                                       const hxq_affine_tensor_t *tensor,
                                       float *const *d_ys, uint32_t n_out,
                                       uint32_t ldy, uint32_t N, void *stream);
/* A batch of n affine matmuls (e.g. a layer's projections) with bf16
 * activations d_xs[i] ([N, in_features of tensor i]) and outputs
 * d_ys[i * n_out + k] ([N, ldys[i]], k < n_out).  Up to 16 tokens the
 * matrices that suit the tensor-core GEMV, and at one token the remaining
 * ones that suit the streaming GEMV, share launches (up to 8 matrices per
 * launch), which pays the per-launch costs once for the batch; any other
 * matrix runs one call of its own.  Returns 0, or -1 on an error. */
/* A batch of n fused VQ matmuls (e.g. a layer's projections), outputs as
 * in hxq_affine_group_matmul_bf16_batch.  Up to HXQ_VQ_MATMUL_TC_MAX
 * tokens the images with matmul tables that suit the tensor-core GEMV share
 * its launches (up to 8 images per launch); up to HXQ_VQ_MATMUL_GEMV_MAX
 * tokens the others share exact-GEMV launches; anything else runs one call
 * per image. */
hxq_error_t hxq_cuda_vq_matmul_batch(uint32_t n, hxq_cuda_image_t *const *imgs,
                                     const uint16_t *const *d_xs, float *const *d_ys,
                                     uint32_t n_out, const uint32_t *ldys, uint32_t N,
                                     void *stream);
int hxq_affine_group_matmul_bf16_batch(uint32_t n, const hxq_affine_tensor_t *tensors,
                                       const uint16_t *const *d_xs, float *const *d_ys,
                                       uint32_t n_out, const uint32_t *ldys, uint32_t N,
                                       void *stream);

/* fp32 activations on a caller stream. */
int hxq_affine_group_matmul_async(const float *d_x,
                                  const hxq_affine_tensor_t *tensor,
                                  float *d_output, uint32_t N, void *stream);

/* -- Lloyd's algorithm on the GPU (compression side) -------------------
 * Device-pointer forms of hxq_lloyd_reassign / hxq_lloyd_assign_only
 * (hxq_lloyd.h; reference src/hxq_lloyd.c:41-308), stream-ordered, no
 * synchronisation: d_weights [n * d] fp32, d_codebook [k * d] fp32,
 * d_indices [n] uint8; k in [1, 256], d in {1, 2, 4, 8}, n < 2^32.
 * Assignment is bit-identical to the reference (fp32 in its order, first
 * minimum wins).  Centroid sums are exact-order-independent 64-bit
 * fixed-point sums (scale: a power of two from the largest |weight|), so
 * the updated codebook is reproducible run to run and within about one fp32
 * ulp of the reference's double sums (whose order depends on its thread
 * count).  *d_n_dead (device int, may be NULL) receives the dead-centroid
 * count.  Returns HXQ_LLOYD_* codes. */
int hxq_cuda_lloyd_assign(const float *d_weights, const float *d_codebook, uint8_t *d_indices, size_t n, int k,
                          int d, void *stream);
int hxq_cuda_lloyd_reassign(const float *d_weights, float *d_codebook, uint8_t *d_indices, size_t n, int k, int d,
                            int *d_n_dead, void *stream);

/* -- PolarQuant rotation on the GPU ---------------------------------------
 * In place on d_values [n_vectors * head_dim]: rotate = each vector times
 * Q^T, unrotate = times Q (d_Q [head_dim * head_dim] row-major, device).
 * Each output is the reference's sequential fp32 sum (reference
 * src/polarquant.c:249-300), so results are bit-identical to it.
 * Stream-ordered.  HXQ_OK, HXQ_ERR_NULL_PTR, HXQ_ERR_INVALID_ARG
 * (head_dim == 0) or HXQ_ERR_CUDA. */
hxq_error_t hxq_cuda_pq_rotate(float *d_values, const float *d_Q, uint64_t n_vectors, uint32_t head_dim,
                               void *stream);
hxq_error_t hxq_cuda_pq_unrotate(float *d_values, const float *d_Q, uint64_t n_vectors, uint32_t head_dim,
                                 void *stream);

#ifdef __cplusplus
}
#endif

#endif /* HXQ_CUDA_H */
