/*
 * hxq_internal.h -- interface between the C host library (hxq_host.c) and
 * the CUDA runtime layer (hxq_cuda_rt.cu).  Internal; not installed.
 */
#ifndef HXQ_INTERNAL_H
#define HXQ_INTERNAL_H

#include "hxq.h"
#include "hxq_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* 1 when a CUDA device is visible. */
int  hxqi_cuda_available(void);
/* 1 when p is device (or managed) memory; never creates a CUDA context. */
int  hxqi_cuda_ptr_is_device(const void *p);
/* Drop the cached device image of t (loaders, free, init). */
void hxqi_cuda_forget_tensor(const hxq_tensor_t *t);
/* Device-arena registry. */
int  hxqi_cuda_is_arena(const hxq_shared_buffer_t *buf);
void hxqi_cuda_arena_forget(const hxq_shared_buffer_t *buf);
void hxqi_cuda_arena_release(hxq_shared_buffer_t *buf);
hxq_error_t hxqi_cuda_arena_reserve(hxq_shared_buffer_t *buf, size_t floats);
/* Synchronous GPU decompress of t into device memory d_out (fp32 when
 * bf16 == 0); *l2 receives the confidence on success. */
hxq_error_t hxqi_cuda_decompress(hxq_tensor_t *t, void *d_out, int bf16, float *l2);
/* GPU decompress, result copied into host memory h_out. */
hxq_error_t hxqi_cuda_decompress_to_host(hxq_tensor_t *t, float *h_out, float *l2);

#ifdef __cplusplus
}
#endif

#endif /* HXQ_INTERNAL_H */
