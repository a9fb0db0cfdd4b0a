/*
 * cuda_wrapper.h -- C memory and upload helpers of libinsitu_b200.so.
 *
 * Same names, argument order and struct layout as the reference's
 * cuda/cuda_wrapper.h:16-77, so C callers built against that header link
 * against this library unchanged.  Differences in behaviour:
 *   - no function exits or resets the device; failures are reported by
 *     cuda_check_last_error() / cuda_get_last_error_string();
 *   - cuda_memcpy_async_* use the calling thread's per-thread default stream.
 */
#ifndef INSITU_B200_CUDA_WRAPPER_H
#define INSITU_B200_CUDA_WRAPPER_H

#include <stdbool.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* cuda_wrapper.h:16 -- vectors per pinned staging buffer */
#define PIPELINE_CHUNK_SIZE 65536

/* cuda_wrapper.h:22-46 -- layout is part of the ABI */
typedef struct GpuPipelineContext {
    int dimensions;
    size_t chunk_capacity;
    size_t total_uploaded;
    float* h_vec_buffers[2];   /* pinned host staging buffers */
    size_t current_counts[2];  /* vectors held by each buffer */
    int active_buf_idx;        /* buffer the host fills next */
    void* events[2];           /* cudaEvent_t per buffer */
    float* d_vectors_base;     /* destination in device memory */
} GpuPipelineContext;

bool cuda_is_available(void);                                  /* :51 */
void** cuda_malloc(void** d_ptr, size_t size);                 /* :54 returns d_ptr, *d_ptr NULL on failure */
void* cuda_alloc_pinned(size_t size);                          /* :55 */
void cuda_free_pinned(void* ptr);                              /* :56 */
void cuda_free(void* d_ptr);                                   /* :57 */
void cuda_memcpy_h2d(void* d_dst, const void* h_src, size_t size);        /* :58 */
void cuda_memcpy_d2h(void* h_dst, const void* d_src, size_t size);        /* :59 */
void cuda_memcpy_async_h2d(void* d_dst, const void* h_src, size_t size);  /* :60 */
void cuda_memcpy_async_d2h(void* h_dst, const void* d_src, size_t size);  /* :61 */
void cuda_cleanup_memory(float* d_query_batch, int* d_cluster_size, float* d_cluster_vectors,
                         float* d_cluster_centers, int* d_initial_indices, float* d_topk_dist,
                         int* d_topk_index);                   /* :64-65 frees the non-NULL ones */

/* :68-72 -- double-buffered pinned upload of fp32 vectors into d_vec_ptr */
void cuda_pipeline_init(GpuPipelineContext* ctx, int dim, size_t total_vectors, float* d_vec_ptr);
void cuda_pipeline_flush(GpuPipelineContext* ctx);
void cuda_pipeline_flush_vectors_only(GpuPipelineContext* ctx);
void cuda_pipeline_free(GpuPipelineContext* ctx);

void cuda_device_synchronize(void);                            /* :75 */
const char* cuda_get_last_error_string(void);                  /* :76 */
bool cuda_check_last_error(void);                              /* :77 true when an error is pending */

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* INSITU_B200_CUDA_WRAPPER_H */
