// cuda_wrapper.cu -- the reference's C memory/upload helpers (cuda/cuda_wrapper.h:16-77).
//
// Semantics kept: cuda_malloc returns its argument, pinned buffers are
// write-combined, the upload pipeline ping-pongs two pinned buffers and
// waits only for the buffer it is about to refill.  Errors never exit; the
// last one is kept per thread for cuda_get_last_error_string().
#include <cuda_runtime.h>
#include <stdio.h>

#include "../../include/cuda_wrapper.h"

namespace {
thread_local cudaError_t g_last = cudaSuccess;
inline void note(cudaError_t e) {
    if (e != cudaSuccess) g_last = e;
}
}  // namespace

extern "C" {

bool cuda_is_available(void) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return n > 0;
}

void** cuda_malloc(void** d_ptr, size_t size) {
    if (!d_ptr) return d_ptr;
    cudaError_t e = cudaMalloc(d_ptr, size);
    if (e != cudaSuccess) {
        *d_ptr = nullptr;
        note(e);
    }
    return d_ptr;
}

void* cuda_alloc_pinned(size_t size) {
    void* p = nullptr;
    cudaError_t e = cudaHostAlloc(&p, size, cudaHostAllocWriteCombined);
    if (e != cudaSuccess) {
        note(e);
        return nullptr;
    }
    return p;
}

void cuda_free_pinned(void* ptr) {
    if (ptr) note(cudaFreeHost(ptr));
}

void cuda_free(void* d_ptr) {
    if (d_ptr) note(cudaFree(d_ptr));
}

void cuda_memcpy_h2d(void* d_dst, const void* h_src, size_t size) {
    note(cudaMemcpy(d_dst, h_src, size, cudaMemcpyHostToDevice));
}

void cuda_memcpy_d2h(void* h_dst, const void* d_src, size_t size) {
    note(cudaMemcpy(h_dst, d_src, size, cudaMemcpyDeviceToHost));
}

void cuda_memcpy_async_h2d(void* d_dst, const void* h_src, size_t size) {
    note(cudaMemcpyAsync(d_dst, h_src, size, cudaMemcpyHostToDevice, cudaStreamPerThread));
}

void cuda_memcpy_async_d2h(void* h_dst, const void* d_src, size_t size) {
    note(cudaMemcpyAsync(h_dst, d_src, size, cudaMemcpyDeviceToHost, cudaStreamPerThread));
}

void cuda_cleanup_memory(float* d_query_batch, int* d_cluster_size, float* d_cluster_vectors,
                         float* d_cluster_centers, int* d_initial_indices, float* d_topk_dist, int* d_topk_index) {
    void* ps[7] = {d_query_batch, d_cluster_size, d_cluster_vectors, d_cluster_centers,
                   d_initial_indices, d_topk_dist, d_topk_index};
    for (void* p : ps)
        if (p) note(cudaFree(p));
}

void cuda_pipeline_init(GpuPipelineContext* ctx, int dim, size_t total_vectors, float* d_vec_ptr) {
    (void)total_vectors;
    if (!ctx) return;
    ctx->dimensions = dim;
    ctx->chunk_capacity = PIPELINE_CHUNK_SIZE;
    ctx->total_uploaded = 0;
    ctx->active_buf_idx = 0;
    ctx->d_vectors_base = d_vec_ptr;
    for (int i = 0; i < 2; ++i) {
        ctx->h_vec_buffers[i] = nullptr;
        ctx->current_counts[i] = 0;
        ctx->events[i] = nullptr;
        void* p = nullptr;
        cudaError_t e = cudaHostAlloc(&p, ctx->chunk_capacity * (size_t)dim * sizeof(float),
                                      cudaHostAllocWriteCombined);
        if (e != cudaSuccess) {
            note(e);
            p = nullptr;
        }
        ctx->h_vec_buffers[i] = (float*)p;
        cudaEvent_t ev = nullptr;
        note(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        if (ev) note(cudaEventRecord(ev, cudaStreamPerThread));
        ctx->events[i] = (void*)ev;
    }
}

void cuda_pipeline_flush_vectors_only(GpuPipelineContext* ctx) {
    if (!ctx) return;
    const int cur = ctx->active_buf_idx;
    if (ctx->current_counts[cur] == 0 || !ctx->h_vec_buffers[cur]) return;
    const size_t bytes = ctx->current_counts[cur] * (size_t)ctx->dimensions * sizeof(float);
    float* dst = ctx->d_vectors_base + ctx->total_uploaded * (size_t)ctx->dimensions;
    note(cudaMemcpyAsync(dst, ctx->h_vec_buffers[cur], bytes, cudaMemcpyHostToDevice, cudaStreamPerThread));
    note(cudaEventRecord((cudaEvent_t)ctx->events[cur], cudaStreamPerThread));
    ctx->total_uploaded += ctx->current_counts[cur];
    ctx->current_counts[cur] = 0;
    const int nxt = 1 - cur;
    if (ctx->events[nxt]) note(cudaEventSynchronize((cudaEvent_t)ctx->events[nxt]));
    ctx->active_buf_idx = nxt;
}

void cuda_pipeline_flush(GpuPipelineContext* ctx) { cuda_pipeline_flush_vectors_only(ctx); }

void cuda_pipeline_free(GpuPipelineContext* ctx) {
    if (!ctx) return;
    note(cudaStreamSynchronize(cudaStreamPerThread));
    for (int i = 0; i < 2; ++i) {
        if (ctx->h_vec_buffers[i]) {
            note(cudaFreeHost(ctx->h_vec_buffers[i]));
            ctx->h_vec_buffers[i] = nullptr;
        }
        if (ctx->events[i]) {
            note(cudaEventDestroy((cudaEvent_t)ctx->events[i]));
            ctx->events[i] = nullptr;
        }
    }
}

void cuda_device_synchronize(void) { note(cudaDeviceSynchronize()); }

const char* cuda_get_last_error_string(void) {
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = g_last;
    g_last = cudaSuccess;
    return e == cudaSuccess ? "no error" : cudaGetErrorString(e);
}

bool cuda_check_last_error(void) {
    cudaError_t e = cudaPeekAtLastError();
    return e != cudaSuccess || g_last != cudaSuccess;
}

}  // extern "C"
