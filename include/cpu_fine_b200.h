/*
 * cpu_fine_b200.h -- the C++-linkage part of the reference's host API,
 * served by libinsitu_b200.so, so that runners compiled against the
 * reference's headers link unchanged.
 *
 *   struct CoarseHandle, CoarseTimingBreakdown, coarse_handle_init/release,
 *   coarse_search, coarse_get_last_timing  -- cuda/search/cpu_fine/cpu_fine.h:232-278
 *   ivftensor::cpu_fine::cpu_fine_kernel_v3_u8[_touched]  -- cpu_fine_u8.h:47-77
 *   ivftensor::cpu_fine::cpu_fine_kernel_pq_resid          -- cpu_fine_pq_resid.h:69-94
 *   ivf_init_streaming_upload, ivf_append_cluster_data,
 *   ivf_finalize_streaming_upload                          -- cuda/search/ivf_search.cuh:330-355
 *
 * Same names, argument order, types and return meaning as the reference
 * (the C++ symbols are mangled identically).  The routing and the fine
 * searches run on the GPU: host arrays in, host arrays out.  The fine-search
 * functions upload the index arrays on every call (they take host arrays, as
 * the reference's CPU kernels do); a caller that searches one index many times
 * should load it once with ivf_u8_load / ivf_pq_load (insitu_b200.h).
 * Differences from the reference, on purpose:
 *   - top-k ties are broken by the smaller position (the reference's heaps
 *     keep whichever the thread schedule saw first);
 *   - bad arguments do not abort: coarse_search leaves its output untouched
 *     and the kernels return -1, with the message in ivf_global_last_error();
 *   - num_threads is accepted and ignored (the work runs on the GPU).
 * The return value of the fine-search functions is the reference's
 * multiply-add count (sum over (query, probed list) of list size x dim for
 * uint8, x pq_M for stage 1 of residual PQ).
 */
#ifndef CPU_FINE_B200_H
#define CPU_FINE_B200_H

#ifndef __cplusplus
#error "cpu_fine_b200.h declares C++-linkage functions; C callers use insitu_b200.h"
#endif

#include <stdint.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

struct CoarseHandle {
    const float* d_centers;
    float* d_centers_norm;
    void* cublas_handle;
    int n_total_clusters;
    int dim;
    int distance_mode_cached;
};

struct CoarseTimingBreakdown {
    double query_h2d_ms = 0.0;
    double seq_init_ms = 0.0;
    double query_norm_ms = 0.0;
    double gemm_ms = 0.0;
    double topk_ms = 0.0;
    double cluster_d2h_ms = 0.0;
    double coarse_compute_ms = 0.0;
    double coarse_total_ms = 0.0;
};

void coarse_handle_init(CoarseHandle* h, const float* d_centers, int n_total_clusters, int dim);
void coarse_handle_release(CoarseHandle* h);
void coarse_search(const CoarseHandle* h, const float* h_query, int n_query_batch, int n_probes, int distance_mode,
                   int* h_cluster_ids_out, double* out_coarse_ms, double* out_h2d_ms, double* out_d2h_ms);
const CoarseTimingBreakdown* coarse_get_last_timing();

/* Streaming upload of an fp32 index -- cuda/search/ivf_search.cuh:330-355 (C++
 * linkage there and here): the rows arrive cluster by cluster from the host,
 * finalize takes the centroids.  The index then serves
 * ivf_pipeline_stage2_compute with distance_mode 0 (L2) or 1 (cosine), routed
 * by cosine as the reference routes this path. */
void ivf_init_streaming_upload(void* idx_ctx_ptr, int n_total_clusters, int n_total_vectors, int n_dim);
void ivf_append_cluster_data(void* idx_ctx_ptr, int cluster_id, float* host_vector_data, int count,
                             int start_offset_idx);
void ivf_finalize_streaming_upload(void* idx_ctx_ptr, float* center_data_flat, int total_vectors_check);

namespace ivftensor {
namespace cpu_fine {

long long cpu_fine_kernel_v3_u8(const uint8_t* h_base_u8, const long long* h_cluster_offsets,
                                const int* h_cluster_counts, const uint8_t* h_query_u8,
                                const int* h_coarse_cluster_ids, int n_query, int dim, int n_total_clusters,
                                int n_probes, int topk, int num_threads, int* h_topk_local_idx, float* h_topk_dist);

long long cpu_fine_kernel_v3_u8_touched(const uint8_t* h_base_u8, const long long* h_cluster_offsets,
                                        const int* h_cluster_counts, const uint8_t* h_query_u8,
                                        const int* h_coarse_cluster_ids, int n_query, int dim, int n_total_clusters,
                                        int n_probes, int topk, int num_threads, int* h_topk_local_idx,
                                        float* h_topk_dist);

long long cpu_fine_kernel_pq_resid(const uint8_t* h_base_u8, const long long* h_cluster_offsets,
                                   const int* h_cluster_counts, const uint8_t* h_pq_codes, const float* h_codebook,
                                   const float* h_centroids, const uint8_t* h_query_u8, const float* h_query_fp32,
                                   const float* h_base_fp32, int use_float_rerank, const int* h_coarse_cluster_ids,
                                   int n_query, int dim, int n_total_clusters, int n_probes, int topk, int rerank_n,
                                   int pq_M, int pq_K, int num_threads, int* h_topk_local_idx, float* h_topk_dist,
                                   double* out_stage1_ms, double* out_stage2_ms);

}  // namespace cpu_fine
}  // namespace ivftensor

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#endif /* CPU_FINE_B200_H */
