// cpp_abi.cu -- the C++-linkage entry points of include/cpu_fine_b200.h: the
// reference's coarse routing handle API (cuda/search/cpu_fine/cpu_fine.h:232-278)
// and its fine-search kernels (cpu_fine_u8.h:47-77, cpu_fine_pq_resid.h:69-94),
// served on the GPU through the C ABI.  Runners compiled against the
// reference's headers resolve to these symbols.
#include <cuda_runtime.h>

#include <chrono>
#include <cstring>
#include <string>
#include <vector>

#define INSITU_B200_NO_COARSE
#include "../../include/insitu_b200.h"
#include "../../include/cpu_fine_b200.h"

namespace isb {
void coarse_init_fwd(void* h, const float* d_centers, int n, int dim);
void coarse_release_fwd(void* h);
void coarse_search_fwd(const void* h, const float* q, int nq, int np, int mode, int* out, double* a, double* b,
                       double* c);
const void* coarse_timing_fwd();
void set_global_error(const std::string& msg);
}  // namespace isb

void coarse_handle_init(CoarseHandle* h, const float* d_centers, int n_total_clusters, int dim) {
    isb::coarse_init_fwd(h, d_centers, n_total_clusters, dim);
}

void coarse_handle_release(CoarseHandle* h) { isb::coarse_release_fwd(h); }

void coarse_search(const CoarseHandle* h, const float* h_query, int n_query_batch, int n_probes, int distance_mode,
                   int* h_cluster_ids_out, double* out_coarse_ms, double* out_h2d_ms, double* out_d2h_ms) {
    isb::coarse_search_fwd(h, h_query, n_query_batch, n_probes, distance_mode, h_cluster_ids_out, out_coarse_ms,
                           out_h2d_ms, out_d2h_ms);
}

const CoarseTimingBreakdown* coarse_get_last_timing() {
    return static_cast<const CoarseTimingBreakdown*>(isb::coarse_timing_fwd());
}

namespace {

double ms_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

// the reference's multiply-add count: every (query, valid probe) pair costs
// list size x per_vector
long long mac_count(const int* counts, const int* probes, int nq, int nprobe, int nlist, long long per_vector) {
    long long s = 0;
    for (size_t i = 0; i < (size_t)nq * nprobe; ++i)
        if (probes[i] >= 0 && probes[i] < nlist) s += (long long)counts[probes[i]] * per_vector;
    return s;
}

// total vectors of a cluster-major layout: the end of the furthest list
long long layout_rows(const long long* offsets, const int* counts, int nlist) {
    long long n = 0;
    for (int l = 0; l < nlist; ++l)
        if (counts[l] > 0) n = std::max(n, offsets[l] + (long long)counts[l]);
    return n;
}

// runs f(idx, batch) with fresh contexts; -1 (message set) on any failure
template <class F>
long long with_contexts(int max_nq, int d, int nprobe, int k, int nlist, F&& f) {
    void* idx = ivf_create_index_context();
    void* b = idx ? ivf_create_batch_context(max_nq, d, nprobe, k, nlist) : nullptr;
    long long rc = -1;
    if (idx && b) {
        rc = f(idx, b);
        if (rc < 0) {
            const char* m = ivf_last_error(b);
            if (!m || !m[0]) m = ivf_last_error(idx);
            isb::set_global_error(std::string("cpu_fine kernel on the GPU: ") + (m ? m : ""));
        }
    } else {
        isb::set_global_error("cpu_fine kernel on the GPU: context creation failed");
    }
    if (b) ivf_destroy_batch_context(b);
    if (idx) ivf_destroy_index_context(idx);
    return rc;
}

long long exact_u8(const uint8_t* base, const long long* offsets, const int* counts, const uint8_t* q_u8,
                   const int* probes, int nq, int dim, int nlist, int nprobe, int topk, int* out_idx,
                   float* out_dist) {
    if (!base || !offsets || !counts || !q_u8 || !probes || !out_idx || !out_dist || nq <= 0 || nprobe <= 0 ||
        topk <= 0 || nlist <= 0) {
        isb::set_global_error("cpu_fine_kernel_v3_u8: bad arguments");
        return -1;
    }
    const long long n = layout_rows(offsets, counts, nlist);
    std::vector<float> qf((size_t)nq * dim);
    for (size_t i = 0; i < qf.size(); ++i) qf[i] = (float)q_u8[i];
    std::vector<float> cent((size_t)nlist * dim, 1.0f);    // routing is not used: probes are given
    return with_contexts(nq, dim, nprobe, topk, nlist, [&](void* idx, void* b) -> long long {
        if (ivf_u8_load(idx, base, offsets, counts, nullptr, cent.data(), nlist, n, dim) != IVF_OK) return -1;
        ivf_pipeline_stage1_prepare(b, qf.data(), nq);
        if (ivf_set_probes(b, probes, nq, nprobe) != IVF_OK) return -1;
        if (ivf_u8_search(b, idx, nq, nprobe, topk, 0) != IVF_OK) return -1;
        ivf_pipeline_get_results(b, out_dist, out_idx, nq, topk);
        if (ivf_last_error(b)[0]) return -1;
        return mac_count(counts, probes, nq, nprobe, nlist, dim);
    });
}

}  // namespace

namespace ivftensor {
namespace cpu_fine {

long long cpu_fine_kernel_v3_u8(const uint8_t* h_base_u8, const long long* h_cluster_offsets,
                                const int* h_cluster_counts, const uint8_t* h_query_u8,
                                const int* h_coarse_cluster_ids, int n_query, int dim, int n_total_clusters,
                                int n_probes, int topk, int num_threads, int* h_topk_local_idx, float* h_topk_dist) {
    (void)num_threads;
    return exact_u8(h_base_u8, h_cluster_offsets, h_cluster_counts, h_query_u8, h_coarse_cluster_ids, n_query, dim,
                    n_total_clusters, n_probes, topk, h_topk_local_idx, h_topk_dist);
}

long long cpu_fine_kernel_v3_u8_touched(const uint8_t* h_base_u8, const long long* h_cluster_offsets,
                                        const int* h_cluster_counts, const uint8_t* h_query_u8,
                                        const int* h_coarse_cluster_ids, int n_query, int dim, int n_total_clusters,
                                        int n_probes, int topk, int num_threads, int* h_topk_local_idx,
                                        float* h_topk_dist) {
    (void)num_threads;
    return exact_u8(h_base_u8, h_cluster_offsets, h_cluster_counts, h_query_u8, h_coarse_cluster_ids, n_query, dim,
                    n_total_clusters, n_probes, topk, h_topk_local_idx, h_topk_dist);
}

long long cpu_fine_kernel_pq_resid(const uint8_t* h_base_u8, const long long* h_cluster_offsets,
                                   const int* h_cluster_counts, const uint8_t* h_pq_codes, const float* h_codebook,
                                   const float* h_centroids, const uint8_t* h_query_u8, const float* h_query_fp32,
                                   const float* h_base_fp32, int use_float_rerank, const int* h_coarse_cluster_ids,
                                   int n_query, int dim, int n_total_clusters, int n_probes, int topk, int rerank_n,
                                   int pq_M, int pq_K, int num_threads, int* h_topk_local_idx, float* h_topk_dist,
                                   double* out_stage1_ms, double* out_stage2_ms) {
    (void)num_threads;
    (void)h_query_u8;      // the u8 rerank rounds the fp32 queries the same way (make_query_u8)
    const bool f32 = use_float_rerank != 0;
    if (!h_cluster_offsets || !h_cluster_counts || !h_pq_codes || !h_codebook || !h_centroids || !h_query_fp32 ||
        !h_coarse_cluster_ids || !h_topk_local_idx || !h_topk_dist || (f32 ? !h_base_fp32 : !h_base_u8) ||
        n_query <= 0 || n_probes <= 0 || topk <= 0 || rerank_n <= 0 || pq_M <= 0 || dim % pq_M != 0) {
        isb::set_global_error("cpu_fine_kernel_pq_resid: bad arguments");
        return -1;
    }
    const long long n = layout_rows(h_cluster_offsets, h_cluster_counts, n_total_clusters);
    const auto t0 = std::chrono::steady_clock::now();
    double load_ms = 0.0;
    const long long rc = with_contexts(n_query, dim, n_probes, topk, n_total_clusters, [&](void* idx, void* b) {
        if (ivf_pq_load(idx, h_centroids, h_codebook, pq_M, pq_K, dim / pq_M, h_pq_codes, h_cluster_offsets,
                        h_cluster_counts, nullptr, f32 ? nullptr : h_base_u8, f32 ? h_base_fp32 : nullptr,
                        n_total_clusters, n, dim) != IVF_OK)
            return -1ll;
        load_ms = ms_since(t0);
        ivf_pipeline_stage1_prepare(b, const_cast<float*>(h_query_fp32), n_query);
        if (ivf_set_probes(b, h_coarse_cluster_ids, n_query, n_probes) != IVF_OK) return -1ll;
        if (ivf_pq_search(b, idx, n_query, n_probes, topk, rerank_n, 0, 0, 0) != IVF_OK) return -1ll;
        ivf_pipeline_get_results(b, h_topk_dist, h_topk_local_idx, n_query, topk);
        if (ivf_last_error(b)[0]) return -1ll;
        return mac_count(h_cluster_counts, h_coarse_cluster_ids, n_query, n_probes, n_total_clusters, pq_M);
    });
    // the GPU search is one pass; the upload is reported as stage 1, the search as stage 2
    if (out_stage1_ms) *out_stage1_ms = load_ms;
    if (out_stage2_ms) *out_stage2_ms = ms_since(t0) - load_ms;
    return rc;
}

}  // namespace cpu_fine
}  // namespace ivftensor
