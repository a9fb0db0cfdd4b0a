// ref_shim.cpp -- extern "C" entry points around the reference's own CPU kernels.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference sources exactly as they lie in the reference tree
//   cuda/search/cpu_fine/cpu_fine_kernels_v3_u8.cpp   (Exact-CPU u8 fine search)
//   cuda/search/cpu_fine/cpu_fine_kernels_pq_resid.cpp (CPU residual PQ + rerank)
// into oracle/_ref/libref_cpu_fine.so.  It is used to pin the oracle
// restatement and as the timed CPU baseline ("kind": "reference").
#include <cstdint>

#include "search/cpu_fine/cpu_fine_u8.h"
#include "search/cpu_fine/cpu_fine_pq_resid.h"

extern "C" {

// cuda/search/cpu_fine/cpu_fine_u8.h:63-77
__attribute__((visibility("default"))) long long ref_cpu_fine_kernel_v3_u8_touched(
    const uint8_t* base_u8, const long long* offsets, const int* counts, const uint8_t* q_u8,
    const int* probes, int nq, int dim, int nlist, int nprobe, int topk, int num_threads,
    int* out_local_idx, float* out_dist) {
    return ivftensor::cpu_fine::cpu_fine_kernel_v3_u8_touched(
        base_u8, offsets, counts, q_u8, probes, nq, dim, nlist, nprobe, topk, num_threads,
        out_local_idx, out_dist);
}

// cuda/search/cpu_fine/cpu_fine_pq_resid.h:69-94
__attribute__((visibility("default"))) long long ref_cpu_fine_kernel_pq_resid(
    const uint8_t* base_u8, const long long* offsets, const int* counts, const uint8_t* codes,
    const float* codebook, const float* centroids, const uint8_t* q_u8, const float* q_f32,
    const float* base_f32, int use_float_rerank, const int* probes, int nq, int dim, int nlist,
    int nprobe, int topk, int rerank_n, int pq_m, int pq_k, int num_threads, int* out_local_idx,
    float* out_dist, double* stage1_ms, double* stage2_ms) {
    return ivftensor::cpu_fine::cpu_fine_kernel_pq_resid(
        base_u8, offsets, counts, codes, codebook, centroids, q_u8, q_f32, base_f32,
        use_float_rerank, probes, nq, dim, nlist, nprobe, topk, rerank_n, pq_m, pq_k, num_threads,
        out_local_idx, out_dist, stage1_ms, stage2_ms);
}

}  // extern "C"
