// ref_coarse_shim.cu -- extern "C" entry point around the reference's own GPU
// coarse routing (coarse_handle_init / coarse_search / coarse_handle_release,
// cuda/search/cpu_fine/cpu_fine.h:252-278).
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile (target ref-coarse) compiles this
// file with the reference's sources as they lie in the reference tree
// (cuda/search/cpu_fine/ivf_search_cpu_fine.cu, cuda/l2norm/l2norm.cu,
// cuda/search/coarse/fusion_{l2,cos}_topk_warpsort.cu, cuda/utils.cu and the
// CPU fine kernels that file links against) and cuBLAS into
// oracle/_ref/libref_coarse.so.  tests/golden/make_route_golden.py runs it on
// a GPU to record the reference's probe lists for seeded inputs; no product
// path loads it.
#include <cuda_runtime.h>

#include "search/cpu_fine/cpu_fine.h"

extern "C" __attribute__((visibility("default"))) int ref_coarse_search(const float* h_centers, int nlist, int dim,
                                                                        const float* h_query, int nq, int nprobe,
                                                                        int* h_ids_out) {
    float* d_centers = nullptr;
    if (cudaMalloc(&d_centers, sizeof(float) * (size_t)nlist * dim) != cudaSuccess) return -1;
    if (cudaMemcpy(d_centers, h_centers, sizeof(float) * (size_t)nlist * dim, cudaMemcpyHostToDevice) !=
        cudaSuccess) {
        cudaFree(d_centers);
        return -2;
    }
    CoarseHandle h{};
    coarse_handle_init(&h, d_centers, nlist, dim);
    double co = 0.0, h2d = 0.0, d2h = 0.0;
    coarse_search(&h, h_query, nq, nprobe, /*distance_mode=*/0, h_ids_out, &co, &h2d, &d2h);
    coarse_handle_release(&h);
    cudaFree(d_centers);
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : -3;
}
