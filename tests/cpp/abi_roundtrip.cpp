// abi_roundtrip.cpp -- a C++ runner of the reference's host API, linked
// against libinsitu_b200.so.
//
// Compiled either against the reference's own headers (-DREF_HEADERS with the
// reference tree's cuda/ directory on the include path: proves that the
// mangled C++ symbols a reference runner needs are the ones this library
// exports) or against include/cpu_fine_b200.h (the same declarations, for
// hosts without the reference tree).  Run as
//     abi_roundtrip <dir>
// it reads an index that tests/test_cpp_abi.py wrote into <dir> in the
// reference's file formats (centroids, assign, codebook, codes, DiskANN u8bin
// base and queries), routes the queries with coarse_search, runs
// cpu_fine_kernel_pq_resid and cpu_fine_kernel_v3_u8_touched on the
// cluster-major arrays, and writes the results as raw int32/float files next
// to the inputs for the test to compare with the oracle.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#ifdef REF_HEADERS
#include "search/cpu_fine/cpu_fine.h"
#include "search/cpu_fine/cpu_fine_pq_resid.h"
#include "search/cpu_fine/cpu_fine_u8.h"
#else
#include "cpu_fine_b200.h"
#endif
#define INSITU_B200_NO_COARSE
#include "insitu_b200.h"

#include <cuda_runtime.h>

static bool write_file(const std::string& path, const void* p, size_t bytes) {
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) return false;
    const bool ok = std::fwrite(p, 1, bytes, f) == bytes;
    std::fclose(f);
    return ok;
}

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s <dir>\n", argv[0]);
        return 2;
    }
    const std::string dir = argv[1];
    int nlist = 0, dim = 0, M = 0, K = 0, dsub = 0, qd = 0, bd = 0;
    long long n = 0, ncodes = 0, nq = 0, nb = 0;
    // sizes first (NULL output), then the data
    if (ivf_read_centroids((dir + "/centroids.bin").c_str(), nullptr, 0, &nlist, &dim) < 0 ||
        ivf_read_assign((dir + "/assign.bin").c_str(), nullptr, 0, &n) < 0 ||
        ivf_read_codebook((dir + "/codebook.bin").c_str(), nullptr, 0, &M, &K, &dsub) < 0 ||
        ivf_read_codes((dir + "/codes.bin").c_str(), nullptr, 0, &ncodes, &M) < 0 ||
        ivf_read_u8bin((dir + "/base.u8bin").c_str(), nullptr, 0, &nb, &bd) < 0 ||
        ivf_read_u8bin((dir + "/query.u8bin").c_str(), nullptr, 0, &nq, &qd) < 0) {
        std::fprintf(stderr, "header: %s\n", ivf_global_last_error());
        return 1;
    }
    std::vector<float> cent((size_t)nlist * dim), cb((size_t)M * K * dsub);
    std::vector<int> assign((size_t)n);
    std::vector<uint8_t> codes((size_t)ncodes * M), base((size_t)nb * bd), qu8((size_t)nq * qd);
    if (ivf_read_centroids((dir + "/centroids.bin").c_str(), cent.data(), (long long)cent.size(), &nlist, &dim) < 0 ||
        ivf_read_assign((dir + "/assign.bin").c_str(), assign.data(), n, &n) < 0 ||
        ivf_read_codebook((dir + "/codebook.bin").c_str(), cb.data(), (long long)cb.size(), &M, &K, &dsub) < 0 ||
        ivf_read_codes((dir + "/codes.bin").c_str(), codes.data(), (long long)codes.size(), &ncodes, &M) < 0 ||
        ivf_read_u8bin((dir + "/base.u8bin").c_str(), base.data(), (long long)base.size(), &nb, &bd) < 0 ||
        ivf_read_u8bin((dir + "/query.u8bin").c_str(), qu8.data(), (long long)qu8.size(), &nq, &qd) < 0) {
        std::fprintf(stderr, "read: %s\n", ivf_global_last_error());
        return 1;
    }
    // the stable cluster-major layout of the assignment (dataset.cuh:559-592)
    std::vector<int> counts(nlist, 0), r2o((size_t)n);
    std::vector<long long> offsets(nlist, 0);
    for (long long i = 0; i < n; ++i) counts[assign[i]]++;
    for (int l = 1; l < nlist; ++l) offsets[l] = offsets[l - 1] + counts[l - 1];
    {
        std::vector<long long> cur(offsets);
        for (long long i = 0; i < n; ++i) r2o[(size_t)cur[assign[i]]++] = (int)i;
    }
    std::vector<uint8_t> base_cm((size_t)n * dim);
    for (long long p = 0; p < n; ++p) std::memcpy(&base_cm[(size_t)p * dim], &base[(size_t)r2o[p] * dim], dim);
    std::vector<float> qf((size_t)nq * dim);
    for (size_t i = 0; i < qf.size(); ++i) qf[i] = (float)qu8[i];

    const int nprobe = 6, topk = 10, rerank_n = 64;
    float* d_cent = nullptr;
    cudaMalloc(&d_cent, sizeof(float) * cent.size());
    cudaMemcpy(d_cent, cent.data(), sizeof(float) * cent.size(), cudaMemcpyHostToDevice);
    CoarseHandle h{};
    coarse_handle_init(&h, d_cent, nlist, dim);
    std::vector<int> probes((size_t)nq * nprobe, -7);
    double tc = 0, th = 0, td = 0;
    coarse_search(&h, qf.data(), (int)nq, nprobe, 0, probes.data(), &tc, &th, &td);
    const CoarseTimingBreakdown* tb = coarse_get_last_timing();
    if (probes[0] < 0 || !tb) {
        std::fprintf(stderr, "coarse_search: %s\n", ivf_global_last_error());
        return 1;
    }
    std::vector<int> pq_ids((size_t)nq * topk), u8_ids((size_t)nq * topk);
    std::vector<float> pq_dist((size_t)nq * topk), u8_dist((size_t)nq * topk);
    double s1 = 0, s2 = 0;
    const long long fma_pq = ivftensor::cpu_fine::cpu_fine_kernel_pq_resid(
        base_cm.data(), offsets.data(), counts.data(), codes.data(), cb.data(), cent.data(), qu8.data(), qf.data(),
        nullptr, 0, probes.data(), (int)nq, dim, nlist, nprobe, topk, rerank_n, M, K, 0, pq_ids.data(),
        pq_dist.data(), &s1, &s2);
    const long long fma_u8 = ivftensor::cpu_fine::cpu_fine_kernel_v3_u8_touched(
        base_cm.data(), offsets.data(), counts.data(), qu8.data(), probes.data(), (int)nq, dim, nlist, nprobe, topk,
        0, u8_ids.data(), u8_dist.data());
    coarse_handle_release(&h);
    cudaFree(d_cent);
    if (fma_pq < 0 || fma_u8 < 0) {
        std::fprintf(stderr, "fine search: %s\n", ivf_global_last_error());
        return 1;
    }
    const bool ok = write_file(dir + "/out_probes.i32", probes.data(), probes.size() * 4) &&
                    write_file(dir + "/out_pq_ids.i32", pq_ids.data(), pq_ids.size() * 4) &&
                    write_file(dir + "/out_pq_dist.f32", pq_dist.data(), pq_dist.size() * 4) &&
                    write_file(dir + "/out_u8_ids.i32", u8_ids.data(), u8_ids.size() * 4) &&
                    write_file(dir + "/out_u8_dist.f32", u8_dist.data(), u8_dist.size() * 4) &&
                    write_file(dir + "/out_r2o.i32", r2o.data(), r2o.size() * 4);
    std::printf("fma_pq %lld fma_u8 %lld\n", fma_pq, fma_u8);
    return ok ? 0 : 1;
}
