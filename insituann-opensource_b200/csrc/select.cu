// select.cu -- per-query top-R over the candidate buffers filled by the scans.
//
// Replaces the reference's group bitonic merges with host syncs between
// rounds (updates/pq_update.cu:91-115, 944-967) and the per-thread heap
// merge of the CPU path (cpu_fine_kernels_v3_u8.cpp:574-592): one CTA per
// query selects the R smallest keys of its buffer and sorts them.
#include "launch.h"

namespace isb {

namespace {

constexpr int kT = 512;
constexpr int kSortMax = 4096;   // buffers up to this size are sorted whole

__global__ void reset_kernel(int32_t* cnt, unsigned long long* thr, int nq) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < nq) {
        cnt[i] = 0;
        thr[i] = kKeyNone;
    }
}

__global__ void __launch_bounds__(kT) select_top_r_kernel(const uint64_t* __restrict__ keys,
                                                          const int32_t* __restrict__ cnt, int cap, int R,
                                                          uint64_t* __restrict__ out) {
    extern __shared__ uint64_t s[];
    __shared__ int hist[256];
    __shared__ int bc[4];
    __shared__ int s_cnt;
    const int q = blockIdx.x, tid = threadIdx.x;
    int n = cnt[q];
    if (n > cap) n = cap;
    const uint64_t* kk = keys + (size_t)q * cap;
    int Rp = 1;
    while (Rp < R) Rp <<= 1;
    if (n <= kSortMax) {
        int np = 1;
        while (np < n) np <<= 1;
        if (np < Rp) np = Rp;
        for (int i = tid; i < np; i += kT) s[i] = i < n ? kk[i] : kKeyNone;
        block_bitonic_sort<kT>(s, np);
    } else {
        auto keyf = [&](int i) -> uint64_t { return kk[i]; };
        uint64_t kap = block_kth_key<kT>(keyf, n, R, kKeyNone, hist, bc);
        if (tid == 0) s_cnt = 0;
        __syncthreads();
        for (int i = tid; i < n; i += kT) {
            uint64_t k = kk[i];
            if (k < kap) s[atomicAdd(&s_cnt, 1)] = k;
        }
        __syncthreads();
        int cl = s_cnt;
        for (int i = cl + tid; i < Rp; i += kT) s[i] = i < R ? kap : kKeyNone;
        block_bitonic_sort<kT>(s, Rp);
    }
    for (int i = tid; i < R; i += kT) out[(size_t)q * R + i] = s[i];
}

__global__ void keys_to_exact_kernel(const uint64_t* __restrict__ keys, int total, int32_t* ids, int32_t* dist,
                                     float* fdist) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    uint64_t k = keys[i];
    bool ok = k != kKeyNone;
    if (ids) ids[i] = ok ? (int32_t)key_lo(k) : -1;
    if (dist) dist[i] = ok ? (int32_t)key_hi(k) : 0x7fffffff;
    if (fdist) fdist[i] = ok ? (float)(int32_t)key_hi(k) : __int_as_float(0x7f800000);
}

}  // namespace

cudaError_t reset_candidates(CandBuf cb, int nq, cudaStream_t st) {
    if (nq <= 0) return cudaSuccess;
    note_launch();
    reset_kernel<<<(nq + 255) / 256, 256, 0, st>>>(cb.cnt, cb.thr, nq);
    return cudaGetLastError();
}

cudaError_t select_top_r(CandBuf cb, int nq, uint64_t* out, cudaStream_t st) {
    if (nq <= 0) return cudaSuccess;
    int Rp = 1;
    while (Rp < cb.R) Rp <<= 1;
    int elems = Rp > kSortMax ? Rp : kSortMax;
    size_t smem = sizeof(uint64_t) * (size_t)elems;
    if (smem > 64 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(select_top_r_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         64 * 1024);
    if (e) return e;
    note_launch();
    select_top_r_kernel<<<nq, kT, smem, st>>>(cb.keys, cb.cnt, cb.cap, cb.R, out);
    return cudaGetLastError();
}

cudaError_t keys_to_exact_results(const uint64_t* keys, int nq, int k, int32_t* ids, int32_t* dist, float* fdist,
                                  cudaStream_t st) {
    int total = nq * k;
    if (total <= 0) return cudaSuccess;
    note_launch();
    keys_to_exact_kernel<<<(total + 255) / 256, 256, 0, st>>>(keys, total, ids, dist, fdist);
    return cudaGetLastError();
}

}  // namespace isb
