// select.cu -- per-query top-R over the candidate buffers filled by the scans.
//
// Replaces the reference's group bitonic merges with host syncs between
// rounds (updates/pq_update.cu:91-115, 944-967) and the per-thread heap
// merge of the CPU path (cpu_fine_kernels_v3_u8.cpp:574-592): one CTA per
// query selects the R smallest keys of its buffer and sorts them (ties at the
// R-th key are filled with copies of it, as a bounded heap would keep them).
#include "launch.h"

namespace isb {

namespace {


__global__ void reset_kernel(int32_t* cnt, unsigned long long* thr, int nq) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < nq) {
        cnt[i] = 0;
        thr[i] = 0x7FFFFFFFFFFFFFFFull;   // no bound yet: above every key, and ordered as a signed int64
                                         // so shards can exchange bounds with an int64 minimum
    }
}

// One CTA per query.  Buffers of up to kSelT * kSelItems keys go to
// registers (one coalesced read) and the R-th key is found by a radix descent
// over the registers; longer buffers are read from global memory on every
// pass.  The keys below the R-th are compacted to shared memory and only
// those R are sorted -- or written as they are when the consumer does not
// need the order (sorted == 0: the single-GPU rerank, which removes repeated
// positions by hashing and selects its top-k itself).
constexpr int kSelT = 256;
constexpr int kSelItems = 16;

__global__ void __launch_bounds__(kSelT) select_top_r_kernel(const uint64_t* __restrict__ keys,
                                                             const int32_t* __restrict__ cnt, int cap, int R,
                                                             uint64_t* __restrict__ out, int sorted) {
    extern __shared__ uint64_t s[];
    __shared__ int hist[256];
    __shared__ int bc[4];
    __shared__ unsigned long long mm[64];
    __shared__ int s_cnt;
    const int q = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
    int n = cnt[q];
    if (n > cap) n = cap;
    const uint64_t* kk = keys + (size_t)q * cap;
    int Rp = 1;
    while (Rp < R) Rp <<= 1;
    if (n <= R) {                     // every key is kept
        if (!sorted) {
            for (int i = tid; i < R; i += kSelT) out[(size_t)q * R + i] = i < n ? kk[i] : kKeyNone;
            return;
        }
        for (int i = tid; i < Rp; i += kSelT) s[i] = i < n ? kk[i] : kKeyNone;
        block_bitonic_sort<kSelT>(s, Rp);
        for (int i = tid; i < R; i += kSelT) out[(size_t)q * R + i] = s[i];
        return;
    }
    if (tid == 0) s_cnt = 0;
    uint64_t kap;
    if (n <= kSelT * kSelItems) {
        uint64_t v[kSelItems];
#pragma unroll
        for (int e = 0; e < kSelItems; ++e) {
            const int i = tid + kSelT * e;
            v[e] = i < n ? kk[i] : kKeyNone;
        }
        kap = block_kth_items<kSelT, kSelItems>([&](int e) { return v[e]; }, R, kKeyNone - 1, hist, bc, mm);
        // keys below kappa (fewer than R), placed with one shared atomic per warp
#pragma unroll
        for (int e = 0; e < kSelItems; ++e) {
            const bool take = v[e] < kap;
            const unsigned ball = __ballot_sync(0xffffffffu, take);
            if (ball == 0) continue;
            int base = 0;
            if (lane == 0) base = atomicAdd(&s_cnt, __popc(ball));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (take) s[base + __popc(ball & ((1u << lane) - 1u))] = v[e];
        }
    } else {
        kap = block_kth_key<kSelT>([&](int i) -> uint64_t { return kk[i]; }, n, R, kKeyNone, hist, bc);
        __syncthreads();
        for (int i = tid; i < n; i += kSelT) {
            const uint64_t k = kk[i];
            if (k < kap) s[atomicAdd(&s_cnt, 1)] = k;
        }
    }
    __syncthreads();
    const int cl = s_cnt;
    for (int i = cl + tid; i < Rp; i += kSelT) s[i] = i < R ? kap : kKeyNone;   // copies of kappa fill to R
    if (sorted) block_bitonic_sort<kSelT>(s, Rp);
    else __syncthreads();
    for (int i = tid; i < R; i += kSelT) out[(size_t)q * R + i] = s[i];
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

cudaError_t select_top_r(CandBuf cb, int nq, uint64_t* out, cudaStream_t st, bool sorted) {
    if (nq <= 0) return cudaSuccess;
    int Rp = 1;
    while (Rp < cb.R) Rp <<= 1;
    const size_t smem = sizeof(uint64_t) * (size_t)Rp;
    if (smem > 64 * 1024) return cudaErrorInvalidValue;
    cudaError_t e =
        cudaFuncSetAttribute(select_top_r_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    if (e) return e;
    note_launch();
    select_top_r_kernel<<<nq, kSelT, smem, st>>>(cb.keys, cb.cnt, cb.cap, cb.R, out, sorted ? 1 : 0);
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
