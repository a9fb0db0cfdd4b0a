// emit.cuh -- block-level candidate filter shared by the exact and PQ scans.
//
// After a CTA has the distances of one chunk of an inverted list for one
// query, only keys that can still be among the query's R best are kept:
//   * keys above the query's running bound thr[q] are dropped;
//   * if more than R keys remain, the R-th smallest (kappa) is found by radix
//     selection, thr[q] is lowered to kappa (atomicMin) and only keys
//     <= kappa are kept.
// Survivors are appended to the query's candidate buffer with one atomic per
// CTA.  thr[q] is always >= the true rank-R key of the query, so no key of
// the final top-R is ever dropped, whatever the order in which chunks run.
#pragma once

#include "internal.cuh"

namespace isb {

struct EmitSmem {
    int hist[256];
    int scratch[4 * 33];
    int bc[4];
    int base;
};

template <int T, class KeyFn>
__device__ void block_filter_emit(KeyFn keyf, int n, const CandBuf& cb, int q, EmitSmem& sm) {
    const int tid = threadIdx.x;
    unsigned long long* thrp = cb.thr + q;
    const uint64_t thr = *((volatile unsigned long long*)thrp);
    int c = 0;
    for (int i = tid; i < n; i += T) c += (keyf(i) <= thr) ? 1 : 0;
    int total = block_sum<T>(c, sm.scratch);
    if (total == 0) return;
    uint64_t cut = thr;
    if (total > cb.R) {
        uint64_t kap = block_kth_key<T>(keyf, n, cb.R, thr, sm.hist, sm.bc);
        cut = kap < thr ? kap : thr;
        if (tid == 0) atomicMin(thrp, (unsigned long long)cut);
        c = 0;
        for (int i = tid; i < n; i += T) c += (keyf(i) <= cut) ? 1 : 0;
    }
    int tot;
    int excl = block_excl_scan<T>(c, sm.scratch, &tot);
    if (tid == 0) sm.base = atomicAdd(cb.cnt + q, tot);
    __syncthreads();
    const int base = sm.base;
    if (base + tot > cb.cap && tid == 0) atomicExch(cb.overflow, 1);
    uint64_t* out = cb.keys + (size_t)q * cb.cap;
    int j = base + excl;
    for (int i = tid; i < n; i += T) {
        uint64_t k = keyf(i);
        if (k <= cut) {
            if (j < cb.cap) out[j] = k;
            ++j;
        }
    }
    __syncthreads();
}

// Sum over the block of four ints per thread.  scratch: >= 4 * 33 ints.
template <int T>
__device__ __forceinline__ int4 block_sum4(int4 v, int* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int W = T / 32;
    v.x = warp_sum(v.x);
    v.y = warp_sum(v.y);
    v.z = warp_sum(v.z);
    v.w = warp_sum(v.w);
    if (lane == 0) {
        scratch[warp] = v.x;
        scratch[32 + warp] = v.y;
        scratch[64 + warp] = v.z;
        scratch[96 + warp] = v.w;
    }
    __syncthreads();
    int4 r = make_int4(0, 0, 0, 0);
#pragma unroll
    for (int w = 0; w < W; ++w) {
        r.x += scratch[w];
        r.y += scratch[32 + w];
        r.z += scratch[64 + w];
        r.w += scratch[96 + w];
    }
    __syncthreads();
    return r;
}

// Appends, warp by warp, every key k(i) <= cut of the items i = threadIdx.x +
// j*T (j < ITEMS, i < n) to the query's candidate buffer: one atomic per warp
// and item round, no block-wide synchronisation.
template <int T, int ITEMS, class KeyFn>
__device__ __forceinline__ void warp_append(KeyFn keyf, int n, uint64_t cut, const CandBuf& cb, int q) {
    const int lane = threadIdx.x & 31;
    uint64_t* out = cb.keys + (size_t)q * cb.cap;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        const int i = threadIdx.x + j * T;
        uint64_t k = kKeyNone;
        bool take = false;
        if (i < n) {
            k = keyf(i);
            take = k <= cut;
        }
        const unsigned ball = __ballot_sync(0xffffffffu, take);
        if (ball == 0) continue;
        int base = 0;
        if (lane == 0) base = atomicAdd(cb.cnt + q, __popc(ball));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (take) {
            const int at = base + __popc(ball & ((1u << lane) - 1u));
            if (at < cb.cap) out[at] = k;
            else atomicExch(cb.overflow, 1);
        }
    }
}

// Next (query, list) pair from the global work counter; -1 when done.
// All threads of the CTA receive the same value.
__device__ __forceinline__ int next_item(int* counter, int total, int* s_item) {
    __syncthreads();
    if (threadIdx.x == 0) *s_item = atomicAdd(counter, 1);
    __syncthreads();
    int it = *s_item;
    return it < total ? it : -1;
}

}  // namespace isb
