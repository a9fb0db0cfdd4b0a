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
    int bc[16];
    int base;
    unsigned long long mm[64];
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

// Ascending bitonic sort of one 64-bit key per lane across the warp.
__device__ __forceinline__ uint64_t warp_sort32(uint64_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const uint64_t o = __shfl_xor_sync(0xffffffffu, v, j);
            const bool up = (lane & k) == 0, lower = (lane & j) == 0;
            v = lower == up ? (o < v ? o : v) : (o > v ? o : v);
        }
    }
    return v;
}

// Appends every key <= cut among ITEMS keys per thread held in registers
// (keyj(j), kKeyNone for none; j is a compile-time index after unrolling, so
// register arrays behind keyj stay in registers) with one atomic per warp:
// the warp's takes are counted by ballots first, then placed item by item.
template <int ITEMS, class KeyJ>
__device__ __forceinline__ void warp_append_items(KeyJ keyj, uint64_t cut, const CandBuf& cb, int q) {
    const int lane = threadIdx.x & 31;
    unsigned ball[ITEMS];
    int n = 0;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        ball[j] = __ballot_sync(0xffffffffu, keyj(j) <= cut);
        n += __popc(ball[j]);
    }
    if (n == 0) return;
    int base = 0;
    if (lane == 0) base = atomicAdd(cb.cnt + q, n);
    base = __shfl_sync(0xffffffffu, base, 0);
    uint64_t* out = cb.keys + (size_t)q * cb.cap;
    const unsigned below = (1u << lane) - 1u;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        if ((ball[j] >> lane) & 1u) {
            const int at = base + __popc(ball[j] & below);
            if (at < cb.cap) out[at] = keyj(j);
            else atomicExch(cb.overflow, 1);
        }
        base += __popc(ball[j]);
    }
}

// Block-wide totals of four per-thread counts with one barrier: each warp
// reduces in hardware and adds into cnt[4] (shared), which the caller zeroed
// before the previous barrier; every thread reads the four totals.
template <int T>
__device__ __forceinline__ int4 block_sum4_once(int4 v, int* cnt) {
    const unsigned a = __reduce_add_sync(0xffffffffu, (unsigned)v.x);
    const unsigned b = __reduce_add_sync(0xffffffffu, (unsigned)v.y);
    const unsigned c = __reduce_add_sync(0xffffffffu, (unsigned)v.z);
    const unsigned d = __reduce_add_sync(0xffffffffu, (unsigned)v.w);
    if ((threadIdx.x & 31) == 0) {
        if (a) atomicAdd(cnt, (int)a);
        if (b) atomicAdd(cnt + 1, (int)b);
        if (c) atomicAdd(cnt + 2, (int)c);
        if (d) atomicAdd(cnt + 3, (int)d);
    }
    __syncthreads();
    return make_int4(cnt[0], cnt[1], cnt[2], cnt[3]);
}

// Cut keys for up to Q = 4 queries at once, over ITEMS keys per thread in
// registers (key(e, q); all threads call it together).  For every query q in
// `active` (bit q), among its participants (keys <= upper[q], at least R of
// them) it finds cut[q] such that at least R participants are <= cut[q] and
// at most R + slack are: a valid new rank-R bound whose keys the caller can
// append without exceeding R + slack per call.
//
// A radix descent as in block_kth_each, but all queries share each pass's
// barriers, the first digit is the 8 bits just below the highest bit in which
// the query's participants differ (block min and max), and a query stops as
// soon as the bin holding its R-th key is small enough (so the cut is the end
// of that bin, not necessarily the R-th key itself).  Passes alternate
// between two histogram buffers so each takes two barriers.  hist: 2 * Q * 256
// ints of shared memory the caller may reuse afterwards only after a barrier;
// bc: 4 * Q ints; mm: 2 * Q * (T / 32) uint64.
template <int T, int ITEMS, int Q, class KeyF>
__device__ void block_cut_items(KeyF key, unsigned active, int R, int slack, const uint64_t (&upper)[Q],
                                int* hist, int* bc, unsigned long long* mm, uint64_t (&cut)[Q]) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int W = T / 32;
    for (int b = tid; b < Q * 256; b += T) hist[b] = 0;
    uint64_t lo[Q], hi[Q];
#pragma unroll
    for (int q = 0; q < Q; ++q) {
        lo[q] = kKeyNone;
        hi[q] = 0;
        if (!((active >> q) & 1u)) continue;
#pragma unroll
        for (int e = 0; e < ITEMS; ++e) {
            const uint64_t k = key(e, q);
            if (k <= upper[q]) {
                lo[q] = k < lo[q] ? k : lo[q];
                hi[q] = k > hi[q] ? k : hi[q];
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint64_t l2 = __shfl_xor_sync(0xffffffffu, lo[q], o);
            const uint64_t h2 = __shfl_xor_sync(0xffffffffu, hi[q], o);
            lo[q] = l2 < lo[q] ? l2 : lo[q];
            hi[q] = h2 > hi[q] ? h2 : hi[q];
        }
        if (lane == 0) {
            mm[(2 * q) * W + warp] = lo[q];
            mm[(2 * q + 1) * W + warp] = hi[q];
        }
    }
    __syncthreads();
    int shift[Q], need[Q];
    uint64_t prefix[Q], mask[Q];
    unsigned todo = 0;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
        shift[q] = 0;
        need[q] = R;
        prefix[q] = 0;
        mask[q] = 0;
        if (!((active >> q) & 1u)) continue;
#pragma unroll
        for (int w = 0; w < W; ++w) {
            const uint64_t l2 = mm[(2 * q) * W + w], h2 = mm[(2 * q + 1) * W + w];
            lo[q] = l2 < lo[q] ? l2 : lo[q];
            hi[q] = h2 > hi[q] ? h2 : hi[q];
        }
        if (lo[q] == hi[q]) {          // every participant holds the same key
            cut[q] = lo[q];
            continue;
        }
        const int top = 63 - __clzll((long long)(lo[q] ^ hi[q]));
        shift[q] = top >= 7 ? top - 7 : 0;
        mask[q] = top >= 63 ? 0ull : ~((2ull << top) - 1ull);
        prefix[q] = lo[q] & mask[q];
        todo |= 1u << q;
    }
    for (int pass = 0; todo; ++pass) {
        int* h = hist + (pass & 1) * (Q * 256);              // zeroed before the last barrier
#pragma unroll
        for (int e = 0; e < ITEMS; ++e) {
#pragma unroll
            for (int q = 0; q < Q; ++q) {
                if (!((todo >> q) & 1u)) continue;       // uniform over the block
                const uint64_t k = key(e, q);
                if (k <= upper[q] && (k & mask[q]) == prefix[q]) atomicAdd(&h[q * 256 + (int)((k >> shift[q]) & 255u)], 1);
            }
        }
        __syncthreads();
        {
            int* hn = hist + ((pass + 1) & 1) * (Q * 256);   // the next pass's buffer
            for (int b = tid; b < Q * 256; b += T) hn[b] = 0;
        }
        if (warp < Q && ((todo >> warp) & 1u)) {      // warp q finds the bin of query q's need-th key
            const int q = warp;
            int needq = 0;
#pragma unroll
            for (int qq = 0; qq < Q; ++qq) needq = qq == q ? need[qq] : needq;   // no dynamic register index
            int loc[8];
            int sum = 0;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                loc[jj] = h[q * 256 + lane * 8 + jj];
                sum += loc[jj];
            }
            const int incl = warp_incl_scan(sum);
            const unsigned ball = __ballot_sync(0xffffffffu, incl >= needq);
            const int src = __ffs(ball) - 1;
            if (lane == src) {
                int acc = incl - sum;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    if (acc + loc[jj] >= needq) {
                        bc[4 * q] = lane * 8 + jj;
                        bc[4 * q + 1] = acc;
                        bc[4 * q + 2] = loc[jj];
                        break;
                    }
                    acc += loc[jj];
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            if (!((todo >> q) & 1u)) continue;
            const int b = bc[4 * q], below = bc[4 * q + 1], cnt = bc[4 * q + 2];
            need[q] -= below;
            prefix[q] |= (uint64_t)b << shift[q];
            mask[q] |= (uint64_t)0xFFu << shift[q];
            if (cnt - need[q] <= slack) {          // keys <= end of this bin: R - need + cnt <= R + slack
                cut[q] = prefix[q] | ~mask[q];
                todo &= ~(1u << q);
            } else if (shift[q] == 0) {            // several participants share the final key
                cut[q] = prefix[q];
                todo &= ~(1u << q);
            } else {
                shift[q] = shift[q] >= 8 ? shift[q] - 8 : 0;
            }
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
