// internal.cuh -- device-side building blocks shared by the hot-path kernels.
//
// Every ranking in this library is a total order on 64-bit keys
//     key = (distance bits << 32) | id
// where the distance is a non-negative float (IEEE bits are then monotone) or a
// non-negative int32, and the id is a list id, a cluster-major position or an
// original vector id.  Ties between equal distances therefore go to the
// smaller id, independent of thread schedule, which is what makes the GPU
// results bit-identical to the CPU restatement.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace isb {

constexpr int kCodes = 256;          // centroids per PQ sub-quantizer (8-bit codes)
constexpr uint64_t kKeyNone = ~0ull; // empty slot / "no bound yet"

__device__ __forceinline__ uint64_t make_key(uint32_t hi, uint32_t lo) {
    return ((uint64_t)hi << 32) | (uint64_t)lo;
}
// Packed fp32x2 add with an explicit round-to-nearest modifier in PTX: each
// half is one IEEE single-precision addition (checked bit for bit against the
// CPU statement).  There is deliberately no packed multiply helper: a packed
// multiply feeding a packed add was measured to differ from separately
// rounded scalar operations in the last bit.
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
    float2 r;
    asm("{\n .reg .b64 ra, rb, rc;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " add.rn.f32x2 rc, ra, rb;\n mov.b64 {%0, %1}, rc;\n}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}

__device__ __forceinline__ uint32_t key_hi(uint64_t k) { return (uint32_t)(k >> 32); }
__device__ __forceinline__ uint32_t key_lo(uint64_t k) { return (uint32_t)k; }

// ---------------------------------------------------------------------------
// warp / block reductions and scans
// ---------------------------------------------------------------------------
__device__ __forceinline__ int warp_incl_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Exclusive block scan of one int per thread.  scratch: >= 33 ints.
// Returns the exclusive prefix; *total receives the block total.
template <int T>
__device__ __forceinline__ int block_excl_scan(int v, int* scratch, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int W = T / 32;
    int incl = warp_incl_scan(v);
    if (lane == 31) scratch[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = lane < W ? scratch[lane] : 0;
        int wi = warp_incl_scan(w);
        if (lane < W) scratch[lane] = wi - w;
        if (lane == W - 1) scratch[32] = wi;
    }
    __syncthreads();
    int r = scratch[warp] + incl - v;
    *total = scratch[32];
    __syncthreads();
    return r;
}

template <int T>
__device__ __forceinline__ int block_sum(int v, int* scratch) {
    int tot;
    (void)block_excl_scan<T>(v, scratch, &tot);
    return tot;
}

// ---------------------------------------------------------------------------
// Radix selection of the need-th smallest 64-bit key (1-based) among the
// participants: the keys <= upper that each(fn) hands to fn(key) (every
// thread passes its own share of the keys).  The caller guarantees at least
// `need` participants.  Returns kappa such that exactly `need` participants
// satisfy key <= min(kappa, upper) when keys are distinct; when several
// participants share the final key, returns that key (the caller takes
// copies as needed).  8 bits per pass from the most significant byte, early
// exit as soon as the bucket that holds the need-th key is needed in full.
// hist: 256 ints of shared memory; bc: 4 ints of shared memory.
// ---------------------------------------------------------------------------
template <int T, class EachFn>
__device__ uint64_t block_kth_each(EachFn each, int need, uint64_t upper, int* hist, int* bc) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint64_t prefix = 0, mask = 0;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int b = tid; b < 256; b += T) hist[b] = 0;
        __syncthreads();
        each([&](uint64_t k) {
            if (k <= upper && (k & mask) == prefix) atomicAdd(&hist[(int)((k >> shift) & 255u)], 1);
        });
        __syncthreads();
        if (warp == 0) {
            int loc[8];
            int s = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                loc[j] = hist[lane * 8 + j];
                s += loc[j];
            }
            int incl = warp_incl_scan(s);
            int excl = incl - s;
            unsigned ball = __ballot_sync(0xffffffffu, incl >= need);
            int src = __ffs(ball) - 1;
            if (lane == src) {
                int acc = excl;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (acc + loc[j] >= need) {
                        bc[0] = lane * 8 + j;
                        bc[1] = acc;
                        bc[2] = loc[j];
                        break;
                    }
                    acc += loc[j];
                }
            }
        }
        __syncthreads();
        const int b = bc[0], below = bc[1], cnt = bc[2];
        __syncthreads();
        need -= below;
        prefix |= (uint64_t)b << shift;
        mask |= (uint64_t)0xFFu << shift;
        if (cnt == need) return prefix | ~mask;
    }
    return prefix;
}

// The selection of block_kth_each over ITEMS keys per thread held in
// registers (keyj(j) for j < ITEMS, kKeyNone for none; all threads call it
// together).  The first pass starts at the highest byte in which the
// participants differ (block-wide min and max), skipping the bytes they all
// share.  mm: 2 * 32 uint64 of shared memory.
template <int T, int ITEMS, class KeyJ>
__device__ uint64_t block_kth_items(KeyJ keyj, int need, uint64_t upper, int* hist, int* bc,
                                    unsigned long long* mm) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int W = T / 32;
    uint64_t lo = kKeyNone, hi = 0;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        const uint64_t k = keyj(j);
        if (k <= upper) {
            lo = k < lo ? k : lo;
            hi = k > hi ? k : hi;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t l2 = __shfl_xor_sync(0xffffffffu, lo, o), h2 = __shfl_xor_sync(0xffffffffu, hi, o);
        lo = l2 < lo ? l2 : lo;
        hi = h2 > hi ? h2 : hi;
    }
    if (lane == 0) {
        mm[warp] = lo;
        mm[32 + warp] = hi;
    }
    __syncthreads();
#pragma unroll
    for (int w = 0; w < W; ++w) {
        const uint64_t l2 = mm[w], h2 = mm[32 + w];
        lo = l2 < lo ? l2 : lo;
        hi = h2 > hi ? h2 : hi;
    }
    if (lo == hi) {               // every participant holds the same key
        __syncthreads();          // mm is read by all before a later call rewrites it
        return lo;
    }
    const int top = 63 - __clzll((long long)(lo ^ hi));
    int shift = (top / 8) * 8;
    uint64_t mask = shift + 8 >= 64 ? 0ull : ~((1ull << (shift + 8)) - 1ull);
    uint64_t prefix = lo & mask;
    for (; shift >= 0; shift -= 8) {
        for (int b = tid; b < 256; b += T) hist[b] = 0;
        __syncthreads();
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
            const uint64_t k = keyj(j);
            if (k <= upper && (k & mask) == prefix) atomicAdd(&hist[(int)((k >> shift) & 255u)], 1);
        }
        __syncthreads();
        if (warp == 0) {
            int loc[8];
            int s = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                loc[j] = hist[lane * 8 + j];
                s += loc[j];
            }
            int incl = warp_incl_scan(s);
            int excl = incl - s;
            unsigned ball = __ballot_sync(0xffffffffu, incl >= need);
            int src = __ffs(ball) - 1;
            if (lane == src) {
                int acc = excl;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (acc + loc[j] >= need) {
                        bc[0] = lane * 8 + j;
                        bc[1] = acc;
                        bc[2] = loc[j];
                        break;
                    }
                    acc += loc[j];
                }
            }
        }
        __syncthreads();
        const int b = bc[0], below = bc[1], cnt = bc[2];
        __syncthreads();
        need -= below;
        prefix |= (uint64_t)b << shift;
        mask |= (uint64_t)0xFFu << shift;
        if (cnt == need) return prefix | ~mask;
    }
    return prefix;
}

// the same over the keys k(i), i < n, strided over the block
template <int T, class KeyFn>
__device__ uint64_t block_kth_key(KeyFn keyf, int n, int need, uint64_t upper, int* hist, int* bc) {
    return block_kth_each<T>(
        [&](auto fn) {
            for (int i = threadIdx.x; i < n; i += T) fn(keyf(i));
        },
        need, upper, hist, bc);
}

// One round of a warp-wide minimum over the E keys per lane in v: the
// smallest key of the warp (high word first, then the low word among the
// lanes that hold the high minimum, both by the warp's min-reduction) is
// returned to every lane and exactly one copy of it -- the lowest lane's first
// slot holding it -- is replaced by kKeyNone, so equal keys of different
// candidates all come out in later rounds.  All 32 lanes call it together.
template <int E>
__device__ __forceinline__ uint64_t warp_take_min(uint64_t (&v)[E]) {
    const int lane = threadIdx.x & 31;
    uint64_t m = v[0];
    int ms = 0;
#pragma unroll
    for (int e = 1; e < E; ++e)
        if (v[e] < m) {
            m = v[e];
            ms = e;
        }
    const uint32_t hi = __reduce_min_sync(0xffffffffu, key_hi(m));
    const uint32_t lo = __reduce_min_sync(0xffffffffu, key_hi(m) == hi ? key_lo(m) : 0xFFFFFFFFu);
    const uint64_t wm = ((uint64_t)hi << 32) | lo;
    const unsigned holders = __ballot_sync(0xffffffffu, m == wm);
    if (lane == __ffs(holders) - 1) {
#pragma unroll
        for (int e = 0; e < E; ++e)
            if (e == ms) v[e] = kKeyNone;
    }
    return wm;
}

// The k smallest of src[0 .. n) (n <= 32 E), ascending, into dst[0 .. k)
// (kKeyNone past the last key), by one warp.
template <int E>
__device__ void warp_smallest_k(const uint64_t* src, int n, int k, uint64_t* dst) {
    const int lane = threadIdx.x & 31;
    uint64_t v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = e * 32 + lane < n ? src[e * 32 + lane] : kKeyNone;
    for (int it = 0; it < k; ++it) {
        const uint64_t wm = warp_take_min<E>(v);
        if (lane == 0) dst[it] = wm;
    }
}

// n <= 128
__device__ __forceinline__ void warp_smallest_k_dispatch(const uint64_t* src, int n, int k, uint64_t* dst) {
    if (n <= 32) warp_smallest_k<1>(src, n, k, dst);
    else if (n <= 64) warp_smallest_k<2>(src, n, k, dst);
    else warp_smallest_k<4>(src, n, k, dst);
}

// ---------------------------------------------------------------------------
// In-place ascending bitonic sort of n (power of two) keys in shared memory.
// ---------------------------------------------------------------------------
template <int T>
__device__ void block_bitonic_sort(uint64_t* s, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < n / 2; i += T) {
                int lo = 2 * i - (i & (stride - 1));
                int hi = lo + stride;
                bool asc = ((lo & size) == 0);
                uint64_t a = s[lo], b = s[hi];
                if ((a > b) == asc) {
                    s[lo] = b;
                    s[hi] = a;
                }
            }
        }
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// device views of the index
// ---------------------------------------------------------------------------
struct ListStore {             // one cluster-major segment (main index or a delta)
    const uint8_t* data;       // PQ codes [n, M] or uint8 vectors [n, d]
    const int64_t* offsets;    // [nlist] first position of each list
    const int32_t* counts;     // [nlist] vectors per list
    const int32_t* ids;        // [n] id reported for each position (nullptr: the position)
    const int64_t* key_off;    // [nlist] position of each list's first vector inside ranking
                               // keys (nullptr: offsets); a shard of a larger index ranks by
                               // the positions of the whole index so shards merge exactly
    const uint8_t* rr_u8;      // [n, d] rerank rows (u8), PQ only
    const float* rr_f32;       // [n, d] rerank rows (fp32), PQ only
    const uint8_t* gring;      // PQ codes in the grouped-ring tile layout (pq.cu), or nullptr
    const int64_t* gring_off;  // [nlist] byte offset of each list's first tile
    int64_t n;
    const int32_t* sqnorm;     // [n] sum of squares of each uint8 row (exact index), or nullptr
    const uint8_t* deleted;    // [n] nonzero = deleted position (not scanned / not reranked), or nullptr
};

struct WorkList {              // probe inversion for one batch: list-major (query, list) pairs
    int32_t* list_cnt;         // [nlist]   pairs per list
    int32_t* list_off;         // [nlist+1] exclusive prefix of list_cnt
    int32_t* cursor;           // [nlist]   fill cursors
    int32_t* pair_q;           // [max_pairs] query of each pair
    int32_t* pair_l;           // [max_pairs] (local) list of each pair
    int32_t* n_pairs;          // -> list_off[nlist]
    int32_t* grp_cnt;          // [nlist+1] query groups per list (optional)
    int32_t* grp_off;          // [nlist+1] exclusive prefix of grp_cnt
    int64_t* groups;           // [max_pairs] (list << 32) | (first pair << S) | group size, list-major
    int32_t* n_groups;         // -> grp_off[nlist]
    int gq;                    // queries per group: 0 = kGroupQueries (4, S = 3); up to 127 (S = 7)
};

__host__ __device__ inline int group_shift(int gq) { return gq <= 7 ? 3 : 7; }

struct CandBuf {               // per-query candidate buffers of one segment
    uint64_t* keys;            // [nq, cap]
    int32_t* cnt;              // [nq]
    unsigned long long* thr;   // [nq] running upper bound of the rank-R key
    int32_t* overflow;         // set when a query's buffer would overflow
    int cap;
    int R;                     // rank budget (rerank_n or delta top-k)
    int slack;                 // a filtered chunk may append up to R + slack keys (0: exactly R)
};

}  // namespace isb
