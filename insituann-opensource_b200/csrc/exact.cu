// exact.cu -- exact uint8 fine search over probed inverted lists.
//
// Semantics follow the reference's deterministic exact path
// (updates/exact_update.cu:632-666 fine_search_scalar_touched_u8 and
// :465-484 finalize_topk): int32 sum_j (q_j - x_j)^2 over every vector of
// every probed list, top-k by (distance, original id).  The reference runs
// this on the CPU with AVX-512 madd_epi16 (cpu_fine_kernels_v3_u8.cpp:49-96).
//
// Here each CTA pulls (query, list) pairs from a global counter; list rows
// are read with 16-byte loads, |q - x| per byte pair comes from one
// __vabsdiffu4 and the squares are summed by __dp4a, exact in int32.  Keys
// (distance, original id) of each chunk go through the shared block filter.
#include "emit.cuh"
#include "launch.h"

namespace isb {

namespace {

constexpr int kET = 256;
constexpr int kEChunk = kExactScanChunk;
constexpr int kEMaxD = 512;

__device__ __forceinline__ uint32_t sqdiff4(uint32_t a, uint32_t b, uint32_t acc) {
    uint32_t ad = __vabsdiffu4(a, b);
    return __dp4a(ad, ad, acc);
}

template <int NW>  // NW = d / 16 when known at compile time, 0 = runtime d
__global__ void __launch_bounds__(kET) exact_scan_kernel(const uint8_t* __restrict__ q_u8, int d, ListStore ls,
                                                         WorkList wl, CandBuf cb, int* counter) {
    __shared__ __align__(16) uint4 sq[kEMaxD / 16];
    __shared__ uint64_t skeys[kEChunk];
    __shared__ EmitSmem esm;
    __shared__ int s_item;
    const int tid = threadIdx.x;
    const int nw = NW > 0 ? NW : d / 16;
    const int P = *wl.n_pairs;
    for (;;) {
        const int it = next_item(counter, P, &s_item);
        if (it < 0) break;
        const int q = wl.pair_q[it], l = wl.pair_l[it];
        const int count = ls.counts[l];
        if (count <= 0) continue;
        const int64_t off = ls.offsets[l];
        for (int w = tid; w < nw; w += kET) sq[w] = reinterpret_cast<const uint4*>(q_u8 + (size_t)q * d)[w];
        __syncthreads();
        for (int cs = 0; cs < count; cs += kEChunk) {
            const int len = min(kEChunk, count - cs);
            for (int v = tid; v < len; v += kET) {
                const int64_t pos = off + cs + v;
                const uint4* row = reinterpret_cast<const uint4*>(ls.data + (size_t)pos * d);
                uint32_t acc = 0;
                if constexpr (NW > 0) {
#pragma unroll
                    for (int w = 0; w < NW; ++w) {
                        uint4 x = __ldg(row + w), y = sq[w];
                        acc = sqdiff4(x.x, y.x, acc);
                        acc = sqdiff4(x.y, y.y, acc);
                        acc = sqdiff4(x.z, y.z, acc);
                        acc = sqdiff4(x.w, y.w, acc);
                    }
                } else {
                    for (int w = 0; w < nw; ++w) {
                        uint4 x = __ldg(row + w), y = sq[w];
                        acc = sqdiff4(x.x, y.x, acc);
                        acc = sqdiff4(x.y, y.y, acc);
                        acc = sqdiff4(x.z, y.z, acc);
                        acc = sqdiff4(x.w, y.w, acc);
                    }
                }
                const uint32_t id = ls.ids ? (uint32_t)ls.ids[pos] : (uint32_t)pos;
                // deleted positions are not scanned (exact_update.cu:89)
                skeys[v] = (ls.deleted && ls.deleted[pos]) ? kKeyNone : make_key(acc, id);
            }
            __syncthreads();
            auto keyf = [&](int i) -> uint64_t { return skeys[i]; };
            block_filter_emit<kET>(keyf, len, cb, q, esm);
        }
    }
}

// ---------------------------------------------------------------------------
// fp32 exact fine search (the reference's GPU path for indexes loaded with
// ivf_load_dataset: cuda/search/ivf_search_separated.cu:417-650,
// fine/indexed_gemm_{l2,cos}.cu): for every vector of every probed list,
//   L2:     sum_j (q_j - x_j)^2 in dimension order (fp32, separately rounded);
//   cosine: 1 - <q, x> / (|q| |x|), <q, x> summed in dimension order, norms as
//           sqrtf of the sequential sum of squares; clamped at 0, and a vector
//           or query of zero norm is at distance 1 (cosine 0);
// keys (distance bits, position) through the shared block filter, so the top-k
// is by (distance, position).
// ---------------------------------------------------------------------------
__global__ void f32_norms_kernel(const float* __restrict__ x, int64_t n, int d, float* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float* r = x + (size_t)i * d;
        float s = 0.f;
        for (int j = 0; j < d; ++j) s = __fadd_rn(s, __fmul_rn(r[j], r[j]));
        out[i] = sqrtf(s);
    }
}

__global__ void __launch_bounds__(kET) f32_scan_kernel(const float* __restrict__ q, int d, const float* __restrict__ x,
                                                       const float* __restrict__ xnorm, ListStore ls, int cosine,
                                                       WorkList wl, CandBuf cb, int* counter) {
    __shared__ float sq[kEMaxD];
    __shared__ uint64_t skeys[kEChunk];
    __shared__ EmitSmem esm;
    __shared__ int s_item;
    __shared__ float s_qn;
    const int tid = threadIdx.x;
    const int P = *wl.n_pairs;
    for (;;) {
        const int it = next_item(counter, P, &s_item);
        if (it < 0) break;
        const int qi = wl.pair_q[it], l = wl.pair_l[it];
        const int count = ls.counts[l];
        if (count <= 0) continue;
        const int64_t off = ls.offsets[l];
        for (int j = tid; j < d; j += kET) sq[j] = q[(size_t)qi * d + j];
        __syncthreads();
        if (tid == 0) {
            float s = 0.f;
            for (int j = 0; j < d; ++j) s = __fadd_rn(s, __fmul_rn(sq[j], sq[j]));
            s_qn = sqrtf(s);
        }
        __syncthreads();
        const float qn = s_qn;
        for (int cs = 0; cs < count; cs += kEChunk) {
            const int len = min(kEChunk, count - cs);
            for (int v = tid; v < len; v += kET) {
                const int64_t pos = off + cs + v;
                const float* row = x + (size_t)pos * d;
                float dist;
                if (cosine) {
                    float dot = 0.f;
                    for (int j = 0; j < d; ++j) dot = __fadd_rn(dot, __fmul_rn(sq[j], __ldg(row + j)));
                    const float den = __fmul_rn(qn, xnorm[pos]);
                    dist = den > 0.f ? fmaxf(__fsub_rn(1.f, __fdiv_rn(dot, den)), 0.f) : 1.f;
                } else {
                    float acc = 0.f;
                    for (int j = 0; j < d; ++j) {
                        const float t = __fsub_rn(sq[j], __ldg(row + j));
                        acc = __fadd_rn(acc, __fmul_rn(t, t));
                    }
                    dist = acc;
                }
                skeys[v] = (ls.deleted && ls.deleted[pos]) ? kKeyNone : make_key(__float_as_uint(dist), (uint32_t)pos);
            }
            __syncthreads();
            auto keyf = [&](int i) -> uint64_t { return skeys[i]; };
            block_filter_emit<kET>(keyf, len, cb, qi, esm);
        }
    }
}

// ---------------------------------------------------------------------------
// Grouped exact scan: one CTA works on a list and up to kXG queries that probe
// it, so every list row is read once per group instead of once per query.
// With |q|^2, |x|^2 and q.x all exact in int32, sum_j (q_j - x_j)^2 =
// |q|^2 + |x|^2 - 2 q.x is the same integer as the reference's sum of squared
// differences; q.x comes from __dp4a on four byte pairs at a time.
//
// A tile of kXT list rows is staged in shared memory (16-byte chunks of a row
// rotated by XOR with row % 8, so the 16 rows a warp reads in one load fall in
// 8 different bank groups).  256 threads cover kXG x kXT (query, row) pairs
// as 16 x 16 blocks of 4 x 4: thread (qb, vb) holds queries 4 qb .. 4 qb + 3
// and rows vb + 16 j, so warp w sees all rows of the tile for its 8 queries
// 8 w .. 8 w + 7.  Each warp keeps the k smallest keys (distance, original
// id) of its queries: a key below the query's current k-th is staged, and
// after the tile the warp merges the staged keys with the query's k (k rounds
// of the warp minimum).  At the end of the list every query's k keys go to its
// candidate buffer (a query probing the list twice appears twice in the group
// and contributes twice, as the reference's per-probe scan does).
constexpr int kXG = 64;             // queries per group
constexpr int kXT = 64;             // list rows per tile
constexpr int kXThreads = 256;
constexpr int kXKMax = 16;          // largest k of the grouped kernel

__host__ __device__ constexpr size_t exact_group_smem(int nw) {
    return sizeof(uint4) * (size_t)(kXG + 2 * kXT) * nw       // queries, two tiles
           + sizeof(uint64_t) * (size_t)kXG * (kXKMax + kXT)   // top-k, staging
           + sizeof(uint64_t) * kXG                            // k-th key per query
           + sizeof(int) * (size_t)(kXG + kXG + 4 * kXT);      // staged counts, |q|^2, two tiles' |x|^2 and ids
}

__global__ void u8_sqnorm_kernel(const uint8_t* __restrict__ x, int64_t n, int nw, int32_t* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint4* r = reinterpret_cast<const uint4*>(x) + i * nw;
        uint32_t s = 0;
        for (int c = 0; c < nw; ++c) {
            const uint4 v = __ldg(r + c);
            s = __dp4a(v.x, v.x, s);
            s = __dp4a(v.y, v.y, s);
            s = __dp4a(v.z, v.z, s);
            s = __dp4a(v.w, v.w, s);
        }
        out[i] = (int32_t)s;
    }
}

template <int NW>  // 16-byte chunks per row, d = 16 NW; NW in {8, 16}
__global__ void __launch_bounds__(kXThreads, 3) exact_group_kernel(const uint8_t* __restrict__ q_u8, ListStore ls,
                                                                WorkList wl, CandBuf cb, int k, int* counter) {
    extern __shared__ __align__(16) unsigned char xsm[];
    uint4* sQ = reinterpret_cast<uint4*>(xsm);                          // [kXG][NW]
    uint4* sX = sQ + kXG * NW;                                          // [2][kXT][NW]
    uint64_t* sTop = reinterpret_cast<uint64_t*>(sX + 2 * kXT * NW);    // [kXG][kXKMax]
    uint64_t* sStage = sTop + kXG * kXKMax;                             // [kXG][kXT]
    uint64_t* sTau = sStage + kXG * kXT;                                // [kXG]
    int* sCnt = reinterpret_cast<int*>(sTau + kXG);                     // [kXG]
    int* sQn = sCnt + kXG;                                              // [kXG]
    int* sXn = sQn + kXG;                                               // [2][kXT]
    uint32_t* sId = reinterpret_cast<uint32_t*>(sXn + 2 * kXT);         // [2][kXT]
    __shared__ int s_item;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qb = tid >> 4, vb = tid & 15;
    constexpr int d = 16 * NW;
    const int NG = *wl.n_groups;
    // tile t0 of list rows from `off` into buffer b: rows, ids, squared norms
    auto stage_tile = [&](int64_t off, int t0, int count, int b) {
        const int nv = min(kXT, count - t0);
        const uint4* src = reinterpret_cast<const uint4*>(ls.data + (size_t)(off + t0) * d);
        uint4* dst = sX + b * kXT * NW;
        for (int e = tid; e < nv * NW; e += kXThreads) {
            const int r = e / NW, c = e % NW;
            dst[r * NW + (c ^ (r & 7))] = __ldg(src + e);
        }
        if (tid < nv) {
            const int64_t pos = off + t0 + tid;
            // a deleted position gets the id 0xFFFFFFFF, which no row passes (exact_update.cu:89)
            sId[b * kXT + tid] = (ls.deleted && ls.deleted[pos]) ? 0xFFFFFFFFu
                                                                 : (ls.ids ? (uint32_t)ls.ids[pos] : (uint32_t)pos);
            sXn[b * kXT + tid] = ls.sqnorm[pos];
        }
    };
    for (;;) {
        __syncthreads();
        if (tid == 0) s_item = atomicAdd(counter, 1);
        __syncthreads();
        const int it = s_item;
        if (it >= NG) break;
        const int64_t pk = wl.groups[it];
        const int l = (int)(pk >> 32), p0 = (int)((pk >> 7) & 0x1FFFFFF), nqg = (int)(pk & 127);
        const int count = ls.counts[l];
        const int64_t off = ls.offsets[l];
        // the group's queries (rows past nqg are zero) and their squared norms
        for (int e = tid; e < kXG * NW; e += kXThreads) {
            const int r = e / NW, c = e % NW;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (r < nqg) v = reinterpret_cast<const uint4*>(q_u8 + (size_t)wl.pair_q[p0 + r] * d)[c];
            sQ[r * NW + (c ^ (r & 7))] = v;
        }
        // a row starts from its query's bound over the lists done so far (the
        // k-th of some k keys already in its buffer): a key at or above it can
        // not be among the query's k smallest -- a second copy of that key
        // would rank k + 1-th at best
        for (int r = tid; r < kXG; r += kXThreads) {
            sTau[r] = r < nqg ? *((volatile unsigned long long*)(cb.thr + wl.pair_q[p0 + r])) : kKeyNone;
            sCnt[r] = 0;
        }
        for (int e = tid; e < kXG * kXKMax; e += kXThreads) sTop[e] = kKeyNone;
        if (count > 0) stage_tile(off, 0, count, 0);
        __syncthreads();
        if (tid < kXG) {
            uint32_t n2 = 0;
#pragma unroll
            for (int c = 0; c < NW; ++c) {
                const uint4 v = sQ[tid * NW + (c ^ (tid & 7))];
                n2 = __dp4a(v.x, v.x, n2);
                n2 = __dp4a(v.y, v.y, n2);
                n2 = __dp4a(v.z, v.z, n2);
                n2 = __dp4a(v.w, v.w, n2);
            }
            sQn[tid] = (int)n2;
        }
        __syncthreads();
        // tile t in buffer t & 1 while tile t + 1 is staged into the other one;
        // one barrier per tile
        for (int t0 = 0, b = 0; t0 < count; t0 += kXT, b ^= 1) {
            const int nv = min(kXT, count - t0);
            if (t0 + kXT < count) stage_tile(off, t0 + kXT, count, b ^ 1);
            const uint4* tile = sX + b * kXT * NW;
            // q.x for this thread's 4 x 4 (query, row) pairs
            uint32_t acc[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = 0u;
#pragma unroll
            for (int c = 0; c < NW; ++c) {
                uint4 qa[4], xa[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = 4 * qb + i;
                    qa[i] = sQ[r * NW + (c ^ (r & 7))];
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) xa[j] = tile[(vb + 16 * j) * NW + (c ^ (vb & 7))];
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc[i][j] = __dp4a(qa[i].x, xa[j].x, acc[i][j]);
                        acc[i][j] = __dp4a(qa[i].y, xa[j].y, acc[i][j]);
                        acc[i][j] = __dp4a(qa[i].z, xa[j].z, acc[i][j]);
                        acc[i][j] = __dp4a(qa[i].w, xa[j].w, acc[i][j]);
                    }
            }
            // keys below the query's current k-th go to its staging list
            bool any = false;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = 4 * qb + i;
                const uint64_t tau = sTau[r];
                const int qn = sQn[r];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int v = vb + 16 * j;
                    if (r < nqg && v < nv && sId[b * kXT + v] != 0xFFFFFFFFu) {
                        const uint32_t dist = (uint32_t)(qn + sXn[b * kXT + v]) - 2u * acc[i][j];
                        const uint64_t key = make_key(dist, sId[b * kXT + v]);
                        if (key < tau) {
                            sStage[r * kXT + atomicAdd(&sCnt[r], 1)] = key;
                            any = true;
                        }
                    }
                }
            }
            __syncwarp();
            if (__any_sync(0xffffffffu, any)) {
                // merge each of this warp's 8 queries with what it staged
                for (int rr = 0; rr < 8; ++rr) {
                    const int r = 8 * warp + rr;
                    const int ns = sCnt[r];
                    if (ns == 0) continue;
                    const int m = k + ns;
                    if (m <= 32) {
                        // few staged keys: lane i takes element i of (top-k, staged) and
                        // writes it at its rank among all m, ties by element index
                        const uint64_t mine = lane < k ? sTop[r * kXKMax + lane]
                                                       : (lane < m ? sStage[r * kXT + (lane - k)] : kKeyNone);
                        int rank = 0;
                        for (int j = 0; j < m; ++j) {
                            const uint64_t o = __shfl_sync(0xffffffffu, mine, j);
                            rank += (o < mine || (o == mine && j < lane)) ? 1 : 0;
                        }
                        __syncwarp();
                        if (lane < m && rank < k) sTop[r * kXKMax + rank] = mine;
                        if (lane < m && rank == k - 1 && mine != kKeyNone && mine < sTau[r]) sTau[r] = mine;
                    } else {
                        uint64_t v4[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int i = e * 32 + lane;
                            v4[e] = i < k ? sTop[r * kXKMax + i]
                                          : (i - k < ns ? sStage[r * kXT + (i - k)] : kKeyNone);
                        }
                        uint64_t kth = kKeyNone;
                        for (int o = 0; o < k; ++o) {
                            const uint64_t mm = warp_take_min<4>(v4);
                            if (lane == o) sTop[r * kXKMax + o] = mm;
                            kth = mm;
                        }
                        __syncwarp();
                        if (lane == 0 && kth != kKeyNone && kth < sTau[r]) sTau[r] = kth;
                    }
                    __syncwarp();
                    if (lane == 0) sCnt[r] = 0;
                    __syncwarp();
                }
            }
            __syncthreads();                               // tile t + 1 staged; tile t no longer read
        }
        __syncthreads();
        // every query's k smallest keys of this list into its candidate buffer
        for (int rr = 0; rr < 8; ++rr) {
            const int r = 8 * warp + rr;
            if (r >= nqg) break;
            const uint64_t key = lane < k ? sTop[r * kXKMax + lane] : kKeyNone;
            const bool ok = key != kKeyNone;
            const unsigned ball = __ballot_sync(0xffffffffu, ok);
            if (!ball) continue;
            const int q = wl.pair_q[p0 + r];
            int base = 0;
            if (lane == 0) {
                base = atomicAdd(cb.cnt + q, __popc(ball));
                // k keys of this list are in the buffer: their k-th bounds the query's k smallest
                const uint64_t kth = sTop[r * kXKMax + k - 1];
                if (kth != kKeyNone) atomicMin(cb.thr + q, (unsigned long long)kth);
            }
            base = __shfl_sync(0xffffffffu, base, 0);
            if (ok) {
                const int at = base + __popc(ball & ((1u << lane) - 1u));
                if (at < cb.cap) cb.keys[(size_t)q * cb.cap + at] = key;
                else atomicExch(cb.overflow, 1);
            }
        }
    }
}

}  // namespace

bool exact_group_usable(int d, int k) { return (d == 128 || d == 256) && k > 0 && k <= kXKMax; }

cudaError_t u8_row_sqnorms(const uint8_t* x, int64_t n, int d, int32_t* out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (d % 16 != 0) return cudaErrorInvalidValue;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    note_launch();
    u8_sqnorm_kernel<<<(int)blocks, 256, 0, st>>>(x, n, d / 16, out);
    return cudaGetLastError();
}

cudaError_t exact_group_scan(const uint8_t* q_u8, int d, int k, ListStore ls, WorkList wl, int max_groups,
                             CandBuf cb, int* work_counter, cudaStream_t st) {
    if (!exact_group_usable(d, k) || !wl.groups || !ls.sqnorm) return cudaErrorInvalidValue;
    if (max_groups <= 0) return cudaSuccess;
    cudaError_t e = cudaMemsetAsync(work_counter, 0, sizeof(int), st);
    if (e) return e;
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int nw = d / 16;
    const size_t smem = exact_group_smem(nw);
    auto go = [&](auto kern) {
        cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e2) return e2;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kXThreads, smem);
        if (per_sm < 1) return cudaErrorInvalidConfiguration;
        long long grid = (long long)sms * per_sm;
        if (grid > max_groups) grid = max_groups;
        note_launch();
        kern<<<(int)grid, kXThreads, smem, st>>>(q_u8, ls, wl, cb, k, work_counter);
        return cudaGetLastError();
    };
    return nw == 8 ? go(exact_group_kernel<8>) : go(exact_group_kernel<16>);
}

cudaError_t exact_scan(const uint8_t* q_u8, int nq, int d, ListStore ls, WorkList wl, int max_pairs, CandBuf cb,
                       int* work_counter, cudaStream_t st) {
    (void)nq;
    if (d <= 0 || d % 16 != 0 || d > kEMaxD) return cudaErrorInvalidValue;
    if (max_pairs <= 0) return cudaSuccess;
    cudaError_t e = cudaMemsetAsync(work_counter, 0, sizeof(int), st);
    if (e) return e;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int grid = sms * 4;
    if (grid > max_pairs) grid = max_pairs;
    switch (d / 16) {
        case 4: note_launch(); exact_scan_kernel<4><<<grid, kET, 0, st>>>(q_u8, d, ls, wl, cb, work_counter); break;
        case 6: note_launch(); exact_scan_kernel<6><<<grid, kET, 0, st>>>(q_u8, d, ls, wl, cb, work_counter); break;
        case 8: note_launch(); exact_scan_kernel<8><<<grid, kET, 0, st>>>(q_u8, d, ls, wl, cb, work_counter); break;
        case 16: note_launch(); exact_scan_kernel<16><<<grid, kET, 0, st>>>(q_u8, d, ls, wl, cb, work_counter); break;
        default: note_launch(); exact_scan_kernel<0><<<grid, kET, 0, st>>>(q_u8, d, ls, wl, cb, work_counter); break;
    }
    return cudaGetLastError();
}

cudaError_t f32_row_norms(const float* x, int64_t n, int d, float* out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    note_launch();
    f32_norms_kernel<<<(int)blocks, 256, 0, st>>>(x, n, d, out);
    return cudaGetLastError();
}

cudaError_t f32_scan(const float* q, int d, const float* x, const float* xnorm, ListStore ls, int cosine, WorkList wl,
                     int max_pairs, CandBuf cb, int* work_counter, cudaStream_t st) {
    if (d <= 0 || d > kEMaxD) return cudaErrorInvalidValue;
    if (max_pairs <= 0) return cudaSuccess;
    cudaError_t e = cudaMemsetAsync(work_counter, 0, sizeof(int), st);
    if (e) return e;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int grid = sms * 4;
    if (grid > max_pairs) grid = max_pairs;
    note_launch();
    f32_scan_kernel<<<grid, kET, 0, st>>>(q, d, x, xnorm, ls, cosine, wl, cb, work_counter);
    return cudaGetLastError();
}

}  // namespace isb
