// route.cu -- coarse routing: top-nprobe inverted lists per query by L2.
//
// Reference behaviour (cuda/search/cpu_fine/ivf_search_cpu_fine.cu:764-1361 and
// cuda/search/coarse/fusion_l2_topk_warpsort.cu:61-157): L2 from
// ||q||^2 + ||c||^2 - 2 q.c with cuBLAS SGEMM, centroids whose norm is below
// 1e-6 skipped, warp top-k.  Its tie order and rounding depend on cuBLAS.
// This library defines routing as the exact fp32 direct-difference distance
// sum_j (q_j - c_j)^2 accumulated in j order without contraction, ranked by
// (distance, list id), so every probe list is reproducible bit for bit on
// the CPU.
#include "launch.h"

namespace isb {

namespace {

__global__ void centroid_valid_kernel(const float* __restrict__ cent, int nlist, int d, uint8_t* valid) {
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= nlist) return;
    const float* row = cent + (size_t)c * d;
    float s = 0.f;
    for (int j = 0; j < d; ++j) s = __fadd_rn(s, __fmul_rn(row[j], row[j]));
    valid[c] = (sqrtf(s) >= 1e-6f) ? 1 : 0;
}

// Cosine routing distance of the reference's fp32 pipeline
// (cuda/search/ivf_search_separated.cu:477-512 with
// coarse/fusion_cos_topk_warpsort.cu:125-135): 1 - <q, c> / (|q| |c|) in fp32,
// <q, c> summed in dimension order, norms sqrtf of the sequential sums;
// centroids below 1e-6 norm are not routed; clamped at 0 so that the bits of
// the distance order as its values.  One thread per (query, centroid); the
// query row of the CTA's queries is read through L1.
__global__ void route_cos_kernel(const float* __restrict__ q, int nq, const float* __restrict__ cent,
                                 const uint8_t* __restrict__ valid, int nlist, int d, uint32_t* __restrict__ out) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x, qi = blockIdx.y;
    if (c >= nlist || qi >= nq) return;
    const float* qr = q + (size_t)qi * d;
    const float* cr = cent + (size_t)c * d;
    float dot = 0.f, qs = 0.f, cs = 0.f;
    for (int j = 0; j < d; ++j) {
        const float a = __ldg(qr + j), b = __ldg(cr + j);
        dot = __fadd_rn(dot, __fmul_rn(a, b));
        qs = __fadd_rn(qs, __fmul_rn(a, a));
        cs = __fadd_rn(cs, __fmul_rn(b, b));
    }
    const float den = __fmul_rn(sqrtf(qs), sqrtf(cs));
    const float dist = den > 0.f ? fmaxf(__fsub_rn(1.f, __fdiv_rn(dot, den)), 0.f) : 1.f;
    out[(size_t)qi * nlist + c] = valid[c] ? __float_as_uint(dist) : 0xFFFFFFFFu;
}

// 128 queries x 128 centroids per CTA, 256 threads, 8x8 pairs per thread, 16
// dimensions staged per step.  The centroid tile is staged negated, so q - c
// is an add (x + (-y) is x - y exactly).  A thread's pairs are float2
// accumulators of two centroids; the subtraction and the accumulation are
// packed fp32x2 add.rn (PTX), the squares scalar __fmul_rn: a packed multiply
// feeding a packed add was measured to differ from the separately rounded CPU
// sums in the last bit, packed adds alone were not.  Packed operations run at
// the same FP32 lane rate as scalar ones on B200 but take half the issue
// slots.  Zero padding beyond d adds exact zeros.
constexpr int kRB = 128, kRK = 16;

__global__ void __launch_bounds__(256) route_dist_kernel(const float* __restrict__ q, int nq,
                                                         const float* __restrict__ cent,
                                                         const uint8_t* __restrict__ valid, int nlist,
                                                         int d, uint32_t* __restrict__ out) {
    __shared__ __align__(16) float sq[kRK][kRB + 4];
    __shared__ __align__(16) float sc[kRK][kRB + 4];     // -centroid
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int q0 = blockIdx.y * kRB, c0 = blockIdx.x * kRB;
    float2 acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.f, 0.f);

    for (int k0 = 0; k0 < d; k0 += kRK) {
        for (int e = tid; e < kRB * kRK; e += 256) {
            const int r = e / kRK, kk = e % kRK;
            const int qi = q0 + r, ci = c0 + r, j = k0 + kk;
            sq[kk][r] = (qi < nq && j < d) ? q[(size_t)qi * d + j] : 0.f;
            sc[kk][r] = (ci < nlist && j < d) ? -cent[(size_t)ci * d + j] : 0.f;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < kRK; ++kk) {
            const float4 a0 = *reinterpret_cast<const float4*>(&sq[kk][ty * 8]);
            const float4 a1 = *reinterpret_cast<const float4*>(&sq[kk][ty * 8 + 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&sc[kk][tx * 8]);
            const float4 b1 = *reinterpret_cast<const float4*>(&sc[kk][tx * 8 + 4]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float2 b[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                                 make_float2(b1.z, b1.w)};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 x = add2_rn(make_float2(a[i], a[i]), b[j]);
                    acc[i][j] = add2_rn(acc[i][j], make_float2(__fmul_rn(x.x, x.x), __fmul_rn(x.y, x.y)));
                }
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int qi = q0 + ty * 8 + i;
        if (qi >= nq) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int ci = c0 + tx * 8 + 2 * j + h;
                if (ci >= nlist) continue;
                const float v = h ? acc[i][j].y : acc[i][j].x;
                out[(size_t)qi * nlist + ci] = valid[ci] ? __float_as_uint(v) : 0xFFFFFFFFu;
            }
        }
    }
}

constexpr int kSelT = 512;
constexpr int kSelMaxL = 2048;

// One CTA per row: keys (dist bits, column) of the row, top-L sorted.
template <class KeyFn>
__device__ void select_row_topl(KeyFn keyf, int n, int L, uint64_t* s, int* hist, int* bc, int* s_cnt) {
    const int tid = threadIdx.x;
    int Lp = 1;
    while (Lp < L) Lp <<= 1;
    int take = n < L ? n : L;
    if (n <= L) {
        for (int i = tid; i < Lp; i += kSelT) s[i] = i < n ? keyf(i) : kKeyNone;
    } else {
        uint64_t kap = block_kth_key<kSelT>(keyf, n, L, kKeyNone, hist, bc);
        if (tid == 0) *s_cnt = 0;
        __syncthreads();
        for (int i = tid; i < n; i += kSelT) {
            uint64_t k = keyf(i);
            if (k < kap) s[atomicAdd(s_cnt, 1)] = k;
        }
        __syncthreads();
        int cl = *s_cnt;
        for (int i = cl + tid; i < Lp; i += kSelT) s[i] = i < take ? kap : kKeyNone;
    }
    block_bitonic_sort<kSelT>(s, Lp);
}

// Rows of up to kRowT * kRowItems keys: one CTA of kRowT threads per row, the
// row's keys in registers, a radix descent for the L-th key, the keys below it
// compacted and only those L sorted.
constexpr int kRowT = 256, kRowItems = 16;

__global__ void __launch_bounds__(kRowT) route_select_reg_kernel(const uint32_t* __restrict__ dist_bits, int n,
                                                                  int L, const int32_t* __restrict__ id_map,
                                                                  int32_t* out_ids, float* out_dist,
                                                                  uint64_t* out_keys) {
    __shared__ uint64_t s[kSelMaxL];
    __shared__ int hist[256];
    __shared__ int bc[4];
    __shared__ unsigned long long mm[64];
    __shared__ int s_cnt;
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
    const uint32_t* r = dist_bits + (size_t)row * n;
    int Lp = 1;
    while (Lp < L) Lp <<= 1;
    uint64_t v[kRowItems];
#pragma unroll
    for (int e = 0; e < kRowItems; ++e) {
        const int i = tid + kRowT * e;
        v[e] = i < n ? make_key(r[i], id_map ? (uint32_t)id_map[i] : (uint32_t)i) : kKeyNone;
    }
    if (tid == 0) s_cnt = 0;
    if (n <= L) {
        __syncthreads();
#pragma unroll
        for (int e = 0; e < kRowItems; ++e) {
            const int i = tid + kRowT * e;
            if (i < n) s[i] = v[e];
        }
        for (int i = n + tid; i < Lp; i += kRowT) s[i] = kKeyNone;
    } else {
        const uint64_t kap =
            block_kth_items<kRowT, kRowItems>([&](int e) { return v[e]; }, L, kKeyNone - 1, hist, bc, mm);
#pragma unroll
        for (int e = 0; e < kRowItems; ++e) {
            const bool take = v[e] < kap;
            const unsigned ball = __ballot_sync(0xffffffffu, take);
            if (ball == 0) continue;
            int base = 0;
            if (lane == 0) base = atomicAdd(&s_cnt, __popc(ball));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (take) s[base + __popc(ball & ((1u << lane) - 1u))] = v[e];
        }
        __syncthreads();
        const int cl = s_cnt;
        for (int i = cl + tid; i < Lp; i += kRowT) s[i] = i < L ? kap : kKeyNone;
    }
    block_bitonic_sort<kRowT>(s, Lp);
    for (int i = tid; i < L; i += kRowT) {
        const uint64_t k = s[i];
        const bool ok = k != kKeyNone && key_hi(k) != 0xFFFFFFFFu;
        if (out_ids) out_ids[(size_t)row * L + i] = ok ? (int32_t)key_lo(k) : -1;
        if (out_dist) out_dist[(size_t)row * L + i] = ok ? __uint_as_float(key_hi(k)) : __int_as_float(0x7f800000);
        if (out_keys) out_keys[(size_t)row * L + i] = k;
    }
}

__global__ void __launch_bounds__(kSelT) route_select_kernel(const uint32_t* __restrict__ dist_bits, int n, int L,
                                                             const int32_t* __restrict__ id_map, int32_t* out_ids,
                                                             float* out_dist, uint64_t* out_keys) {
    __shared__ uint64_t s[kSelMaxL];
    __shared__ int hist[256];
    __shared__ int bc[4];
    __shared__ int s_cnt;
    const int row = blockIdx.x;
    const uint32_t* r = dist_bits + (size_t)row * n;
    auto keyf = [&](int i) -> uint64_t { return make_key(r[i], id_map ? (uint32_t)id_map[i] : (uint32_t)i); };
    select_row_topl(keyf, n, L, s, hist, bc, &s_cnt);
    for (int i = threadIdx.x; i < L; i += kSelT) {
        uint64_t k = s[i];
        bool ok = k != kKeyNone && key_hi(k) != 0xFFFFFFFFu;
        if (out_ids) out_ids[(size_t)row * L + i] = ok ? (int32_t)key_lo(k) : -1;
        if (out_dist) out_dist[(size_t)row * L + i] = ok ? __uint_as_float(key_hi(k)) : __int_as_float(0x7f800000);
        if (out_keys) out_keys[(size_t)row * L + i] = k;
    }
}

__global__ void __launch_bounds__(kSelT) merge_keys_kernel(const uint64_t* __restrict__ keys, int n, int L,
                                                           int int_dist, int32_t* out_ids, float* out_dist,
                                                           int32_t* out_idist) {
    __shared__ uint64_t s[kSelMaxL];
    __shared__ int hist[256];
    __shared__ int bc[4];
    __shared__ int s_cnt;
    const int row = blockIdx.x;
    const uint64_t* r = keys + (size_t)row * n;
    auto keyf = [&](int i) -> uint64_t { return r[i]; };
    select_row_topl(keyf, n, L, s, hist, bc, &s_cnt);
    for (int i = threadIdx.x; i < L; i += kSelT) {
        uint64_t k = s[i];
        bool ok = k != kKeyNone && key_hi(k) != 0xFFFFFFFFu;
        out_ids[(size_t)row * L + i] = ok ? (int32_t)key_lo(k) : -1;
        if (out_dist) {
            float f = int_dist ? (float)key_hi(k) : __uint_as_float(key_hi(k));
            out_dist[(size_t)row * L + i] = ok ? f : __int_as_float(0x7f800000);
        }
        if (out_idist) out_idist[(size_t)row * L + i] = ok ? (int32_t)key_hi(k) : 0x7fffffff;
    }
}

// One warp per query over the shards' sorted routing keys as all-gathered,
// [S][nq][L]: the query's S * L keys (at most 32 E) go to registers and L
// rounds of the warp minimum give its global top-L; lane j writes the j-th.
template <int E>
__global__ void __launch_bounds__(256) merge_shard_keys_kernel(const uint64_t* __restrict__ keys, int S, int nq,
                                                               int L, int32_t* __restrict__ out_ids) {
    const int q = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (q >= nq) return;                   // whole warps only
    const int n = S * L;
    uint64_t v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int i = e * 32 + lane;
        v[e] = i < n ? keys[((size_t)(i / L) * nq + q) * L + (i % L)] : kKeyNone;
    }
    uint64_t mine = kKeyNone;
    for (int it = 0; it < L; ++it) {
        const uint64_t wm = warp_take_min<E>(v);
        if (lane == it) mine = wm;
    }
    if (lane < L) {
        const bool ok = mine != kKeyNone && key_hi(mine) != 0xFFFFFFFFu;
        out_ids[(size_t)q * L + lane] = ok ? (int32_t)key_lo(mine) : -1;
    }
}

__global__ void make_u8_kernel(const float* __restrict__ q, size_t n, uint8_t* __restrict__ out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float x = fminf(fmaxf(q[i], 0.f), 255.f);
        out[i] = (uint8_t)lroundf(x);
    }
}

}  // namespace

cudaError_t route_centroid_valid(const float* cent, int nlist, int d, uint8_t* valid, cudaStream_t st) {
    note_launch();
    centroid_valid_kernel<<<(nlist + 255) / 256, 256, 0, st>>>(cent, nlist, d, valid);
    return cudaGetLastError();
}

cudaError_t route_distances(const float* q, int nq, const float* cent, const uint8_t* valid, int nlist, int d,
                            uint32_t* out, cudaStream_t st) {
    if (nq <= 0) return cudaSuccess;
    dim3 grid((nlist + kRB - 1) / kRB, (nq + kRB - 1) / kRB);
    note_launch();
    route_dist_kernel<<<grid, 256, 0, st>>>(q, nq, cent, valid, nlist, d, out);
    return cudaGetLastError();
}

cudaError_t route_distances_cos(const float* q, int nq, const float* cent, const uint8_t* valid, int nlist, int d,
                                uint32_t* out, cudaStream_t st) {
    if (nq <= 0) return cudaSuccess;
    dim3 grid((nlist + 255) / 256, nq);
    note_launch();
    route_cos_kernel<<<grid, 256, 0, st>>>(q, nq, cent, valid, nlist, d, out);
    return cudaGetLastError();
}

cudaError_t route_select(const uint32_t* dist_bits, int nq, int n, int L, const int32_t* id_map, int32_t* out_ids,
                         float* out_dist, uint64_t* out_keys, cudaStream_t st) {
    if (L > kSelMaxL || L <= 0) return cudaErrorInvalidValue;
    if (nq <= 0) return cudaSuccess;
    note_launch();
    if (n <= kRowT * kRowItems)
        route_select_reg_kernel<<<nq, kRowT, 0, st>>>(dist_bits, n, L, id_map, out_ids, out_dist, out_keys);
    else
        route_select_kernel<<<nq, kSelT, 0, st>>>(dist_bits, n, L, id_map, out_ids, out_dist, out_keys);
    return cudaGetLastError();
}

cudaError_t merge_keys(const uint64_t* keys, int nq, int n, int L, int int_dist, int32_t* out_ids, float* out_dist,
                       int32_t* out_idist, cudaStream_t st) {
    if (L > kSelMaxL || L <= 0) return cudaErrorInvalidValue;
    if (nq <= 0) return cudaSuccess;
    note_launch();
    merge_keys_kernel<<<nq, kSelT, 0, st>>>(keys, n, L, int_dist, out_ids, out_dist, out_idist);
    return cudaGetLastError();
}

cudaError_t merge_shard_keys(const uint64_t* keys, int S, int nq, int L, int32_t* out_ids, cudaStream_t st) {
    if (S <= 0 || L <= 0 || L > 32 || S * L > 256) return cudaErrorInvalidValue;
    if (nq <= 0) return cudaSuccess;
    const int n = S * L;
    const unsigned blocks = (unsigned)(((size_t)nq * 32 + 255) / 256);
    note_launch();
    if (n <= 32) merge_shard_keys_kernel<1><<<blocks, 256, 0, st>>>(keys, S, nq, L, out_ids);
    else if (n <= 64) merge_shard_keys_kernel<2><<<blocks, 256, 0, st>>>(keys, S, nq, L, out_ids);
    else if (n <= 128) merge_shard_keys_kernel<4><<<blocks, 256, 0, st>>>(keys, S, nq, L, out_ids);
    else merge_shard_keys_kernel<8><<<blocks, 256, 0, st>>>(keys, S, nq, L, out_ids);
    return cudaGetLastError();
}

cudaError_t make_query_u8(const float* q, size_t n, uint8_t* out, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    size_t blocks = (n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    note_launch();
    make_u8_kernel<<<(int)blocks, 256, 0, st>>>(q, n, out);
    return cudaGetLastError();
}

}  // namespace isb
