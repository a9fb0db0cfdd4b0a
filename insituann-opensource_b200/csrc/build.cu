// build.cu -- index build on the GPU: stable cluster-major reorder, k-means
// centroid update, residual-PQ codebook training and encoding.  The exact
// nearest-centroid assignment is the routing path with n_probes = 1
// (ivf_assign in capi.cu).
//
// The reference builds its indexes offline (k-means in
// cuda/clustering/kmeans/kmeans.cu, the stable reorder in
// cuda/dataset/dataset.cuh:559-592, residual PQ with faiss in
// scripts/train_ivfpq_residual.py:151-310).  Here every reduction runs in a
// fixed order -- rows of a list (or of a sub-space code) in increasing row
// order, summed in fp64 -- so a build is deterministic: the same input gives
// the same centroids, codebook and codes on every run and every GPU.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include <algorithm>

#include "launch.h"

namespace isb {

namespace {

__device__ __forceinline__ float row_val(const void* x, int is_u8, size_t i) {
    return is_u8 ? (float)static_cast<const uint8_t*>(x)[i] : static_cast<const float*>(x)[i];
}

__global__ void count_assign_kernel(const int32_t* __restrict__ a, int64_t n, int nlist, int32_t* counts,
                                    int* bad) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int l = a[i];
        if (l >= 0 && l < nlist) atomicAdd(&counts[l], 1);
        else atomicOr(bad, 1);
    }
}

__global__ void iota_kernel(int32_t* v, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        v[i] = (int32_t)i;
}

__global__ void i32_to_i64_kernel(const int32_t* in, int64_t* out, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = in[i];
}

// one block per list, one thread per dimension: the mean of the list's rows
// (in increasing row order, fp64); a list without rows keeps its centroid
__global__ void list_mean_kernel(const void* __restrict__ x, int is_u8, int d, const int64_t* __restrict__ offsets,
                                 const int32_t* __restrict__ counts, const int32_t* __restrict__ order,
                                 float* __restrict__ cent) {
    const int l = blockIdx.x;
    const int cnt = counts[l];
    if (cnt == 0) return;
    const int64_t off = offsets[l];
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        double s = 0.0;
        for (int i = 0; i < cnt; ++i) s += (double)row_val(x, is_u8, (size_t)order[off + i] * d + j);
        cent[(size_t)l * d + j] = (float)(s / (double)cnt);
    }
}

// codes of one sub-space: nearest of K = 256 codewords to the residual
// sub-vector (squared L2 summed in dimension order, ties to the smaller code)
template <int DSUB>
__global__ void __launch_bounds__(256) pq_encode_kernel(const void* __restrict__ x, int is_u8, int64_t n, int d,
                                                        const int32_t* __restrict__ rows,
                                                        const float* __restrict__ cent,
                                                        const int32_t* __restrict__ assign,
                                                        const float* __restrict__ cb, int M,
                                                        uint8_t* __restrict__ codes) {
    __shared__ float scb[kCodes * DSUB];
    const int m = blockIdx.y;
    for (int i = threadIdx.x; i < kCodes * DSUB; i += blockDim.x) scb[i] = cb[(size_t)m * kCodes * DSUB + i];
    __syncthreads();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = rows ? (int64_t)rows[i] : i;
        const int l = assign[row];
        float r[DSUB];
#pragma unroll
        for (int e = 0; e < DSUB; ++e) {
            const int j = m * DSUB + e;
            r[e] = __fsub_rn(row_val(x, is_u8, (size_t)row * d + j), cent[(size_t)l * d + j]);
        }
        float best = __int_as_float(0x7f800000);
        int bc = 0;
        for (int c = 0; c < kCodes; ++c) {
            float s = 0.f;
#pragma unroll
            for (int e = 0; e < DSUB; ++e) {
                const float t = __fsub_rn(r[e], scb[c * DSUB + e]);
                s = __fadd_rn(s, __fmul_rn(t, t));
            }
            if (s < best) {
                best = s;
                bc = c;
            }
        }
        codes[(size_t)i * M + m] = (uint8_t)bc;
    }
}

// (m, code) keys of every (row, sub-space) pair: key = m * 256 + code
__global__ void pq_pair_keys_kernel(const uint8_t* __restrict__ codes, int64_t n, int M, int32_t* keys) {
    const int64_t total = n * M;
    for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < total;
         p += (int64_t)gridDim.x * blockDim.x)
        keys[p] = (int32_t)((p % M) * kCodes + codes[p]);
}

// one warp per (m, code): the mean residual sub-vector of its pairs (sorted
// by pair index, i.e. by row), fp64; a code without pairs keeps its codeword
__global__ void pq_code_mean_kernel(const void* __restrict__ x, int is_u8, int d, int M, int dsub,
                                    const float* __restrict__ cent, const int32_t* __restrict__ assign,
                                    const int32_t* __restrict__ pair_of, const int64_t* __restrict__ off,
                                    const int32_t* __restrict__ cnt, float* __restrict__ cb) {
    const int seg = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (seg >= M * kCodes) return;
    const int c = cnt[seg];
    if (c == 0) return;
    const int m = seg / kCodes;
    const int64_t o = off[seg];
    for (int e = 0; e < dsub; ++e) {
        const int j = m * dsub + e;
        double s = 0.0;
        for (int i = lane; i < c; i += 32) {
            const int64_t row = pair_of[o + i] / M;
            s += (double)row_val(x, is_u8, (size_t)row * d + j) - (double)cent[(size_t)assign[row] * d + j];
        }
#pragma unroll
        for (int w = 16; w > 0; w >>= 1) s += __shfl_xor_sync(0xffffffffu, s, w);
        if (lane == 0) cb[(size_t)seg * dsub + e] = (float)(s / (double)c);
    }
}

int grid_for(int64_t n, int threads = 256) {
    int64_t b = (n + threads - 1) / threads;
    return (int)(b < 1 ? 1 : (b > 65535 ? 65535 : b));
}

// stable sort of `keys` [n] (values = 0..n-1) -> order; counts / offsets per key in [0, nkeys)
cudaError_t stable_groups(const int32_t* keys, int64_t n, int nkeys, int32_t* counts, int64_t* offsets,
                          int32_t* order, cudaStream_t st) {
    if (n >= (int64_t)INT32_MAX) return cudaErrorInvalidValue;
    cudaError_t e;
    int* bad = nullptr;
    int32_t *vals = nullptr, *kout = nullptr, *off32 = nullptr;
    void* tmp = nullptr;
    size_t tb = 0, tb2 = 0;
    int bits = 1;
    while ((1ll << bits) < nkeys) ++bits;
    if ((e = cudaMallocAsync(&bad, sizeof(int), st))) return e;
    if ((e = cudaMallocAsync(&vals, sizeof(int32_t) * (size_t)std::max<int64_t>(n, 1), st))) goto out;
    if ((e = cudaMallocAsync(&kout, sizeof(int32_t) * (size_t)std::max<int64_t>(n, 1), st))) goto out;
    if ((e = cudaMallocAsync(&off32, sizeof(int32_t) * ((size_t)nkeys + 1), st))) goto out;
    cudaMemsetAsync(bad, 0, sizeof(int), st);
    cudaMemsetAsync(counts, 0, sizeof(int32_t) * (size_t)nkeys, st);
    note_launch(2);
    count_assign_kernel<<<grid_for(n), 256, 0, st>>>(keys, n, nkeys, counts, bad);
    iota_kernel<<<grid_for(n), 256, 0, st>>>(vals, n);
    cub::DeviceRadixSort::SortPairs(nullptr, tb, (const int32_t*)nullptr, (int32_t*)nullptr,
                                    (const int32_t*)nullptr, (int32_t*)nullptr, (int)n, 0, bits, st);
    cub::DeviceScan::ExclusiveSum(nullptr, tb2, (int32_t*)nullptr, (int32_t*)nullptr, nkeys, st);
    if ((e = cudaMallocAsync(&tmp, std::max(tb, tb2), st))) goto out;
    // LSD radix sort is stable: equal keys keep increasing row order
    if ((e = cub::DeviceRadixSort::SortPairs(tmp, tb, keys, kout, vals, order, (int)n, 0, bits, st))) goto out;
    if ((e = cub::DeviceScan::ExclusiveSum(tmp, tb2, counts, off32, nkeys, st))) goto out;
    note_launch(1);
    i32_to_i64_kernel<<<grid_for(nkeys), 256, 0, st>>>(off32, offsets, nkeys);
    {
        int hbad = 0;
        if ((e = cudaMemcpyAsync(&hbad, bad, sizeof(int), cudaMemcpyDeviceToHost, st))) goto out;
        if ((e = cudaStreamSynchronize(st))) goto out;
        if (hbad) e = cudaErrorInvalidValue;       // a key outside [0, nkeys)
    }
out:
    cudaFreeAsync(tmp, st);
    cudaFreeAsync(off32, st);
    cudaFreeAsync(kout, st);
    cudaFreeAsync(vals, st);
    cudaFreeAsync(bad, st);
    return e ? e : cudaGetLastError();
}

}  // namespace

namespace {
__global__ void stage_rows_kernel(const void* __restrict__ x, int is_u8, size_t offset, size_t n,
                                  float* __restrict__ out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = row_val(x, is_u8, offset + i);
}
}  // namespace

cudaError_t stage_rows_f32(const void* x, int is_u8, size_t offset, size_t n, float* out, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    note_launch();
    stage_rows_kernel<<<grid_for((int64_t)n), 256, 0, st>>>(x, is_u8, offset, n, out);
    return cudaGetLastError();
}

cudaError_t build_reorder(const int32_t* assign, int64_t n, int nlist, int32_t* counts, int64_t* offsets,
                          int32_t* order, cudaStream_t st) {
    return stable_groups(assign, n, nlist, counts, offsets, order, st);
}

cudaError_t kmeans_update(const void* x, int is_u8, int64_t n, int d, const int32_t* assign, int nlist, float* cent,
                          cudaStream_t st) {
    cudaError_t e;
    int32_t *counts = nullptr, *order = nullptr;
    int64_t* offsets = nullptr;
    if ((e = cudaMallocAsync(&counts, sizeof(int32_t) * (size_t)nlist, st))) return e;
    if ((e = cudaMallocAsync(&offsets, sizeof(int64_t) * (size_t)nlist, st))) goto out;
    if ((e = cudaMallocAsync(&order, sizeof(int32_t) * (size_t)std::max<int64_t>(n, 1), st))) goto out;
    if ((e = stable_groups(assign, n, nlist, counts, offsets, order, st))) goto out;
    note_launch();
    list_mean_kernel<<<nlist, d < 256 ? ((d + 31) / 32) * 32 : 256, 0, st>>>(x, is_u8, d, offsets, counts, order,
                                                                            cent);
    e = cudaGetLastError();
out:
    cudaFreeAsync(order, st);
    cudaFreeAsync(offsets, st);
    cudaFreeAsync(counts, st);
    return e;
}

cudaError_t pq_encode_rows(const void* x, int is_u8, int64_t n, int d, const int32_t* rows, const float* cent,
                           const int32_t* assign, const float* cb, int M, uint8_t* codes, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (M <= 0 || d % M) return cudaErrorInvalidValue;
    const int dsub = d / M;
    const dim3 grid((unsigned)std::min<int64_t>((n + 255) / 256, 4096), (unsigned)M);
    note_launch();
    switch (dsub) {
        case 1: pq_encode_kernel<1><<<grid, 256, 0, st>>>(x, is_u8, n, d, rows, cent, assign, cb, M, codes); break;
        case 2: pq_encode_kernel<2><<<grid, 256, 0, st>>>(x, is_u8, n, d, rows, cent, assign, cb, M, codes); break;
        case 4: pq_encode_kernel<4><<<grid, 256, 0, st>>>(x, is_u8, n, d, rows, cent, assign, cb, M, codes); break;
        case 8: pq_encode_kernel<8><<<grid, 256, 0, st>>>(x, is_u8, n, d, rows, cent, assign, cb, M, codes); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t pq_train(const void* x, int is_u8, int64_t n, int d, const float* cent, const int32_t* assign, int M,
                     int iters, float* cb, cudaStream_t st) {
    if (n <= 0 || iters <= 0) return cudaSuccess;
    if (M <= 0 || d % M || n * M >= (int64_t)INT32_MAX) return cudaErrorInvalidValue;
    const int dsub = d / M, nseg = M * kCodes;
    cudaError_t e;
    uint8_t* codes = nullptr;
    int32_t *keys = nullptr, *cnt = nullptr, *pair_of = nullptr;
    int64_t* off = nullptr;
    const int64_t np = n * M;
    if ((e = cudaMallocAsync(&codes, (size_t)np, st))) return e;
    if ((e = cudaMallocAsync(&keys, sizeof(int32_t) * (size_t)np, st))) goto out;
    if ((e = cudaMallocAsync(&pair_of, sizeof(int32_t) * (size_t)np, st))) goto out;
    if ((e = cudaMallocAsync(&cnt, sizeof(int32_t) * (size_t)nseg, st))) goto out;
    if ((e = cudaMallocAsync(&off, sizeof(int64_t) * (size_t)nseg, st))) goto out;
    for (int it = 0; it < iters; ++it) {
        if ((e = pq_encode_rows(x, is_u8, n, d, nullptr, cent, assign, cb, M, codes, st))) goto out;
        note_launch();
        pq_pair_keys_kernel<<<grid_for(np), 256, 0, st>>>(codes, n, M, keys);
        if ((e = stable_groups(keys, np, nseg, cnt, off, pair_of, st))) goto out;
        note_launch();
        pq_code_mean_kernel<<<(unsigned)(((size_t)nseg * 32 + 255) / 256), 256, 0, st>>>(
            x, is_u8, d, M, dsub, cent, assign, pair_of, off, cnt, cb);
        if ((e = cudaGetLastError())) goto out;
    }
out:
    cudaFreeAsync(off, st);
    cudaFreeAsync(cnt, st);
    cudaFreeAsync(pair_of, st);
    cudaFreeAsync(keys, st);
    cudaFreeAsync(codes, st);
    return e;
}

}  // namespace isb
