// worklist.cu -- query -> list inversion built entirely on the device.
//
// The reference builds (query, list, chunk) descriptors with three CUB scans
// and a host read-back after each (updates/pq_update.cu:181-244, 907-936) and,
// on the CPU path, a per-batch hash map of touched clusters
// (cpu_fine_kernels_v3_u8.cpp:373-403).  Here one count pass, one device
// scan and one fill pass produce list-major (query, list) pairs with no host
// round trip; the scan kernels then pull pairs from a global counter.
#include <cub/device/device_scan.cuh>

#include "launch.h"

namespace isb {

namespace {

// pair index i (over nq x ncol) -> probe table entry: query i / ncol, column col0 + i % ncol
__device__ __forceinline__ size_t probe_at(size_t i, int nprobe, int col0, int ncol) {
    return (i / (size_t)ncol) * (size_t)nprobe + (size_t)col0 + i % (size_t)ncol;
}

__device__ __forceinline__ int local_list(const int32_t* probes, size_t i, int nlist_global,
                                          const int32_t* list_map) {
    int g = probes[i];
    if (g < 0 || g >= nlist_global) return -1;
    return list_map ? list_map[g] : g;
}

__global__ void count_pairs_kernel(const int32_t* probes, size_t total, int nprobe, int col0, int ncol,
                                   int nlist_global, const int32_t* list_map, int32_t* list_cnt) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        int l = local_list(probes, probe_at(i, nprobe, col0, ncol), nlist_global, list_map);
        if (l >= 0) atomicAdd(&list_cnt[l], 1);
    }
}

// Seeded two-pass split by local lists (thread per query): part 0 = the
// query's first probe column whose list is local, part 1 = its other local
// probes.  On an unsharded index that is column 0 and the rest.
__device__ __forceinline__ int first_local_col(const int32_t* probes, int q, int nprobe, int nlist_global,
                                               const int32_t* list_map) {
    for (int c = 0; c < nprobe; ++c)
        if (local_list(probes, (size_t)q * nprobe + c, nlist_global, list_map) >= 0) return c;
    return nprobe;
}

__global__ void count_seed_kernel(const int32_t* probes, int nq, int nprobe, int part, int nlist_global,
                                  const int32_t* list_map, int32_t* list_cnt) {
    for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < nq; q += gridDim.x * blockDim.x) {
        const int c0 = first_local_col(probes, q, nprobe, nlist_global, list_map);
        if (c0 >= nprobe) continue;
        const int cb = part == 0 ? c0 : c0 + 1, ce = part == 0 ? c0 + 1 : nprobe;
        for (int c = cb; c < ce; ++c) {
            const int l = local_list(probes, (size_t)q * nprobe + c, nlist_global, list_map);
            if (l >= 0) atomicAdd(&list_cnt[l], 1);
        }
    }
}

__global__ void fill_seed_kernel(const int32_t* probes, int nq, int nprobe, int part, int nlist_global,
                                 const int32_t* list_map, const int32_t* list_off, int32_t* cursor, int32_t* pair_q,
                                 int32_t* pair_l) {
    for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < nq; q += gridDim.x * blockDim.x) {
        const int c0 = first_local_col(probes, q, nprobe, nlist_global, list_map);
        if (c0 >= nprobe) continue;
        const int cb = part == 0 ? c0 : c0 + 1, ce = part == 0 ? c0 + 1 : nprobe;
        for (int c = cb; c < ce; ++c) {
            const int l = local_list(probes, (size_t)q * nprobe + c, nlist_global, list_map);
            if (l < 0) continue;
            const int p = list_off[l] + atomicAdd(&cursor[l], 1);
            pair_q[p] = q;
            pair_l[p] = l;
        }
    }
}

__global__ void fill_pairs_kernel(const int32_t* probes, size_t total, int nprobe, int col0, int ncol,
                                  int nlist_global, const int32_t* list_map, const int32_t* list_off,
                                  int32_t* cursor, int32_t* pair_q, int32_t* pair_l) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        int l = local_list(probes, probe_at(i, nprobe, col0, ncol), nlist_global, list_map);
        if (l < 0) continue;
        int slot = atomicAdd(&cursor[l], 1);
        int p = list_off[l] + slot;
        pair_q[p] = (int32_t)(i / (size_t)ncol);
        pair_l[p] = l;
    }
}

__global__ void group_count_kernel(const int32_t* list_cnt, int nlist, int gq, int32_t* grp_cnt) {
    int l = blockIdx.x * blockDim.x + threadIdx.x;
    if (l < nlist) grp_cnt[l] = (list_cnt[l] + gq - 1) / gq;
    else if (l == nlist) grp_cnt[l] = 0;
}

__global__ void group_fill_kernel(const int32_t* list_off, const int32_t* grp_off, int nlist, int gq, int shift,
                                  int64_t* groups) {
    int l = blockIdx.x * blockDim.x + threadIdx.x;
    if (l >= nlist) return;
    const int first = list_off[l], n = list_off[l + 1] - first;
    int g = grp_off[l];
    for (int o = 0; o < n; o += gq) {
        const int sz = n - o < gq ? n - o : gq;
        groups[g++] = ((int64_t)l << 32) | (int64_t)(((int64_t)(first + o) << shift) | sz);
    }
}

int grid_for(size_t total, int threads) {
    size_t b = (total + threads - 1) / threads;
    if (b < 1) b = 1;
    if (b > 148 * 16) b = 148 * 16;
    return (int)b;
}

}  // namespace

size_t worklist_scan_bytes(int nlist) {
    size_t bytes = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, bytes, (int32_t*)nullptr, (int32_t*)nullptr, nlist + 1);
    return bytes;
}

cudaError_t build_worklist(const int32_t* probes, int nq, int nprobe, int nlist_global,
                           const int32_t* list_map, int nlist_local, WorkList wl,
                           void* scan_tmp, size_t scan_bytes, cudaStream_t st, int col0, int ncol, int seed_part) {
    cudaError_t e;
    if (ncol <= 0) ncol = nprobe - col0;
    if ((e = cudaMemsetAsync(wl.list_cnt, 0, sizeof(int32_t) * (nlist_local + 1), st))) return e;
    if ((e = cudaMemsetAsync(wl.cursor, 0, sizeof(int32_t) * nlist_local, st))) return e;
    size_t total = (size_t)nq * (ncol > 0 ? ncol : 0);
    if (seed_part >= 0) {
        total = 0;
        if (nq > 0) {
            note_launch();
            count_seed_kernel<<<grid_for(nq, 256), 256, 0, st>>>(probes, nq, nprobe, seed_part, nlist_global,
                                                                 list_map, wl.list_cnt);
            if ((e = cudaGetLastError())) return e;
        }
    }
    if (total > 0) {
        note_launch();
        count_pairs_kernel<<<grid_for(total, 256), 256, 0, st>>>(probes, total, nprobe, col0, ncol, nlist_global,
                                                                 list_map, wl.list_cnt);
        if ((e = cudaGetLastError())) return e;
    }
    if ((e = cub::DeviceScan::ExclusiveSum(scan_tmp, scan_bytes, wl.list_cnt, wl.list_off, nlist_local + 1, st)))
        return e;
    if (total > 0) {
        note_launch();
        fill_pairs_kernel<<<grid_for(total, 256), 256, 0, st>>>(probes, total, nprobe, col0, ncol, nlist_global,
                                                                list_map, wl.list_off, wl.cursor, wl.pair_q,
                                                                wl.pair_l);
        if ((e = cudaGetLastError())) return e;
    }
    if (seed_part >= 0 && nq > 0) {
        note_launch();
        fill_seed_kernel<<<grid_for(nq, 256), 256, 0, st>>>(probes, nq, nprobe, seed_part, nlist_global, list_map,
                                                            wl.list_off, wl.cursor, wl.pair_q, wl.pair_l);
        if ((e = cudaGetLastError())) return e;
    }
    if (wl.groups) {
        note_launch();
        const int gq = wl.gq > 0 ? wl.gq : kGroupQueries;
        group_count_kernel<<<(nlist_local + 256) / 256, 256, 0, st>>>(wl.list_cnt, nlist_local, gq, wl.grp_cnt);
        if ((e = cudaGetLastError())) return e;
        if ((e = cub::DeviceScan::ExclusiveSum(scan_tmp, scan_bytes, wl.grp_cnt, wl.grp_off, nlist_local + 1, st)))
            return e;
        note_launch();
        group_fill_kernel<<<(nlist_local + 255) / 256, 256, 0, st>>>(wl.list_off, wl.grp_off, nlist_local, gq,
                                                                       group_shift(gq), wl.groups);
        if ((e = cudaGetLastError())) return e;
    }
    return cudaSuccess;
}

}  // namespace isb
