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
                skeys[v] = make_key(acc, id);
            }
            __syncthreads();
            auto keyf = [&](int i) -> uint64_t { return skeys[i]; };
            block_filter_emit<kET>(keyf, len, cb, q, esm);
        }
    }
}

}  // namespace

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
        note_launch();
        default: exact_scan_kernel<0><<<grid, kET, 0, st>>>(q_u8, d, ls, wl, cb, work_counter); break;
    }
    return cudaGetLastError();
}

}  // namespace isb
