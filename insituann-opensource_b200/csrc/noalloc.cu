// noalloc.cu -- exact uint8 fine search that allocates no memory.
//
// Some hosts of this library cannot call cudaMalloc on the query path: a
// database backend that runs inside a memory-accounted worker (each worker's
// device allocations are budgeted up front, so a search that grows its own
// buffers would be refused or would have to be accounted elsewhere), a
// real-time service that must not hit the allocator (and its implicit
// device-wide synchronisation) per request, or a caller that only has a raw
// stream and pre-allocated buffers from its own pool.  For them this file
// offers ivf_u8_search_noalloc: the same exact search as ivf_u8_search on a
// given probe table, but all of its scratch lives in one fixed file-scope
// device array, so the call itself allocates nothing.
//
// The array is a __device__ variable: every GPU that loads the library holds
// its kNoAllocScratchBytes until the process exits.  Host code cannot use its
// name as a device address (that is a host-side stand-in), so the first call
// on each device looks the real address up with cudaGetSymbolAddress, with
// that device current, and caches it.  That first call should happen before
// any stream capture.  All calls share the array and it keeps the previous
// call's contents; every counter the search relies on is cleared by the call
// itself.  Two calls whose work overlaps on the GPU (different streams, or
// different host threads without ordering) race on the array.  The cached
// address lives as long as the device's primary context: a caller that runs
// cudaDeviceReset while the library is loaded must not call this entry point
// again in that process.  The call leaves the caller's current device as it
// found it.
#include <cuda_runtime.h>

#include <mutex>
#include <shared_mutex>
#include <string>

#include "../../include/insitu_b200.h"
#include "launch.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB per device

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// device address of g_noalloc_scratch on the current device (set up once per device)
cudaError_t scratch_address(int dev, void** out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

// carves aligned sub-arrays out of the scratch; returns false when it does not fit
struct Carver {
    unsigned char* base;
    size_t used = 0, cap;
    template <class T>
    T* take(size_t n) {
        used = (used + 255) & ~(size_t)255;
        T* p = reinterpret_cast<T*>(base + used);
        used += sizeof(T) * (n ? n : 1);
        return p;
    }
    bool fits() const { return used <= cap; }
};

}  // namespace

// Defined in capi.cu: layout facts of a loaded uint8 index, and the calling
// thread's error message read by ivf_global_last_error().
namespace isb {
bool u8_index_view(void* idx_ctx, ListStore* ls, int* nlist, int* nlist_global, const int32_t** g2l, int* d,
                   int* max_count, int* device);
void set_global_error(const std::string& msg);
// shared hold on the index's arrays: a concurrent call that replaces them
// (delete mask, delta segment) waits until this call has queued its work
std::shared_lock<std::shared_mutex> index_read_lock(void* idx_ctx);
}  // namespace isb

namespace {
int fail(int code, const std::string& msg) {
    isb::set_global_error(msg);
    return code;
}

// makes `dev` current for the lifetime of the guard, then restores the
// caller's device
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};
}  // namespace

extern "C" int ivf_u8_search_noalloc(void* idx_ctx, const uint8_t* d_query_u8, const int* d_probes, int n_query,
                                     int n_probes, int k, int* d_out_ids, int* d_out_dist, void* stream) {
    using namespace isb;
    ListStore ls{};
    int nlist = 0, nlist_global = 0, d = 0, max_count = 0, dev = 0;
    const int32_t* g2l = nullptr;
    auto rd = index_read_lock(idx_ctx);
    if (!u8_index_view(idx_ctx, &ls, &nlist, &nlist_global, &g2l, &d, &max_count, &dev))
        return fail(IVF_ESTATE, "ivf_u8_search_noalloc: not a loaded uint8 exact index");
    if (n_query < 0 || n_probes <= 0 || k <= 0 || k > 4096)
        return fail(IVF_EINVAL, "ivf_u8_search_noalloc: need n_query >= 0, n_probes > 0, 0 < k <= 4096");
    if ((n_query > 0) && (!d_query_u8 || !d_probes || !d_out_ids || !d_out_dist))
        return fail(IVF_EINVAL, "ivf_u8_search_noalloc: null device pointer");
    if (n_query == 0) return IVF_OK;
    if (dev < 0 || dev >= kMaxDevices) return fail(IVF_EINVAL, "ivf_u8_search_noalloc: device index out of range");
    DeviceGuard guard(dev);
    int cur = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess || cur != dev)
        return fail(IVF_ECUDA, std::string("could not make the index's device current: ") + cudaGetErrorString(e));
    void* base = nullptr;
    e = scratch_address(dev, &base);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(IVF_ECUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    // every chunk of kExactScanChunk vectors keeps at most k keys per query, so
    // this capacity cannot overflow
    const long long chunks = ((long long)(max_count > 0 ? max_count : 1) + kExactScanChunk - 1) / kExactScanChunk;
    const long long cap = (long long)n_probes * chunks * (k < kExactScanChunk ? k : kExactScanChunk);
    Carver cv{static_cast<unsigned char*>(base), 0, kNoAllocScratchBytes};
    WorkList wl{};
    wl.list_cnt = cv.take<int32_t>((size_t)nlist + 1);
    wl.list_off = cv.take<int32_t>((size_t)nlist + 1);
    wl.cursor = cv.take<int32_t>((size_t)nlist + 1);
    wl.pair_q = cv.take<int32_t>((size_t)n_query * n_probes);
    wl.pair_l = cv.take<int32_t>((size_t)n_query * n_probes);
    wl.n_pairs = wl.list_off + nlist;
    // the grouped kernel (one read of a list per 64 probing queries) where the
    // shape allows it, as ivf_u8_search chooses; its group words hold pair
    // indices below 2^25
    const bool grouped = exact_group_usable(d, k) && ls.sqnorm != nullptr &&
                         (size_t)n_query * n_probes < ((size_t)1 << 25);
    if (grouped) {
        wl.grp_cnt = cv.take<int32_t>((size_t)nlist + 1);
        wl.grp_off = cv.take<int32_t>((size_t)nlist + 1);
        wl.groups = cv.take<int64_t>((size_t)n_query * n_probes);
        wl.n_groups = wl.grp_off + nlist;
        wl.gq = 64;
    }
    const size_t scan_bytes = worklist_scan_bytes(nlist);
    void* scan_tmp = cv.take<unsigned char>(scan_bytes);
    CandBuf cb{};
    cb.keys = cv.take<uint64_t>((size_t)n_query * (size_t)cap);
    cb.cnt = cv.take<int32_t>((size_t)n_query);
    cb.thr = cv.take<unsigned long long>((size_t)n_query);
    cb.overflow = cv.take<int32_t>(1);
    cb.cap = (int)cap;
    cb.R = k;
    int* counter = cv.take<int>(1);
    uint64_t* topk = cv.take<uint64_t>((size_t)n_query * k);
    if (!cv.fits() || cap > (1ll << 30))
        return fail(IVF_EINVAL, "ivf_u8_search_noalloc: this batch needs " + std::to_string(cv.used) +
                                    " bytes of scratch, more than the fixed " +
                                    std::to_string(kNoAllocScratchBytes) +
                                    "; use fewer queries or probes per call, or ivf_u8_search");

    if ((e = cudaMemsetAsync(cb.overflow, 0, sizeof(int32_t), st)) ||
        (e = build_worklist(d_probes, n_query, n_probes, nlist_global, g2l, nlist, wl, scan_tmp, scan_bytes, st)) ||
        (e = reset_candidates(cb, n_query, st)) ||
        (e = grouped ? exact_group_scan(d_query_u8, d, k, ls, wl, n_query * n_probes, cb, counter, st)
                     : exact_scan(d_query_u8, n_query, d, ls, wl, n_query * n_probes, cb, counter, st)) ||
        (e = select_top_r(cb, n_query, topk, st)) ||
        (e = keys_to_exact_results(topk, n_query, k, d_out_ids, d_out_dist, nullptr, st))) {
        cudaGetLastError();
        return fail(IVF_ECUDA, std::string("ivf_u8_search_noalloc: ") + cudaGetErrorString(e));
    }
    isb::set_global_error("");
    return IVF_OK;
}
