// capi.cu -- index / batch contexts and the C ABI declared in include/insitu_b200.h.
//
// Contexts mirror the reference's IVFIndexContext / IVFQueryBatchContext
// (cuda/search/ivf_search_separated.cu:31-93): the index context owns the
// device-resident lists, the batch context owns one stream and the scratch of
// a query batch.  Unlike the reference, no call allocates per batch once the
// scratch has grown to the batch shape, no call synchronises the host in the
// middle of a search, and no call exits or resets the device.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <shared_mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/insitu_b200.h"
#include "launch.h"

using namespace isb;

namespace {

constexpr uint32_t kIdxMagic = 0x31584449u;  // "IDX1"
constexpr uint32_t kBatMagic = 0x31544142u;  // "BAT1"
constexpr int kKindEmpty = 0, kKindF32 = 1, kKindU8 = 2, kKindPQ = 3, kKindRoute = 4;

struct ApiError : std::runtime_error {
    int code;
    ApiError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int code, const std::string& msg) { throw ApiError(code, msg); }

void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(e == cudaErrorMemoryAllocation ? IVF_ENOMEM : IVF_ECUDA,
             std::string(what) + ": " + cudaGetErrorString(e));
    }
}

void require(bool ok, const std::string& msg, int code = IVF_EINVAL) {
    if (!ok) fail(code, msg);
}

template <class T>
T* dalloc(size_t n, std::vector<void*>& owned) {
    void* p = nullptr;
    ck(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)), "cudaMalloc");
    owned.push_back(p);
    return static_cast<T*>(p);
}

// copies n elements from host or device memory (the runtime infers which from
// the pointer) into a new device array owned by `owned`
template <class T>
T* dcopy(const T* h, size_t n, std::vector<void*>& owned) {
    T* d = dalloc<T>(n, owned);
    if (n) ck(cudaMemcpy(d, h, n * sizeof(T), cudaMemcpyDefault), "cudaMemcpy to device");
    return d;
}

void free_all(std::vector<void*>& owned) {
    for (void* p : owned) cudaFree(p);
    owned.clear();
}

struct Segment {
    uint8_t* data = nullptr;
    int64_t* offsets = nullptr;
    int32_t* counts = nullptr;
    int32_t* ids = nullptr;
    int64_t* key_off = nullptr;
    uint8_t* rr_u8 = nullptr;
    float* rr_f32 = nullptr;
    uint8_t* gring = nullptr;      // PQ codes in the grouped-ring tile layout
    int64_t* gring_off = nullptr;  // [nlist] byte offset of each list's tiles
    int32_t* sqnorm = nullptr;     // [n] squared norm of each uint8 row (exact index)
    uint8_t* deleted = nullptr;    // [n] delete mask by position (ivf_set_deleted), or nullptr
    // delta segment only: each list's main rows then its delta rows as one
    // grouped-ring tile stream (pq_build_gring_mix), or nullptr
    uint8_t* mix = nullptr;
    int64_t* mix_off = nullptr;
    int64_t n = 0;
    int max_count = 0;
    std::vector<void*> owned;

    void release() {
        free_all(owned);
        *this = Segment();
    }
    ListStore view() const {
        return ListStore{data, offsets, counts, ids, key_off, rr_u8, rr_f32, gring, gring_off, n, sqnorm, deleted};
    }
};

struct IndexCtx {
    uint32_t magic = kIdxMagic;
    int device = 0;
    int kind = kKindEmpty;
    int nlist = 0, d = 0;
    int64_t n = 0;
    float* cent = nullptr;
    uint8_t* valid = nullptr;
    uint16_t* tc_ops = nullptr;  // tensor-core routing operand of the centroids (null: exact kernels only)
    float* tc_cn = nullptr;      // [nlist] squared centroid norms
    float* tc_cne = nullptr;     // the same per tile row, +inf for invalid lists and padding
    float* tc_cnmax = nullptr;   // largest squared norm of a valid centroid
    // tensor map over the uint8 rows of an exact index (exact_tc.cu); tc_rows_ok
    // false: the exact search uses the CUDA-core kernels
    alignas(64) unsigned char tc_rows_map[128] = {};
    bool tc_rows_ok = false;
    int M = 0, dsub = 0;
    float* f32_rows = nullptr;   // fp32 index (ivf_load_dataset / streaming upload): cluster-major rows
    float* f32_norms = nullptr;  // and their L2 norms (cosine)
    // streaming upload in progress (ivf_init_streaming_upload .. finalize)
    bool su_active = false;
    std::vector<int32_t> su_counts;
    std::vector<int64_t> su_offsets;
    float* codebook = nullptr;
    float* codebook_t = nullptr;   // [256, M, dsub]
    Segment main, delta;
    bool has_delta = false;
    int delta_search = 0;        // ivf_pq_delta_mode: 0 none, 1 direct, 2 combined stream, 3 own tiles
    // host copy of the published delta segment in delta-position order (list
    // major), kept so ivf_pq_insert can grow it
    std::vector<uint8_t> h_dcodes, h_draw_u8;
    std::vector<float> h_draw_f32;
    std::vector<int32_t> h_dids, h_dcounts;
    int nlist_global = 0;        // == nlist unless the index is a shard
    int32_t* l2g = nullptr;      // [nlist] local -> global list id (shards)
    int32_t* g2l = nullptr;      // [nlist_global] global -> local list id or -1 (shards)
    std::vector<void*> owned;    // centroids, validity, codebook, shard maps, adopted arrays
    std::mutex mu;
    // Searches hold rw shared from reading the device arrays until their
    // launches are queued; calls that replace arrays (delete mask, delta
    // segment, loads) hold it exclusively, then synchronise the device before
    // freeing, so no queued or later kernel reads freed memory.
    std::shared_mutex rw;
    std::string err;
};

struct Grow {
    void* p = nullptr;
    size_t bytes = 0;
};

struct BatchCtx {
    uint32_t magic = kBatMagic;
    int device = 0;
    cudaStream_t st = nullptr;
    int max_nq = 0, d = 0, max_nprobe = 0, max_k = 0, nlist = 0;
    float* q = nullptr;
    uint8_t* q_u8 = nullptr;
    int32_t* probes = nullptr;
    int32_t* out_ids = nullptr;
    float* out_dist = nullptr;
    int32_t* out_idist = nullptr;
    int* counter = nullptr;
    int* overflow = nullptr;      // device flags: [0] candidate overflow, [1] routing wait gave up,
                                  // [2] fine-search (tensor-core) wait gave up
    int* h_overflow = nullptr;    // pinned mirror, read after the stream syncs
    int res_nq = 0, res_k = 0;
    int probes_nq = 0, probes_np = 0;
    Grow route_dist, route_rowfb, route_split, route_bound, wl_cnt, wl_off, wl_cursor, pair_q, pair_l, scan_tmp, grp_cnt, grp_off, groups;
    Grow cand_m, cand_d, cnt_m, cnt_d, thr_m, thr_d, s1m, s1d, exk;
    std::vector<void*> owned;
    std::string err;
    // optional per-stage CUDA-event timing (ivf_batch_profile / ivf_batch_stage_ms)
    bool prof = false;
    std::vector<cudaEvent_t> stage_ev[IVF_STAGE_COUNT];
    size_t stage_used[IVF_STAGE_COUNT] = {};
};

// Brackets the launches of one stage with events on the batch stream when
// profiling is on; elapsed times are summed by ivf_batch_stage_ms().
struct StageScope {
    BatchCtx* b;
    int s;
    StageScope(BatchCtx* b_, int s_) : b(b_), s(s_) { mark(); }
    ~StageScope() { mark(); }
    void mark() {
        if (!b->prof) return;
        auto& v = b->stage_ev[s];
        if (b->stage_used[s] >= v.size()) {
            cudaEvent_t e = nullptr;
            if (cudaEventCreate(&e) != cudaSuccess) {
                cudaGetLastError();
                return;
            }
            v.push_back(e);
        }
        cudaEventRecord(v[b->stage_used[s]++], b->st);
    }
};

thread_local std::string g_err;
std::atomic<unsigned long long> g_launches{0};

// device memory budget for per-batch candidate / routing scratch
// INSITU_SCRATCH_MB, else an eighth of the current device's memory, at most
// 24 GB and at least 1 GB (22.9 GB on a 183 GB B200: a 10k-query batch of
// the 100M-row index runs as one sub-batch, whose groups share each list's
// LUT and tile reads among more queries than two half batches would)
size_t scratch_budget() {
    const char* e = getenv("INSITU_SCRATCH_MB");
    long mb = e ? atol(e) : 0;
    if (mb > 0) return (size_t)mb << 20;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) {
        cudaGetLastError();
        total_b = (size_t)48 << 30;
    }
    return std::min<size_t>((size_t)24 << 30, std::max<size_t>((size_t)1 << 30, total_b / 8));
}

template <class T>
T* ensure(BatchCtx* b, Grow& g, size_t n) {
    size_t bytes = std::max<size_t>(n, 1) * sizeof(T);
    if (bytes <= g.bytes) return static_cast<T*>(g.p);
    if (g.p) {
        ck(cudaStreamSynchronize(b->st), "cudaStreamSynchronize");
        cudaFree(g.p);
        g.p = nullptr;
        g.bytes = 0;
    }
    ck(cudaMalloc(&g.p, bytes), "cudaMalloc (scratch)");
    g.bytes = bytes;
    return static_cast<T*>(g.p);
}

IndexCtx* as_index(void* p) {
    auto* c = static_cast<IndexCtx*>(p);
    require(c && c->magic == kIdxMagic, "not an index context");
    return c;
}

BatchCtx* as_batch(void* p) {
    auto* c = static_cast<BatchCtx*>(p);
    require(c && c->magic == kBatMagic, "not a batch context");
    return c;
}

// runs f, converting exceptions into (status, message on ctx)
template <class F>
int guarded(std::string* err, F&& f) {
    try {
        f();
        if (err) err->clear();
        g_err.clear();
        return IVF_OK;
    } catch (const ApiError& e) {
        if (err) *err = e.what();
        g_err = e.what();
        return e.code;
    } catch (const std::exception& e) {
        if (err) *err = e.what();
        g_err = e.what();
        return IVF_EINVAL;
    }
}

std::string* err_of(void* ctx) {
    if (!ctx) return nullptr;
    uint32_t m = *static_cast<uint32_t*>(ctx);
    if (m == kIdxMagic) return &static_cast<IndexCtx*>(ctx)->err;
    if (m == kBatMagic) return &static_cast<BatchCtx*>(ctx)->err;
    return nullptr;
}

int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// ---------------------------------------------------------------------------
// index loading helpers
// ---------------------------------------------------------------------------
void load_lists(IndexCtx* x, Segment& s, const uint8_t* data, size_t row_bytes, const long long* offsets,
                const int* counts, const int* ids, const long long* key_off, int nlist, long long n) {
    require(offsets && counts, "offsets and counts are required");
    int max_count = 0;
    for (int l = 0; l < nlist; ++l) {
        require(counts[l] >= 0, "negative list count");
        require(offsets[l] >= 0 && offsets[l] + counts[l] <= n, "list outside [0, n)");
        max_count = std::max(max_count, counts[l]);
    }
    require(n < (1ll << 32) - 1, "more than 2^32-2 vectors in one segment");
    (void)x;
    s.data = dcopy(data, (size_t)n * row_bytes, s.owned);
    s.offsets = dcopy(reinterpret_cast<const int64_t*>(offsets), (size_t)nlist, s.owned);
    s.counts = dcopy(reinterpret_cast<const int32_t*>(counts), (size_t)nlist, s.owned);
    s.ids = ids ? dcopy(reinterpret_cast<const int32_t*>(ids), (size_t)n, s.owned) : nullptr;
    s.key_off = key_off ? dcopy(reinterpret_cast<const int64_t*>(key_off), (size_t)nlist, s.owned) : nullptr;
    s.n = n;
    s.max_count = max_count;
}

// Re-lays a segment's PQ codes out as grouped-ring tiles when the grouped
// kernel scans this shape; the row-major copy is then dropped from the device
// unless keep_rows (a delta segment scanned by pq_delta_direct).
void build_gring(Segment& s, const int* counts, int nlist, int M, int d, bool keep_rows = false) {
    if (!pq_group_usable(M, d)) return;
    std::vector<int64_t> toff((size_t)nlist);
    int64_t acc = 0;
    for (int l = 0; l < nlist; ++l) {
        toff[(size_t)l] = acc;
        acc += pq_gring_list_bytes(counts[l], M);
    }
    s.gring_off = dcopy(toff.data(), toff.size(), s.owned);
    s.gring = dalloc<uint8_t>((size_t)acc + 64, s.owned);
    ck(pq_build_gring(s.data, s.offsets, s.counts, s.gring_off, nlist, M, s.gring, 0), "pq_build_gring");
    ck(cudaDeviceSynchronize(), "pq_build_gring");
    if (keep_rows) return;
    auto it = std::find(s.owned.begin(), s.owned.end(), (void*)s.data);
    if (it != s.owned.end()) {
        cudaFree(*it);
        s.owned.erase(it);
    }
    s.data = nullptr;
}

// tensor-core routing operands of the loaded centroids (when the shape allows)
void prepare_route_tc(IndexCtx* x, int nlist, int d) {
    if (!route_tc_usable(d, nlist)) return;
    x->tc_ops = dalloc<uint16_t>(route_tc_ops_elems(nlist, d), x->owned);
    x->tc_cn = dalloc<float>((size_t)nlist, x->owned);
    x->tc_cne = dalloc<float>(route_tc_cne_len(nlist), x->owned);
    x->tc_cnmax = dalloc<float>(1, x->owned);
    ck(route_tc_prepare(x->cent, x->valid, nlist, d, x->tc_ops, x->tc_cn, x->tc_cne, x->tc_cnmax, 0),
       "routing operands");
}

// Routing kernels (all give the same lists bit for bit), INSITU_ROUTE_TC:
//   0  the exact CUDA-core kernels only;
//   1  (default) the fused tensor-core kernel wherever it applies (nprobe <=
//      32, operands within shared memory), else the tensor-core matrix +
//      rescoring for 8192 lists or more, else the exact kernels;
//   2  the fused kernel where it applies, else the tensor-core matrix;
//   3  the tensor-core matrix + rescoring for every shape it covers.
// Read on every call.
// Exact uint8 groups, INSITU_EXACT_TC: 1 (default) the tensor-core kernel
// where it applies, 0 the CUDA-core grouped kernel.  Read on every call.
int exact_tc_mode() {
    const char* v = std::getenv("INSITU_EXACT_TC");
    return (v && v[0] == '0') ? 0 : 1;
}

int route_tc_mode() {
    const char* v = std::getenv("INSITU_ROUTE_TC");
    if (!v || !v[0]) return 1;
    return (v[0] >= '0' && v[0] <= '3') ? v[0] - '0' : 1;
}

void load_centroids(IndexCtx* x, const float* centroids, int nlist, int d) {
    require(centroids != nullptr, "centroids are required");
    x->cent = dcopy(centroids, (size_t)nlist * d, x->owned);
    x->valid = dalloc<uint8_t>((size_t)nlist, x->owned);
    ck(route_centroid_valid(x->cent, nlist, d, x->valid, 0), "centroid validity");
    prepare_route_tc(x, nlist, d);
    ck(cudaDeviceSynchronize(), "centroid validity");
    x->nlist = nlist;
    x->nlist_global = nlist;
    x->d = d;
}

// ---------------------------------------------------------------------------
// search drivers
// ---------------------------------------------------------------------------
void check_shape(BatchCtx* b, IndexCtx* x, int nq, int nprobe, int k) {
    require(x->kind != kKindEmpty, "index context holds no index", IVF_ESTATE);
    require(nq >= 0 && nq <= b->max_nq, "n_query outside [0, max_n_query]");
    require(nprobe > 0 && nprobe <= b->max_nprobe, "n_probes outside [1, max_n_probes]");
    require(k > 0 && k <= b->max_k, "k outside [1, max_k]");
    require(b->d == x->d, "batch and index dimensions differ");
}

// top-nprobe of the staged queries over the index's (local) centroids.
// keys != nullptr: write sorted keys with global list ids instead of probes.
void do_route(BatchCtx* b, IndexCtx* x, int nq, int nprobe, uint64_t* keys, bool cosine = false) {
    require(x->nlist_global >= nprobe || keys, "n_probes > n_total_clusters");
    const int L = std::min(nprobe, 2048);
    require(L == nprobe, "n_probes > 2048 is not supported");
    StageScope stage(b, IVF_STAGE_ROUTE);
    // the routing kernels report a bounded wait that gave up in flag word 1,
    // which the fine-search stages do not reset
    int* rflag = b->overflow + 1;
    ck(cudaMemsetAsync(rflag, 0, sizeof(int), b->st), "memset");
    const int mode = (x->tc_ops && !cosine) ? route_tc_mode() : 0;
    if ((mode == 1 || mode == 2) && route_tc_fused_usable(x->d, x->nlist, nprobe)) {
        // one tcgen05 sweep, no distance matrix; the per-split keys bound the sub-batch
        const int splits = route_tc_fused_splits(nq, x->nlist);
        const size_t per_q = (size_t)splits * nprobe * sizeof(uint64_t) + 2 * sizeof(int32_t);
        const int nsub = (int)std::max<size_t>(1, std::min<size_t>((size_t)std::max(nq, 1), scratch_budget() / per_q));
        int32_t* fb = ensure<int32_t>(b, b->route_rowfb, (size_t)nsub);
        uint32_t* rbnd = ensure<uint32_t>(b, b->route_bound, (size_t)nsub);
        uint64_t* sk = splits > 1 ? ensure<uint64_t>(b, b->route_split, (size_t)nsub * splits * nprobe) : nullptr;
        for (int s = 0; s < nq; s += nsub) {
            const int n = std::min(nsub, nq - s);
            ck(route_tc_fused(b->q + (size_t)s * x->d, n, x->tc_ops, x->tc_cne, x->tc_cnmax, x->valid, x->nlist,
                              x->d, x->cent, nprobe, x->l2g, keys ? nullptr : b->probes + (size_t)s * nprobe,
                              keys ? keys + (size_t)s * nprobe : nullptr, fb, sk, rbnd, splits, rflag, b->st),
               "route_tc_fused");
        }
    } else {
        size_t row = (size_t)x->nlist * sizeof(uint32_t);
        int nsub = (int)std::max<size_t>(1, std::min<size_t>((size_t)nq, scratch_budget() / 4 / row));
        uint32_t* dist = ensure<uint32_t>(b, b->route_dist, (size_t)nsub * x->nlist);
        const bool tc = mode >= 2 || (mode == 1 && x->nlist >= 8192);
        for (int s = 0; s < nq; s += nsub) {
            int n = std::min(nsub, nq - s);
            const float* qs = b->q + (size_t)s * x->d;
            if (tc) {
                ck(route_tc(qs, n, x->tc_ops, x->tc_cn, x->valid, x->nlist, x->d, dist, rflag, b->st),
                   "route_tc");
                ck(route_rescore(dist, qs, n, x->cent, x->tc_cnmax, x->valid, x->nlist, x->d, nprobe, x->l2g,
                                 keys ? nullptr : b->probes + (size_t)s * nprobe, nullptr,
                                 keys ? keys + (size_t)s * nprobe : nullptr, b->st),
                   "route_rescore");
                continue;
            }
            if (cosine)
                ck(route_distances_cos(qs, n, x->cent, x->valid, x->nlist, x->d, dist, b->st), "route_distances_cos");
            else
                ck(route_distances(qs, n, x->cent, x->valid, x->nlist, x->d, dist, b->st), "route_distances");
            if (keys) {
                ck(route_select(dist, n, x->nlist, nprobe, x->l2g, nullptr, nullptr, keys + (size_t)s * nprobe,
                                b->st),
                   "route_select");
            } else {
                ck(route_select(dist, n, x->nlist, nprobe, x->l2g, b->probes + (size_t)s * nprobe, nullptr,
                                nullptr, b->st),
                   "route_select");
            }
        }
    }
    ck(cudaMemcpyAsync(b->h_overflow + 1, rflag, sizeof(int), cudaMemcpyDeviceToHost, b->st), "flag D2H");
    if (!keys) {
        b->probes_nq = nq;
        b->probes_np = nprobe;
    }
}

WorkList worklist_for(BatchCtx* b, IndexCtx* x, int nsub, int nprobe, void** tmp, size_t* tmp_bytes,
                      bool groups = false) {
    WorkList wl{};
    if (groups) {
        wl.grp_cnt = ensure<int32_t>(b, b->grp_cnt, (size_t)x->nlist + 1);
        wl.grp_off = ensure<int32_t>(b, b->grp_off, (size_t)x->nlist + 1);
        wl.groups = ensure<int64_t>(b, b->groups, (size_t)nsub * nprobe);
        wl.n_groups = wl.grp_off + x->nlist;
    }
    wl.list_cnt = ensure<int32_t>(b, b->wl_cnt, (size_t)x->nlist + 1);
    wl.list_off = ensure<int32_t>(b, b->wl_off, (size_t)x->nlist + 1);
    wl.cursor = ensure<int32_t>(b, b->wl_cursor, (size_t)x->nlist + 1);
    wl.pair_q = ensure<int32_t>(b, b->pair_q, (size_t)nsub * nprobe);
    wl.pair_l = ensure<int32_t>(b, b->pair_l, (size_t)nsub * nprobe);
    wl.n_pairs = wl.list_off + x->nlist;
    *tmp_bytes = worklist_scan_bytes(x->nlist);
    *tmp = ensure<uint8_t>(b, b->scan_tmp, *tmp_bytes);
    return wl;
}

void require_probes(BatchCtx* b, int nq, int nprobe) {
    require(b->probes_nq >= nq && b->probes_np == nprobe,
            "no probe table for this (n_query, n_probes): route or set probes first", IVF_ESTATE);
}

// clears the flags a fine search raises (candidate overflow, tensor-core wait)
void reset_fine_flags(BatchCtx* b) {
    ck(cudaMemsetAsync(b->overflow, 0, sizeof(int), b->st), "memset");
    ck(cudaMemsetAsync(b->overflow + 2, 0, sizeof(int), b->st), "memset");
}

void queue_overflow_check(BatchCtx* b) {
    ck(cudaMemcpyAsync(b->h_overflow, b->overflow, sizeof(int), cudaMemcpyDeviceToHost, b->st), "overflow D2H");
    ck(cudaMemcpyAsync(b->h_overflow + 2, b->overflow + 2, sizeof(int), cudaMemcpyDeviceToHost, b->st),
       "flag D2H");
}

// exact uint8 search on the batch probes; keys_out: per-query sorted top-k keys instead of results
void run_u8(BatchCtx* b, IndexCtx* x, int nq, int nprobe, int k, uint64_t* keys_out) {
    require(x->kind == kKindU8, "index is not a uint8 exact index", IVF_ESTATE);
    require_probes(b, nq, nprobe);
    ck(make_query_u8(b->q, (size_t)nq * x->d, b->q_u8, b->st), "make_query_u8");
    const int cap = nprobe * ceil_div(std::max(x->main.max_count, 1), kExactScanChunk) *
                    std::min(k, kExactScanChunk);
    size_t per_q = (size_t)cap * 8 + (size_t)k * 8 + 16;
    int nsub = (int)std::max<size_t>(1, std::min<size_t>((size_t)std::max(nq, 1), scratch_budget() / per_q));
    void* tmp;
    size_t tmp_bytes;
    // the grouped kernel reads every list once per 64 queries; its group words
    // hold pair indices below 2^25
    const bool grouped = exact_group_usable(x->d, k) && x->main.sqnorm != nullptr &&
                         (size_t)nsub * nprobe < ((size_t)1 << 25);
    WorkList wl = worklist_for(b, x, nsub, nprobe, &tmp, &tmp_bytes, grouped);
    if (grouped) wl.gq = 64;
    // groups on the tensor cores (exact_tc.cu) unless INSITU_EXACT_TC=0
    const bool use_tc = grouped && x->tc_rows_ok && exact_tc_usable(x->d, k) && exact_tc_mode() != 0;
    if (use_tc) wl.gq = 127;     // the tensor-core kernel takes up to 127 queries per group
    CandBuf cb{};
    cb.keys = ensure<uint64_t>(b, b->cand_m, (size_t)nsub * cap);
    cb.cnt = ensure<int32_t>(b, b->cnt_m, (size_t)nsub);
    cb.thr = ensure<unsigned long long>(b, b->thr_m, (size_t)nsub);
    cb.overflow = b->overflow;
    cb.cap = cap;
    cb.R = k;
    uint64_t* topk = ensure<uint64_t>(b, b->exk, (size_t)nsub * k);
    reset_fine_flags(b);
    for (int s = 0; s < nq; s += nsub) {
        int n = std::min(nsub, nq - s);
        {
            StageScope stage(b, IVF_STAGE_WORKLIST);
            ck(reset_candidates(cb, n, b->st), "reset_candidates");
        }
        // Two passes over the probe table, as in the residual-PQ search: every
        // query's nearest list first, whose k smallest bound the query tightly,
        // then its other probes, of which few rows then pass.  The result does
        // not depend on the order.
        const int npass = nprobe > 1 ? 2 : 1;
        for (int pass = 0; pass < npass; ++pass) {
            const int ncol = npass == 1 ? nprobe : (pass == 0 ? 1 : nprobe - 1);   // bound on pairs per query
            {
                StageScope stage(b, IVF_STAGE_WORKLIST);
                ck(build_worklist(b->probes + (size_t)s * nprobe, n, nprobe, x->nlist_global, x->g2l, x->nlist, wl,
                                  tmp, tmp_bytes, b->st, 0, npass == 1 ? nprobe : 0, npass == 1 ? -1 : pass),
                   "build_worklist");
            }
            StageScope stage(b, IVF_STAGE_SCAN);
            if (use_tc)
                ck(exact_tc_scan(x->tc_rows_map, b->q_u8 + (size_t)s * x->d, x->d, k, x->main.view(), wl,
                                 n * ncol, cb, b->counter, b->overflow + 2, b->st),
                   "exact_tc_scan");
            else if (grouped)
                ck(exact_group_scan(b->q_u8 + (size_t)s * x->d, x->d, k, x->main.view(), wl, n * ncol, cb,
                                    b->counter, b->st),
                   "exact_group_scan");
            else
                ck(exact_scan(b->q_u8 + (size_t)s * x->d, n, x->d, x->main.view(), wl, n * ncol, cb, b->counter,
                              b->st),
                   "exact_scan");
        }
        uint64_t* dst = keys_out ? keys_out + (size_t)s * k : topk;
        {
            StageScope stage(b, IVF_STAGE_SELECT);
            ck(select_top_r(cb, n, dst, b->st), "select_top_r");
            if (!keys_out)
                ck(keys_to_exact_results(topk, n, k, b->out_ids + (size_t)s * k, b->out_idist + (size_t)s * k,
                                         b->out_dist + (size_t)s * k, b->st),
                   "keys_to_exact_results");
        }
    }
    queue_overflow_check(b);
    b->res_nq = nq;
    b->res_k = k;
}

// exact fp32 search (L2, or cosine) on the batch probes of an fp32 index
void run_f32(BatchCtx* b, IndexCtx* x, int nq, int nprobe, int k, bool cosine) {
    require(x->kind == kKindF32 && x->f32_rows, "index is not an fp32 index", IVF_ESTATE);
    require(x->d <= 512, "fp32 search needs d <= 512");
    require_probes(b, nq, nprobe);
    const int cap = nprobe * ceil_div(std::max(x->main.max_count, 1), kExactScanChunk) *
                    std::min(k, kExactScanChunk);
    size_t per_q = (size_t)cap * 8 + (size_t)k * 8 + 16;
    int nsub = (int)std::max<size_t>(1, std::min<size_t>((size_t)std::max(nq, 1), scratch_budget() / per_q));
    void* tmp;
    size_t tmp_bytes;
    WorkList wl = worklist_for(b, x, nsub, nprobe, &tmp, &tmp_bytes, false);
    CandBuf cb{};
    cb.keys = ensure<uint64_t>(b, b->cand_m, (size_t)nsub * cap);
    cb.cnt = ensure<int32_t>(b, b->cnt_m, (size_t)nsub);
    cb.thr = ensure<unsigned long long>(b, b->thr_m, (size_t)nsub);
    cb.overflow = b->overflow;
    cb.cap = cap;
    cb.R = k;
    uint64_t* topk = ensure<uint64_t>(b, b->exk, (size_t)nsub * k);
    reset_fine_flags(b);
    for (int s = 0; s < nq; s += nsub) {
        int n = std::min(nsub, nq - s);
        {
            StageScope stage(b, IVF_STAGE_WORKLIST);
            ck(build_worklist(b->probes + (size_t)s * nprobe, n, nprobe, x->nlist_global, x->g2l, x->nlist, wl,
                              tmp, tmp_bytes, b->st),
               "build_worklist");
            ck(reset_candidates(cb, n, b->st), "reset_candidates");
        }
        {
            StageScope stage(b, IVF_STAGE_SCAN);
            ck(f32_scan(b->q + (size_t)s * x->d, x->d, x->f32_rows, x->f32_norms, x->main.view(), cosine ? 1 : 0, wl,
                        n * nprobe, cb, b->counter, b->st),
               "f32_scan");
        }
        StageScope stage(b, IVF_STAGE_SELECT);
        ck(select_top_r(cb, n, topk, b->st), "select_top_r");
        ck(merge_keys(topk, n, k, k, 0, b->out_ids + (size_t)s * k, b->out_dist + (size_t)s * k, nullptr, b->st),
           "merge_keys");
    }
    queue_overflow_check(b);
    b->res_nq = nq;
    b->res_k = k;
}

PQParams pq_params(IndexCtx* x, const float* q, bool use_delta) {
    PQParams p{};
    p.q = q;
    p.cent = x->cent;
    p.codebook = x->codebook;
    p.codebook_t = x->codebook_t;
    p.d = x->d;
    p.M = x->M;
    p.dsub = x->dsub;
    p.main = x->main.view();
    p.delta = x->delta.view();
    p.has_delta = use_delta ? 1 : 0;
    p.mix = use_delta ? x->delta.mix : nullptr;
    p.mix_off = use_delta ? x->delta.mix_off : nullptr;
    return p;
}

// residual-PQ search on the batch probes.  shard outputs (all device, may be null):
//   adc/exact [nq, R], dadc/dexact [nq, Rd]; when adc is given no final top-k is formed.
void run_pq(BatchCtx* b, IndexCtx* x, int nq, int nprobe, int k, int rerank_n, bool overlay, int delta_topk,
            uint64_t* adc, uint64_t* exact, uint64_t* dadc, uint64_t* dexact) {
    require(x->kind == kKindPQ, "index is not a residual-PQ index", IVF_ESTATE);
    require_probes(b, nq, nprobe);
    const int R = std::max(rerank_n, adc ? 1 : k);
    const bool use_delta = overlay && x->has_delta && delta_topk > 0;
    const int Rd = use_delta ? delta_topk : 0;
    // the delta rows by their own kernel after the main scan (row-major delta
    // codes kept at publish), or in the scan's launches (candidate buffer cd)
    const bool direct = use_delta && x->delta.data != nullptr && pq_delta_direct_usable(x->M, x->d, Rd);
    const bool scan_delta = use_delta && !direct;
    require(R <= 4096 && R + Rd <= 4096, "rerank_n + delta_topk must be <= 4096");
    // every filtered chunk of a probed list appends at most min(R, chunk items) keys
    const int items = pq_scan_chunk_items(x->M, x->d);
    const int slack_m = pq_chunk_slack(x->M, x->d, R), slack_d = pq_chunk_slack(x->M, x->d, Rd);
    const int64_t cap_m64 = (int64_t)nprobe * std::max(1, pq_scan_chunks(x->M, x->d, x->main.max_count)) *
                            std::min(R + slack_m, items);
    // with the combined tile stream a probed list appends all of its delta rows
    const int64_t cap_d64 =
        scan_delta ? (int64_t)nprobe * std::max<int64_t>(x->delta.mix ? x->delta.max_count : 0,
                                                        std::max(1, pq_scan_chunks(x->M, x->d, x->delta.max_count)) *
                                                            std::min(Rd + slack_d, items))
                  : 0;
    require(cap_m64 <= (1ll << 30) && cap_d64 <= (1ll << 30),
            "candidate buffer of one query would exceed 2^30 keys (lists too long for this nprobe)", IVF_EOVERFLOW);
    const int cap_m = (int)cap_m64, cap_d = (int)cap_d64;
    size_t per_q = ((size_t)cap_m + cap_d + R + Rd) * 8 + 32;
    int nsub = (int)std::max<size_t>(1, std::min<size_t>((size_t)std::max(nq, 1), scratch_budget() / per_q));
    void* tmp;
    size_t tmp_bytes;
    WorkList wl = worklist_for(b, x, nsub, nprobe, &tmp, &tmp_bytes, pq_group_usable(x->M, x->d));
    CandBuf cm{}, cd{};
    cm.keys = ensure<uint64_t>(b, b->cand_m, (size_t)nsub * cap_m);
    cm.cnt = ensure<int32_t>(b, b->cnt_m, (size_t)nsub);
    cm.thr = ensure<unsigned long long>(b, b->thr_m, (size_t)nsub);
    cm.overflow = b->overflow;
    cm.cap = cap_m;
    cm.R = R;
    cm.slack = slack_m;
    uint64_t* s1m = ensure<uint64_t>(b, b->s1m, (size_t)nsub * R);
    uint64_t* s1d = use_delta ? ensure<uint64_t>(b, b->s1d, (size_t)nsub * Rd) : nullptr;
    if (scan_delta) {
        cd.keys = ensure<uint64_t>(b, b->cand_d, (size_t)nsub * cap_d);
        cd.cnt = ensure<int32_t>(b, b->cnt_d, (size_t)nsub);
        cd.thr = ensure<unsigned long long>(b, b->thr_d, (size_t)nsub);
        cd.overflow = b->overflow;
        cd.cap = cap_d;
        cd.R = Rd;
        cd.slack = slack_d;
    }
    reset_fine_flags(b);
    for (int s = 0; s < nq; s += nsub) {
        int n = std::min(nsub, nq - s);
        PQParams p = pq_params(x, b->q + (size_t)s * x->d, scan_delta);
        {
            StageScope stage(b, IVF_STAGE_WORKLIST);
            ck(reset_candidates(cm, n, b->st), "reset_candidates");
            if (scan_delta) ck(reset_candidates(cd, n, b->st), "reset_candidates");
        }
        // Two passes over the probe table: every query's nearest local list first,
        // which sets a tight rank-R bound, then its other local probes, which then
        // emit few candidates.  The result does not depend on the order.
        const int npass = nprobe > 1 ? 2 : 1;
        for (int pass = 0; pass < npass; ++pass) {
            const int ncol = npass == 1 ? nprobe : (pass == 0 ? 1 : nprobe - 1);   // bound on pairs per query
            {
                StageScope stage(b, IVF_STAGE_WORKLIST);
                ck(build_worklist(b->probes + (size_t)s * nprobe, n, nprobe, x->nlist_global, x->g2l, x->nlist, wl,
                                  tmp, tmp_bytes, b->st, 0, npass == 1 ? nprobe : 0, npass == 1 ? -1 : pass),
                   "build_worklist");
            }
            StageScope stage(b, IVF_STAGE_SCAN);
            ck(pq_scan(p, wl, n * ncol, cm, cd, b->counter, b->st), "pq_scan");
        }
        uint64_t* m_out = adc ? adc + (size_t)s * R : s1m;
        uint64_t* d_out = use_delta ? (dadc ? dadc + (size_t)s * Rd : s1d) : nullptr;
        if (direct) {
            StageScope stage(b, IVF_STAGE_SCAN);
            const PQParams pd = pq_params(x, b->q + (size_t)s * x->d, true);
            ck(pq_delta_direct(pd, b->probes + (size_t)s * nprobe, n, nprobe, x->nlist_global, x->g2l, Rd, d_out,
                               b->st),
               "pq_delta_direct");
        }
        {
            StageScope stage(b, IVF_STAGE_SELECT);
            // sorted stage-1 lists only where they leave the library (shard outputs)
            ck(select_top_r(cm, n, m_out, b->st, adc != nullptr), "select_top_r");
            if (scan_delta) ck(select_top_r(cd, n, d_out, b->st, adc != nullptr), "select_top_r (delta)");
        }
        StageScope stage(b, IVF_STAGE_RERANK);
        if (adc) {
            ck(pq_rerank(p, x->nlist, m_out, R, d_out, Rd, n, k, nullptr, nullptr, exact + (size_t)s * R,
                         use_delta ? dexact + (size_t)s * Rd : nullptr, b->st),
               "pq_rerank");
        } else {
            ck(pq_rerank(p, x->nlist, m_out, R, d_out, Rd, n, k, b->out_ids + (size_t)s * k,
                         b->out_dist + (size_t)s * k, nullptr, nullptr, b->st),
               "pq_rerank");
        }
    }
    if (adc && dadc && !use_delta) {
        // caller asked for delta outputs but there is no delta segment: empty lists
        ck(cudaMemsetAsync(dadc, 0xFF, sizeof(uint64_t) * (size_t)nq * std::max(delta_topk, 0), b->st), "memset");
        ck(cudaMemsetAsync(dexact, 0xFF, sizeof(uint64_t) * (size_t)nq * std::max(delta_topk, 0), b->st), "memset");
    }
    queue_overflow_check(b);
    if (!adc) {
        b->res_nq = nq;
        b->res_k = k;
    }
}

void check_overflow_after_sync(BatchCtx* b) {
    if ((b->h_overflow[0] | b->h_overflow[1] | b->h_overflow[2]) & 4)
        fail(IVF_ECUDA, "a bounded device wait of a tensor-core kernel gave up");
    if (*b->h_overflow)
        fail(IVF_EOVERFLOW, "a candidate buffer overflowed; raise INSITU_SCRATCH_MB or lower n_probes");
}

void copy_results(BatchCtx* b, float* dist, int* idx, int32_t* idist, int nq, int k, cudaMemcpyKind kind) {
    require(nq <= b->res_nq && k == b->res_k, "results of this shape are not available", IVF_ESTATE);
    size_t n = (size_t)nq * k;
    if (dist) ck(cudaMemcpyAsync(dist, b->out_dist, n * sizeof(float), kind, b->st), "results copy");
    if (idx) ck(cudaMemcpyAsync(idx, b->out_ids, n * sizeof(int32_t), kind, b->st), "results copy");
    if (idist) ck(cudaMemcpyAsync(idist, b->out_idist, n * sizeof(int32_t), kind, b->st), "results copy");
}

// ---------------------------------------------------------------------------
// registry (ivf_search_wrapper.cpp:329-427; a mutex makes it thread-safe)
// ---------------------------------------------------------------------------
constexpr int kMaxIndices = 64;
struct RegEntry {
    unsigned oid;
    void* handle;
    bool active;
};
RegEntry g_reg[kMaxIndices];
std::mutex g_reg_mu;

// ---------------------------------------------------------------------------
// coarse handle state (stored behind CoarseHandle::cublas_handle)
// ---------------------------------------------------------------------------
struct RouteState {
    int device = 0;
    cudaStream_t st = nullptr;
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    BatchCtx* b = nullptr;     // scratch reuse through a private batch context
    IndexCtx* x = nullptr;     // view of the borrowed centroids
};
thread_local CoarseTimingBreakdown g_coarse_timing;

}  // namespace

namespace isb {
void note_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

bool u8_index_view(void* idx_ctx, ListStore* ls, int* nlist, int* nlist_global, const int32_t** g2l, int* d,
                   int* max_count, int* device) {
    auto* x = static_cast<IndexCtx*>(idx_ctx);
    if (!x || x->magic != kIdxMagic || x->kind != kKindU8) return false;
    *ls = x->main.view();
    *nlist = x->nlist;
    *nlist_global = x->nlist_global;
    *g2l = x->g2l;
    *d = x->d;
    *max_count = x->main.max_count;
    *device = x->device;
    return true;
}

void set_global_error(const std::string& msg) { g_err = msg; }

std::shared_lock<std::shared_mutex> index_read_lock(void* idx_ctx) {
    auto* x = static_cast<IndexCtx*>(idx_ctx);
    if (!x || x->magic != kIdxMagic) return std::shared_lock<std::shared_mutex>();
    return std::shared_lock<std::shared_mutex>(x->rw);
}
}  // namespace isb

// ===========================================================================
// C ABI
// ===========================================================================
namespace {

struct ShardPlan {
    CandBuf cm{};
    WorkList wl{};
    void* tmp = nullptr;
    size_t tmp_bytes = 0;
};

// the candidate buffers and work list of one phased search (one sub-batch)
ShardPlan shard_plan(BatchCtx* b, IndexCtx* x, int nq, int nprobe, int R) {
    require(x->kind == kKindPQ, "index is not a residual-PQ index", IVF_ESTATE);
    require(R > 0 && R <= 4096, "rerank_n must be in [1, 4096]");
    const int items = pq_scan_chunk_items(x->M, x->d);
    const int slack = pq_chunk_slack(x->M, x->d, R);
    const int64_t cap64 =
        (int64_t)nprobe * std::max(1, pq_scan_chunks(x->M, x->d, x->main.max_count)) * std::min(R + slack, items);
    require(cap64 <= (1ll << 30), "candidate buffer of one query would exceed 2^30 keys", IVF_EOVERFLOW);
    const size_t per_q = (size_t)cap64 * 8 + 32;
    require((size_t)std::max(nq, 1) <= std::max<size_t>(1, scratch_budget() / per_q),
            "the phased shard search takes one sub-batch: lower n_query or raise INSITU_SCRATCH_MB");
    ShardPlan sp;
    sp.wl = worklist_for(b, x, std::max(nq, 1), nprobe, &sp.tmp, &sp.tmp_bytes, pq_group_usable(x->M, x->d));
    sp.cm.keys = ensure<uint64_t>(b, b->cand_m, (size_t)std::max(nq, 1) * cap64);
    sp.cm.cnt = ensure<int32_t>(b, b->cnt_m, (size_t)std::max(nq, 1));
    sp.cm.thr = ensure<unsigned long long>(b, b->thr_m, (size_t)std::max(nq, 1));
    sp.cm.overflow = b->overflow;
    sp.cm.cap = (int)cap64;
    sp.cm.R = R;
    sp.cm.slack = slack;
    return sp;
}

}  // namespace

namespace {

// An fp32 index over cluster-major rows already on the device (the reference's
// ivf_load_dataset / streaming upload): counts [nlist] (device, adopted),
// offsets as the running sum of counts, per-row norms, centroid validity and
// the routing operands.
void adopt_f32_lists(IndexCtx* x, int* d_counts, float* d_rows, int nlist, long long n, int d,
                     const int64_t* h_offsets = nullptr) {
    std::vector<int32_t> hc((size_t)nlist);
    ck(cudaMemcpy(hc.data(), d_counts, sizeof(int32_t) * hc.size(), cudaMemcpyDeviceToHost), "counts D2H");
    std::vector<int64_t> off((size_t)nlist, 0);
    int maxc = 0;
    for (int l = 0; l < nlist; ++l) {
        require(hc[l] >= 0, "negative list size");
        if (h_offsets) off[l] = h_offsets[l];
        else if (l) off[l] = off[l - 1] + hc[l - 1];
        require(off[l] >= 0 && off[l] + hc[l] <= n, "a list lies outside [0, n_total_vectors)");
        maxc = std::max(maxc, hc[l]);
    }
    x->main.counts = d_counts;
    x->main.offsets = dcopy(off.data(), off.size(), x->owned);
    x->main.n = n;
    x->main.max_count = maxc;
    x->f32_rows = d_rows;
    x->f32_norms = dalloc<float>((size_t)std::max<long long>(n, 1), x->owned);
    ck(f32_row_norms(d_rows, n, d, x->f32_norms, 0), "row norms");
    x->valid = dalloc<uint8_t>((size_t)nlist, x->owned);
    ck(route_centroid_valid(x->cent, nlist, d, x->valid, 0), "centroid validity");
    prepare_route_tc(x, nlist, d);
    ck(cudaDeviceSynchronize(), "fp32 index");
    x->nlist = x->nlist_global = nlist;
    x->d = d;
    x->n = n;
    x->kind = kKindF32;
}

// How a published delta segment is searched (INSITU_PQ_DELTA, read when the
// delta is published): "direct" -- its rows by pq_delta_direct, a kernel of
// its own after the main scan, which computes each row's distance without a
// LUT (delta ranks above 32 fall back to "seg"); "mix" -- each list's main and
// delta rows in one combined tile stream, scanned in one pass with the main
// rows' LUT (a second copy of the main tiles); "seg" -- the delta rows in
// their own tiles, scanned after each list's main rows with the same LUT.
// Unset: "direct" for deltas of at most kDirectRowsPerList rows per list on
// average (a LUT would cost more than it saves), else "mix".
enum DeltaMode { kDeltaAuto = -1, kDeltaDirect = 0, kDeltaMix = 1, kDeltaSeg = 2 };
constexpr long long kDirectRowsPerList = 100;
DeltaMode delta_mode() {
    const char* e = std::getenv("INSITU_PQ_DELTA");
    if (e && std::strcmp(e, "direct") == 0) return kDeltaDirect;
    if (e && std::strcmp(e, "mix") == 0) return kDeltaMix;
    if (e && std::strcmp(e, "seg") == 0) return kDeltaSeg;
    return kDeltaAuto;
}

// Lays out every list's main rows followed by its delta rows (the delta
// segment s, already in grouped-ring tiles) as one tile stream, so that a
// search scans both in one pass over the list.
void build_mix(IndexCtx* x, Segment& s, const int* dcounts) {
    std::vector<int32_t> mc((size_t)x->nlist);
    ck(cudaMemcpy(mc.data(), x->main.counts, sizeof(int32_t) * mc.size(), cudaMemcpyDeviceToHost), "main counts");
    std::vector<int64_t> off((size_t)x->nlist);
    int64_t acc = 0;
    for (int l = 0; l < x->nlist; ++l) {
        off[(size_t)l] = acc;
        acc += pq_mix_list_bytes(mc[(size_t)l], dcounts[l], x->M);
    }
    s.mix_off = dcopy(off.data(), off.size(), s.owned);
    s.mix = dalloc<uint8_t>((size_t)acc + 64, s.owned);
    ck(pq_build_gring_mix(x->main.gring, x->main.gring_off, x->main.counts, s.gring, s.gring_off, s.counts, s.mix_off,
                          x->nlist, x->M, s.mix, 0),
       "pq_build_gring_mix");
    ck(cudaDeviceSynchronize(), "pq_build_gring_mix");
}

// Publishes a delta segment (the caller holds x->mu): the new segment is built
// in full first, then swapped in under the exclusive index lock after the
// device has finished every queued search, so a search sees either the old
// segment or the new one.  Keeps a host copy for ivf_pq_insert (the arrays may
// be host or device pointers).
void publish_delta_locked(IndexCtx* x, const uint8_t* codes, const int* ids, const int* counts,
                          const long long* offsets, const long long* key_offsets, const uint8_t* raw_u8,
                          const float* raw_f32, long long n_delta) {
    require(x->kind == kKindPQ, "publish needs a residual-PQ index", IVF_ESTATE);
    require(n_delta >= 0, "negative n_delta");
    require(ids != nullptr || n_delta == 0, "delta ids are required");
    require(counts && offsets, "delta counts and offsets are required");
    const bool f32 = x->main.rr_f32 != nullptr;
    require(n_delta == 0 || (f32 ? raw_f32 != nullptr : raw_u8 != nullptr),
            "delta rerank rows must match the base type");
    cudaSetDevice(x->device);
    Segment s;
    std::vector<uint8_t> hc((size_t)n_delta * x->M), hu;
    std::vector<float> hf;
    std::vector<int32_t> hi((size_t)n_delta), hcnt(counts, counts + x->nlist);
    DeltaMode mode = kDeltaSeg;
    try {
        load_lists(x, s, codes, (size_t)x->M, offsets, counts, ids, key_offsets, x->nlist, n_delta);
        if (f32) s.rr_f32 = dcopy(raw_f32, (size_t)n_delta * x->d, s.owned);
        else s.rr_u8 = dcopy(raw_u8, (size_t)n_delta * x->d, s.owned);
        if (n_delta) {
            ck(cudaMemcpy(hc.data(), s.data, hc.size(), cudaMemcpyDeviceToHost), "delta copy");
            ck(cudaMemcpy(hi.data(), s.ids, sizeof(int32_t) * hi.size(), cudaMemcpyDeviceToHost), "delta copy");
            if (f32) {
                hf.resize((size_t)n_delta * x->d);
                ck(cudaMemcpy(hf.data(), s.rr_f32, sizeof(float) * hf.size(), cudaMemcpyDeviceToHost), "delta copy");
            } else {
                hu.resize((size_t)n_delta * x->d);
                ck(cudaMemcpy(hu.data(), s.rr_u8, hu.size(), cudaMemcpyDeviceToHost), "delta copy");
            }
        }
        mode = delta_mode();
        if (mode == kDeltaAuto) mode = n_delta <= kDirectRowsPerList * x->nlist ? kDeltaDirect : kDeltaMix;
        build_gring(s, counts, x->nlist, x->M, x->d, mode == kDeltaDirect);
        if (n_delta > 0 && s.gring && x->main.gring && mode == kDeltaMix) build_mix(x, s, counts);
    } catch (...) {
        s.release();
        throw;
    }
    std::unique_lock<std::shared_mutex> wr(x->rw);
    cudaError_t e = cudaDeviceSynchronize();                // no queued search still reads the old segment
    if (e != cudaSuccess) {
        s.release();
        ck(e, "cudaDeviceSynchronize");
    }
    x->delta.release();
    x->delta = std::move(s);
    x->has_delta = n_delta > 0;
    // how run_pq will search it (the direct kernel needs its shapes and the
    // row-major codes; the combined stream needs its tiles)
    x->delta_search = n_delta <= 0                                                       ? 0
                      : mode == kDeltaDirect && x->delta.data && pq_group_usable(x->M, x->d) ? 1
                      : x->delta.mix                                                      ? 2
                                                                                          : 3;
    x->h_dcodes.swap(hc);
    x->h_dids.swap(hi);
    x->h_dcounts.swap(hcnt);
    x->h_draw_u8.swap(hu);
    x->h_draw_f32.swap(hf);
}

}  // namespace

extern "C" {

void* ivf_create_index_context(void) {
    try {
        auto* x = new IndexCtx();
        cudaGetDevice(&x->device);
        return x;
    } catch (...) {
        g_err = "out of host memory";
        return nullptr;
    }
}

void ivf_destroy_index_context(void* idx_ctx) {
    if (!idx_ctx) return;
    auto* x = static_cast<IndexCtx*>(idx_ctx);
    if (x->magic != kIdxMagic) return;
    cudaSetDevice(x->device);
    cudaDeviceSynchronize();
    x->main.release();
    x->delta.release();
    free_all(x->owned);
    x->magic = 0;
    delete x;
}

int ivf_load_dataset(void* idx_ctx, int* d_cluster_size, float* d_cluster_vectors, float* d_cluster_centers,
                     int n_total_clusters, int n_total_vectors, int n_dim) {
    int ret = 0;
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx);
    } catch (...) {
        return 0;
    }
    int st = guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);
        std::unique_lock<std::shared_mutex> wr(x->rw);
        if (x->kind != kKindEmpty) {
            ret = 0;
            return;
        }
        require(d_cluster_size && d_cluster_vectors && d_cluster_centers, "null device array");
        require(n_total_clusters > 0 && n_total_vectors >= 0 && n_dim > 0, "bad sizes");
        cudaSetDevice(x->device);
        // ownership passes to the context (ivf_search_separated.cu:141-143)
        x->owned.push_back(d_cluster_size);
        x->owned.push_back(d_cluster_vectors);
        x->cent = d_cluster_centers;
        x->owned.push_back(d_cluster_centers);
        adopt_f32_lists(x, d_cluster_size, d_cluster_vectors, n_total_clusters, n_total_vectors, n_dim);
        ret = 1;
    });
    return st == IVF_OK ? ret : 0;
}

void* ivf_create_batch_context(int max_n_query, int n_dim, int max_n_probes, int max_k, int n_total_clusters) {
    BatchCtx* b = nullptr;
    int st = guarded(nullptr, [&] {
        require(max_n_query > 0 && n_dim > 0 && max_n_probes > 0 && max_k > 0 && n_total_clusters > 0,
                "bad batch limits");
        require(n_dim <= 512, "n_dim > 512 is not supported");
        b = new BatchCtx();
        try {
            cudaGetDevice(&b->device);
            b->max_nq = max_n_query;
            b->d = n_dim;
            b->max_nprobe = max_n_probes;
            b->max_k = max_k;
            b->nlist = n_total_clusters;
            ck(cudaStreamCreateWithFlags(&b->st, cudaStreamNonBlocking), "cudaStreamCreate");
            b->q = dalloc<float>((size_t)max_n_query * n_dim, b->owned);
            b->q_u8 = dalloc<uint8_t>((size_t)max_n_query * n_dim, b->owned);
            b->probes = dalloc<int32_t>((size_t)max_n_query * max_n_probes, b->owned);
            b->out_ids = dalloc<int32_t>((size_t)max_n_query * max_k, b->owned);
            b->out_dist = dalloc<float>((size_t)max_n_query * max_k, b->owned);
            b->out_idist = dalloc<int32_t>((size_t)max_n_query * max_k, b->owned);
            b->counter = dalloc<int>(4, b->owned);
            b->overflow = dalloc<int>(4, b->owned);
            ck(cudaMemset(b->overflow, 0, sizeof(int) * 4), "memset");
            ck(cudaMallocHost(&b->h_overflow, sizeof(int) * 4), "cudaMallocHost");
            b->h_overflow[0] = b->h_overflow[1] = b->h_overflow[2] = 0;
        } catch (...) {
            if (b->st) cudaStreamDestroy(b->st);
            free_all(b->owned);
            if (b->h_overflow) cudaFreeHost(b->h_overflow);
            delete b;
            b = nullptr;
            throw;
        }
    });
    return st == IVF_OK ? b : nullptr;
}

void ivf_destroy_batch_context(void* batch_ctx) {
    if (!batch_ctx) return;
    auto* b = static_cast<BatchCtx*>(batch_ctx);
    if (b->magic != kBatMagic) return;
    cudaSetDevice(b->device);
    cudaStreamSynchronize(b->st);
    Grow* gs[] = {&b->route_dist, &b->route_rowfb, &b->wl_cnt, &b->wl_off, &b->wl_cursor, &b->pair_q, &b->pair_l,
                  &b->scan_tmp,
                  &b->grp_cnt, &b->grp_off, &b->groups,
                  &b->cand_m, &b->cand_d, &b->cnt_m, &b->cnt_d, &b->thr_m, &b->thr_d, &b->s1m, &b->s1d, &b->exk};
    for (Grow* g : gs)
        if (g->p) cudaFree(g->p);
    free_all(b->owned);
    if (b->h_overflow) cudaFreeHost(b->h_overflow);
    for (auto& v : b->stage_ev)
        for (cudaEvent_t e : v) cudaEventDestroy(e);
    cudaStreamDestroy(b->st);
    b->magic = 0;
    delete b;
}

void ivf_pipeline_stage1_prepare(void* batch_ctx, float* query_batch_host, int n_query) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return;
    }
    guarded(&b->err, [&] {
        require(query_batch_host != nullptr || n_query == 0, "null query pointer");
        require(n_query >= 0 && n_query <= b->max_nq, "batch size exceeds capacity");
        cudaSetDevice(b->device);
        ck(cudaMemcpyAsync(b->q, query_batch_host, sizeof(float) * (size_t)n_query * b->d, cudaMemcpyHostToDevice,
                           b->st),
           "query H2D");
        b->probes_nq = 0;
    });
}

int ivf_pipeline_stage1_prepare_device(void* batch_ctx, const float* d_query, int n_query) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        require(d_query != nullptr || n_query == 0, "null query pointer");
        require(n_query >= 0 && n_query <= b->max_nq, "batch size exceeds capacity");
        cudaSetDevice(b->device);
        ck(cudaMemcpyAsync(b->q, d_query, sizeof(float) * (size_t)n_query * b->d, cudaMemcpyDeviceToDevice, b->st),
           "query D2D");
        b->probes_nq = 0;
    });
}

void ivf_pipeline_stage2_compute(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int k,
                                 int distance_mode) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return;
    }
    guarded(&b->err, [&] {
        IndexCtx* x = as_index(idx_ctx);
        std::shared_lock<std::shared_mutex> rd(x->rw);
        require(distance_mode == IVF_DISTANCE_L2 || distance_mode == IVF_DISTANCE_COSINE, "bad distance_mode");
        check_shape(b, x, n_query, n_probes, k);
        cudaSetDevice(b->device);
        if (x->kind == kKindF32) {
            // the reference routes this path by cosine in both modes
            // (ivf_search_separated.cu:477-512), then scans by L2 or cosine
            do_route(b, x, n_query, n_probes, nullptr, true);
            run_f32(b, x, n_query, n_probes, k, distance_mode == IVF_DISTANCE_COSINE);
            return;
        }
        require(distance_mode == IVF_DISTANCE_L2, "cosine is served on fp32 indexes (ivf_load_dataset) only",
                IVF_EUNSUPPORTED);
        do_route(b, x, n_query, n_probes, nullptr);
        if (x->kind == kKindU8) run_u8(b, x, n_query, n_probes, k, nullptr);
        else run_pq(b, x, n_query, n_probes, k, 512, true, 16, nullptr, nullptr, nullptr, nullptr);
    });
}

void ivf_pipeline_get_results(void* batch_ctx, float* topk_dist, int* topk_index, int n_query, int k) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return;
    }
    guarded(&b->err, [&] {
        cudaSetDevice(b->device);
        copy_results(b, topk_dist, topk_index, nullptr, n_query, k, cudaMemcpyDeviceToHost);
        ck(cudaStreamSynchronize(b->st), "cudaStreamSynchronize");
        check_overflow_after_sync(b);
    });
}

int ivf_get_results_i32(void* batch_ctx, int* ids, int* dist, int n_query, int k) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        cudaSetDevice(b->device);
        copy_results(b, nullptr, ids, dist, n_query, k, cudaMemcpyDeviceToHost);
        ck(cudaStreamSynchronize(b->st), "cudaStreamSynchronize");
        check_overflow_after_sync(b);
    });
}

int ivf_get_results_device(void* batch_ctx, float* d_dist, int* d_index, int n_query, int k) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        cudaSetDevice(b->device);
        copy_results(b, d_dist, d_index, nullptr, n_query, k, cudaMemcpyDeviceToDevice);
    });
}

void ivf_pipeline_sync_batch(void* batch_ctx) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return;
    }
    guarded(&b->err, [&] {
        cudaSetDevice(b->device);
        ck(cudaStreamSynchronize(b->st), "cudaStreamSynchronize");
    });
}

void* ivf_batch_stream(void* batch_ctx) {
    auto* b = static_cast<BatchCtx*>(batch_ctx);
    if (!b || b->magic != kBatMagic) return nullptr;
    return (void*)b->st;
}

// ---------------------------------------------------------------------------
// loading
// ---------------------------------------------------------------------------
int ivf_u8_load(void* idx_ctx, const uint8_t* base_u8, const long long* offsets, const int* counts,
                const int* reorder_to_original, const float* centroids, int nlist, long long n, int d) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);
        std::unique_lock<std::shared_mutex> wr(x->rw);
        require(x->kind == kKindEmpty, "index context already holds an index", IVF_ESTATE);
        require(nlist > 0 && n >= 0 && d > 0 && d % 16 == 0 && d <= 512, "need nlist > 0, d % 16 == 0, d <= 512");
        require(base_u8 != nullptr || n == 0, "null base");
        cudaSetDevice(x->device);
        try {
            load_lists(x, x->main, base_u8, (size_t)d, offsets, counts, reorder_to_original, nullptr, nlist, n);
            load_centroids(x, centroids, nlist, d);
            if (n > 0) {
                x->main.sqnorm = dalloc<int32_t>((size_t)n, x->main.owned);
                ck(u8_row_sqnorms(x->main.data, n, d, x->main.sqnorm, 0), "u8_row_sqnorms");
                ck(cudaDeviceSynchronize(), "u8_row_sqnorms");
                x->tc_rows_ok =
                    exact_tc_usable(d, 1) && exact_tc_map(x->main.data, n, d, x->tc_rows_map) == cudaSuccess;
                cudaGetLastError();
            }
        } catch (...) {
            x->main.release();
            free_all(x->owned);
            throw;
        }
        x->n = n;
        x->kind = kKindU8;
    });
}

int ivf_set_deleted(void* idx_ctx, const unsigned char* deleted, long long n) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);
        std::unique_lock<std::shared_mutex> wr(x->rw);
        require(x->kind != kKindEmpty, "no index loaded", IVF_ESTATE);
        cudaSetDevice(x->device);
        ck(cudaDeviceSynchronize(), "cudaDeviceSynchronize");   // no search may still read the old mask
        if (x->main.deleted) {
            for (auto it = x->main.owned.begin(); it != x->main.owned.end(); ++it)
                if (*it == x->main.deleted) {
                    x->main.owned.erase(it);
                    break;
                }
            cudaFree(x->main.deleted);
            x->main.deleted = nullptr;
        }
        if (!deleted) return;
        require(n == x->main.n, "the delete mask must have one byte per position of the index");
        x->main.deleted = dcopy(deleted, (size_t)n, x->main.owned);
    });
}

int ivf_pq_load(void* idx_ctx, const float* centroids, const float* codebook, int M, int K, int dsub,
                const uint8_t* codes, const long long* offsets, const int* counts, const int* reorder_to_original,
                const uint8_t* base_u8, const float* base_f32, int nlist, long long n, int d) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);
        std::unique_lock<std::shared_mutex> wr(x->rw);
        require(x->kind == kKindEmpty, "index context already holds an index", IVF_ESTATE);
        require(nlist > 0 && n >= 0 && d > 0 && d <= 512, "bad sizes");
        require(K == 256, "only K = 256 (8-bit codes) is supported");
        require(pq_supported_m(M), "M must be a multiple of 8 and <= 64");
        require(dsub > 0 && M * dsub == d, "M * dsub must equal d");
        require(codebook && (codes || n == 0), "null codebook or codes");
        require((base_u8 != nullptr) != (base_f32 != nullptr), "exactly one of base_u8 / base_f32 is required");
        require(base_f32 ? d % 4 == 0 : d % 16 == 0, "rerank rows need d % 16 == 0 (u8) or d % 4 == 0 (fp32)");
        cudaSetDevice(x->device);
        try {
            load_lists(x, x->main, codes, (size_t)M, offsets, counts, reorder_to_original, nullptr, nlist, n);
            if (base_u8) x->main.rr_u8 = dcopy(base_u8, (size_t)n * d, x->main.owned);
            else x->main.rr_f32 = dcopy(base_f32, (size_t)n * d, x->main.owned);
            load_centroids(x, centroids, nlist, d);
            x->codebook = dcopy(codebook, (size_t)M * K * dsub, x->owned);
            std::vector<float> cbt((size_t)M * K * dsub);
            for (int m = 0; m < M; ++m)
                for (int c = 0; c < K; ++c)
                    for (int e = 0; e < dsub; ++e)
                        cbt[((size_t)c * M + m) * dsub + e] = codebook[((size_t)m * K + c) * dsub + e];
            x->codebook_t = dcopy(cbt.data(), cbt.size(), x->owned);
            build_gring(x->main, counts, nlist, M, d);
        } catch (...) {
            x->main.release();
            free_all(x->owned);
            throw;
        }
        x->M = M;
        x->dsub = dsub;
        x->n = n;
        x->kind = kKindPQ;
    });
}

// ---------------------------------------------------------------------------
// index build (build.cu kernels; assignment through the routing path)
// ---------------------------------------------------------------------------
int ivf_load_centroids(void* idx_ctx, const float* centroids, int nlist, int d) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);
        std::unique_lock<std::shared_mutex> wr(x->rw);
        require(x->kind == kKindEmpty, "index context already holds an index", IVF_ESTATE);
        require(nlist > 0 && d > 0 && d % 4 == 0 && d <= 512, "need nlist > 0, d % 4 == 0, d <= 512");
        cudaSetDevice(x->device);
        try {
            load_centroids(x, centroids, nlist, d);
        } catch (...) {
            free_all(x->owned);
            throw;
        }
        x->kind = kKindRoute;
    });
}

int ivf_assign(void* batch_ctx, void* idx_ctx, const void* d_x, int x_is_u8, long long n, int* d_assign) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        IndexCtx* x = as_index(idx_ctx);
        std::shared_lock<std::shared_mutex> rd(x->rw);
        require(x->kind != kKindEmpty, "index context holds no centroids", IVF_ESTATE);
        require(b->d == x->d, "batch and index dimensions differ");
        require(n >= 0 && (d_x || n == 0) && (d_assign || n == 0), "bad rows or output");
        require(x->nlist_global == x->nlist, "assignment needs the whole centroid set, not a shard");
        cudaSetDevice(b->device);
        for (long long s = 0; s < n; s += b->max_nq) {
            const int m = (int)std::min<long long>(b->max_nq, n - s);
            ck(stage_rows_f32(d_x, x_is_u8, (size_t)s * x->d, (size_t)m * x->d, b->q, b->st), "stage rows");
            b->probes_nq = 0;
            do_route(b, x, m, 1, nullptr);
            ck(cudaMemcpyAsync(d_assign + s, b->probes, sizeof(int32_t) * (size_t)m, cudaMemcpyDeviceToDevice,
                               b->st),
               "assign D2D");
        }
        b->probes_nq = 0;
    });
}

int ivf_build_reorder(const int* d_assign, long long n, int nlist, int* d_counts, long long* d_offsets, int* d_order,
                      void* stream) {
    return guarded(nullptr, [&] {
        require(n >= 0 && n < 2147483647ll && nlist > 0, "need 0 <= n < 2^31, nlist > 0");
        require(d_assign && d_counts && d_offsets && d_order, "null pointer");
        ck(build_reorder(d_assign, n, nlist, d_counts, reinterpret_cast<int64_t*>(d_offsets), d_order,
                         static_cast<cudaStream_t>(stream)),
           "build_reorder (an assignment outside [0, nlist)?)");
    });
}

int ivf_kmeans_update(const void* d_x, int x_is_u8, long long n, int d, const int* d_assign, int nlist,
                      float* d_centroids, void* stream) {
    return guarded(nullptr, [&] {
        require(n >= 0 && n < 2147483647ll && d > 0 && nlist > 0 && d_x && d_assign && d_centroids, "bad arguments");
        ck(kmeans_update(d_x, x_is_u8, n, d, d_assign, nlist, d_centroids, static_cast<cudaStream_t>(stream)),
           "kmeans_update (an assignment outside [0, nlist)?)");
    });
}

int ivf_pq_train(const void* d_x, int x_is_u8, long long n, int d, const float* d_centroids, const int* d_assign,
                 int M, int iters, float* d_codebook, void* stream) {
    return guarded(nullptr, [&] {
        require(n >= 0 && d > 0 && M > 0 && d % M == 0 && (d / M == 1 || d / M == 2 || d / M == 4 || d / M == 8),
                "need d % M == 0 and d / M in {1, 2, 4, 8}");
        require((long long)n * M < 2147483647ll, "n * M must be below 2^31");
        ck(pq_train(d_x, x_is_u8, n, d, d_centroids, d_assign, M, iters, d_codebook,
                    static_cast<cudaStream_t>(stream)),
           "pq_train");
    });
}

int ivf_pq_encode(const void* d_x, int x_is_u8, long long n, int d, const int* d_rows, const float* d_centroids,
                  const int* d_assign, const float* d_codebook, int M, unsigned char* d_codes, void* stream) {
    return guarded(nullptr, [&] {
        require(n >= 0 && d > 0 && M > 0 && d % M == 0 && (d / M == 1 || d / M == 2 || d / M == 4 || d / M == 8),
                "need d % M == 0 and d / M in {1, 2, 4, 8}");
        ck(pq_encode_rows(d_x, x_is_u8, n, d, d_rows, d_centroids, d_assign, d_codebook, M, d_codes,
                          static_cast<cudaStream_t>(stream)),
           "pq_encode");
    });
}

int ivf_set_shard(void* idx_ctx, int nlist_global, const int* local_to_global, const long long* key_offsets) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);
        std::unique_lock<std::shared_mutex> wr(x->rw);
        require(x->kind == kKindU8 || x->kind == kKindPQ, "load the shard's lists first", IVF_ESTATE);
        require(x->l2g == nullptr, "shard mapping already set", IVF_ESTATE);
        require(nlist_global >= x->nlist && local_to_global, "bad shard mapping");
        std::vector<int32_t> g2l((size_t)nlist_global, -1);
        for (int l = 0; l < x->nlist; ++l) {
            int g = local_to_global[l];
            require(g >= 0 && g < nlist_global, "global list id out of range");
            require(l == 0 || g > local_to_global[l - 1], "local lists must be in increasing global order");
            g2l[(size_t)g] = l;
        }
        cudaSetDevice(x->device);
        x->l2g = dcopy(reinterpret_cast<const int32_t*>(local_to_global), (size_t)x->nlist, x->owned);
        x->g2l = dcopy(g2l.data(), g2l.size(), x->owned);
        if (key_offsets)
            x->main.key_off = dcopy(reinterpret_cast<const int64_t*>(key_offsets), (size_t)x->nlist, x->main.owned);
        x->nlist_global = nlist_global;
    });
}

int ivf_pq_publish_delta(void* idx_ctx, const uint8_t* codes, const int* ids, const int* counts,
                         const long long* offsets, const long long* key_offsets, const uint8_t* raw_u8,
                         const float* raw_f32, long long n_delta) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);
        publish_delta_locked(x, codes, ids, counts, offsets, key_offsets, raw_u8, raw_f32, n_delta);
    });
}

int ivf_pq_clear_delta(void* idx_ctx) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);
        std::unique_lock<std::shared_mutex> wr(x->rw);
        cudaSetDevice(x->device);
        ck(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        x->delta.release();
        x->has_delta = false;
        x->delta_search = 0;
        x->h_dcodes.clear();
        x->h_dids.clear();
        x->h_dcounts.clear();
        x->h_draw_u8.clear();
        x->h_draw_f32.clear();
    });
}

int ivf_pq_delta_mode(void* idx_ctx) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    std::shared_lock<std::shared_mutex> rd(x->rw);
    return x->delta_search;
}

int ivf_pq_insert(void* idx_ctx, const void* d_x, int x_is_u8, const int* ids, long long n) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);          // one insert or publish at a time
        require(x->kind == kKindPQ, "insert needs a residual-PQ index", IVF_ESTATE);
        require(x->nlist_global == x->nlist, "insert into a shard is not supported: insert into the whole index");
        require(n >= 0 && (n == 0 || (d_x && ids)), "bad rows or ids");
        const bool f32 = x->main.rr_f32 != nullptr;
        require(f32 ? !x_is_u8 : x_is_u8 != 0, "inserted rows must have the type of the index's rerank rows");
        if (n == 0) return;
        cudaSetDevice(x->device);
        const int d = x->d, M = x->M, nlist = x->nlist;
        // 1. exact nearest centroid (the routing kernels, n_probes = 1) and 2. the
        // residual codes, on a private stream; searches keep running meanwhile
        std::vector<void*> tmp;
        int32_t* d_assign = dalloc<int32_t>((size_t)n, tmp);
        uint8_t* d_codes = dalloc<uint8_t>((size_t)n * M, tmp);
        void* b = ivf_create_batch_context((int)std::min<long long>(n, 65536), d, 1, 1, nlist);
        std::vector<int32_t> ha((size_t)n);
        std::vector<uint8_t> hc((size_t)n * M);
        try {
            require(b != nullptr, "batch context: " + g_err, IVF_ENOMEM);
            BatchCtx* bc = static_cast<BatchCtx*>(b);
            {
                std::shared_lock<std::shared_mutex> rd(x->rw);
                for (long long s0 = 0; s0 < n; s0 += bc->max_nq) {
                    const int m = (int)std::min<long long>(bc->max_nq, n - s0);
                    ck(stage_rows_f32(d_x, x_is_u8, (size_t)s0 * d, (size_t)m * d, bc->q, bc->st), "stage rows");
                    do_route(bc, x, m, 1, nullptr);
                    ck(cudaMemcpyAsync(d_assign + s0, bc->probes, sizeof(int32_t) * (size_t)m,
                                       cudaMemcpyDeviceToDevice, bc->st),
                       "assign D2D");
                }
                ck(pq_encode_rows(d_x, x_is_u8, n, d, nullptr, x->cent, d_assign, x->codebook, M, d_codes, bc->st),
                   "pq_encode");
                ck(cudaMemcpyAsync(ha.data(), d_assign, sizeof(int32_t) * ha.size(), cudaMemcpyDeviceToHost,
                                   bc->st),
                   "assign D2H");
                ck(cudaMemcpyAsync(hc.data(), d_codes, hc.size(), cudaMemcpyDeviceToHost, bc->st), "codes D2H");
                ck(cudaStreamSynchronize(bc->st), "cudaStreamSynchronize");
                check_overflow_after_sync(bc);
            }
        } catch (...) {
            if (b) ivf_destroy_batch_context(b);
            free_all(tmp);
            throw;
        }
        ivf_destroy_batch_context(b);
        free_all(tmp);
        const size_t rb = f32 ? sizeof(float) : 1;
        std::vector<uint8_t> hraw((size_t)n * d * rb);
        ck(cudaMemcpy(hraw.data(), d_x, hraw.size(), cudaMemcpyDefault), "rows D2H");
        // 3. the grown segment, list-major; a list keeps its older delta rows
        // first, then the new ones in insertion order
        const long long n_old = (long long)x->h_dids.size();
        std::vector<int32_t> cnt((size_t)nlist, 0);
        if (n_old) cnt = x->h_dcounts;
        std::vector<long long> old_off((size_t)nlist, 0);
        for (int l = 1; l < nlist; ++l) old_off[l] = old_off[l - 1] + cnt[l - 1];
        std::vector<int32_t> add((size_t)nlist, 0);
        for (long long i = 0; i < n; ++i) add[ha[i]]++;
        std::vector<int32_t> ncnt((size_t)nlist);
        std::vector<long long> noff((size_t)nlist, 0);
        for (int l = 0; l < nlist; ++l) ncnt[l] = cnt[l] + add[l];
        for (int l = 1; l < nlist; ++l) noff[l] = noff[l - 1] + ncnt[l - 1];
        const long long nt = n_old + n;
        require(nt < (1ll << 31), "delta segment above 2^31 rows");
        std::vector<uint8_t> codes((size_t)nt * M), raw((size_t)nt * d * rb);
        std::vector<int32_t> nid((size_t)nt);
        const uint8_t* oraw = f32 ? reinterpret_cast<const uint8_t*>(x->h_draw_f32.data()) : x->h_draw_u8.data();
        for (int l = 0; l < nlist; ++l) {
            const size_t src = (size_t)old_off[l], dst = (size_t)noff[l], c = (size_t)cnt[l];
            if (!c) continue;
            std::memcpy(&codes[dst * M], &x->h_dcodes[src * M], c * M);
            std::memcpy(&raw[dst * d * rb], &oraw[src * d * rb], c * d * rb);
            std::memcpy(&nid[dst], &x->h_dids[src], c * sizeof(int32_t));
        }
        std::vector<long long> cur(noff);
        for (int l = 0; l < nlist; ++l) cur[l] += cnt[l];
        for (long long i = 0; i < n; ++i) {
            const size_t dst = (size_t)cur[ha[i]]++;
            std::memcpy(&codes[dst * M], &hc[(size_t)i * M], M);
            std::memcpy(&raw[dst * d * rb], &hraw[(size_t)i * d * rb], d * rb);
            nid[dst] = ids[i];
        }
        // 4. published in one step
        publish_delta_locked(x, codes.data(), nid.data(), ncnt.data(), noff.data(), nullptr,
                             f32 ? nullptr : raw.data(), f32 ? reinterpret_cast<const float*>(raw.data()) : nullptr,
                             nt);
    });
}

// ---------------------------------------------------------------------------
// search
// ---------------------------------------------------------------------------
int ivf_route(void* batch_ctx, void* idx_ctx, int n_query, int n_probes) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        IndexCtx* x = as_index(idx_ctx);
        std::shared_lock<std::shared_mutex> rd(x->rw);
        check_shape(b, x, n_query, n_probes, 1);
        cudaSetDevice(b->device);
        do_route(b, x, n_query, n_probes, nullptr);
    });
}

int ivf_set_probes(void* batch_ctx, const int* h_probes, int n_query, int n_probes) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        require(h_probes != nullptr, "null probes");
        require(n_query >= 0 && n_query <= b->max_nq && n_probes > 0 && n_probes <= b->max_nprobe,
                "probe table shape exceeds the batch limits");
        cudaSetDevice(b->device);
        ck(cudaMemcpyAsync(b->probes, h_probes, sizeof(int32_t) * (size_t)n_query * n_probes,
                           cudaMemcpyHostToDevice, b->st),
           "probes H2D");
        ck(cudaStreamSynchronize(b->st), "cudaStreamSynchronize");
        b->probes_nq = n_query;
        b->probes_np = n_probes;
    });
}

int ivf_get_probes(void* batch_ctx, int* h_probes, int n_query, int n_probes) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        require(h_probes != nullptr, "null probes");
        require_probes(b, n_query, n_probes);
        cudaSetDevice(b->device);
        ck(cudaMemcpyAsync(h_probes, b->probes, sizeof(int32_t) * (size_t)n_query * n_probes,
                           cudaMemcpyDeviceToHost, b->st),
           "probes D2H");
        ck(cudaStreamSynchronize(b->st), "cudaStreamSynchronize");
        if (b->h_overflow[1] & 4) fail(IVF_ECUDA, "a bounded device wait of the tensor-core routing gave up");
    });
}

int ivf_u8_search(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int k, int route) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        IndexCtx* x = as_index(idx_ctx);
        std::shared_lock<std::shared_mutex> rd(x->rw);
        check_shape(b, x, n_query, n_probes, k);
        cudaSetDevice(b->device);
        if (route) do_route(b, x, n_query, n_probes, nullptr);
        run_u8(b, x, n_query, n_probes, k, nullptr);
    });
}

int ivf_pq_search(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int k, int rerank_n, int use_overlay,
                  int delta_topk, int route) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        IndexCtx* x = as_index(idx_ctx);
        std::shared_lock<std::shared_mutex> rd(x->rw);
        check_shape(b, x, n_query, n_probes, k);
        require(rerank_n > 0, "rerank_n must be > 0");
        require(delta_topk >= 0, "delta_topk must be >= 0");
        cudaSetDevice(b->device);
        if (route) do_route(b, x, n_query, n_probes, nullptr);
        run_pq(b, x, n_query, n_probes, k, rerank_n, use_overlay != 0, delta_topk, nullptr, nullptr, nullptr,
               nullptr);
    });
}

int ivf_route_keys(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, unsigned long long* d_keys) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        IndexCtx* x = as_index(idx_ctx);
        std::shared_lock<std::shared_mutex> rd(x->rw);
        check_shape(b, x, n_query, n_probes, 1);
        require(d_keys != nullptr, "null key output");
        cudaSetDevice(b->device);
        do_route(b, x, n_query, n_probes, reinterpret_cast<uint64_t*>(d_keys));
    });
}

int ivf_route_merge(void* batch_ctx, const unsigned long long* d_keys, int n_in, int n_query, int n_probes) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        require(d_keys != nullptr && n_in > 0, "bad key input");
        require(n_query >= 0 && n_query <= b->max_nq && n_probes > 0 && n_probes <= b->max_nprobe,
                "shape exceeds the batch limits");
        cudaSetDevice(b->device);
        ck(merge_keys(reinterpret_cast<const uint64_t*>(d_keys), n_query, n_in, n_probes, 0, b->probes, nullptr,
                      nullptr, b->st),
           "merge_keys");
        b->probes_nq = n_query;
        b->probes_np = n_probes;
    });
}

int ivf_route_merge_shards(void* batch_ctx, const unsigned long long* d_keys, int n_shards, int n_query,
                           int n_probes) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        require(d_keys != nullptr && n_shards > 0, "bad key input");
        require(n_query >= 0 && n_query <= b->max_nq && n_probes > 0 && n_probes <= b->max_nprobe,
                "shape exceeds the batch limits");
        require(n_probes <= 32 && n_shards * n_probes <= 256, "n_probes <= 32 and n_shards * n_probes <= 256");
        cudaSetDevice(b->device);
        ck(merge_shard_keys(reinterpret_cast<const uint64_t*>(d_keys), n_shards, n_query, n_probes, b->probes, b->st),
           "merge_shard_keys");
        b->probes_nq = n_query;
        b->probes_np = n_probes;
    });
}

int ivf_pq_search_shard(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int rerank_n, int delta_topk,
                        unsigned long long* d_adc, unsigned long long* d_exact, unsigned long long* d_dadc,
                        unsigned long long* d_dexact) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        IndexCtx* x = as_index(idx_ctx);
        std::shared_lock<std::shared_mutex> rd(x->rw);
        check_shape(b, x, n_query, n_probes, 1);
        require(d_adc && d_exact && rerank_n > 0, "adc and exact outputs are required");
        require(!d_dadc == !d_dexact, "give both or neither delta outputs");
        cudaSetDevice(b->device);
        run_pq(b, x, n_query, n_probes, 1, rerank_n, d_dadc != nullptr, d_dadc ? delta_topk : 0,
               reinterpret_cast<uint64_t*>(d_adc), reinterpret_cast<uint64_t*>(d_exact),
               reinterpret_cast<uint64_t*>(d_dadc), reinterpret_cast<uint64_t*>(d_dexact));
    });
}

int ivf_pq_merge_shards(void* batch_ctx, const unsigned long long* d_adc, const unsigned long long* d_exact,
                        int n_main, int rerank_n, const unsigned long long* d_dadc,
                        const unsigned long long* d_dexact, int n_delta, int delta_topk, int n_query, int k,
                        int exact_is_int) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        require(d_adc && d_exact && n_main > 0 && rerank_n > 0, "bad main inputs");
        require(n_query >= 0 && n_query <= b->max_nq && k > 0 && k <= b->max_k, "shape exceeds the batch limits");
        cudaSetDevice(b->device);
        ck(pq_merge_shards(reinterpret_cast<const uint64_t*>(d_adc), reinterpret_cast<const uint64_t*>(d_exact),
                           n_main, rerank_n, reinterpret_cast<const uint64_t*>(d_dadc),
                           reinterpret_cast<const uint64_t*>(d_dexact), d_dadc ? n_delta : 0,
                           d_dadc ? delta_topk : 0, n_query, k, exact_is_int, b->out_ids, b->out_dist, b->st),
           "pq_merge_shards");
        b->res_nq = n_query;
        b->res_k = k;
    });
}

// ---------------------------------------------------------------------------
// Sharded residual-PQ search in phases (no counterpart in the reference): the
// caller exchanges the rank-R bounds after the nearest-probe pass, and the
// shards rerank only the stage-1 prefix each query's owner asks for.
// ---------------------------------------------------------------------------
int ivf_pq_shard_scan(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int rerank_n, int pass) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        IndexCtx* x = as_index(idx_ctx);
        std::shared_lock<std::shared_mutex> rd(x->rw);
        check_shape(b, x, n_query, n_probes, 1);
        require(pass == 0 || pass == 1, "pass must be 0 (nearest probe) or 1 (the other probes)");
        require_probes(b, n_query, n_probes);
        cudaSetDevice(b->device);
        ShardPlan sp = shard_plan(b, x, n_query, n_probes, rerank_n);
        PQParams p = pq_params(x, b->q, false);
        if (pass == 0) {
            StageScope stage(b, IVF_STAGE_WORKLIST);
            reset_fine_flags(b);
            ck(reset_candidates(sp.cm, n_query, b->st), "reset_candidates");
        }
        const int col0 = pass == 0 ? 0 : 1, ncol = pass == 0 ? 1 : n_probes - 1;
        if (ncol <= 0 || n_query == 0) return;
        {
            StageScope stage(b, IVF_STAGE_WORKLIST);
            ck(build_worklist(b->probes, n_query, n_probes, x->nlist_global, x->g2l, x->nlist, sp.wl, sp.tmp,
                              sp.tmp_bytes, b->st, col0, ncol),
               "build_worklist");
        }
        StageScope stage(b, IVF_STAGE_SCAN);
        CandBuf none{};
        ck(pq_scan(p, sp.wl, n_query * ncol, sp.cm, none, b->counter, b->st), "pq_scan");
        queue_overflow_check(b);
    });
}

unsigned long long* ivf_pq_shard_bounds(void* batch_ctx) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return nullptr;
    }
    return reinterpret_cast<unsigned long long*>(b->thr_m.p);
}

int ivf_pq_shard_select(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int rerank_n,
                        unsigned long long* d_adc) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        IndexCtx* x = as_index(idx_ctx);
        std::shared_lock<std::shared_mutex> rd(x->rw);
        check_shape(b, x, n_query, n_probes, 1);
        require(d_adc != nullptr, "adc output is required");
        cudaSetDevice(b->device);
        ShardPlan sp = shard_plan(b, x, n_query, n_probes, rerank_n);
        StageScope stage(b, IVF_STAGE_SELECT);
        ck(select_top_r(sp.cm, n_query, reinterpret_cast<uint64_t*>(d_adc), b->st, false), "select_top_r");
    });
}

int ivf_pq_shard_kappa(void* batch_ctx, const unsigned long long* d_adc_all, int n_shards, int n_owned,
                       int rerank_n, unsigned long long* d_kappa) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        require(d_adc_all && d_kappa && n_shards > 0 && n_owned >= 0 && rerank_n > 0, "bad shard-kappa arguments");
        cudaSetDevice(b->device);
        ck(pq_shard_kappa(reinterpret_cast<const uint64_t*>(d_adc_all), n_shards, n_owned, rerank_n,
                          reinterpret_cast<uint64_t*>(d_kappa), b->st),
           "pq_shard_kappa");
    });
}

int ivf_pq_shard_rerank(void* batch_ctx, void* idx_ctx, int n_query, int rerank_n,
                        const unsigned long long* d_adc, const unsigned long long* d_kappa, int k,
                        unsigned long long* d_topk) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        IndexCtx* x = as_index(idx_ctx);
        std::shared_lock<std::shared_mutex> rd(x->rw);
        require(x->kind == kKindPQ, "index is not a residual-PQ index", IVF_ESTATE);
        require(d_adc && d_kappa && d_topk && rerank_n > 0, "bad shard-rerank arguments");
        require(n_query >= 0 && n_query <= b->max_nq && b->d == x->d, "shape exceeds the batch limits");
        require(k > 0 && k <= b->max_k && k <= 32, "k must be in 1 .. min(32, the batch k)");
        cudaSetDevice(b->device);
        PQParams p = pq_params(x, b->q, false);
        StageScope stage(b, IVF_STAGE_RERANK);
        ck(pq_rerank(p, x->nlist, reinterpret_cast<const uint64_t*>(d_adc), rerank_n, nullptr, 0, n_query, k, nullptr,
                     nullptr, nullptr, nullptr, b->st, reinterpret_cast<const uint64_t*>(d_kappa),
                     reinterpret_cast<uint64_t*>(d_topk)),
           "pq_rerank");
    });
}

int ivf_pq_shard_final(void* batch_ctx, const unsigned long long* d_topk_all, int n_shards, int n_owned, int k,
                       int exact_is_int) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        require(d_topk_all && n_shards > 0, "bad shard-final arguments");
        require(n_owned >= 0 && n_owned <= b->max_nq && k > 0 && k <= b->max_k, "shape exceeds the batch limits");
        require(k <= 32 && n_shards * k <= 256, "k <= 32 and n_shards * k <= 256");
        cudaSetDevice(b->device);
        ck(pq_shard_final(reinterpret_cast<const uint64_t*>(d_topk_all), n_shards, n_owned, k, exact_is_int,
                          b->out_ids, b->out_dist, b->st),
           "pq_shard_final");
        b->res_nq = n_owned;
        b->res_k = k;
    });
}

int ivf_u8_search_shard(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int k,
                        unsigned long long* d_keys) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        IndexCtx* x = as_index(idx_ctx);
        std::shared_lock<std::shared_mutex> rd(x->rw);
        check_shape(b, x, n_query, n_probes, k);
        require(d_keys != nullptr, "null key output");
        cudaSetDevice(b->device);
        run_u8(b, x, n_query, n_probes, k, reinterpret_cast<uint64_t*>(d_keys));
    });
}

int ivf_u8_merge_shards(void* batch_ctx, const unsigned long long* d_keys, int n_in, int n_query, int k) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        require(d_keys != nullptr && n_in > 0, "bad key input");
        require(n_query >= 0 && n_query <= b->max_nq && k > 0 && k <= b->max_k, "shape exceeds the batch limits");
        cudaSetDevice(b->device);
        ck(merge_keys(reinterpret_cast<const uint64_t*>(d_keys), n_query, n_in, k, 1, b->out_ids, b->out_dist,
                      b->out_idist, b->st),
           "merge_keys");
        b->res_nq = n_query;
        b->res_k = k;
    });
}

unsigned long long ivf_kernel_launches(void) { return g_launches.load(); }

int ivf_batch_profile(void* batch_ctx, int enable) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    return guarded(&b->err, [&] {
        cudaSetDevice(b->device);
        ck(cudaStreamSynchronize(b->st), "cudaStreamSynchronize");
        b->prof = enable != 0;
        for (auto& u : b->stage_used) u = 0;
    });
}

int ivf_batch_stage_ms(void* batch_ctx, double* out_ms, int n) {
    BatchCtx* b = nullptr;
    try {
        b = as_batch(batch_ctx);
    } catch (...) {
        return IVF_EINVAL;
    }
    int st = guarded(&b->err, [&] {
        require(out_ms != nullptr && n >= 0, "null output");
        cudaSetDevice(b->device);
        ck(cudaStreamSynchronize(b->st), "cudaStreamSynchronize");
        for (int s = 0; s < IVF_STAGE_COUNT; ++s) {
            double acc = 0;
            for (size_t i = 0; i + 1 < b->stage_used[s]; i += 2) {
                float ms = 0;
                ck(cudaEventElapsedTime(&ms, b->stage_ev[s][i], b->stage_ev[s][i + 1]), "cudaEventElapsedTime");
                acc += ms;
            }
            if (s < n) out_ms[s] = acc;
            b->stage_used[s] = 0;
        }
    });
    return st == IVF_OK ? IVF_STAGE_COUNT : st;
}

const char* ivf_last_error(void* ctx) {
    std::string* e = err_of(ctx);
    return e ? e->c_str() : "not a context";
}

const char* ivf_global_last_error(void) { return g_err.c_str(); }

// ---------------------------------------------------------------------------
// *_wrapper exports (ivf_search_wrapper.cpp:85-321) and the registry
// ---------------------------------------------------------------------------
void* ivf_create_index_context_wrapper(void) { return ivf_create_index_context(); }
void ivf_destroy_index_context_wrapper(void* idx_ctx) { ivf_destroy_index_context(idx_ctx); }
int ivf_load_dataset_wrapper(void* idx_ctx, int* d_cluster_size, float* d_cluster_vectors, float* d_cluster_centers,
                             int n_total_clusters, int n_total_vectors, int n_dim) {
    auto* x = static_cast<IndexCtx*>(idx_ctx);
    if (!x || x->magic != kIdxMagic) return -1;
    int r = ivf_load_dataset(idx_ctx, d_cluster_size, d_cluster_vectors, d_cluster_centers, n_total_clusters,
                             n_total_vectors, n_dim);
    return (r == 0 && !x->err.empty()) ? -1 : r;
}
void* ivf_create_batch_context_wrapper(int max_n_query, int n_dim, int max_n_probes, int max_k, int n_total_clusters) {
    return ivf_create_batch_context(max_n_query, n_dim, max_n_probes, max_k, n_total_clusters);
}
void ivf_destroy_batch_context_wrapper(void* batch_ctx) { ivf_destroy_batch_context(batch_ctx); }
void ivf_pipeline_stage1_prepare_wrapper(void* batch_ctx, float* q, int n_query) {
    ivf_pipeline_stage1_prepare(batch_ctx, q, n_query);
}
void ivf_pipeline_stage2_compute_wrapper(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int k,
                                         int distance_mode) {
    ivf_pipeline_stage2_compute(batch_ctx, idx_ctx, n_query, n_probes, k, distance_mode);
}
void ivf_pipeline_get_results_wrapper(void* batch_ctx, float* topk_dist, int* topk_index, int n_query, int k) {
    ivf_pipeline_get_results(batch_ctx, topk_dist, topk_index, n_query, k);
}
void ivf_pipeline_sync_batch_wrapper(void* batch_ctx) { ivf_pipeline_sync_batch(batch_ctx); }
int ivf_check_index_initialized_wrapper(void* idx_ctx) {
    auto* x = static_cast<IndexCtx*>(idx_ctx);
    if (!x || x->magic != kIdxMagic) return 0;
    return x->kind != kKindEmpty ? 1 : 0;
}

void ivf_register_index_instance(unsigned int index_oid, void* gpu_handle) {
    if (!gpu_handle) return;
    void* old = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_reg_mu);
        for (auto& e : g_reg)
            if (e.active && e.oid == index_oid) {
                old = e.handle == gpu_handle ? nullptr : e.handle;
                e.handle = gpu_handle;
                goto done;
            }
        for (auto& e : g_reg)
            if (!e.active) {
                e = RegEntry{index_oid, gpu_handle, true};
                goto done;
            }
        g_err = "index registry full (64 entries)";
    done:;
    }
    if (old) ivf_destroy_index_context(old);
}

void* ivf_get_index_instance(unsigned int index_oid) {
    std::lock_guard<std::mutex> lk(g_reg_mu);
    for (auto& e : g_reg)
        if (e.active && e.oid == index_oid) return e.handle;
    return nullptr;
}

void ivf_unregister_index_instance(unsigned int index_oid) {
    void* old = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_reg_mu);
        for (auto& e : g_reg)
            if (e.active && e.oid == index_oid) {
                old = e.handle;
                e = RegEntry{0, nullptr, false};
                break;
            }
    }
    if (old) ivf_destroy_index_context(old);
}

// ---------------------------------------------------------------------------
// coarse handle (cpu_fine.h:232-278)
// ---------------------------------------------------------------------------
void coarse_handle_init(CoarseHandle* h, const float* d_centers, int n_total_clusters, int dim) {
    if (!h) return;
    std::memset(h, 0, sizeof(*h));
    guarded(nullptr, [&] {
        require(d_centers && n_total_clusters > 0 && dim > 0 && dim <= 512, "bad coarse handle arguments");
        auto* rs = new RouteState();
        try {
            cudaGetDevice(&rs->device);
            rs->x = new IndexCtx();
            rs->x->device = rs->device;
            rs->x->cent = const_cast<float*>(d_centers);  // borrowed, never freed
            rs->x->valid = dalloc<uint8_t>((size_t)n_total_clusters, rs->x->owned);
            ck(route_centroid_valid(d_centers, n_total_clusters, dim, rs->x->valid, 0), "centroid validity");
            ck(cudaDeviceSynchronize(), "centroid validity");
            rs->x->nlist = rs->x->nlist_global = n_total_clusters;
            rs->x->d = dim;
            rs->x->kind = kKindF32;
            prepare_route_tc(rs->x, n_total_clusters, dim);      // tensor-core routing where the shape allows
            ck(cudaDeviceSynchronize(), "routing operands");
            for (auto& e : rs->ev) ck(cudaEventCreate(&e), "cudaEventCreate");
        } catch (...) {
            if (rs->x) {
                free_all(rs->x->owned);
                delete rs->x;
            }
            delete rs;
            throw;
        }
        h->d_centers = d_centers;
        h->d_centers_norm = reinterpret_cast<float*>(rs->x->valid);
        h->cublas_handle = rs;
        h->n_total_clusters = n_total_clusters;
        h->dim = dim;
        h->distance_mode_cached = IVF_DISTANCE_L2;
    });
}

void coarse_handle_release(CoarseHandle* h) {
    if (!h || !h->cublas_handle) return;
    auto* rs = static_cast<RouteState*>(h->cublas_handle);
    cudaSetDevice(rs->device);
    if (rs->b) ivf_destroy_batch_context(rs->b);
    for (auto& e : rs->ev)
        if (e) cudaEventDestroy(e);
    free_all(rs->x->owned);
    rs->x->magic = 0;
    delete rs->x;
    delete rs;
    std::memset(h, 0, sizeof(*h));
}

void coarse_search(const CoarseHandle* h, const float* h_query, int n_query_batch, int n_probes, int distance_mode,
                   int* h_cluster_ids_out, double* out_coarse_ms, double* out_h2d_ms, double* out_d2h_ms) {
    g_coarse_timing = CoarseTimingBreakdown{};
    guarded(nullptr, [&] {
        require(h && h->cublas_handle, "invalid coarse handle");
        require(distance_mode == IVF_DISTANCE_L2, "only distance_mode 0 (L2) is supported", IVF_EUNSUPPORTED);
        require(n_query_batch > 0 && n_probes > 0 && n_probes <= h->n_total_clusters,
                "bad args: need n_query > 0 and 0 < n_probes <= n_total_clusters");
        require(h_query && h_cluster_ids_out, "null host pointer");
        auto* rs = static_cast<RouteState*>(h->cublas_handle);
        cudaSetDevice(rs->device);
        if (!rs->b || rs->b->max_nq < n_query_batch || rs->b->max_nprobe < n_probes) {
            if (rs->b) ivf_destroy_batch_context(rs->b);
            rs->b = static_cast<BatchCtx*>(ivf_create_batch_context(
                std::max(n_query_batch, rs->b ? rs->b->max_nq : 0), h->dim,
                std::max(n_probes, rs->b ? rs->b->max_nprobe : 0), 1, h->n_total_clusters));
            require(rs->b != nullptr, "batch scratch allocation failed: " + g_err, IVF_ENOMEM);
        }
        BatchCtx* b = rs->b;
        ck(cudaEventRecord(rs->ev[0], b->st), "event");
        ck(cudaMemcpyAsync(b->q, h_query, sizeof(float) * (size_t)n_query_batch * h->dim, cudaMemcpyHostToDevice,
                           b->st),
           "query H2D");
        ck(cudaEventRecord(rs->ev[1], b->st), "event");
        do_route(b, rs->x, n_query_batch, n_probes, nullptr);
        ck(cudaEventRecord(rs->ev[2], b->st), "event");
        ck(cudaMemcpyAsync(h_cluster_ids_out, b->probes, sizeof(int32_t) * (size_t)n_query_batch * n_probes,
                           cudaMemcpyDeviceToHost, b->st),
           "ids D2H");
        ck(cudaEventRecord(rs->ev[3], b->st), "event");
        ck(cudaEventSynchronize(rs->ev[3]), "cudaEventSynchronize");
        float t01 = 0, t12 = 0, t23 = 0, t03 = 0;
        cudaEventElapsedTime(&t01, rs->ev[0], rs->ev[1]);
        cudaEventElapsedTime(&t12, rs->ev[1], rs->ev[2]);
        cudaEventElapsedTime(&t23, rs->ev[2], rs->ev[3]);
        cudaEventElapsedTime(&t03, rs->ev[0], rs->ev[3]);
        g_coarse_timing.query_h2d_ms = t01;
        g_coarse_timing.topk_ms = t12;
        g_coarse_timing.coarse_compute_ms = t12;
        g_coarse_timing.cluster_d2h_ms = t23;
        g_coarse_timing.coarse_total_ms = t03;
        if (out_coarse_ms) *out_coarse_ms = t12;
        if (out_h2d_ms) *out_h2d_ms = t01;
        if (out_d2h_ms) *out_d2h_ms = t23;
    });
}

const CoarseTimingBreakdown* coarse_get_last_timing(void) { return &g_coarse_timing; }

}  // extern "C"

// The C++-linkage names of the same functions (cpp_abi.cu) forward here; the
// handle and timing structs have the same layout in both headers.
namespace isb {
void coarse_init_fwd(void* h, const float* d_centers, int n, int dim) {
    coarse_handle_init(static_cast<CoarseHandle*>(h), d_centers, n, dim);
}
void coarse_release_fwd(void* h) { coarse_handle_release(static_cast<CoarseHandle*>(h)); }
void coarse_search_fwd(const void* h, const float* q, int nq, int np, int mode, int* out, double* a, double* b2,
                       double* c) {
    coarse_search(static_cast<const CoarseHandle*>(h), q, nq, np, mode, out, a, b2, c);
}
const void* coarse_timing_fwd() { return coarse_get_last_timing(); }
}  // namespace isb

extern "C" {

}  // extern "C"

// ===========================================================================
// Streaming upload of an fp32 index, cuda/search/ivf_search.cuh:330-355 and
// ivf_search_separated.cu:166-270 (C++ linkage, as in the reference).  The
// functions return nothing; failures are recorded on the index context
// (ivf_last_error) and in ivf_global_last_error().
// ===========================================================================
__attribute__((visibility("default"))) void ivf_init_streaming_upload(void* idx_ctx_ptr, int n_total_clusters, int n_total_vectors, int n_dim) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx_ptr);
    } catch (...) {
        g_err = "not an index context";
        return;
    }
    guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);
        std::unique_lock<std::shared_mutex> wr(x->rw);
        require(x->kind == kKindEmpty && !x->su_active, "index context already holds an index", IVF_ESTATE);
        require(n_total_clusters > 0 && n_total_vectors >= 0 && n_dim > 0 && n_dim <= 512, "bad sizes");
        cudaSetDevice(x->device);
        x->f32_rows = dalloc<float>((size_t)n_total_vectors * n_dim, x->owned);
        x->su_counts.assign((size_t)n_total_clusters, 0);
        x->su_offsets.assign((size_t)n_total_clusters, 0);
        x->nlist = x->nlist_global = n_total_clusters;
        x->d = n_dim;
        x->n = n_total_vectors;
        x->su_active = true;
    });
}

__attribute__((visibility("default"))) void ivf_append_cluster_data(void* idx_ctx_ptr, int cluster_id, float* host_vector_data, int count,
                             int start_offset_idx) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx_ptr);
    } catch (...) {
        g_err = "not an index context";
        return;
    }
    guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);
        require(x->su_active, "no streaming upload in progress", IVF_ESTATE);
        require(cluster_id >= 0 && cluster_id < x->nlist, "cluster_id outside [0, n_total_clusters)");
        require(start_offset_idx >= 0, "negative start offset");
        const int c = (count > 0 && host_vector_data) ? count : 0;    // no data: an empty cluster
        require((long long)start_offset_idx + c <= x->n, "cluster data beyond n_total_vectors");
        cudaSetDevice(x->device);
        if (c)
            ck(cudaMemcpy(x->f32_rows + (size_t)start_offset_idx * x->d, host_vector_data,
                          sizeof(float) * (size_t)c * x->d, cudaMemcpyHostToDevice),
               "cluster data H2D");
        x->su_counts[(size_t)cluster_id] = c;
        x->su_offsets[(size_t)cluster_id] = start_offset_idx;
    });
}

__attribute__((visibility("default"))) void ivf_finalize_streaming_upload(void* idx_ctx_ptr, float* center_data_flat, int total_vectors_check) {
    IndexCtx* x = nullptr;
    try {
        x = as_index(idx_ctx_ptr);
    } catch (...) {
        g_err = "not an index context";
        return;
    }
    guarded(&x->err, [&] {
        std::lock_guard<std::mutex> lk(x->mu);
        std::unique_lock<std::shared_mutex> wr(x->rw);
        require(x->su_active, "no streaming upload in progress", IVF_ESTATE);
        require(center_data_flat != nullptr, "null centroids");
        require(total_vectors_check >= 0 && total_vectors_check <= x->n, "total_vectors_check beyond n_total_vectors");
        cudaSetDevice(x->device);
        x->cent = dcopy(center_data_flat, (size_t)x->nlist * x->d, x->owned);
        int32_t* d_counts = dcopy(x->su_counts.data(), x->su_counts.size(), x->owned);
        adopt_f32_lists(x, d_counts, x->f32_rows, x->nlist, x->n, x->d, x->su_offsets.data());
        x->su_active = false;
    });
}
