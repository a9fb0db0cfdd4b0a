// launch.h -- host-side launchers of the hot-path kernels (internal to the library).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "internal.cuh"

namespace isb {

// Counts this library's own kernel launches (reported by ivf_kernel_launches()).
void note_launch(int n = 1);

constexpr int kPQScanChunk = 2048;    // vectors per filtered chunk in the PQ scan
constexpr int kExactScanChunk = 1024; // vectors per filtered chunk in the exact scan

// ---- probe inversion (worklist.cu) ----------------------------------------
// Scratch for the device-wide scan; query with bytes=0 first.
size_t worklist_scan_bytes(int nlist);
// Builds list-major (query, list) pairs from probes [nq, nprobe] (global list
// ids; list_map maps them to local lists or -1, nullptr = identity).
// When wl.groups is set, also packs the pairs of every list into groups of up
// to wl.gq (0: kGroupQueries) consecutive pairs:
// groups[g] = (list << 32) | (first pair << group_shift(gq)) | size.
// Only probe-table columns col0 .. col0+ncol-1 are used (ncol <= 0: to the end).
// seed_part >= 0 replaces the column range: 0 = each query's first probe whose
// list is local, 1 = its other local probes.
cudaError_t build_worklist(const int32_t* probes, int nq, int nprobe, int nlist_global,
                           const int32_t* list_map, int nlist_local, WorkList wl,
                           void* scan_tmp, size_t scan_bytes, cudaStream_t st, int col0 = 0, int ncol = 0,
                           int seed_part = -1);
constexpr int kGroupQueries = 4;

// ---- exact uint8 search on the tensor cores (exact_tc.cu) ------------------
// d in {128, 256}, 0 < k <= 16
bool exact_tc_usable(int d, int k);
// the tensor map (128 bytes, 64-byte aligned) over rows [n, d] of an exact index
cudaError_t exact_tc_map(const uint8_t* rows, int64_t n, int d, void* map_out);
// the grouped exact search (groups of up to 127 queries, wl.gq = 127) with q.x
// on the tensor cores; the same candidate keys as exact_group_scan.  flag is
// raised (4) when a bounded wait gave up.
cudaError_t exact_tc_scan(const void* map, const uint8_t* q_u8, int d, int k, ListStore ls, WorkList wl,
                          int max_groups, CandBuf cb, int* work_counter, int* flag, cudaStream_t st);

// ---- coarse routing (route.cu) --------------------------------------------
// valid[c] = 1 when the centroid's L2 norm is >= 1e-6, else 0.
cudaError_t route_centroid_valid(const float* cent, int nlist, int d, uint8_t* valid, cudaStream_t st);
// Exact fp32 squared L2 of every (query, centroid) pair as sortable bits
// (0xFFFFFFFF for centroids that are not valid): out [nq, nlist].
cudaError_t route_distances(const float* q, int nq, const float* cent, const uint8_t* valid,
                            int nlist, int d, uint32_t* out, cudaStream_t st);
// the same for the cosine distance 1 - <q, c> / (|q| |c|) (clamped at 0)
cudaError_t route_distances_cos(const float* q, int nq, const float* cent, const uint8_t* valid, int nlist, int d,
                                uint32_t* out, cudaStream_t st);
// Top-L (dist, id) per row of dist_bits [nq, n] -> ids [nq, L] (+ dist [nq, L] and/or
// sorted keys [nq, L], each optional).  Column c has id id_map[c] (nullptr: c).
cudaError_t route_select(const uint32_t* dist_bits, int nq, int n, int L, const int32_t* id_map,
                         int32_t* out_ids, float* out_dist, uint64_t* out_keys, cudaStream_t st);
// Top-L of n keys per query [nq, n] -> ids [nq, L]; distances as float bits
// (int_dist = 0) or as int32 (int_dist = 1, written to out_idist and out_dist).
cudaError_t merge_keys(const uint64_t* keys, int nq, int n, int L, int int_dist, int32_t* out_ids,
                       float* out_dist, int32_t* out_idist, cudaStream_t st);
// Top-L ids per query from S shards' sorted keys laid out [S][nq][L] (an
// all-gather of per-shard [nq, L]); L <= 32, S * L <= 256.
cudaError_t merge_shard_keys(const uint64_t* keys, int S, int nq, int L, int32_t* out_ids, cudaStream_t st);
// out[i] = clamp(round(q[i]), 0, 255) (updates/exact_update.cu:410-418)
// Tensor-core routing (route_tc.cu): approximate distances from one tcgen05
// GEMM over bf16 hi/lo splits, then exact rescoring of the candidates within
// the error bound of the approximation -- the same top-L as route_distances +
// route_select.  Usable for d % 16 == 0, d <= 144.
bool route_tc_usable(int d, int nlist);
int route_tc_tile(int d);
size_t route_tc_ops_elems(int nlist, int d);     // bf16 elements of the centroid operand
// cn: [nlist] squared norms; cne: [route_tc_cne_len] the same, +inf for
// invalid lists and tile padding
size_t route_tc_cne_len(int nlist);
cudaError_t route_tc_prepare(const float* cent, const uint8_t* valid, int nlist, int d, uint16_t* ops, float* cn,
                             float* cne, float* cn_max, cudaStream_t st);
// approximate distance bits [nq, nlist] (invalid lists 0xFFFFFFFF); flag bit 2
// is raised when a bounded wait gave up
cudaError_t route_tc(const float* q, int nq, const uint16_t* ops, const float* cn, const uint8_t* valid, int nlist,
                     int d, uint32_t* out, int* flag, cudaStream_t st);
// nprobe <= 32: one fused kernel (one tcgen05 sweep over the split operands,
// candidates and exact rescoring on chip; the centroids split over `splits`
// CTAs per 128 queries, whose sorted top-L keys [splits][nq][L] go to
// split_keys and are merged), plus an exact pass over the rare rows it hands
// back.  row_fallback, row_bound: [nq] scratch (row_bound may be null: then the
// CTAs of a query do not share their running bounds).
bool route_tc_fused_usable(int d, int nlist, int L);
// column splits that balance nq queries x nlist centroids over the device's SMs
int route_tc_fused_splits(int nq, int nlist);
cudaError_t route_tc_fused(const float* q, int nq, const uint16_t* ops, const float* cne, const float* cn_max,
                           const uint8_t* valid, int nlist, int d, const float* cent, int L, const int32_t* id_map,
                           int32_t* out_ids, uint64_t* out_keys, int32_t* row_fallback, uint64_t* split_keys,
                           uint32_t* row_bound, int splits, int* flag, cudaStream_t st);
cudaError_t route_rescore(const uint32_t* approx, const float* q, int nq, const float* cent, const float* cn_max,
                          const uint8_t* valid, int nlist, int d, int L, const int32_t* id_map, int32_t* out_ids,
                          float* out_dist, uint64_t* out_keys, cudaStream_t st);
cudaError_t make_query_u8(const float* q, size_t n, uint8_t* out, cudaStream_t st);

// ---- candidate selection (select.cu) ---------------------------------------
cudaError_t reset_candidates(CandBuf cb, int nq, cudaStream_t st);
// Top-R keys per query from a candidate buffer -> out [nq, R] (padding ~0), ascending
// when sorted, else the same keys in no particular order.
cudaError_t select_top_r(CandBuf cb, int nq, uint64_t* out, cudaStream_t st, bool sorted = true);
// Sorted exact keys -> (ids, int32 distances): for the exact path.
cudaError_t keys_to_exact_results(const uint64_t* keys, int nq, int k, int32_t* ids, int32_t* dist,
                                  float* fdist, cudaStream_t st);

// ---- exact uint8 fine search (exact.cu) -------------------------------------
// out[i] = sum_j x[i][j]^2 for n uint8 rows of d bytes (d % 16 == 0), exact int32.
cudaError_t u8_row_sqnorms(const uint8_t* x, int64_t n, int d, int32_t* out, cudaStream_t st);
// Grouped exact scan (d = 128 or 256, k <= 16): groups of up to 64 queries per
// list from wl.groups (wl.gq = 64); every (query, list) pair appends its k
// smallest keys to the query's candidate buffer.
bool exact_group_usable(int d, int k);
cudaError_t exact_group_scan(const uint8_t* q_u8, int d, int k, ListStore ls, WorkList wl, int max_groups,
                             CandBuf cb, int* work_counter, cudaStream_t st);
cudaError_t exact_scan(const uint8_t* q_u8, int nq, int d, ListStore ls, WorkList wl, int max_pairs,
                       CandBuf cb, int* work_counter, cudaStream_t st);
// fp32 rows: out[i] = sqrtf(sum_j x[i][j]^2) (sequential fp32 sum)
cudaError_t f32_row_norms(const float* x, int64_t n, int d, float* out, cudaStream_t st);
// exact fp32 fine search over the probed lists of x (cluster-major [n, d]):
// L2 or (cosine != 0) 1 - cos, keys (distance, position) into cb
cudaError_t f32_scan(const float* q, int d, const float* x, const float* xnorm, ListStore ls, int cosine, WorkList wl,
                     int max_pairs, CandBuf cb, int* work_counter, cudaStream_t st);

// ---- index build (build.cu) ---------------------------------------------------
// out[i] = x[offset + i] as fp32 for i < n (x uint8 when is_u8, else fp32)
cudaError_t stage_rows_f32(const void* x, int is_u8, size_t offset, size_t n, float* out, cudaStream_t st);
// stable cluster-major order of n rows by assignment: counts / offsets per
// list, order[p] = row at position p (rows of a list in increasing order);
// cudaErrorInvalidValue when an assignment is outside [0, nlist)
cudaError_t build_reorder(const int32_t* assign, int64_t n, int nlist, int32_t* counts, int64_t* offsets,
                          int32_t* order, cudaStream_t st);
// cent[l] = mean of the rows assigned to l (fp64 sums in row order; empty lists keep their centroid)
cudaError_t kmeans_update(const void* x, int is_u8, int64_t n, int d, const int32_t* assign, int nlist, float* cent,
                          cudaStream_t st);
// codes[i][m] = nearest of the 256 codewords of sub-space m to the residual of
// row rows[i] (nullptr: i) against its centroid cent[assign[row]]
cudaError_t pq_encode_rows(const void* x, int is_u8, int64_t n, int d, const int32_t* rows, const float* cent,
                           const int32_t* assign, const float* cb, int M, uint8_t* codes, cudaStream_t st);
// `iters` Lloyd iterations per sub-space on n rows, codebook cb [M, 256, d / M] updated in place
cudaError_t pq_train(const void* x, int is_u8, int64_t n, int d, const float* cent, const int32_t* assign, int M,
                     int iters, float* cb, cudaStream_t st);

// ---- residual PQ (pq.cu) -----------------------------------------------------
struct PQParams {
    const float* q;          // [nq, d] fp32 queries
    const float* cent;       // [nlist, d]
    const float* codebook;   // [M, 256, dsub]
    const float* codebook_t; // [256, M, dsub] (the same codebook, code-major, for coalesced LUT builds)
    int d, M, dsub;
    ListStore main;
    ListStore delta;
    int has_delta;
    // with a delta: every list's main rows followed by its delta rows in one
    // grouped-ring tile stream (pq_build_gring_mix), or nullptr
    const uint8_t* mix;
    const int64_t* mix_off;  // [nlist] byte offset of each list's combined tiles
};
bool pq_supported_m(int M);
// true when the query-grouped kernel scans (M, d); other shapes use the row kernel
bool pq_group_usable(int M, int d);
// bytes of the grouped-ring tile layout of one list of `count` vectors
int64_t pq_gring_list_bytes(int count, int M);
// builds the grouped-ring tile layout of every list from row-major codes [n, M]
cudaError_t pq_build_gring(const uint8_t* codes, const int64_t* offsets, const int32_t* counts,
                           const int64_t* tile_off, int nlist, int M, uint8_t* out, cudaStream_t st);
// the Rd (<= 32) smallest delta keys of each query over the delta rows of its
// probed lists, sorted, computed directly from the row-major delta codes
// (PQParams::delta.data) without LUTs; probes [nq, nprobe] hold global list
// ids mapped through list_map (nullptr: identity) like build_worklist's
bool pq_delta_direct_usable(int M, int d, int Rd);
cudaError_t pq_delta_direct(const PQParams& p, const int32_t* probes, int nq, int nprobe, int nlist_global,
                            const int32_t* list_map, int Rd, uint64_t* out, cudaStream_t st);
// the combined tile stream of every list (pq.cu, mix_stripes): each of the
// 32 stripes holds its share of the list's main rows, then its share of the
// delta rows, from the main and delta tiles; list l's bytes at mix_off[l],
// pq_mix_list_bytes of them
int64_t pq_mix_list_bytes(int count_main, int count_delta, int M);
cudaError_t pq_build_gring_mix(const uint8_t* main_tiles, const int64_t* main_off, const int32_t* main_counts,
                               const uint8_t* delta_tiles, const int64_t* delta_off, const int32_t* delta_counts,
                               const int64_t* mix_off, int nlist, int M, uint8_t* out, cudaStream_t st);
// vectors per filtered chunk of the kernel that scans (M, d); each chunk keeps at
// most R candidates per query, which bounds the candidate buffers
// filtered chunks the scan of one list of `count` vectors takes, and the most
// vectors one chunk holds: a query's candidates from one probed list number at
// most chunks * min(R + slack, chunk items)
int pq_scan_chunks(int M, int d, int count);
int pq_scan_chunk_items(int M, int d);
// keys beyond R one filtered chunk of the PQ scan may append (its cut is a
// bound that admits between R and R + slack keys)
int pq_chunk_slack(int M, int d, int R);
cudaError_t pq_scan(const PQParams& p, WorkList wl, int max_pairs, CandBuf cm, CandBuf cd, int* work_counter,
                    cudaStream_t st);
// Exact rerank of the stage-1 keys of both segments -> top-k (ids, dist).
// When out_exact_main is given, the per-candidate exact keys are written instead
// of (ids, dist) being selected: [nq, R] and [nq, Rd] aligned with the inputs.
// kmax (device [nq], may be null): main keys above kmax[q] are not candidates.
// out_topk (device [nq, k], may be null): the top-k exact keys instead of (ids, dist).
cudaError_t pq_rerank(const PQParams& p, int nlist, const uint64_t* s1_main, int R, const uint64_t* s1_delta,
                      int Rd, int nq, int k, int32_t* out_ids, float* out_dist, uint64_t* out_exact_main,
                      uint64_t* out_exact_delta, cudaStream_t st, const uint64_t* kmax = nullptr,
                      uint64_t* out_topk = nullptr);
// Sharded search, owner side: adc_all [G][qo][R] stage-1 lists of the G shards
// (any order) -> kappa [qo], the R-th smallest key of their union (kKeyNone
// when the union has fewer than R keys); top_all [G][qo][k] the shards' exact
// top-k of their keys <= kappa -> the top-k.
cudaError_t pq_shard_kappa(const uint64_t* adc_all, int G, int qo, int R, uint64_t* kappa, cudaStream_t st);
cudaError_t pq_shard_final(const uint64_t* top_all, int G, int qo, int k, int exact_is_int, int32_t* out_ids,
                           float* out_dist, cudaStream_t st);
// Final merge of sharded stage-1 results: per query, G shards each give R
// (ADC key, exact key) pairs for the main segment and Rd for the delta.
cudaError_t pq_merge_shards(const uint64_t* adc_main, const uint64_t* exact_main, int n_main, int R,
                            const uint64_t* adc_delta, const uint64_t* exact_delta, int n_delta, int Rd,
                            int nq, int k, int exact_is_int, int32_t* out_ids, float* out_dist,
                            cudaStream_t st);

}  // namespace isb
