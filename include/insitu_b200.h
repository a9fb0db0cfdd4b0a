/*
 * insitu_b200.h -- C ABI of libinsitu_b200.so, the B200 (sm_100a) IVF query
 * hot path of InSituANN: coarse routing, exact uint8 fine search, residual-PQ
 * ADC search with exact rerank, the update overlay (published delta
 * segments) and the entry points a cluster-sharded multi-GPU driver needs.
 *
 * Plain C types only.  Every function may be called from any host thread;
 * one batch context is one CUDA stream and must not be used by two threads at
 * once.  Index contexts are immutable after loading except for the delete
 * mask and the delta segment, so several batch contexts may search one index
 * concurrently.  ivf_set_deleted, ivf_pq_publish_delta and
 * ivf_pq_clear_delta may run while other threads search the same index: they
 * wait until every search that has started reading the index has queued its
 * work, synchronise the device, and only then free the replaced arrays;
 * searches that start later see the new arrays.  An index context must not be
 * destroyed while a search on it is in flight.
 *
 * Return conventions
 *   - names taken from the reference keep the reference's return types and
 *     meaning (cited per function);
 *   - the entry points the reference does not have return 0 on success and a
 *     negative IVF_E* code on failure; the message is kept per context and is
 *     read with ivf_last_error().
 * No function aborts, exits or resets the device.
 *
 * Environment (read on every call; every choice gives the same results bit
 * for bit):
 *   INSITU_SCRATCH_MB   per-batch scratch budget in MB (default: an eighth
 *                       of the device's memory, 1 to 24 GB); larger batches
 *                       run in query sub-batches inside one call
 *   INSITU_ROUTE_TC     routing kernels: 1 (default) fused tensor-core
 *                       kernel where it applies, 2 fused or tensor-core
 *                       matrix, 3 tensor-core matrix, 0 CUDA cores only
 *   INSITU_EXACT_TC     exact uint8 groups (d = 128 / 256, k <= 16): 1
 *                       (default) on the tensor cores, 0 on the CUDA cores
 *   INSITU_PQ_DELTA     read by ivf_pq_publish_delta / ivf_pq_insert: how
 *                       the published delta rows are searched -- "direct"
 *                       by a kernel of their own after the main scan
 *                       (delta_topk above 32 as "seg"), "mix" in one tile
 *                       stream with each list's main rows, "seg" in their
 *                       own tiles after each list's main rows; unset:
 *                       "direct" up to 100 delta rows per list on average,
 *                       else "mix"
 *
 * Citations are paths inside the reference project
 * (mindtravel/InSituANN-OpenSource).
 */
#ifndef INSITU_B200_H
#define INSITU_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* status codes of the entry points that are new in this library */
#define IVF_OK 0
#define IVF_EINVAL -1       /* bad argument (null pointer, size, unsupported shape) */
#define IVF_ECUDA -2        /* a CUDA call failed (message has the CUDA error string) */
#define IVF_ESTATE -3       /* wrong context state (nothing loaded, wrong index type) */
#define IVF_ENOMEM -4       /* device allocation failed */
#define IVF_EOVERFLOW -5    /* a candidate buffer overflowed (results would be wrong) */
#define IVF_EUNSUPPORTED -6 /* metric / layout outside the hot path (e.g. cosine) */

/* distance_mode values, cuda/pch.h:36-39 */
#define IVF_DISTANCE_L2 0
#define IVF_DISTANCE_COSINE 1

/* ======================================================================
 * Index and batch contexts -- cuda/search/ivf_search.cuh:204-321
 * ====================================================================== */

/* ivf_search.cuh:215 -- new, empty index context (NULL on failure). */
void* ivf_create_index_context(void);
/* ivf_search.cuh:222 -- frees the context and every device buffer it owns. */
void ivf_destroy_index_context(void* idx_ctx);

/*
 * ivf_search.cuh:236-244 -- adopt caller-allocated device arrays of an fp32
 * index (ownership passes to the context, as in ivf_search_separated.cu:141-143):
 * list sizes [nlist], cluster-major rows [n, d] (list l starts at the sum of
 * the sizes before it), centroids [nlist, d].  Returns 1 when loaded, 0 when
 * the context already holds an index.  ivf_pipeline_stage2_compute on such an
 * index routes by cosine (as the reference does on this path) and scans by
 * exact L2 (distance_mode 0) or 1 - cosine (distance_mode 1); results are
 * row positions.  The streaming upload (cpu_fine_b200.h) builds the same index
 * from host data.
 */
int ivf_load_dataset(void* idx_ctx, int* d_cluster_size, float* d_cluster_vectors, float* d_cluster_centers,
                     int n_total_clusters, int n_total_vectors, int n_dim);

/* ivf_search.cuh:258 -- batch context: one stream, scratch sized for these limits. */
void* ivf_create_batch_context(int max_n_query, int n_dim, int max_n_probes, int max_k, int n_total_clusters);
/* ivf_search.cuh:265 */
void ivf_destroy_batch_context(void* batch_ctx);

/* ivf_search.cuh:276-280 -- async H2D of the fp32 query batch on the batch stream. */
void ivf_pipeline_stage1_prepare(void* batch_ctx, float* query_batch_host, int n_query);

/*
 * ivf_search.cuh:294-301 -- routing + fine search of the staged queries:
 *   uint8 index: exact int32 search, top-k by (distance, original id);
 *   PQ index:    residual-PQ stage 1 (rerank_n = 512) + exact rerank, with
 *                the published delta segment when one exists.
 *   fp32 index:  cosine routing, exact L2 or cosine scan (see ivf_load_dataset).
 * distance_mode IVF_DISTANCE_COSINE is served on fp32 indexes only (the others
 * record IVF_EUNSUPPORTED).
 */
void ivf_pipeline_stage2_compute(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int k,
                                 int distance_mode);

/* ivf_search.cuh:314-320 -- D2H of the results, then stream sync. */
void ivf_pipeline_get_results(void* batch_ctx, float* topk_dist, int* topk_index, int n_query, int k);
/* ivf_search.cuh:327 */
void ivf_pipeline_sync_batch(void* batch_ctx);

/* ======================================================================
 * Exception-safe *_wrapper exports and the per-OID registry --
 * cuda/search/ivf_search_wrapper.cpp:85-427.  Same meaning as above; the
 * int-returning wrappers give -1 on failure.
 * ====================================================================== */
void* ivf_create_index_context_wrapper(void);
void ivf_destroy_index_context_wrapper(void* idx_ctx);
int ivf_load_dataset_wrapper(void* idx_ctx, int* d_cluster_size, float* d_cluster_vectors,
                             float* d_cluster_centers, int n_total_clusters, int n_total_vectors, int n_dim);
void* ivf_create_batch_context_wrapper(int max_n_query, int n_dim, int max_n_probes, int max_k,
                                       int n_total_clusters);
void ivf_destroy_batch_context_wrapper(void* batch_ctx);
void ivf_pipeline_stage1_prepare_wrapper(void* batch_ctx, float* query_batch_host, int n_query);
void ivf_pipeline_stage2_compute_wrapper(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int k,
                                         int distance_mode);
void ivf_pipeline_get_results_wrapper(void* batch_ctx, float* topk_dist, int* topk_index, int n_query, int k);
void ivf_pipeline_sync_batch_wrapper(void* batch_ctx);
/* ivf_search_wrapper.cpp:313-320 -- 1 when the context holds a loaded index. */
int ivf_check_index_initialized_wrapper(void* idx_ctx);
/* ivf_search_wrapper.cpp:346-427 -- 64-slot OID -> index registry (thread-safe here). */
void ivf_register_index_instance(unsigned int index_oid, void* gpu_handle);
void* ivf_get_index_instance(unsigned int index_oid);
void ivf_unregister_index_instance(unsigned int index_oid);

/* ======================================================================
 * Coarse routing handle -- cuda/search/cpu_fine/cpu_fine.h:232-278
 * (C++ linkage there; C linkage here, same layout and argument meaning).
 * The library exports both: C callers use these declarations, C++ runners
 * the reference's own cpu_fine.h or cpu_fine_b200.h.  A C++ file that
 * includes cpu_fine_b200.h (or the reference's cpu_fine.h) and this header
 * defines INSITU_B200_NO_COARSE first, since a function cannot be declared
 * with both linkages.
 * ====================================================================== */
#ifndef INSITU_B200_NO_COARSE
typedef struct CoarseHandle {
    const float* d_centers;   /* borrowed device centroids [n_total_clusters, dim] */
    float* d_centers_norm;    /* owned: here the per-centroid validity (norm >= 1e-6) */
    void* cublas_handle;      /* owned: here the routing state (stream, scratch) */
    int n_total_clusters;
    int dim;
    int distance_mode_cached;
} CoarseHandle;

typedef struct CoarseTimingBreakdown {
    double query_h2d_ms;
    double seq_init_ms;
    double query_norm_ms;
    double gemm_ms;
    double topk_ms;
    double cluster_d2h_ms;
    double coarse_compute_ms;
    double coarse_total_ms;
} CoarseTimingBreakdown;

/* cpu_fine.h:252-257 */
void coarse_handle_init(CoarseHandle* h, const float* d_centers, int n_total_clusters, int dim);
/* cpu_fine.h:259 */
void coarse_handle_release(CoarseHandle* h);
/*
 * cpu_fine.h:266-276 -- top-n_probes lists per query, host in / host out,
 * ranked by exact fp32 L2 (ties: smaller list id).  Bad arguments are
 * reported through ivf_global_last_error() and leave the output untouched
 * (the reference aborts, ivf_search_cpu_fine.cu:775-784).
 */
void coarse_search(const CoarseHandle* h, const float* h_query, int n_query_batch, int n_probes, int distance_mode,
                   int* h_cluster_ids_out, double* out_coarse_ms, double* out_h2d_ms, double* out_d2h_ms);
/* cpu_fine.h:278 -- timing of the calling thread's last coarse_search. */
const CoarseTimingBreakdown* coarse_get_last_timing(void);
#endif /* INSITU_B200_NO_COARSE */

/* ======================================================================
 * Index loading (new: the reference loads these inside its runners,
 * updates/pq_update.cu:676-713 and updates/exact_update.cu:2229).  Arrays
 * are in the reference file layouts and are copied into memory the index
 * owns; positions are cluster-major (stable reorder).  offsets, counts,
 * centroids and the codebook are host arrays; the bulk arrays (base rows,
 * codes, reorder_to_original, rerank rows) may be host arrays or device
 * arrays on the index's device (the copy direction is inferred).
 * ====================================================================== */

/*
 * uint8 exact index.  base_u8 [n, d] cluster-major; offsets [nlist] (first
 * position of each list), counts [nlist]; reorder_to_original [n] (NULL =
 * identity); centroids [nlist, d].  d must be a multiple of 16, <= 512.
 */
int ivf_u8_load(void* idx_ctx, const uint8_t* base_u8, const long long* offsets, const int* counts,
                const int* reorder_to_original, const float* centroids, int nlist, long long n, int d);

/*
 * Residual-PQ index (formats of scripts/train_ivfpq_residual.py:6-15):
 * codebook [M, K, dsub] fp32 with K = 256 and M*dsub = d, M a multiple of 8
 * and <= 64; codes [n, M] cluster-major; rerank rows base_u8 [n, d] or
 * base_f32 [n, d] (exactly one non-NULL) in the same cluster-major order.
 */
int ivf_pq_load(void* idx_ctx, const float* centroids, const float* codebook, int M, int K, int dsub,
                const uint8_t* codes, const long long* offsets, const int* counts, const int* reorder_to_original,
                const uint8_t* base_u8, const float* base_f32, int nlist, long long n, int d);

/*
 * Marks a loaded index as one shard of a larger index: local list l is
 * global list local_to_global[l] (of nlist_global), and its vectors occupy
 * global positions key_offsets[l] .. key_offsets[l]+counts[l]-1 of the whole
 * index.  Routing then reports global list ids, fine search accepts global
 * probe ids (lists of other shards are skipped) and ranking keys use global
 * positions, so per-shard results merge into exactly the unsharded result.
 */
int ivf_set_shard(void* idx_ctx, int nlist_global, const int* local_to_global, const long long* key_offsets);

/*
 * Query-time deletes (the reference applies them inside its runners,
 * updates/exact_update.cu:54, 89, 354-407 and updates/pq_update.cu:45,
 * 503-523): deleted [n] holds one byte per cluster-major position of the
 * loaded index (nonzero = deleted; NULL clears the mask).  The exact search
 * does not scan deleted positions; the residual-PQ search keeps them in stage
 * 1 (they take candidate slots, as in the reference) and does not rerank them.
 * The delta segment has no deletes.  Waits for the device before replacing
 * the mask.
 */
int ivf_set_deleted(void* idx_ctx, const unsigned char* deleted, long long n);

/* ======================================================================
 * The reference's index file formats (host code):
 *   centroids [nlist:i32][dim:i32][f32 ...]            updates/pq_update.cu:46
 *   assign    [n:i64][i32 ...]                         updates/pq_update.cu:47
 *   codebook  [M:i32][K:i32][dsub:i32][pad:i32][f32 M*K*dsub]
 *                                        scripts/train_ivfpq_residual.py:209-213
 *   codes     [n:i64][M:i32][pad:i32][u8 n*M], cluster-major  (:304-307)
 *   u8bin / fbin [n:i32][d:i32][payload]  (DiskANN)    updates/io.h:183-294
 *   gt        [n:i32][k:i32][i32 n*k]                  scripts/gen_gt_fast.py:34-38
 * Readers return the payload's element count; with out == NULL they read the
 * header only, else out must hold cap >= count elements.  -1 on error
 * (message in ivf_global_last_error()).  Writers return IVF_OK or -1.
 * ====================================================================== */
long long ivf_read_centroids(const char* path, float* out, long long cap, int* nlist, int* dim);
long long ivf_read_assign(const char* path, int* out, long long cap, long long* n);
long long ivf_read_codebook(const char* path, float* out, long long cap, int* M, int* K, int* dsub);
long long ivf_read_codes(const char* path, unsigned char* out, long long cap, long long* n, int* M);
long long ivf_read_u8bin(const char* path, unsigned char* out, long long cap, long long* n, int* d);
long long ivf_read_fbin(const char* path, float* out, long long cap, long long* n, int* d);
long long ivf_read_gt(const char* path, int* out, long long cap, long long* n, int* k);
int ivf_write_centroids(const char* path, const float* centroids, int nlist, int dim);
int ivf_write_assign(const char* path, const int* assign, long long n);
int ivf_write_codebook(const char* path, const float* codebook, int M, int K, int dsub);
int ivf_write_codes(const char* path, const unsigned char* codes, long long n, int M);
/* residual-PQ index straight from the reference's files: centroids, codebook,
 * cluster-major codes, assignment and the uint8 base rows (u8bin, original
 * order), laid out by the stable reorder of the assignment -- what
 * updates/pq_update.cu:676-713 loads; reported ids are original ids */
int ivf_pq_load_files(void* idx_ctx, const char* centroids_path, const char* codebook_path, const char* codes_path,
                      const char* assign_path, const char* base_u8bin_path);

/* ======================================================================
 * Index build on the GPU (the reference builds offline: k-means in
 * cuda/clustering/kmeans/kmeans.cu, the stable reorder in
 * cuda/dataset/dataset.cuh:559-592, residual PQ with faiss in
 * scripts/train_ivfpq_residual.py:151-310).  Device pointers; every
 * reduction runs in a fixed order (fp64 sums, rows in increasing order), so
 * a build is deterministic.  The calls without a batch context queue their
 * work on `stream` (a cudaStream_t, NULL = legacy default stream) and may
 * allocate temporary device memory; they report failures through
 * ivf_global_last_error().
 * ====================================================================== */
/* a routing-only index context: the centroids [nlist, d] (host or device),
 * for ivf_assign and ivf_route */
int ivf_load_centroids(void* idx_ctx, const float* centroids, int nlist, int d);
/* exact nearest centroid of n rows d_x [n, d] (fp32, or uint8 when x_is_u8):
 * the routing kernels with n_probes = 1 (exact fp32 L2, ties to the smaller
 * list id), in sub-batches of the batch context's max_n_query rows, on the
 * batch stream; d_assign [n] int32 */
int ivf_assign(void* batch_ctx, void* idx_ctx, const void* d_x, int x_is_u8, long long n, int* d_assign);
/* stable cluster-major order: d_counts [nlist], d_offsets [nlist], d_order
 * [n] = the row at each position (a list's rows in increasing row order, as
 * dataset.cuh:559-592 and the reorder_to_original array of the loaders) */
int ivf_build_reorder(const int* d_assign, long long n, int nlist, int* d_counts, long long* d_offsets, int* d_order,
                      void* stream);
/* one k-means update: centroid l = mean of the rows assigned to l (lists
 * without rows keep their centroid) */
int ivf_kmeans_update(const void* d_x, int x_is_u8, long long n, int d, const int* d_assign, int nlist,
                      float* d_centroids, void* stream);
/* residual-PQ training: `iters` Lloyd iterations per sub-space (K = 256,
 * dsub = d / M in {1, 2, 4, 8}) on the residuals x_i - centroid[assign_i] of
 * n sample rows, starting from and updating d_codebook [M, 256, dsub] */
int ivf_pq_train(const void* d_x, int x_is_u8, long long n, int d, const float* d_centroids, const int* d_assign,
                 int M, int iters, float* d_codebook, void* stream);
/* residual-PQ encoding: d_codes [n, M], code m of row d_rows[i] (NULL: i) =
 * the nearest codeword (squared L2 in dimension order, ties to the smaller
 * code) of sub-space m to its residual against centroid[assign[row]] */
int ivf_pq_encode(const void* d_x, int x_is_u8, long long n, int d, const int* d_rows, const float* d_centroids,
                  const int* d_assign, const float* d_codebook, int M, unsigned char* d_codes, void* stream);

/* ======================================================================
 * Update overlay (new: runner-internal in the reference,
 * updates/pq_update.cu:396-494, 975-1055)
 * ====================================================================== */
/*
 * Publishes one delta segment of n_delta vectors over the same lists:
 * codes [n_delta, M] list-major, offsets/counts [nlist] (local lists),
 * ids [n_delta] (reported ids, disjoint from the base), rerank rows raw_u8
 * or raw_f32 [n_delta, d] in delta-position order (same type as the base
 * rerank rows).  key_offsets [nlist] may be NULL (= offsets); shards pass the
 * global delta positions.  Replaces a previously published segment.
 */
int ivf_pq_publish_delta(void* idx_ctx, const uint8_t* codes, const int* ids, const int* counts,
                         const long long* offsets, const long long* key_offsets, const uint8_t* raw_u8,
                         const float* raw_f32, long long n_delta);
int ivf_pq_clear_delta(void* idx_ctx);
/*
 * How the published delta is searched, fixed when it was published
 * (INSITU_PQ_DELTA, else by its size): 0 none published, 1 a delta kernel of
 * its own after the main scan (a delta_topk above 32 is searched as 3), 2 in
 * one tile stream with each list's main rows, 3 in its own tiles after each
 * list's main rows; IVF_EINVAL for a bad context.  Every mode returns the same
 * results.
 */
int ivf_pq_delta_mode(void* idx_ctx);
/*
 * Online insert (the pipeline the reference's README describes as not
 * released, README.md:16-24): n new vectors d_x [n, d] -- device rows, uint8
 * (x_is_u8 = 1) or fp32 as the index's rerank rows -- with reported ids
 * (host [n]) join the delta segment.  Each row is assigned to its nearest
 * centroid by the exact routing (n_probes = 1), its residual is encoded with
 * the index's codebook (the build kernels of ivf_pq_encode), and the grown
 * segment is published in one step: a concurrent search sees all of an
 * insert or none of it.  Within a list, older delta rows come first, then
 * the new ones in insertion order.  Whole (unsharded) indexes only.
 */
int ivf_pq_insert(void* idx_ctx, const void* d_x, int x_is_u8, const int* ids, long long n);

/* ======================================================================
 * Search (new, explicit parameters)
 * ====================================================================== */
/* routing of the staged queries into the batch's probe table (device). */
int ivf_route(void* batch_ctx, void* idx_ctx, int n_query, int n_probes);
/* copies probe ids in or out of the batch's probe table [n_query, n_probes] (host). */
int ivf_set_probes(void* batch_ctx, const int* h_probes, int n_query, int n_probes);
int ivf_get_probes(void* batch_ctx, int* h_probes, int n_query, int n_probes);

/* exact uint8 search: routing (if route != 0) + fine search on the batch probes. */
int ivf_u8_search(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int k, int route);
/*
 * residual-PQ search: routing (if route != 0) + stage 1 with rerank_n
 * candidates (+ delta_topk from the delta segment when use_overlay != 0 and
 * one is published; the reference uses 16, pq_update.cu:25) + exact rerank
 * (int32 on uint8 rows; fp32 rows in the reference's AVX-512 order of
 * operations, cpu_fine_kernels_pq_resid.cpp:106-131, so distances equal the
 * reference's bit for bit).  A position that stage 1 holds twice (a list
 * probed twice) is reranked once.
 */
int ivf_pq_search(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int k, int rerank_n,
                  int use_overlay, int delta_topk, int route);

/* results of the last search: ids [n_query, k]; float or int32 distances. */
int ivf_get_results_i32(void* batch_ctx, int* ids, int* dist, int n_query, int k);

/* ======================================================================
 * Device-resident variants (pointers are device pointers on the batch's
 * device; used when the caller keeps queries and results in HBM)
 * ====================================================================== */
int ivf_pipeline_stage1_prepare_device(void* batch_ctx, const float* d_query, int n_query);
int ivf_get_results_device(void* batch_ctx, float* d_dist, int* d_index, int n_query, int k);
/* the batch's CUDA stream (cudaStream_t) so callers can order their own work */
void* ivf_batch_stream(void* batch_ctx);

/* ======================================================================
 * Shard exchange (new; inverted lists sharded by cluster over GPUs).  All
 * pointers are device pointers; the caller moves them between GPUs (NCCL).
 * ====================================================================== */
/* local routing keys [n_query, n_probes]: (fp32 distance bits << 32) | global list id */
int ivf_route_keys(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, unsigned long long* d_keys);
/* merges n_in keys per query [n_query, n_in] into the batch probe table */
int ivf_route_merge(void* batch_ctx, const unsigned long long* d_keys, int n_in, int n_query, int n_probes);
/* merges n_shards sorted key lists laid out as all-gathered, [n_shards][n_query][n_probes]
 * (no transpose), into the batch probe table; n_probes <= 32, n_shards * n_probes <= 256 */
int ivf_route_merge_shards(void* batch_ctx, const unsigned long long* d_keys, int n_shards, int n_query,
                           int n_probes);
/*
 * stage 1 + exact scoring of this shard's candidates for the batch probes:
 * d_adc [n_query, rerank_n] sorted (ADC bits << 32 | global position),
 * d_exact [n_query, rerank_n] aligned (exact bits << 32 | reported id);
 * the same for the delta segment when d_dadc/d_dexact are non-NULL.
 */
int ivf_pq_search_shard(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int rerank_n, int delta_topk,
                        unsigned long long* d_adc, unsigned long long* d_exact, unsigned long long* d_dadc,
                        unsigned long long* d_dexact);
/* merges per-query concatenations of shard outputs into the batch results */
int ivf_pq_merge_shards(void* batch_ctx, const unsigned long long* d_adc, const unsigned long long* d_exact,
                        int n_main, int rerank_n, const unsigned long long* d_dadc,
                        const unsigned long long* d_dexact, int n_delta, int delta_topk, int n_query, int k,
                        int exact_is_int);
/* exact uint8 shard search: sorted top-k keys (distance << 32 | original id) per query */
int ivf_u8_search_shard(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int k,
                        unsigned long long* d_keys);
/* merges n_in exact keys per query into the batch results (top-k) */
int ivf_u8_merge_shards(void* batch_ctx, const unsigned long long* d_keys, int n_in, int n_query, int k);

/* ======================================================================
 * Phased sharded residual-PQ search (no counterpart in the reference)
 * ====================================================================== */
/*
 * The same results as ivf_pq_search_shard + ivf_pq_merge_shards, with less
 * work and traffic per shard: every shard scans each query's nearest probe
 * first, the shards exchange their rank-R bounds (int64 minimum over
 * shards), then scan the other probes with the exchanged bounds; the query's
 * owner finds kappa, the R-th smallest stage-1 key over all shards, and each
 * shard reranks only its keys <= kappa and returns its exact top-k.  Per
 * batch (queries broadcast, block-partitioned owners, G shards):
 *   ivf_pq_shard_scan(pass 0)
 *   all-reduce MIN (int64) over ivf_pq_shard_bounds(batch)[0 .. n_query)
 *   ivf_pq_shard_scan(pass 1)
 *   ivf_pq_shard_select -> d_adc [n_query, rerank_n] (this shard's stage-1
 *       keys with global positions, in no particular order);  all-to-all to
 *       the owners -> [G][n_owned][R]
 *   ivf_pq_shard_kappa (owner) -> d_kappa [n_owned];  all-to-all back ->
 *       each shard's [n_query] key limits in global query order
 *   ivf_pq_shard_rerank -> d_topk [n_query, k] (exact keys, ascending,
 *       kKeyNone-padded);  all-to-all to the owners -> [G][n_owned][k]
 *   ivf_pq_shard_final (owner) -> the batch results of its n_owned queries
 * Probes come from ivf_set_probes / ivf_route_merge / ivf_route_merge_shards.
 * One sub-batch only (IVF_EINVAL when the candidate buffers of n_query
 * queries exceed INSITU_SCRATCH_MB).  Main segment only (no overlay);
 * k <= 32 and G * k <= 256.
 */
int ivf_pq_shard_scan(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int rerank_n, int pass);
/* device array [n_query] of the rank-R bounds, as int64 (no bound: INT64_MAX) */
unsigned long long* ivf_pq_shard_bounds(void* batch_ctx);
int ivf_pq_shard_select(void* batch_ctx, void* idx_ctx, int n_query, int n_probes, int rerank_n,
                        unsigned long long* d_adc);
int ivf_pq_shard_kappa(void* batch_ctx, const unsigned long long* d_adc_all, int n_shards, int n_owned,
                       int rerank_n, unsigned long long* d_kappa);
int ivf_pq_shard_rerank(void* batch_ctx, void* idx_ctx, int n_query, int rerank_n,
                        const unsigned long long* d_adc, const unsigned long long* d_kappa, int k,
                        unsigned long long* d_topk);
int ivf_pq_shard_final(void* batch_ctx, const unsigned long long* d_topk_all, int n_shards, int n_owned, int k,
                       int exact_is_int);

/* ======================================================================
 * Allocation-free search (no counterpart in the reference)
 * ====================================================================== */
/*
 * Exact uint8 search for callers that must not allocate device memory while
 * they serve queries (a database worker whose device memory is budgeted up
 * front, a real-time service that must avoid the allocator and its implicit
 * synchronisation, a caller that brings its own stream and buffer pool).
 * Same results as ivf_u8_search on the probe table d_probes; every argument
 * is a device pointer on the index's device and the work is queued on
 * `stream` (a cudaStream_t; NULL = legacy default stream), so the outputs are
 * ready once that stream has synchronised.
 *
 * All scratch comes from one fixed 16 MiB array compiled into the library,
 * held by every GPU that loads the library until the process exits.  The
 * call allocates nothing; a batch whose scratch would exceed 16 MiB is
 * rejected with IVF_EINVAL (message in ivf_global_last_error()) -- split it
 * into smaller batches.  The first call on each device looks up the array's
 * device address; make that first call before any stream capture.  Calls
 * share the array: two calls that overlap on the GPU race, so order them on
 * one stream or synchronise between them.  The call returns with the
 * caller's current device unchanged; the cached array address is valid for
 * the life of the device's primary context (no cudaDeviceReset in between).
 */
int ivf_u8_search_noalloc(void* idx_ctx, const uint8_t* d_query_u8, const int* d_probes, int n_query, int n_probes,
                          int k, int* d_out_ids, int* d_out_dist, void* stream);

/* ======================================================================
 * observability
 * ====================================================================== */
/* number of kernels this library has launched in this process (all devices) */
unsigned long long ivf_kernel_launches(void);

/* stages timed by ivf_batch_profile; ivf_batch_stage_ms returns IVF_STAGE_COUNT */
#define IVF_STAGE_ROUTE 0     /* coarse routing: distances + top-nprobe */
#define IVF_STAGE_WORKLIST 1  /* probe inversion + candidate reset */
#define IVF_STAGE_SCAN 2      /* fine scan (ADC or exact) with the block filter */
#define IVF_STAGE_SELECT 3    /* per-query top-R / top-k selection */
#define IVF_STAGE_RERANK 4    /* exact rerank of the PQ candidates */
#define IVF_STAGE_COUNT 5
/* enable (1) / disable (0) CUDA-event timing of the stages of later searches */
int ivf_batch_profile(void* batch_ctx, int enable);
/* syncs the batch stream, writes the summed ms of each stage since the last
 * call into out_ms[0..n), resets the sums; returns IVF_STAGE_COUNT or < 0 */
int ivf_batch_stage_ms(void* batch_ctx, double* out_ms, int n);

/* ======================================================================
 * errors
 * ====================================================================== */
/* last error message of an index or batch context ("" when none) */
const char* ivf_last_error(void* ctx);
/* last error of the calling thread for calls without a context (coarse_search) */
const char* ivf_global_last_error(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* INSITU_B200_H */
