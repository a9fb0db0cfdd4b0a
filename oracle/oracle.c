/*
 * oracle.c -- CPU restatement of the InSituANN IVF query hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this file.  It is imported by tests/, by __graft_entry__.smoke() and
 * by bench.py's cpu_baseline / --impl reference legs, always as the checker.
 *
 * Parity is pinned two ways (see tests/test_oracle.py):
 *   - hand-computed known-answer cases (tests/golden/kat_*.json);
 *   - the reference's own CPU kernels, compiled unmodified from the reference
 *     tree into oracle/_ref/libref_cpu_fine.so, run on the committed seeded
 *     fixtures (tests/golden/ npz files produced by tests/golden/make_golden.py).
 *
 * Arithmetic rules (compile with -O2 -ffp-contract=off, never -ffast-math):
 *   - every float sum is sequential in index order, products are rounded
 *     before they are added (no fused multiply-add), except the fp32 rerank
 *     distance, which restates the reference's AVX-512 arithmetic (16 lane
 *     accumulators with explicit fmaf, then a pairwise tree; l2_f32_rerank);
 *   - every top-k / top-R is a total order on (distance, id) pairs, so ties
 *     are broken by the smaller id (or position) and results are
 *     schedule-independent.
 *
 * Reference files followed (paths inside the reference project):
 *   routing      cuda/search/cpu_fine/ivf_search_cpu_fine.cu:764-1361 (coarse_search)
 *                cuda/search/coarse/fusion_l2_topk_warpsort.cu:127-135 (L2 epilogue,
 *                centroids with norm < 1e-6 are skipped)
 *   exact u8     updates/exact_update.cu:632-666 (fine_search_scalar_touched_u8)
 *                updates/exact_update.cu:465-484 (finalize_topk, (dist, id) order)
 *                updates/exact_update.cu:410-418 (make_query_u8)
 *   residual PQ  cuda/search/cpu_fine/cpu_fine_kernels_pq_resid.cpp:146-213 (LUT, ADC)
 *                cuda/search/cpu_fine/cpu_fine_kernels_pq_resid.cpp:259-525 (stage 1
 *                top-rerank_n, dedup, exact rerank -> top-k)
 *   overlay      updates/pq_update.cu:25, 1045-1055 (main top-512 + delta top-16)
 *                updates/pq_update.cu:496-561 (rerank over main + delta candidates)
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ */
/* bounded max-heap over uint64 keys: keeps the `cap` smallest keys     */
/* ------------------------------------------------------------------ */
typedef struct {
    uint64_t* k;
    int n, cap;
} kheap;

static void kheap_push(kheap* h, uint64_t key) {
    if (h->cap <= 0) return;
    if (h->n < h->cap) {
        int i = h->n++;
        h->k[i] = key;
        while (i > 0) {
            int p = (i - 1) >> 1;
            if (h->k[p] >= h->k[i]) break;
            uint64_t t = h->k[p]; h->k[p] = h->k[i]; h->k[i] = t;
            i = p;
        }
    } else if (key < h->k[0]) {
        h->k[0] = key;
        int i = 0;
        for (;;) {
            int l = 2 * i + 1, r = l + 1, m = i;
            if (l < h->n && h->k[l] > h->k[m]) m = l;
            if (r < h->n && h->k[r] > h->k[m]) m = r;
            if (m == i) break;
            uint64_t t = h->k[m]; h->k[m] = h->k[i]; h->k[i] = t;
            i = m;
        }
    }
}

static int cmp_u64(const void* a, const void* b) {
    uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return (x > y) - (x < y);
}

/* heap contents -> ascending order */
static void kheap_sort(kheap* h) { qsort(h->k, (size_t)h->n, sizeof(uint64_t), cmp_u64); }

static inline uint32_t fbits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bitsf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* (non-negative float distance, unsigned id) -> order-preserving key */
static inline uint64_t fkey(float d, uint32_t id) { return ((uint64_t)fbits(d) << 32) | id; }
static inline uint64_t ikey(int32_t d, uint32_t id) { return ((uint64_t)(uint32_t)d << 32) | id; }

/* ------------------------------------------------------------------ */
/* make_query_u8: clamp to [0,255] and round half away from zero        */
/* (updates/exact_update.cu:410-418)                                    */
/* ------------------------------------------------------------------ */
ORACLE_API void oracle_make_query_u8(const float* q, int64_t n, uint8_t* out) {
    for (int64_t i = 0; i < n; ++i) {
        float x = q[i];
        if (x < 0.0f) x = 0.0f;
        if (x > 255.0f) x = 255.0f;
        out[i] = (uint8_t)lroundf(x);
    }
}

/* ------------------------------------------------------------------ */
/* routing                                                              */
/* ------------------------------------------------------------------ */
/* squared L2 by direct differences, sequential in j, no contraction */
static inline float l2_f32(const float* a, const float* b, int d) {
    float s = 0.0f;
    for (int j = 0; j < d; ++j) {
        float x = a[j] - b[j];
        float p = x * x;
        s = s + p;
    }
    return s;
}

/*
 * A centroid takes part in routing only when its L2 norm is >= 1e-6
 * (fusion_l2_topk_warpsort.cu:131).  valid[c] = 1 for usable centroids.
 */
ORACLE_API void oracle_centroid_valid(const float* cent, int nlist, int d, uint8_t* valid) {
    for (int c = 0; c < nlist; ++c) {
        float s = 0.0f;
        for (int j = 0; j < d; ++j) {
            float p = cent[(size_t)c * d + j] * cent[(size_t)c * d + j];
            s = s + p;
        }
        valid[c] = (sqrtf(s) >= 1e-6f) ? 1 : 0;
    }
}

/*
 * Top-nprobe lists per query by exact fp32 L2 with (dist, list id) order.
 * Slots beyond the number of usable centroids get id -1 and dist +inf.
 */
ORACLE_API int oracle_route_l2(const float* q, int nq, const float* cent, int nlist, int d,
                               int nprobe, int32_t* out_ids, float* out_dist) {
    if (nq < 0 || nlist <= 0 || d <= 0 || nprobe <= 0) return -1;
    uint8_t* valid = (uint8_t*)malloc((size_t)nlist);
    uint64_t* buf = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)nprobe);
    if (!valid || !buf) { free(valid); free(buf); return -2; }
    oracle_centroid_valid(cent, nlist, d, valid);
    for (int qi = 0; qi < nq; ++qi) {
        kheap h = {buf, 0, nprobe};
        const float* qq = q + (size_t)qi * d;
        for (int c = 0; c < nlist; ++c) {
            if (!valid[c]) continue;
            kheap_push(&h, fkey(l2_f32(qq, cent + (size_t)c * d, d), (uint32_t)c));
        }
        kheap_sort(&h);
        for (int p = 0; p < nprobe; ++p) {
            if (p < h.n) {
                out_ids[(size_t)qi * nprobe + p] = (int32_t)(uint32_t)h.k[p];
                if (out_dist) out_dist[(size_t)qi * nprobe + p] = bitsf((uint32_t)(h.k[p] >> 32));
            } else {
                out_ids[(size_t)qi * nprobe + p] = -1;
                if (out_dist) out_dist[(size_t)qi * nprobe + p] = INFINITY;
            }
        }
    }
    free(valid);
    free(buf);
    return 0;
}

/*
 * The reference's own routing formula (cuda/search/cpu_fine/ivf_search_cpu_fine.cu:857-944
 * with cuda/search/coarse/fusion_l2_topk_warpsort.cu:127-135): per query and
 * centroid, dist = -2 * <q, c> + |q| * |q| + |c| * |c|, the norms as
 * sqrtf of the sum of squares (cuda/l2norm/l2norm.cu), evaluated left to right
 * in fp32; centroids with |c| < 1e-6 are skipped.  The reference takes <q, c>
 * from cuBLAS SGEMM, whose summation order is not documented; here it is the
 * sequential fp32 sum, one admissible order.  Used only to measure how often
 * this formula and the direct-difference routing above disagree (near-ties).
 * Top-nprobe by (dist, list id); negative distances (cancellation) order
 * below zero.
 */
static inline uint64_t fkey_signed(float v, uint32_t id) {
    uint32_t b;
    memcpy(&b, &v, 4);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((uint64_t)b << 32) | id;
}

static inline float unfkey_signed(uint32_t b) {
    b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
    float v;
    memcpy(&v, &b, 4);
    return v;
}

ORACLE_API int oracle_route_l2_normexp(const float* q, int nq, const float* cent, int nlist, int d,
                                       int nprobe, int32_t* out_ids, float* out_dist) {
    if (nq < 0 || nlist <= 0 || d <= 0 || nprobe <= 0) return -1;
    float* cn = (float*)malloc(sizeof(float) * (size_t)nlist);
    uint64_t* buf = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)nprobe);
    if (!cn || !buf) { free(cn); free(buf); return -2; }
    for (int c = 0; c < nlist; ++c) {
        float s = 0.0f;
        for (int j = 0; j < d; ++j) {
            float p = cent[(size_t)c * d + j] * cent[(size_t)c * d + j];
            s = s + p;
        }
        cn[c] = sqrtf(s);
    }
    for (int qi = 0; qi < nq; ++qi) {
        kheap h = {buf, 0, nprobe};
        const float* qq = q + (size_t)qi * d;
        float s = 0.0f;
        for (int j = 0; j < d; ++j) {
            float p = qq[j] * qq[j];
            s = s + p;
        }
        const float qn = sqrtf(s);
        for (int c = 0; c < nlist; ++c) {
            if (!(cn[c] >= 1e-6f)) continue;
            const float* cc = cent + (size_t)c * d;
            float ip = 0.0f;
            for (int j = 0; j < d; ++j) {
                float p = qq[j] * cc[j];
                ip = ip + p;
            }
            float t = -2.0f * ip;
            float qq2 = qn * qn;
            float cc2 = cn[c] * cn[c];
            t = t + qq2;
            t = t + cc2;
            kheap_push(&h, fkey_signed(t, (uint32_t)c));
        }
        kheap_sort(&h);
        for (int p = 0; p < nprobe; ++p) {
            if (p < h.n) {
                out_ids[(size_t)qi * nprobe + p] = (int32_t)(uint32_t)h.k[p];
                if (out_dist) out_dist[(size_t)qi * nprobe + p] = unfkey_signed((uint32_t)(h.k[p] >> 32));
            } else {
                out_ids[(size_t)qi * nprobe + p] = -1;
                if (out_dist) out_dist[(size_t)qi * nprobe + p] = INFINITY;
            }
        }
    }
    free(cn);
    free(buf);
    return 0;
}

/*
 * The reference's fp32 pipeline (ivf_load_dataset + ivf_pipeline_stage2_compute,
 * cuda/search/ivf_search_separated.cu:417-650): routing by cosine distance
 * 1 - <q, c> / (|q| |c|) in both distance modes (:477-512,
 * coarse/fusion_cos_topk_warpsort.cu:125-135; centroids below 1e-6 norm are
 * skipped), then an exact scan of the probed lists by L2 (mode 0) or 1 - cosine
 * (mode 1, fine/indexed_gemm_cos.cu:114-116).  Sums in dimension order, norms
 * sqrtf of sequential sums, cosine distances clamped at 0 and 1 for a zero
 * norm; ties by list id (routing) and by row position (scan).
 */
static inline float cos_dist(const float* a, const float* b, int d, float an, float bn) {
    float dot = 0.0f;
    for (int j = 0; j < d; ++j) {
        float p = a[j] * b[j];
        dot = dot + p;
    }
    float den = an * bn;
    if (!(den > 0.0f)) return 1.0f;
    float v = 1.0f - dot / den;
    return v > 0.0f ? v : 0.0f;
}

static inline float norm_f32(const float* a, int d) {
    float s = 0.0f;
    for (int j = 0; j < d; ++j) {
        float p = a[j] * a[j];
        s = s + p;
    }
    return sqrtf(s);
}

ORACLE_API int oracle_f32_search(const float* rows, const int64_t* offsets, const int32_t* counts, int nlist, int d,
                                 const float* cent, const float* q, int nq, int nprobe, int k, int cosine,
                                 int32_t* out_probes, int32_t* out_ids, float* out_dist) {
    if (nq < 0 || nlist <= 0 || d <= 0 || nprobe <= 0 || k <= 0) return -1;
    uint64_t* pb = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)nprobe);
    uint64_t* kb = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)k);
    float* cn = (float*)malloc(sizeof(float) * (size_t)nlist);
    if (!pb || !kb || !cn) { free(pb); free(kb); free(cn); return -2; }
    for (int c = 0; c < nlist; ++c) cn[c] = norm_f32(cent + (size_t)c * d, d);
    for (int qi = 0; qi < nq; ++qi) {
        const float* qq = q + (size_t)qi * d;
        const float qn = norm_f32(qq, d);
        kheap hp = {pb, 0, nprobe};
        for (int c = 0; c < nlist; ++c) {
            if (!(cn[c] >= 1e-6f)) continue;
            kheap_push(&hp, fkey(cos_dist(qq, cent + (size_t)c * d, d, qn, cn[c]), (uint32_t)c));
        }
        kheap_sort(&hp);
        kheap hk = {kb, 0, k};
        for (int p = 0; p < nprobe; ++p) {
            const int l = p < hp.n ? (int)(uint32_t)hp.k[p] : -1;
            out_probes[(size_t)qi * nprobe + p] = l;
            if (l < 0) continue;
            for (int v = 0; v < counts[l]; ++v) {
                const int64_t pos = offsets[l] + v;
                const float* x = rows + (size_t)pos * d;
                float dist;
                if (cosine) {
                    dist = cos_dist(qq, x, d, qn, norm_f32(x, d));
                } else {
                    float s = 0.0f;
                    for (int j = 0; j < d; ++j) {
                        float t = qq[j] - x[j];
                        float p2 = t * t;
                        s = s + p2;
                    }
                    dist = s;
                }
                kheap_push(&hk, fkey(dist, (uint32_t)pos));
            }
        }
        kheap_sort(&hk);
        for (int j = 0; j < k; ++j) {
            if (j < hk.n) {
                out_ids[(size_t)qi * k + j] = (int32_t)(uint32_t)hk.k[j];
                out_dist[(size_t)qi * k + j] = bitsf((uint32_t)(hk.k[j] >> 32));
            } else {
                out_ids[(size_t)qi * k + j] = -1;
                out_dist[(size_t)qi * k + j] = INFINITY;
            }
        }
    }
    free(pb);
    free(kb);
    free(cn);
    return 0;
}

/* ------------------------------------------------------------------ */
/* exact uint8 fine search                                              */
/* ------------------------------------------------------------------ */
static inline int32_t l2_u8(const uint8_t* a, const uint8_t* b, int d) {
    int32_t s = 0;
    for (int j = 0; j < d; ++j) {
        int32_t x = (int32_t)a[j] - (int32_t)b[j];
        s += x * x;
    }
    return s;
}

/*
 * fp32 rerank distance as the reference computes it on AVX-512 hosts
 * (cuda/search/cpu_fine/cpu_fine_kernels_pq_resid.cpp:106-131, l2_sq_fp32):
 * for each full block of 16 dimensions, lane l (0..15) accumulates
 * acc[l] = fma(x, x, acc[l]) with x = q[i + l] - v[i + l] rounded first; the
 * 16 lanes are then summed as a pairwise tree -- lane l with lane l + 8, then
 * + 4, + 2, + 1 -- which is the order of the 512-bit horizontal add it calls
 * (checked bit for bit against that intrinsic, with and without -ffast-math,
 * over 2M random vectors).  Dimensions past the last full block are added
 * sequentially with fma (the reference's scalar tail under contraction; the
 * device library accepts only d % 16 == 0, where there is no tail).
 */
static inline float l2_f32_rerank(const float* q, const float* v, int d) {
    float acc[16];
    for (int l = 0; l < 16; ++l) acc[l] = 0.0f;
    int i = 0;
    for (; i + 16 <= d; i += 16) {
        for (int l = 0; l < 16; ++l) {
            float x = q[i + l] - v[i + l];
            acc[l] = fmaf(x, x, acc[l]);
        }
    }
    for (int w = 8; w >= 1; w >>= 1)
        for (int l = 0; l < w; ++l) acc[l] = acc[l] + acc[l + w];
    float s = acc[0];
    for (; i < d; ++i) {
        float x = q[i] - v[i];
        s = fmaf(x, x, s);
    }
    return s;
}

/*
 * Exact int32 L2 over the probed lists -> top-k by (dist, original id).
 * Probe ids outside [0, nlist) are skipped; a list probed twice contributes
 * its vectors twice (as the reference does); positions with deleted[pos] != 0
 * (deleted may be NULL) are not scanned (exact_update.cu:54, 89).  Output:
 * original ids and int32 distances; empty slots are id -1 / INT32_MAX.
 */
ORACLE_API int oracle_exact_u8(const uint8_t* base_u8, const int64_t* offsets, const int32_t* counts,
                               const int32_t* r2o, int nlist, int d,
                               const uint8_t* q_u8, const int32_t* probes, int nq, int nprobe, int k,
                               const uint8_t* deleted, int32_t* out_ids, int32_t* out_dist) {
    if (k <= 0 || d <= 0) return -1;
    uint64_t* buf = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)k);
    if (!buf) return -2;
    for (int qi = 0; qi < nq; ++qi) {
        kheap h = {buf, 0, k};
        const uint8_t* qq = q_u8 + (size_t)qi * d;
        for (int p = 0; p < nprobe; ++p) {
            int c = probes[(size_t)qi * nprobe + p];
            if (c < 0 || c >= nlist) continue;
            int64_t off = offsets[c];
            for (int32_t v = 0; v < counts[c]; ++v) {
                int64_t pos = off + v;
                if (deleted && deleted[pos]) continue;   /* exact_update.cu:89 */
                int32_t dist = l2_u8(qq, base_u8 + (size_t)pos * d, d);
                uint32_t id = r2o ? (uint32_t)r2o[pos] : (uint32_t)pos;
                kheap_push(&h, ikey(dist, id));
            }
        }
        kheap_sort(&h);
        for (int j = 0; j < k; ++j) {
            if (j < h.n) {
                out_ids[(size_t)qi * k + j] = (int32_t)(uint32_t)h.k[j];
                out_dist[(size_t)qi * k + j] = (int32_t)(uint32_t)(h.k[j] >> 32);
            } else {
                out_ids[(size_t)qi * k + j] = -1;
                out_dist[(size_t)qi * k + j] = INT32_MAX;
            }
        }
    }
    free(buf);
    return 0;
}

/* ------------------------------------------------------------------ */
/* residual PQ                                                          */
/* ------------------------------------------------------------------ */
/*
 * LUT[m][c] = sum_j ((q_j - cent_j) - cb[m][c][j])^2 for the j of sub-space m,
 * in j order (cpu_fine_kernels_pq_resid.cpp:176-189, pq_update.cu:130-134).
 */
ORACLE_API void oracle_pq_lut(const float* q, const float* centroid, const float* codebook,
                              int M, int K, int dsub, float* lut) {
    for (int m = 0; m < M; ++m) {
        for (int c = 0; c < K; ++c) {
            const float* cb = codebook + ((size_t)m * K + c) * dsub;
            float s = 0.0f;
            for (int j = 0; j < dsub; ++j) {
                float r = q[m * dsub + j] - centroid[m * dsub + j];
                float x = r - cb[j];
                float p = x * x;
                s = s + p;
            }
            lut[(size_t)m * K + c] = s;
        }
    }
}

/* ADC distance: sum over m in order (cpu_fine_kernels_pq_resid.cpp:200-213) */
static inline float pq_adc(const float* lut, const uint8_t* code, int M, int K) {
    float s = 0.0f;
    for (int m = 0; m < M; ++m) s = s + lut[(size_t)m * K + code[m]];
    return s;
}

ORACLE_API float oracle_pq_adc(const float* lut, const uint8_t* code, int M, int K) {
    return pq_adc(lut, code, M, K);
}

/* one inverted-list segment (main index or a published delta) */
typedef struct {
    const uint8_t* codes;    /* [n, M] cluster-major */
    const int64_t* offsets;  /* [nlist] */
    const int32_t* counts;   /* [nlist] */
    const int32_t* ids;      /* [n] final id of each position (NULL: id = position) */
    const uint8_t* raw_u8;   /* [n, d] rerank vectors by position (u8 rerank) */
    const float* raw_f32;    /* [n, d] rerank vectors by position (fp32 rerank) */
} pq_segment;

/*
 * Stage 1 for one query over one segment: every vector of every probed list
 * gets its ADC distance; the R smallest (ADC, position) keys are kept.
 */
static void pq_stage1(const pq_segment* s, const float* q, const float* cent, int nlist, int d,
                      const float* codebook, int M, int K, int dsub, const int32_t* probes, int nprobe,
                      float* lut, kheap* h) {
    for (int p = 0; p < nprobe; ++p) {
        int c = probes[p];
        if (c < 0 || c >= nlist) continue;
        int32_t cnt = s->counts[c];
        if (cnt <= 0) continue;
        oracle_pq_lut(q, cent + (size_t)c * d, codebook, M, K, dsub, lut);
        int64_t off = s->offsets[c];
        for (int32_t v = 0; v < cnt; ++v) {
            int64_t pos = off + v;
            float a = pq_adc(lut, s->codes + (size_t)pos * M, M, K);
            kheap_push(h, fkey(a, (uint32_t)pos));
        }
    }
}

/*
 * Residual-PQ search with optional delta overlay.
 *
 *  stage 1: main top-rerank_n by (ADC, position); delta top-delta_topk by
 *           (ADC, delta position) when a delta segment is given;
 *  stage 2: unique candidates reranked exactly -- int32 L2 on u8 vectors
 *           (query = make_query_u8(q)) or fp32 L2 (l2_f32_rerank) -- and the top-k
 *           kept by (exact distance, final id); main positions with
 *           deleted[pos] != 0 (deleted may be NULL) keep their stage-1 slots
 *           but are not reranked.
 *
 * Final ids: main -> r2o[position] (or position), delta -> delta ids[position].
 * Outputs: out_ids/out_dist [nq, k] (empty slots -1 / +inf); optionally the
 * sorted stage-1 keys [nq, rerank_n] and [nq, delta_topk] (empty = ~0).
 */
ORACLE_API int oracle_pq_search(
    const float* cent, int nlist, int d,
    const float* codebook, int M, int K, int dsub,
    const uint8_t* codes, const int64_t* offsets, const int32_t* counts, const int32_t* r2o,
    const uint8_t* base_u8, const float* base_f32, int use_f32_rerank,
    const uint8_t* dcodes, const int64_t* doffsets, const int32_t* dcounts, const int32_t* dids,
    const uint8_t* draw_u8, const float* draw_f32, int delta_topk,
    const float* q, int nq, const int32_t* probes, int nprobe, int rerank_n, int k, const uint8_t* deleted,
    int32_t* out_ids, float* out_dist, uint64_t* out_stage1, uint64_t* out_delta1) {
    if (M <= 0 || K <= 0 || K > 256 || dsub <= 0 || M * dsub != d || k <= 0) return -1;
    if (rerank_n < k) rerank_n = k;
    const int use_delta = (dcodes && doffsets && dcounts && delta_topk > 0);
    pq_segment main_seg = {codes, offsets, counts, r2o, base_u8, base_f32};
    pq_segment delta_seg = {dcodes, doffsets, dcounts, dids, draw_u8, draw_f32};
    float* lut = (float*)malloc(sizeof(float) * (size_t)M * K);
    uint64_t* h1 = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)rerank_n);
    uint64_t* hd = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(delta_topk > 0 ? delta_topk : 1));
    uint64_t* hk = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)k);
    uint8_t* qu8 = (uint8_t*)malloc((size_t)d);
    if (!lut || !h1 || !hd || !hk || !qu8) {
        free(lut); free(h1); free(hd); free(hk); free(qu8);
        return -2;
    }
    for (int qi = 0; qi < nq; ++qi) {
        const float* qq = q + (size_t)qi * d;
        const int32_t* pr = probes + (size_t)qi * nprobe;
        kheap H1 = {h1, 0, rerank_n};
        pq_stage1(&main_seg, qq, cent, nlist, d, codebook, M, K, dsub, pr, nprobe, lut, &H1);
        kheap_sort(&H1);
        kheap HD = {hd, 0, use_delta ? delta_topk : 0};
        if (use_delta) {
            pq_stage1(&delta_seg, qq, cent, nlist, d, codebook, M, K, dsub, pr, nprobe, lut, &HD);
            kheap_sort(&HD);
        }
        if (out_stage1)
            for (int j = 0; j < rerank_n; ++j)
                out_stage1[(size_t)qi * rerank_n + j] = j < H1.n ? h1[j] : ~(uint64_t)0;
        if (out_delta1 && delta_topk > 0)
            for (int j = 0; j < delta_topk; ++j)
                out_delta1[(size_t)qi * delta_topk + j] = j < HD.n ? hd[j] : ~(uint64_t)0;

        oracle_make_query_u8(qq, d, qu8);
        kheap HK = {hk, 0, k};
        for (int seg = 0; seg < 2; ++seg) {
            const pq_segment* s = seg == 0 ? &main_seg : &delta_seg;
            const kheap* S = seg == 0 ? &H1 : &HD;
            for (int j = 0; j < S->n; ++j) {
                uint32_t pos = (uint32_t)S->k[j];
                /* sorted keys: a repeated position (list probed twice) is adjacent */
                if (j > 0 && (uint32_t)S->k[j - 1] == pos) continue;
                /* deleted main positions stay in stage 1 but are not reranked
                 * (pq_update.cu:503-523) */
                if (seg == 0 && deleted && deleted[pos]) continue;
                uint32_t id = s->ids ? (uint32_t)s->ids[pos] : pos;
                float e;
                if (use_f32_rerank) {
                    e = l2_f32_rerank(qq, s->raw_f32 + (size_t)pos * d, d);
                } else {
                    e = (float)l2_u8(qu8, s->raw_u8 + (size_t)pos * d, d);
                }
                kheap_push(&HK, fkey(e, id));
            }
        }
        kheap_sort(&HK);
        for (int j = 0; j < k; ++j) {
            if (j < HK.n) {
                out_ids[(size_t)qi * k + j] = (int32_t)(uint32_t)HK.k[j];
                out_dist[(size_t)qi * k + j] = bitsf((uint32_t)(HK.k[j] >> 32));
            } else {
                out_ids[(size_t)qi * k + j] = -1;
                out_dist[(size_t)qi * k + j] = INFINITY;
            }
        }
    }
    free(lut); free(h1); free(hd); free(hk); free(qu8);
    return 0;
}

/* ------------------------------------------------------------------ */
/* layout helpers                                                       */
/* ------------------------------------------------------------------ */
/*
 * Stable cluster-major reorder (dataset.cuh:559-592, train_ivfpq_residual.py:138-148):
 * counts[c], offsets[c] (exclusive prefix) and r2o[pos] = original id, with
 * positions inside a list increasing with the original id.
 */
ORACLE_API void oracle_reorder(const int32_t* assign, int64_t n, int nlist,
                               int32_t* counts, int64_t* offsets, int32_t* r2o) {
    memset(counts, 0, sizeof(int32_t) * (size_t)nlist);
    for (int64_t i = 0; i < n; ++i) counts[assign[i]]++;
    int64_t acc = 0;
    for (int c = 0; c < nlist; ++c) { offsets[c] = acc; acc += counts[c]; }
    int64_t* next = (int64_t*)malloc(sizeof(int64_t) * (size_t)nlist);
    memcpy(next, offsets, sizeof(int64_t) * (size_t)nlist);
    for (int64_t i = 0; i < n; ++i) r2o[next[assign[i]]++] = (int32_t)i;
    free(next);
}

/* recall@k as updates/io.h:151-168 (hits of the first k ids among the first k GT ids) */
ORACLE_API double oracle_recall_at_k(const int32_t* ids, const int32_t* gt, int nq, int k,
                                     int ids_row, int gt_row) {
    if (k > ids_row) k = ids_row;
    if (k > gt_row) k = gt_row;
    long long hit = 0, total = (long long)nq * k;
    for (int q = 0; q < nq; ++q)
        for (int i = 0; i < k; ++i) {
            int c = ids[(size_t)q * ids_row + i];
            for (int j = 0; j < k; ++j)
                if (c == gt[(size_t)q * gt_row + j]) { ++hit; break; }
        }
    return total > 0 ? (double)hit / (double)total : 0.0;
}
