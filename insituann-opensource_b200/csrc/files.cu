// files.cu -- readers and writers of the reference's index file formats, and a
// loader that builds a residual-PQ index straight from them.
//
//   centroids  [nlist:i32][dim:i32][f32 nlist*dim]          updates/pq_update.cu:46
//   assign     [n:i64][i32 n]                               updates/pq_update.cu:47
//   codebook   [M:i32][K:i32][dsub:i32][pad:i32][f32 M*K*dsub]   scripts/train_ivfpq_residual.py:209-213
//              (dsub = -1, pad = 1 marks the variable-subdims variant, :231-233, not served here)
//   codes      [n:i64][M:i32][pad:i32][u8 n*M], cluster-major     scripts/train_ivfpq_residual.py:304-307
//   u8bin/fbin [n:i32][d:i32][u8|f32 n*d]  (DiskANN)              updates/io.h:183-294
//   gt         [n:i32][k:i32][i32 n*k] (+ an optional f32 distance block)   scripts/gen_gt_fast.py:34-38
//
// Host code only.  Every reader returns the element count of the payload;
// with out == NULL it reads only the header (sizes), otherwise out must hold
// cap >= that many elements.  Errors return -1 with the message in
// ivf_global_last_error().
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/insitu_b200.h"

namespace isb {
void set_global_error(const std::string& msg);
}

namespace {

struct File {
    FILE* f = nullptr;
    explicit File(const char* path, const char* mode) : f(path ? std::fopen(path, mode) : nullptr) {}
    ~File() {
        if (f) std::fclose(f);
    }
};

long long fail(const std::string& msg) {
    isb::set_global_error(msg);
    return -1;
}

template <class T>
bool get(FILE* f, T* v, size_t n = 1) {
    return std::fread(v, sizeof(T), n, f) == n;
}

template <class T>
bool put(FILE* f, const T* v, size_t n = 1) {
    return std::fwrite(v, sizeof(T), n, f) == n;
}

// reads `count` elements of T when out is given (cap checked); returns count or -1
template <class T>
long long payload(FILE* f, const char* path, T* out, long long cap, long long count) {
    if (count < 0) return fail(std::string(path) + ": negative size in the header");
    if (!out) return count;
    if (cap < count) return fail(std::string(path) + ": output buffer holds fewer elements than the file");
    if (count && !get(f, out, (size_t)count)) return fail(std::string(path) + ": file shorter than its header says");
    return count;
}

}  // namespace

extern "C" {

long long ivf_read_centroids(const char* path, float* out, long long cap, int* nlist, int* dim) {
    File fl(path, "rb");
    if (!fl.f) return fail(std::string("cannot open ") + (path ? path : "(null)"));
    int32_t nl = 0, d = 0;
    if (!get(fl.f, &nl) || !get(fl.f, &d)) return fail(std::string(path) + ": short header");
    if (nlist) *nlist = nl;
    if (dim) *dim = d;
    return payload(fl.f, path, out, cap, (long long)nl * d);
}

long long ivf_read_assign(const char* path, int* out, long long cap, long long* n) {
    File fl(path, "rb");
    if (!fl.f) return fail(std::string("cannot open ") + (path ? path : "(null)"));
    int64_t nn = 0;
    if (!get(fl.f, &nn)) return fail(std::string(path) + ": short header");
    if (n) *n = nn;
    return payload(fl.f, path, out, cap, (long long)nn);
}

long long ivf_read_codebook(const char* path, float* out, long long cap, int* M, int* K, int* dsub) {
    File fl(path, "rb");
    if (!fl.f) return fail(std::string("cannot open ") + (path ? path : "(null)"));
    int32_t h[4];
    if (!get(fl.f, h, 4)) return fail(std::string(path) + ": short header");
    if (h[2] <= 0) return fail(std::string(path) + ": variable-subdims codebooks (dsub = -1) are not served");
    if (M) *M = h[0];
    if (K) *K = h[1];
    if (dsub) *dsub = h[2];
    return payload(fl.f, path, out, cap, (long long)h[0] * h[1] * h[2]);
}

long long ivf_read_codes(const char* path, unsigned char* out, long long cap, long long* n, int* M) {
    File fl(path, "rb");
    if (!fl.f) return fail(std::string("cannot open ") + (path ? path : "(null)"));
    int64_t nn = 0;
    int32_t m = 0, pad = 0;
    if (!get(fl.f, &nn) || !get(fl.f, &m) || !get(fl.f, &pad)) return fail(std::string(path) + ": short header");
    if (n) *n = nn;
    if (M) *M = m;
    return payload(fl.f, path, out, cap, (long long)nn * m);
}

long long ivf_read_u8bin(const char* path, unsigned char* out, long long cap, long long* n, int* d) {
    File fl(path, "rb");
    if (!fl.f) return fail(std::string("cannot open ") + (path ? path : "(null)"));
    int32_t nn = 0, dd = 0;
    if (!get(fl.f, &nn) || !get(fl.f, &dd)) return fail(std::string(path) + ": short header");
    if (n) *n = nn;
    if (d) *d = dd;
    return payload(fl.f, path, out, cap, (long long)nn * dd);
}

long long ivf_read_fbin(const char* path, float* out, long long cap, long long* n, int* d) {
    File fl(path, "rb");
    if (!fl.f) return fail(std::string("cannot open ") + (path ? path : "(null)"));
    int32_t nn = 0, dd = 0;
    if (!get(fl.f, &nn) || !get(fl.f, &dd)) return fail(std::string(path) + ": short header");
    if (n) *n = nn;
    if (d) *d = dd;
    return payload(fl.f, path, out, cap, (long long)nn * dd);
}

long long ivf_read_gt(const char* path, int* out, long long cap, long long* n, int* k) {
    File fl(path, "rb");
    if (!fl.f) return fail(std::string("cannot open ") + (path ? path : "(null)"));
    int32_t nn = 0, kk = 0;
    if (!get(fl.f, &nn) || !get(fl.f, &kk)) return fail(std::string(path) + ": short header");
    if (n) *n = nn;
    if (k) *k = kk;
    return payload(fl.f, path, out, cap, (long long)nn * kk);     // a trailing distance block is not read
}

int ivf_write_centroids(const char* path, const float* cent, int nlist, int dim) {
    File fl(path, "wb");
    const int32_t h[2] = {nlist, dim};
    if (!fl.f || !put(fl.f, h, 2) || !put(fl.f, cent, (size_t)nlist * dim))
        return (int)fail(std::string("cannot write ") + (path ? path : "(null)"));
    return IVF_OK;
}

int ivf_write_assign(const char* path, const int* assign, long long n) {
    File fl(path, "wb");
    const int64_t nn = n;
    if (!fl.f || !put(fl.f, &nn) || !put(fl.f, assign, (size_t)n))
        return (int)fail(std::string("cannot write ") + (path ? path : "(null)"));
    return IVF_OK;
}

int ivf_write_codebook(const char* path, const float* codebook, int M, int K, int dsub) {
    File fl(path, "wb");
    const int32_t h[4] = {M, K, dsub, 0};
    if (!fl.f || !put(fl.f, h, 4) || !put(fl.f, codebook, (size_t)M * K * dsub))
        return (int)fail(std::string("cannot write ") + (path ? path : "(null)"));
    return IVF_OK;
}

int ivf_write_codes(const char* path, const unsigned char* codes, long long n, int M) {
    File fl(path, "wb");
    const int64_t nn = n;
    const int32_t h[2] = {M, 0};
    if (!fl.f || !put(fl.f, &nn) || !put(fl.f, h, 2) || !put(fl.f, codes, (size_t)n * M))
        return (int)fail(std::string("cannot write ") + (path ? path : "(null)"));
    return IVF_OK;
}

int ivf_pq_load_files(void* idx_ctx, const char* centroids_path, const char* codebook_path, const char* codes_path,
                      const char* assign_path, const char* base_u8bin_path) {
    int nlist = 0, dim = 0, M = 0, K = 0, dsub = 0, bd = 0, Mc = 0;
    long long n = 0, nc = 0, nb = 0;
    if (ivf_read_centroids(centroids_path, nullptr, 0, &nlist, &dim) < 0 ||
        ivf_read_codebook(codebook_path, nullptr, 0, &M, &K, &dsub) < 0 ||
        ivf_read_codes(codes_path, nullptr, 0, &nc, &Mc) < 0 || ivf_read_assign(assign_path, nullptr, 0, &n) < 0 ||
        ivf_read_u8bin(base_u8bin_path, nullptr, 0, &nb, &bd) < 0)
        return IVF_EINVAL;
    if (nc != n || nb != n || Mc != M || bd != dim || M * dsub != dim || nlist <= 0) {
        fail("index files disagree on n, M or dim");
        return IVF_EINVAL;
    }
    std::vector<float> cent((size_t)nlist * dim), cb((size_t)M * K * dsub);
    std::vector<int> assign((size_t)n);
    std::vector<unsigned char> codes((size_t)n * M), base((size_t)n * dim);
    if (ivf_read_centroids(centroids_path, cent.data(), (long long)cent.size(), &nlist, &dim) < 0 ||
        ivf_read_codebook(codebook_path, cb.data(), (long long)cb.size(), &M, &K, &dsub) < 0 ||
        ivf_read_codes(codes_path, codes.data(), (long long)codes.size(), &nc, &Mc) < 0 ||
        ivf_read_assign(assign_path, assign.data(), n, &n) < 0 ||
        ivf_read_u8bin(base_u8bin_path, base.data(), (long long)base.size(), &nb, &bd) < 0)
        return IVF_EINVAL;
    // stable cluster-major layout of the assignment (dataset.cuh:559-592); the
    // codes file is already in this order (train_ivfpq_residual.py:293-307),
    // the base rows are in original order and are gathered here
    std::vector<int> counts((size_t)nlist, 0), r2o((size_t)n);
    std::vector<long long> offsets((size_t)nlist, 0);
    for (long long i = 0; i < n; ++i) {
        if (assign[i] < 0 || assign[i] >= nlist) {
            fail("assignment outside [0, nlist)");
            return IVF_EINVAL;
        }
        counts[assign[i]]++;
    }
    for (int l = 1; l < nlist; ++l) offsets[l] = offsets[l - 1] + counts[l - 1];
    std::vector<long long> cur(offsets);
    for (long long i = 0; i < n; ++i) r2o[(size_t)cur[assign[i]]++] = (int)i;
    std::vector<unsigned char> base_cm((size_t)n * dim);
    for (long long p = 0; p < n; ++p) std::memcpy(&base_cm[(size_t)p * dim], &base[(size_t)r2o[p] * dim], dim);
    return ivf_pq_load(idx_ctx, cent.data(), cb.data(), M, K, dsub, codes.data(), offsets.data(), counts.data(),
                       r2o.data(), base_cm.data(), nullptr, nlist, n, dim);
}

}  // extern "C"
