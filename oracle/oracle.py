"""ctypes bindings for the CPU checker libraries (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module.  It exposes
  * the C restatement in oracle/oracle.c (``liboracle.so``), and
  * the reference's own CPU kernels compiled unmodified into
    ``oracle/_ref/libref_cpu_fine*.so`` (``ref_*`` functions), when present.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def ref_root() -> str:
    """The reference checkout: $REF_ROOT, else `reference` beside this repository's checkout."""
    return os.environ.get("REF_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
_LIB = None
_REF = None

u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
u64p = np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")


def build(ref: bool = False) -> None:
    """Compile liboracle.so (and, when the reference tree exists, the reference kernels)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref and os.path.isdir(ref_root()):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF_ROOT={ref_root()}"], check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.oracle_make_query_u8.argtypes = [f32p, C.c_int64, u8p]
        L.oracle_centroid_valid.argtypes = [f32p, C.c_int, C.c_int, u8p]
        L.oracle_route_l2.argtypes = [f32p, C.c_int, f32p, C.c_int, C.c_int, C.c_int, i32p, f32p]
        L.oracle_route_l2.restype = C.c_int
        L.oracle_route_l2_normexp.argtypes = [f32p, C.c_int, f32p, C.c_int, C.c_int, C.c_int, i32p, f32p]
        L.oracle_f32_search.argtypes = [f32p, i64p, i32p, C.c_int, C.c_int, f32p, f32p, C.c_int, C.c_int,
                                        C.c_int, C.c_int, i32p, i32p, f32p]
        L.oracle_f32_search.restype = C.c_int
        L.oracle_route_l2_normexp.restype = C.c_int
        L.oracle_exact_u8.argtypes = [u8p, i64p, i32p, C.c_void_p, C.c_int, C.c_int,
                                      u8p, i32p, C.c_int, C.c_int, C.c_int, C.c_void_p, i32p, i32p]
        L.oracle_exact_u8.restype = C.c_int
        L.oracle_pq_lut.argtypes = [f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, f32p]
        L.oracle_pq_adc.argtypes = [f32p, u8p, C.c_int, C.c_int]
        L.oracle_pq_adc.restype = C.c_float
        vp = C.c_void_p
        L.oracle_pq_search.argtypes = [
            f32p, C.c_int, C.c_int,
            f32p, C.c_int, C.c_int, C.c_int,
            u8p, i64p, i32p, vp,
            vp, vp, C.c_int,
            vp, vp, vp, vp, vp, vp, C.c_int,
            f32p, C.c_int, i32p, C.c_int, C.c_int, C.c_int, vp,
            i32p, f32p, vp, vp]
        L.oracle_pq_search.restype = C.c_int
        L.oracle_reorder.argtypes = [i32p, C.c_int64, C.c_int, i32p, i64p, i32p]
        L.oracle_recall_at_k.argtypes = [i32p, i32p, C.c_int, C.c_int, C.c_int, C.c_int]
        L.oracle_recall_at_k.restype = C.c_double
        _LIB = L
    return _LIB


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dt):
    return None if a is None else np.ascontiguousarray(a, dtype=dt)


# ----------------------------------------------------------------------------
# restatement
# ----------------------------------------------------------------------------
def make_query_u8(q: np.ndarray) -> np.ndarray:
    q = _c(q, np.float32)
    out = np.empty(q.shape, dtype=np.uint8)
    lib().oracle_make_query_u8(q.reshape(-1), q.size, out.reshape(-1))
    return out


def centroid_valid(cent: np.ndarray) -> np.ndarray:
    cent = _c(cent, np.float32)
    out = np.empty(cent.shape[0], dtype=np.uint8)
    lib().oracle_centroid_valid(cent, cent.shape[0], cent.shape[1], out)
    return out


def route_l2(q, cent, nprobe):
    q = _c(q, np.float32)
    cent = _c(cent, np.float32)
    nq, d = q.shape
    ids = np.empty((nq, nprobe), np.int32)
    dist = np.empty((nq, nprobe), np.float32)
    rc = lib().oracle_route_l2(q, nq, cent, cent.shape[0], d, nprobe, ids, dist)
    assert rc == 0, rc
    return ids, dist


def exact_u8(base_u8, offsets, counts, r2o, q_u8, probes, k, deleted=None):
    """Exact uint8 search; ``deleted`` [n] (per cluster-major position, nonzero = deleted) or None."""
    base_u8 = _c(base_u8, np.uint8)
    deleted = _c(deleted, np.uint8)
    offsets = _c(offsets, np.int64)
    counts = _c(counts, np.int32)
    r2o = _c(r2o, np.int32)
    q_u8 = _c(q_u8, np.uint8)
    probes = _c(probes, np.int32)
    nq, nprobe = probes.shape
    ids = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.int32)
    rc = lib().oracle_exact_u8(base_u8, offsets, counts, _ptr(r2o), counts.shape[0], base_u8.shape[1],
                               q_u8, probes, nq, nprobe, k, _ptr(deleted), ids, dist)
    assert rc == 0, rc
    return ids, dist


def pq_lut(q, centroid, codebook):
    q = _c(q, np.float32)
    centroid = _c(centroid, np.float32)
    codebook = _c(codebook, np.float32)
    M, K, dsub = codebook.shape
    out = np.empty((M, K), np.float32)
    lib().oracle_pq_lut(q, centroid, codebook, M, K, dsub, out)
    return out


def pq_search(cent, codebook, codes, offsets, counts, r2o, q, probes, k, rerank_n=512,
              base_u8=None, base_f32=None, delta=None, delta_topk=16, return_stage1=False, deleted=None):
    """Residual-PQ search; ``delta`` is a dict with codes/offsets/counts/ids/raw_u8|raw_f32;
    ``deleted`` [n] (per main position, nonzero = not reranked) or None."""
    deleted = _c(deleted, np.uint8)
    cent = _c(cent, np.float32)
    codebook = _c(codebook, np.float32)
    codes = _c(codes, np.uint8)
    offsets = _c(offsets, np.int64)
    counts = _c(counts, np.int32)
    r2o = _c(r2o, np.int32)
    q = _c(q, np.float32)
    probes = _c(probes, np.int32)
    base_u8 = _c(base_u8, np.uint8)
    base_f32 = _c(base_f32, np.float32)
    M, K, dsub = codebook.shape
    nq, nprobe = probes.shape
    d = q.shape[1]
    use_f32 = 1 if base_f32 is not None else 0
    ids = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.float32)
    s1 = np.empty((nq, max(rerank_n, k)), np.uint64) if return_stage1 else None
    dt = 0
    dargs = [None] * 6
    keep = []
    if delta is not None:
        dt = delta_topk
        dc = [_c(delta["codes"], np.uint8), _c(delta["offsets"], np.int64), _c(delta["counts"], np.int32),
              _c(delta.get("ids"), np.int32), _c(delta.get("raw_u8"), np.uint8),
              _c(delta.get("raw_f32"), np.float32)]
        keep = dc
        dargs = [_ptr(a) for a in dc]
    sd = np.empty((nq, max(dt, 1)), np.uint64) if (return_stage1 and dt) else None
    rc = lib().oracle_pq_search(cent, cent.shape[0], d, codebook, M, K, dsub, codes, offsets, counts,
                                _ptr(r2o), _ptr(base_u8), _ptr(base_f32), use_f32,
                                *dargs, dt, q, nq, probes, nprobe, rerank_n, k, _ptr(deleted), ids, dist,
                                _ptr(s1), _ptr(sd))
    del keep
    assert rc == 0, rc
    if return_stage1:
        return ids, dist, s1, sd
    return ids, dist


def f32_search(rows, offsets, counts, cent, q, nprobe, k, cosine=False):
    """The reference's fp32 pipeline restated: cosine routing, exact L2 / cosine
    scan; returns (probes, ids = row positions, distances)."""
    rows, cent, q = _c(rows, np.float32), _c(cent, np.float32), _c(q, np.float32)
    offsets, counts = _c(offsets, np.int64), _c(counts, np.int32)
    nq, d = q.shape
    probes = np.empty((nq, nprobe), np.int32)
    ids = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.float32)
    rc = lib().oracle_f32_search(rows, offsets, counts, counts.shape[0], d, cent, q, nq, nprobe, k,
                                 1 if cosine else 0, probes, ids, dist)
    assert rc == 0, rc
    return probes, ids, dist


def route_l2_normexp(q, cent, nprobe, threads=0):
    """Routing by the reference's formula -2 q.c + |q|^2 + |c|^2 (fp32, norms
    through sqrtf), over query slices on host threads; see oracle.c."""
    from concurrent.futures import ThreadPoolExecutor

    q = _c(q, np.float32)
    cent = _c(cent, np.float32)

    def one(r):
        qs = np.ascontiguousarray(q[r[0]:r[1]])
        ids = np.empty((qs.shape[0], nprobe), np.int32)
        dist = np.empty((qs.shape[0], nprobe), np.float32)
        rc = lib().oracle_route_l2_normexp(qs, qs.shape[0], cent, cent.shape[0], q.shape[1], nprobe, ids, dist)
        assert rc == 0, rc
        return ids, dist
    parts = _split_queries(q.shape[0], threads)
    with ThreadPoolExecutor(len(parts)) as ex:
        res = list(ex.map(one, parts))
    return np.concatenate([a for a, _ in res]), np.concatenate([b for _, b in res])


def route_disagreement(q, cent, ours, theirs, d_bound_factor=None):
    """Compares two top-nprobe probe tables of the same queries.

    Returns (n_queries_differing, max_gap_ratio): for every query whose sets
    differ, every list only in `theirs` must not be farther (exact fp64
    distance) than our nprobe-th list by more than B, and every list only in
    `ours` not nearer than it by more than B, with
    B = 2 (2 d + 10) 2^-24 (|q|^2 + max |c|^2), the rounding bound of an fp32
    evaluation of -2 q.c + |q|^2 + |c|^2 in any summation order;
    max_gap_ratio is the largest such excess over B seen (<= 1 when every
    disagreement is a rounding-level near-tie)."""
    q = np.asarray(q, np.float64)
    cent = np.asarray(cent, np.float64)
    d = q.shape[1]
    f = d_bound_factor if d_bound_factor is not None else 2.0 * (2 * d + 10) * 2.0 ** -24
    cmax = float((cent * cent).sum(1).max())
    n_diff, worst = 0, 0.0
    for i in range(q.shape[0]):
        a, b = set(ours[i][ours[i] >= 0].tolist()), set(theirs[i][theirs[i] >= 0].tolist())
        if a == b:
            continue
        n_diff += 1
        ids = np.array(sorted(a | b))
        dd = ((cent[ids] - q[i]) ** 2).sum(1)
        dist = dict(zip(ids.tolist(), dd.tolist()))
        T = max(dist[x] for x in a)
        B = f * (float((q[i] * q[i]).sum()) + cmax)
        for x in b - a:
            worst = max(worst, (dist[x] - T) / B)
        for x in a - b:
            worst = max(worst, (T - dist[x]) / B if dist[x] < T else 0.0)
    return n_diff, worst


def _split_queries(nq, threads):
    threads = max(1, min(threads or (os.cpu_count() or 1), nq))
    step = (nq + threads - 1) // threads
    return [(s, min(nq, s + step)) for s in range(0, nq, step)]


def route_l2_par(q, cent, nprobe, threads=0):
    """route_l2 over query slices on host threads (the C calls release the GIL)."""
    from concurrent.futures import ThreadPoolExecutor

    q = _c(q, np.float32)
    cent = _c(cent, np.float32)
    parts = _split_queries(q.shape[0], threads)
    with ThreadPoolExecutor(len(parts)) as ex:
        res = list(ex.map(lambda r: route_l2(q[r[0]:r[1]], cent, nprobe), parts))
    return np.concatenate([a for a, _ in res]), np.concatenate([b for _, b in res])


def pq_search_par(cent, codebook, codes, offsets, counts, r2o, q, probes, k, threads=0, **kw):
    """pq_search over query slices on host threads (results are per query, so equal to one call)."""
    from concurrent.futures import ThreadPoolExecutor

    parts = _split_queries(q.shape[0], threads)
    with ThreadPoolExecutor(len(parts)) as ex:
        res = list(ex.map(lambda r: pq_search(cent, codebook, codes, offsets, counts, r2o, q[r[0]:r[1]],
                                              probes[r[0]:r[1]], k, **kw), parts))
    return tuple(None if res[0][i] is None else np.concatenate([x[i] for x in res]) for i in range(len(res[0])))


def reorder(assign, nlist):
    assign = _c(assign, np.int32)
    n = assign.shape[0]
    counts = np.empty(nlist, np.int32)
    offsets = np.empty(nlist, np.int64)
    r2o = np.empty(n, np.int32)
    lib().oracle_reorder(assign, n, nlist, counts, offsets, r2o)
    return counts, offsets, r2o


def recall_at_k(ids, gt, k):
    ids = _c(ids, np.int32)
    gt = _c(gt, np.int32)
    return float(lib().oracle_recall_at_k(ids, gt, ids.shape[0], k, ids.shape[1], gt.shape[1]))


# ----------------------------------------------------------------------------
# the reference's own CPU kernels (oracle/_ref)
# ----------------------------------------------------------------------------
def _cpu_has_avx512bw() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
        return " avx512bw" in flags and " avx512f" in flags
    except OSError:
        return False


_REF_STOCK = None


def ref_lib(stock=False):
    """The reference's CPU kernels, or None when oracle/_ref was not built.

    stock=False: the build without -ffast-math that pins the oracle;
    stock=True: the reference's own flags (-O3 -ffast-math -funroll-loops,
    AVX-512), the timed baseline (AVX-512 hosts; else the first build)."""
    global _REF, _REF_STOCK
    if stock:
        if _REF_STOCK is None:
            path = os.path.join(HERE, "_ref", "libref_cpu_fine_stock.so")
            if not (_cpu_has_avx512bw() and os.path.exists(path)):
                return ref_lib(False)
            _REF_STOCK = _bind_ref(C.CDLL(path), path)
        return _REF_STOCK
    if _REF is None:
        name = "libref_cpu_fine.so" if _cpu_has_avx512bw() else "libref_cpu_fine_avx2.so"
        path = os.path.join(HERE, "_ref", name)
        if not os.path.exists(path):
            return None
        _REF = _bind_ref(C.CDLL(path), path)
    return _REF


def _bind_ref(L, path):
    if True:
        L.ref_cpu_fine_kernel_v3_u8_touched.argtypes = [
            u8p, i64p, i32p, u8p, i32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, i32p, f32p]
        L.ref_cpu_fine_kernel_v3_u8_touched.restype = C.c_longlong
        vp = C.c_void_p
        L.ref_cpu_fine_kernel_pq_resid.argtypes = [
            vp, i64p, i32p, u8p, f32p, f32p, vp, f32p, vp, C.c_int, i32p,
            C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
            i32p, f32p, C.POINTER(C.c_double), C.POINTER(C.c_double)]
        L.ref_cpu_fine_kernel_pq_resid.restype = C.c_longlong
        L.library_path = path
    return L


_REF_COARSE = None


def ref_coarse_lib():
    """The reference's GPU coarse_search (oracle/_ref/libref_coarse.so, built by
    `make ref-coarse`), or None when it was not built.  Needs a CUDA device."""
    global _REF_COARSE
    if _REF_COARSE is None:
        path = os.path.join(HERE, "_ref", "libref_coarse.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        L.ref_coarse_search.argtypes = [f32p, C.c_int, C.c_int, f32p, C.c_int, C.c_int, i32p]
        L.ref_coarse_search.restype = C.c_int
        _REF_COARSE = L
    return _REF_COARSE


def ref_coarse_search(cent, q_f32, nprobe):
    """Probe lists [nq, nprobe] of the reference's own coarse_search
    (cuda/search/cpu_fine/ivf_search_cpu_fine.cu:764-1361: norms, cuBLAS SGEMM
    ||q||^2 + ||c||^2 - 2 q.c, warp-sort top-nprobe) run on the GPU."""
    L = ref_coarse_lib()
    assert L is not None, "oracle/_ref/libref_coarse.so not built"
    cent = _c(cent, np.float32)
    q_f32 = _c(q_f32, np.float32)
    ids = np.full((q_f32.shape[0], nprobe), -1, np.int32)
    rc = L.ref_coarse_search(cent, cent.shape[0], cent.shape[1], q_f32, q_f32.shape[0], nprobe, ids)
    assert rc == 0, f"ref_coarse_search returned {rc}"
    return ids


def ref_exact_u8_touched(base_u8, offsets, counts, q_u8, probes, k, threads=0, stock=False):
    """Reference cpu_fine_kernel_v3_u8_touched: returns (local positions, float dists)."""
    L = ref_lib(stock)
    assert L is not None, "oracle/_ref not built"
    base_u8 = _c(base_u8, np.uint8)
    offsets = _c(offsets, np.int64)
    counts = _c(counts, np.int32)
    q_u8 = _c(q_u8, np.uint8)
    probes = _c(probes, np.int32)
    nq, nprobe = probes.shape
    idx = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.float32)
    L.ref_cpu_fine_kernel_v3_u8_touched(base_u8, offsets, counts, q_u8, probes, nq, base_u8.shape[1],
                                        counts.shape[0], nprobe, k, threads, idx, dist)
    return idx, dist


def ref_pq_resid(cent, codebook, codes, offsets, counts, q_f32, probes, k, rerank_n=512,
                 base_u8=None, q_u8=None, base_f32=None, threads=0, stock=False):
    """Reference cpu_fine_kernel_pq_resid: returns (local positions, float exact dists, s1_ms, s2_ms)."""
    L = ref_lib(stock)
    assert L is not None, "oracle/_ref not built"
    cent = _c(cent, np.float32)
    codebook = _c(codebook, np.float32)
    codes = _c(codes, np.uint8)
    offsets = _c(offsets, np.int64)
    counts = _c(counts, np.int32)
    q_f32 = _c(q_f32, np.float32)
    probes = _c(probes, np.int32)
    base_u8 = _c(base_u8, np.uint8)
    base_f32 = _c(base_f32, np.float32)
    q_u8 = _c(q_u8, np.uint8)
    M, K, _ = codebook.shape
    nq, nprobe = probes.shape
    d = q_f32.shape[1]
    idx = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.float32)
    s1 = C.c_double(0)
    s2 = C.c_double(0)
    L.ref_cpu_fine_kernel_pq_resid(_ptr(base_u8), offsets, counts, codes, codebook, cent, _ptr(q_u8), q_f32,
                                   _ptr(base_f32), 1 if base_f32 is not None else 0, probes, nq, d,
                                   counts.shape[0], nprobe, k, rerank_n, M, K, threads, idx, dist,
                                   C.byref(s1), C.byref(s2))
    return idx, dist, s1.value, s2.value
