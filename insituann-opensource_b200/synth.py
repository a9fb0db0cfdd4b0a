"""Seeded synthetic datasets and offline index building for the benchmark configs.

The reference measures on SIFT1B / DEEP / SPACEV, which are not available
here; seeded Gaussian mixtures with the shapes, sizes and value ranges of the
benchmark configs stand in for them.  Index building (k-means, stable
cluster-major reorder, residual-PQ training and encoding) is the offline
part of the reference (cuda/clustering/, scripts/train_ivfpq_residual.py).
The torch functions here serve the small CPU-side cases of the tests;
build_pq_shard can instead drive the library's GPU build entry points
(insitu_b200.Builder: exact assignment by the routing kernels, fixed-order
means), which the benchmark uses.  None of it is part of the measured query
path.

Counter-based seeding: every chunk of rows draws from its own generator
seeded by (seed, chunk index), so any shard can generate its rows alone.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

GOLDEN = 0x9E3779B97F4A7C15
MASK64 = (1 << 64) - 1


# ----------------------------------------------------------------------------
# hashing helpers (the reference's delta generators, updates/pq_update.cu:42, 431-446)
# ----------------------------------------------------------------------------
def splitmix64(x: np.ndarray) -> np.ndarray:
    """splitmix64 finaliser on uint64 arrays (wrapping arithmetic)."""
    x = np.asarray(x, dtype=np.uint64)
    with np.errstate(over="ignore"):
        x = x + np.uint64(GOLDEN)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        x = x ^ (x >> np.uint64(31))
    return x


def delta_list_of(local_ids: np.ndarray, nlist: int) -> np.ndarray:
    """list = local * 11400714819323198485 mod 2^64 mod nlist (pq_update.cu:431-433)."""
    x = np.asarray(local_ids, dtype=np.uint64)
    with np.errstate(over="ignore"):
        h = x * np.uint64(11400714819323198485)
    return (h % np.uint64(nlist)).astype(np.int64)


def delta_codes_of(local_ids: np.ndarray, M: int) -> np.ndarray:
    """code[m] = splitmix64(local ^ (0x9e37...*(m+1))) & 255 (pq_update.cu:444-446)."""
    x = np.asarray(local_ids, dtype=np.uint64)[:, None]
    with np.errstate(over="ignore"):
        salt = np.uint64(GOLDEN) * (np.arange(M, dtype=np.uint64) + np.uint64(1))
    return (splitmix64(x ^ salt[None, :]) & np.uint64(255)).astype(np.uint8)


def delete_mask(position_ids: np.ndarray, ratio: float, protected_ids=None) -> np.ndarray:
    """Per-position delete mask (1 = deleted) in the reference's form
    (updates/exact_update.cu:354-407): an id is deleted when
    splitmix64(id) < ratio * (2^64 - 1), compared in x86 extended precision
    (long double), unless it is protected; ratio <= 0 deletes nothing and
    ratio >= 1 every id >= 0.  position_ids[pos] is the original id of each
    cluster-major position (reorder_to_original)."""
    ids = np.asarray(position_ids, dtype=np.int64)
    out = np.zeros(ids.shape[0], np.uint8)
    if ratio <= 0.0:
        return out
    ok = ids >= 0
    if ratio >= 1.0:
        out[ok] = 1
    else:
        threshold = np.longdouble(ratio) * np.longdouble(np.iinfo(np.uint64).max)
        h = splitmix64(ids.astype(np.uint64))
        out[ok & (h.astype(np.longdouble) < threshold)] = 1
    if protected_ids is not None:
        prot = np.zeros(max(int(ids.max(initial=0)) + 1, 1), bool)
        p = np.asarray(protected_ids, dtype=np.int64)
        p = p[(p >= 0) & (p < prot.shape[0])]
        prot[p] = True
        out[ok & prot[np.clip(ids, 0, prot.shape[0] - 1)]] = 0
    return out


def _gen(seed: int, stream: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(splitmix64(np.uint64((seed * 1_000_003 + stream) & MASK64))) & ((1 << 63) - 1))
    return g


# ----------------------------------------------------------------------------
# data
# ----------------------------------------------------------------------------
def _component_ids(n, ncomp, seed, stream, device, zipf: Optional[float]):
    g = _gen(seed, stream, device)
    if zipf is None:
        return torch.randint(0, ncomp, (n,), generator=g, device=device)
    w = 1.0 / torch.arange(1, ncomp + 1, device=device, dtype=torch.float64) ** zipf
    return torch.multinomial(w.float(), n, replacement=True, generator=g)


def u8_centers(d, ncomp, seed, device="cpu", lo=32.0, hi=224.0):
    """Mixture centers of mixture_u8: uniform in [lo, hi] per dimension."""
    gc = _gen(seed, 1 << 40, device)
    return lo + (hi - lo) * torch.rand((ncomp, d), generator=gc, device=device)


def f32_centers(d, ncomp, seed, device="cpu"):
    """Mixture centers of mixture_f32_unit: Gaussian directions on the unit sphere."""
    gc = _gen(seed, 1 << 40, device)
    centers = torch.randn((ncomp, d), generator=gc, device=device)
    return centers / centers.norm(dim=1, keepdim=True)


def mixture_u8(n, d, ncomp, sigma, seed, device="cpu", start=0, zipf=None, lo=32.0, hi=224.0, chunk=1 << 20,
               stream_base=0, centers=None):
    """uint8 rows from a Gaussian mixture: centers U[lo, hi], per-dim sigma, rounded and clipped.

    Rows start .. start+n-1 of the seeded sequence (start a multiple of chunk);
    centers (from u8_centers) may be passed to skip recomputing them."""
    if centers is None:
        centers = u8_centers(d, ncomp, seed, device, lo, hi)
    out = torch.empty((n, d), dtype=torch.uint8, device=device)
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        s = stream_base + (start + c0) // chunk
        comp = _component_ids(c1 - c0, ncomp, seed, 2 * s, device, zipf)
        g = _gen(seed, 2 * s + 1, device)
        x = centers[comp] + sigma * torch.randn((c1 - c0, d), generator=g, device=device)
        out[c0:c1] = torch.clamp(torch.round(x), 0, 255).to(torch.uint8)
    return out


def mixture_f32_unit(n, d, ncomp, sigma, seed, device="cpu", start=0, chunk=1 << 20, stream_base=0,
                     centers=None):
    """fp32 rows from a Gaussian mixture (centers on the unit sphere, per-dim sigma), unit-normalised."""
    if centers is None:
        centers = f32_centers(d, ncomp, seed, device)
    out = torch.empty((n, d), dtype=torch.float32, device=device)
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        s = stream_base + (start + c0) // chunk
        comp = _component_ids(c1 - c0, ncomp, seed, 2 * s, device, None)
        g = _gen(seed, 2 * s + 1, device)
        x = centers[comp] + sigma * torch.randn((c1 - c0, d), generator=g, device=device)
        out[c0:c1] = x / x.norm(dim=1, keepdim=True).clamp_min(1e-12)
    return out


# ----------------------------------------------------------------------------
# k-means / assignment
# ----------------------------------------------------------------------------
def _rows_per_batch(nc, budget_bytes=1 << 31):
    return max(1024, budget_bytes // max(1, nc * 4 * 3))


def assign(x: torch.Tensor, cent: torch.Tensor, batch: Optional[int] = None) -> torch.Tensor:
    """Nearest centroid (L2) of every row; int64 [n]."""
    cent = cent.float()
    cn = (cent * cent).sum(1)
    bs = batch or _rows_per_batch(cent.shape[0])
    out = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    for i in range(0, x.shape[0], bs):
        xb = x[i:i + bs].float()
        dd = cn[None, :] - 2.0 * (xb @ cent.T)
        out[i:i + bs] = dd.argmin(1)
    return out


def kmeans(x: torch.Tensor, k: int, iters: int, seed: int, sample: Optional[int] = None) -> torch.Tensor:
    """Lloyd k-means with a seeded sample init; empty clusters keep their centroid."""
    dev = x.device
    g = _gen(seed, 7, dev)
    if sample is not None and sample < x.shape[0]:
        idx = torch.randperm(x.shape[0], generator=g, device=dev)[:sample]
        xs = x[idx].float()
    else:
        xs = x.float()
    init = torch.randperm(xs.shape[0], generator=g, device=dev)[:k]
    cent = xs[init].clone()
    for _ in range(iters):
        a = assign(xs, cent)
        sums = torch.zeros_like(cent).index_add_(0, a, xs)
        cnt = torch.bincount(a, minlength=k).float()
        nz = cnt > 0
        cent[nz] = sums[nz] / cnt[nz, None]
    return cent.contiguous()


def reorder(assign_ids: np.ndarray, nlist: int):
    """Stable cluster-major reorder (dataset.cuh:559-592): counts, offsets, reorder_to_original."""
    a = np.asarray(assign_ids, dtype=np.int64)
    counts = np.bincount(a, minlength=nlist).astype(np.int32)
    offsets = np.zeros(nlist, dtype=np.int64)
    offsets[1:] = np.cumsum(counts, dtype=np.int64)[:-1]
    r2o = np.argsort(a, kind="stable").astype(np.int32)
    return counts, offsets, r2o


# ----------------------------------------------------------------------------
# residual PQ
# ----------------------------------------------------------------------------
def _pq_dist(r: torch.Tensor, cb: torch.Tensor) -> torch.Tensor:
    """r [T, M, dsub], cb [M, 256, dsub] -> squared L2 [M, T, 256]."""
    rm = r.permute(1, 0, 2)  # [M, T, dsub]
    return (rm * rm).sum(-1, keepdim=True) - 2.0 * torch.bmm(rm, cb.transpose(1, 2)) + (cb * cb).sum(-1)[:, None, :]


def train_pq(resid: torch.Tensor, M: int, iters: int, seed: int, K: int = 256) -> torch.Tensor:
    """Per-sub-space k-means (K centroids) on residuals -> codebook [M, K, dsub]."""
    T, d = resid.shape
    dsub = d // M
    r = resid.float().reshape(T, M, dsub)
    g = _gen(seed, 11, resid.device)
    init = torch.randperm(T, generator=g, device=resid.device)[:K]
    cb = r[init].permute(1, 0, 2).contiguous()  # [M, K, dsub]
    bs = max(1024, (1 << 30) // (M * K * 4))
    for _ in range(iters):
        sums = torch.zeros_like(cb)
        cnt = torch.zeros((M, K), device=resid.device)
        for i in range(0, T, bs):
            rb = r[i:i + bs]
            a = _pq_dist(rb, cb).argmin(-1)  # [M, t]
            for m in range(M):
                sums[m].index_add_(0, a[m], rb[:, m, :])
                cnt[m] += torch.bincount(a[m], minlength=K).float()
        nz = cnt > 0
        cb[nz] = sums[nz] / cnt[nz][:, None]
    return cb.contiguous()


def encode_pq(resid: torch.Tensor, cb: torch.Tensor) -> torch.Tensor:
    M, K, dsub = cb.shape
    n = resid.shape[0]
    out = torch.empty((n, M), dtype=torch.uint8, device=resid.device)
    bs = max(1024, (1 << 30) // (M * K * 4))
    for i in range(0, n, bs):
        rb = resid[i:i + bs].float().reshape(-1, M, dsub)
        out[i:i + bs] = _pq_dist(rb, cb).argmin(-1).T.to(torch.uint8)
    return out


def build_pq_index(base: torch.Tensor, nlist: int, M: int, seed: int, kmeans_iters: int = 20, pq_iters: int = 12,
                   train_n: int = 500_000, kmeans_sample: Optional[int] = None):
    """Residual-PQ index in the reference file layouts (numpy arrays, cluster-major).

    Returns dict(centroids, codebook, codes, offsets, counts, r2o, base_rr) where
    base_rr is the rerank matrix in cluster-major order (uint8 or fp32 like base).
    """
    dev = base.device
    n, d = base.shape
    cent = kmeans(base, nlist, kmeans_iters, seed, sample=kmeans_sample or min(n, 64 * nlist))
    a = assign(base, cent)
    g = _gen(seed, 13, dev)
    tr = torch.randperm(n, generator=g, device=dev)[:min(train_n, n)]
    resid_tr = base[tr].float() - cent[a[tr]]
    cb = train_pq(resid_tr, M, pq_iters, seed)
    del resid_tr
    counts, offsets, r2o = reorder(a.cpu().numpy(), nlist)
    r2o_t = torch.from_numpy(r2o).to(dev).long()
    codes = torch.empty((n, M), dtype=torch.uint8, device=dev)
    bs = 1 << 20
    for i in range(0, n, bs):
        ids = r2o_t[i:i + bs]
        resid = base[ids].float() - cent[a[ids]]
        codes[i:i + bs] = encode_pq(resid, cb)
    base_rr = base[r2o_t]
    return dict(centroids=cent.cpu().numpy(), codebook=cb.cpu().numpy(), codes=codes.cpu().numpy(),
                offsets=offsets, counts=counts, r2o=r2o, base_rr=base_rr.cpu().numpy(),
                assign=a.cpu().numpy().astype(np.int32))


def build_u8_index(base_u8: torch.Tensor, nlist: int, seed: int, iters: int = 20, kmeans_sample=None):
    """Exact uint8 index: centroids, stable cluster-major base, offsets/counts/r2o (numpy)."""
    dev = base_u8.device
    n = base_u8.shape[0]
    cent = kmeans(base_u8, nlist, iters, seed, sample=kmeans_sample)
    a = assign(base_u8, cent)
    counts, offsets, r2o = reorder(a.cpu().numpy(), nlist)
    base_cm = base_u8[torch.from_numpy(r2o).to(dev).long()]
    return dict(centroids=cent.cpu().numpy(), base_cm=base_cm.cpu().numpy(), offsets=offsets, counts=counts,
                r2o=r2o, assign=a.cpu().numpy().astype(np.int32))


def delta_segment(n_delta: int, nlist: int, M: int, base_id: int, d: int, seed: int, f32: bool = False):
    """Published delta segment built like build_delta_pq_mutable_publish (pq_update.cu:448-489).

    Lists and code bytes come from the reference's hash generators; the raw
    rerank rows are seeded uniform bytes (the reference draws them with
    mt19937_64, pq_update.cu:435-442).  Returned arrays are in delta-position
    order (list-major, local id ascending within a list).
    """
    local = np.arange(n_delta, dtype=np.int64)
    lists = delta_list_of(local, nlist)
    order = np.argsort(lists, kind="stable")
    counts = np.bincount(lists, minlength=nlist).astype(np.int32)
    offsets = np.zeros(nlist, dtype=np.int64)
    offsets[1:] = np.cumsum(counts, dtype=np.int64)[:-1]
    codes = np.empty((n_delta, M), dtype=np.uint8)
    step = 1 << 20
    for i in range(0, n_delta, step):
        codes[i:i + step] = delta_codes_of(local[order[i:i + step]], M)
    ids = (base_id + local[order]).astype(np.int32)
    g = np.random.default_rng(seed)
    raw_by_local = g.integers(0, 256, size=(n_delta, d), dtype=np.uint8)
    raw = raw_by_local[order]
    out = dict(codes=codes, offsets=offsets, counts=counts, ids=ids, local=local[order])
    if f32:
        out["raw_f32"] = raw.astype(np.float32)
    else:
        out["raw_u8"] = raw
    return out


def gt_keys(base: torch.Tensor, q: torch.Tensor, k: int, ids: Optional[torch.Tensor] = None,
            batch_rows: int = 1 << 15) -> torch.Tensor:
    """Exact top-k of q against the rows of base as keys (distance bits << 32) | id, ascending.

    uint8 rows: the distance is the exact integer |q|^2 + |x|^2 - 2 q.x; on a
    GPU q.x comes from an int8 tensor-core GEMM of the values shifted by -128
    (exact int32), elsewhere from an fp32 GEMM of integer operands, which is
    exact too (every partial sum is an integer below 128 * 255^2 < 2^24 and
    TF32 is off); the terms are combined in int64.  fp32 rows: fp32 |q|^2 + |x|^2 -
    2 q.x, clamped at 0.  ids [n] are the rows' original ids (default: the
    row index).  Ties go to the smaller id."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        nq = q.shape[0]
        is_u8 = base.dtype == torch.uint8
        d = q.shape[1]
        # uint8 on a GPU: q.x from an int8 tensor-core GEMM of the values shifted
        # by -128, exact in int32: q.x = q'.x' + 128 (sum q' + sum x') + 128^2 d
        int8 = (is_u8 and q.is_cuda and hasattr(torch, "_int_mm") and nq > 16 and d % 8 == 0
                and bool((q == q.round()).all()) and batch_rows % 8 == 0)
        if int8:
            q8 = (q.round().clamp(0, 255).to(torch.int32) - 128).to(torch.int8).contiguous()
            sq = q8.to(torch.int64).sum(1)
        qf = q.float()
        if is_u8:
            qn = (qf * qf).sum(1).round().long()
        else:
            qn = (qf * qf).sum(1)
        best = torch.full((nq, k), (1 << 63) - 1, dtype=torch.int64, device=q.device)
        for i in range(0, base.shape[0], batch_rows):
            nb = min(batch_rows, base.shape[0] - i)
            if int8 and nb % 8 == 0:
                x8 = (base[i:i + nb].to(torch.int32) - 128).to(torch.int8).contiguous()
                sx = x8.to(torch.int64).sum(1)
                dot = torch._int_mm(q8, x8.T).to(torch.int64) + 128 * (sq[:, None] + sx[None, :]) + 128 * 128 * d
                xw = base[i:i + nb].to(torch.int64)
                dd = qn[:, None] + (xw * xw).sum(1)[None, :] - 2 * dot
            else:
                xb = base[i:i + nb].float()
                dot = qf @ xb.T
                if is_u8:
                    xn = (xb * xb).sum(1).round().long()
                    dd = qn[:, None] + xn[None, :] - 2 * dot.round().long()          # exact, < 2^31
                else:
                    dd = (qn[:, None] + (xb * xb).sum(1)[None, :] - 2.0 * dot).clamp_min(0.0)
                    dd = dd.view(torch.int32).long()                             # non-negative: bits order as values
            rid = (torch.arange(i, i + nb, device=q.device) if ids is None else ids[i:i + nb].long())
            key = (dd << 32) | rid[None, :]
            kb = min(k, nb)
            vk, _ = torch.topk(key, kb, dim=1, largest=False)
            best, _ = torch.sort(torch.cat([best, vk], 1), dim=1)
            best = best[:, :k].contiguous()
        return best
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def merge_gt_keys(keys: torch.Tensor, k: int) -> np.ndarray:
    """keys [..., nq, m] from several parts (e.g. gathered from ranks) -> top-k original ids [nq, k]."""
    if keys.dim() == 3:
        keys = keys.permute(1, 0, 2).reshape(keys.shape[1], -1)
    best, _ = torch.sort(keys, dim=1)
    best = best[:, :k]
    ids = (best & 0xFFFFFFFF).int()
    ids[best == (1 << 63) - 1] = -1
    return ids.cpu().numpy()


def brute_force_gt(base: torch.Tensor, q: torch.Tensor, k: int, batch_rows: int = 1 << 15) -> np.ndarray:
    """Exact top-k original ids by L2 (ties by smaller id), for recall (see gt_keys)."""
    return merge_gt_keys(gt_keys(base, q, k, batch_rows=batch_rows), k)


# ----------------------------------------------------------------------------
# shard-local index build (every rank builds only its own lists)
# ----------------------------------------------------------------------------
class RowSource:
    """The seeded rows of one benchmark config, generated chunk by chunk.

    Counter-based: chunk i (rows i*chunk .. ) is drawn from generators keyed by
    (seed, i) alone, so any rank can produce any chunk without the others; the
    bytes equal mixture_u8 / mixture_f32_unit over the whole range."""

    def __init__(self, kind: str, n: int, d: int, ncomp: int, sigma: float, seed: int, device,
                 zipf: Optional[float] = None, chunk: int = 1 << 20, stream_base: int = 0):
        self.kind, self.n, self.d, self.ncomp, self.sigma, self.seed = kind, n, d, ncomp, sigma, seed
        self.device, self.zipf, self.chunk, self.stream_base = device, zipf, chunk, stream_base
        self.centers = (u8_centers(d, ncomp, seed, device) if kind == "u8" else f32_centers(d, ncomp, seed, device))
        self.nchunks = (n + chunk - 1) // chunk

    def rows(self, start: int, n: int) -> torch.Tensor:
        """rows start .. start+n-1 (start a multiple of the chunk)."""
        if self.kind == "u8":
            return mixture_u8(n, self.d, self.ncomp, self.sigma, self.seed, device=self.device, start=start,
                              zipf=self.zipf, chunk=self.chunk, stream_base=self.stream_base, centers=self.centers)
        return mixture_f32_unit(n, self.d, self.ncomp, self.sigma, self.seed, device=self.device, start=start,
                                chunk=self.chunk, stream_base=self.stream_base, centers=self.centers)

    def chunk_range(self, i: int):
        return i * self.chunk, min(self.n, (i + 1) * self.chunk)

    def chunk_rows(self, i: int) -> torch.Tensor:
        r0, r1 = self.chunk_range(i)
        return self.rows(r0, r1 - r0)


def build_pq_shard(src: RowSource, nlist: int, M: int, seed: int, rank: int = 0, world: int = 1, dist=None,
                   kmeans_iters: int = 20, pq_iters: int = 12, train_n: int = 500_000,
                   kmeans_sample: Optional[int] = None, row_bytes: Optional[int] = None, assign_fn=None,
                   log=None, builder=None):
    """Residual-PQ index of src, built so that each rank holds only its own lists.

    1. rank 0 runs k-means on the first kmeans_sample rows (an i.i.d. sample of
       the mixture) and broadcasts the centroids;
    2. each rank assigns the chunks i with i % world == rank to their nearest
       centroid; an all-reduce completes the assignment on every rank;
    3. rank 0 trains the PQ codebook on the residuals of the first train_n rows
       and broadcasts it;
    4. lists go to ranks by LPT on bytes (shard.lpt_shards; one rank owns all
       at world == 1); every rank regenerates the chunks, keeps the rows of
       its lists, orders them cluster-major (stable: by list, then original
       id, as dataset.cuh:559-592) and encodes their residuals.
    builder: an insitu_b200.Builder -- k-means, assignment, PQ training and
    encoding then run in the library's GPU build kernels (exact nearest
    centroids, fixed-order means) instead of torch.
    Returns device tensors (centroids, codebook, codes, r2o, base_rr) and
    numpy maps (my_lists, local offsets/counts, global offsets/counts)."""
    import shard

    dev = src.device
    say = log or (lambda *_: None)
    n, d = src.n, src.d
    S = min(n, kmeans_sample or 64 * nlist)
    if rank == 0:
        xs = src.rows(0, S)
        if builder is not None:
            g = _gen(seed, 7, dev)
            init = torch.randperm(S, generator=g, device=dev)[:nlist]
            cent = builder.kmeans(xs, xs[init].float(), kmeans_iters)
        else:
            cent = kmeans(xs, nlist, kmeans_iters, seed)
        del xs
    else:
        cent = torch.empty((nlist, d), dtype=torch.float32, device=dev)
    if world > 1:
        dist.broadcast(cent, src=0)
    say("k-means")
    if assign_fn is None:
        assign_fn = (lambda x, c: builder.assign(x, c)) if builder is not None else (lambda x, c: assign(x, c))
    a = torch.zeros(n, dtype=torch.int32, device=dev)
    for i in range(rank, src.nchunks, world):
        r0, r1 = src.chunk_range(i)
        a[r0:r1] = assign_fn(src.chunk_rows(i), cent).int()
    if world > 1:
        dist.all_reduce(a)
    say("assignment")
    T = min(train_n, n)
    if rank == 0:
        if builder is not None:
            xt = src.rows(0, T)
            g = _gen(seed, 11, dev)
            init = torch.randperm(T, generator=g, device=dev)[:256]
            cb = (xt[init].float() - cent[a[init].long()]).reshape(256, M, -1).permute(1, 0, 2).contiguous()
            cb = builder.pq_train(xt, cent, a[:T].contiguous(), cb, pq_iters)
            del xt
        else:
            resid = src.rows(0, T).float() - cent[a[:T].long()]
            cb = train_pq(resid, M, pq_iters, seed)
            del resid
    else:
        cb = torch.empty((M, 256, d // M), dtype=torch.float32, device=dev)
    if world > 1:
        dist.broadcast(cb, src=0)
    say("codebook")
    counts_g = torch.bincount(a.long(), minlength=nlist).cpu().numpy().astype(np.int32)
    offsets_g = np.zeros(nlist, np.int64)
    offsets_g[1:] = np.cumsum(counts_g, dtype=np.int64)[:-1]
    rb = row_bytes or (M + (1 if src.kind == "u8" else 4) * d)
    owner = shard.lpt_shards(counts_g, rb, world) if world > 1 else np.zeros(nlist, np.int32)
    my_lists = np.where(owner == rank)[0].astype(np.int32)
    mine = torch.from_numpy(owner == rank).to(dev)
    parts, pids = [], []
    for i in range(src.nchunks):
        r0, r1 = src.chunk_range(i)
        sel = torch.nonzero(mine[a[r0:r1].long()]).squeeze(1)
        if sel.numel():
            parts.append(src.chunk_rows(i)[sel])
            pids.append(sel + r0)
    rows = torch.cat(parts) if parts else torch.empty((0, d), dtype=torch.uint8 if src.kind == "u8" else
                                                      torch.float32, device=dev)
    ids = torch.cat(pids) if pids else torch.empty(0, dtype=torch.int64, device=dev)
    del parts, pids
    order = torch.argsort((a[ids].long() << 32) | ids)
    rows = rows[order].contiguous()
    ids = ids[order]
    del order
    say("rows")
    if builder is not None:
        la = a[ids].contiguous()
        codes = builder.pq_encode(rows, cent, la, cb) if rows.shape[0] else \
            torch.empty((0, M), dtype=torch.uint8, device=dev)
        del la
    else:
        codes = torch.empty((rows.shape[0], M), dtype=torch.uint8, device=dev)
        bs = 1 << 20
        for i in range(0, rows.shape[0], bs):
            resid = rows[i:i + bs].float() - cent[a[ids[i:i + bs]].long()]
            codes[i:i + bs] = encode_pq(resid, cb)
    say("codes")
    cnt = counts_g[my_lists].astype(np.int32)
    off = np.zeros(len(my_lists), np.int64)
    if len(my_lists):
        off[1:] = np.cumsum(cnt, dtype=np.int64)[:-1]
    return dict(centroids=cent, codebook=cb, codes=codes, r2o=ids.int(), base_rr=rows, my_lists=my_lists,
                offsets=off, counts=cnt, offsets_global=offsets_g, counts_global=counts_g)


def recall_at_k(ids: np.ndarray, gt: np.ndarray, k: int) -> float:
    """updates/io.h:151-168: hits of the first k ids among the first k GT ids."""
    ids = np.asarray(ids)[:, :k]
    gt = np.asarray(gt)[:, :k]
    hit = sum(len(np.intersect1d(a[a >= 0], b)) for a, b in zip(ids, gt))
    return hit / float(ids.shape[0] * k)
