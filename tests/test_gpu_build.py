"""GPU index build (ivf_assign, ivf_build_reorder, ivf_kmeans_update,
ivf_pq_train, ivf_pq_encode) against NumPy restatements of the same steps:
assignment = the oracle's exact routing with n_probes = 1, reorder = a
stable argsort, k-means update = sequential fp64 means in row order, PQ
encode = fp32 sums in dimension order with the first minimum, PQ training =
the same Lloyd step on the residuals."""
import numpy as np
import pytest
import torch

import insitu_b200 as ib
import oracle
import synth

pytestmark = pytest.mark.gpu


def _data(n, d, ncomp, nlist, seed):
    base = synth.mixture_u8(n, d, ncomp, 10.0, seed=seed)
    g = np.random.default_rng(seed)
    cent = base[torch.from_numpy(g.choice(n, nlist, replace=False))].float().numpy() + 0.37
    cent[3] = cent[5]                       # identical centroids: ties go to the smaller id
    return base.numpy(), cent.astype(np.float32)


@pytest.mark.parametrize("d,nlist", [(128, 700), (32, 64)])
def test_assign_and_reorder(cuda_ok, d, nlist):
    x, cent = _data(30000, d, 40, nlist, 9 + d)
    b = ib.Builder(d, batch_rows=4096)
    xd = torch.from_numpy(x).cuda()
    a = b.assign(xd, torch.from_numpy(cent).cuda()).cpu().numpy()
    exp, _ = oracle.route_l2_par(x.astype(np.float32), cent, 1)
    assert np.array_equal(a, exp[:, 0])
    # fp32 rows give the same assignment
    a32 = b.assign(xd.float(), torch.from_numpy(cent).cuda()).cpu().numpy()
    assert np.array_equal(a32, a)
    counts, offsets, order = b.reorder(torch.from_numpy(a).cuda(), nlist)
    c_np, o_np, r_np = synth.reorder(a, nlist)
    assert np.array_equal(counts.cpu().numpy(), c_np)
    assert np.array_equal(offsets.cpu().numpy(), o_np)
    assert np.array_equal(order.cpu().numpy(), r_np)


def test_kmeans_update_is_the_sequential_mean(cuda_ok):
    d, nlist = 64, 300
    x, cent = _data(20000, d, 30, nlist, 21)
    b = ib.Builder(d, batch_rows=8192)
    xd = torch.from_numpy(x).cuda()
    cd = torch.from_numpy(cent).cuda()
    a = b.assign(xd, cd)
    a[:50] = 7                              # a crowded list
    a[a == 11] = 12                         # an empty list keeps its centroid
    got = b.kmeans_update(xd, a, cd.clone()).cpu().numpy()
    an = a.cpu().numpy()
    exp = cent.copy()
    for l in range(nlist):
        rows = np.where(an == l)[0]
        if len(rows):
            s = np.cumsum(x[rows].astype(np.float64), axis=0)[-1]
            exp[l] = (s / len(rows)).astype(np.float32)
    assert np.array_equal(got, exp)
    # two runs give the same centroids (fixed summation order)
    again = b.kmeans(xd, cd, 3).cpu().numpy()
    assert np.array_equal(again, b.kmeans(xd, cd, 3).cpu().numpy())


@pytest.mark.parametrize("d,M", [(128, 32), (96, 48)])
def test_pq_encode_and_train(cuda_ok, d, M):
    nlist, n = 64, 12000
    x, cent = _data(n, d, 30, nlist, 31 + M)
    dsub = d // M
    b = ib.Builder(d, batch_rows=8192)
    xd = torch.from_numpy(x).cuda()
    cd = torch.from_numpy(cent).cuda()
    a = b.assign(xd, cd)
    an = a.cpu().numpy()
    resid = (x.astype(np.float32) - cent[an]).reshape(n, M, dsub)
    g = np.random.default_rng(5)
    cb0 = resid[g.choice(n, 256, replace=False)].transpose(1, 0, 2).copy()      # [M, 256, dsub]

    def encode(cb):
        s = np.zeros((n, M, 256), np.float32)
        for e in range(dsub):
            t = resid[:, :, e][:, :, None] - cb[None, :, :, e]
            s = s + t * t
        return s.argmin(-1).astype(np.uint8)
    codes = b.pq_encode(xd, cd, a, torch.from_numpy(cb0).cuda()).cpu().numpy()
    assert np.array_equal(codes, encode(cb0))
    # rows in a given order (the cluster-major positions)
    _, _, order = b.reorder(a, nlist)
    codes_cm = b.pq_encode(xd, cd, a, torch.from_numpy(cb0).cuda(), rows=order).cpu().numpy()
    assert np.array_equal(codes_cm, encode(cb0)[order.cpu().numpy()])
    # one Lloyd step per sub-space
    cb1 = b.pq_train(xd, cd, a, torch.from_numpy(cb0).cuda().clone(), 1).cpu().numpy()
    c0 = encode(cb0)
    exp = cb0.copy()
    for m in range(M):
        for c in range(256):
            rows = np.where(c0[:, m] == c)[0]
            if len(rows):
                exp[m, c] = (resid[rows, m, :].astype(np.float64).sum(0) / len(rows)).astype(np.float32)
    np.testing.assert_allclose(cb1, exp, rtol=1e-6, atol=1e-6)


def test_ground_truth_int8_path_equals_exact(cuda_ok):
    """synth.gt_keys on a GPU (int8 tensor-core q.x) equals the CPU keys
    (fp32 products of integers) bit for bit, ties included."""
    base = synth.mixture_u8(20000, 128, 20, 10.0, seed=91)
    base[100:140] = base[99]
    q = synth.mixture_u8(64, 128, 20, 10.0, seed=91, stream_base=1 << 20).float()
    cpu = synth.gt_keys(base, q, 10, batch_rows=4096)
    gpu = synth.gt_keys(base.cuda(), q.cuda(), 10, batch_rows=4096).cpu()
    assert torch.equal(cpu, gpu)


def _np_encode(x, cent, a, cb):
    """residual PQ codes in the kernel's arithmetic: fp32 terms in dimension order, first minimum"""
    M, _, dsub = cb.shape
    resid = (x.astype(np.float32) - cent[a]).reshape(x.shape[0], M, dsub)
    s = np.zeros((x.shape[0], M, 256), np.float32)
    for e in range(dsub):
        t = resid[:, :, e][:, :, None] - cb[None, :, :, e]
        s = s + t * t
    return s.argmin(-1).astype(np.uint8)


def test_online_insert_matches_the_oracle(cuda_ok):
    """ivf_pq_insert: three batches of new uint8 rows are assigned, encoded
    and published into the delta segment; after each, the overlay search
    equals the oracle on the delta built in NumPy (list-major, older rows
    first, new rows in insertion order)."""
    n, d, nlist, M, nq, nprobe, k, R = 8000, 64, 32, 16, 60, 6, 10, 64
    base = synth.mixture_u8(n, d, 30, 10.0, seed=101)
    idx = synth.build_pq_index(base, nlist, M, seed=101, kmeans_iters=5, pq_iters=4, train_n=5000)
    q = synth.mixture_u8(nq, d, 30, 10.0, seed=101, stream_base=1 << 20).float().numpy()
    index = ib.Index().load_pq(idx["centroids"], idx["codebook"], idx["codes"], idx["offsets"], idx["counts"],
                               idx["r2o"], base_u8=idx["base_rr"])
    b = ib.Batch(nq, d, nprobe, k, nlist)
    probes, _ = oracle.route_l2(q, idx["centroids"], nprobe)
    rows_all, ids_all, lists_all = [], [], []
    next_id = n
    for step, m in enumerate((500, 1, 1300)):
        new = synth.mixture_u8(m, d, 30, 10.0, seed=101, stream_base=(1 << 21) + step).numpy()
        ids = np.arange(next_id, next_id + m, dtype=np.int32)
        next_id += m
        index.insert(torch.from_numpy(new).cuda(), ids)
        a, _ = oracle.route_l2(new.astype(np.float32), idx["centroids"], 1)
        rows_all.append(new)
        ids_all.append(ids)
        lists_all.append(a[:, 0])
        rows = np.concatenate(rows_all)
        lists = np.concatenate(lists_all)
        order = np.argsort(lists, kind="stable")               # older inserts first within a list
        counts = np.bincount(lists, minlength=nlist).astype(np.int32)
        offsets = np.zeros(nlist, np.int64)
        offsets[1:] = np.cumsum(counts)[:-1]
        codes = _np_encode(rows, idx["centroids"], lists, idx["codebook"])
        delta = dict(codes=codes[order], offsets=offsets, counts=counts, ids=np.concatenate(ids_all)[order],
                     raw_u8=rows[order])
        b.stage1_prepare(q)
        b.set_probes(probes)
        b.pq_search(index, nq, nprobe, k, rerank_n=R, overlay=True, delta_topk=16, route=False)
        gi, gd = b.get_results(nq, k)
        oi, od = oracle.pq_search(idx["centroids"], idx["codebook"], idx["codes"], idx["offsets"], idx["counts"],
                                  idx["r2o"], q, probes, k, rerank_n=R, base_u8=idx["base_rr"], delta=delta,
                                  delta_topk=16)
        assert np.array_equal(gi, oi) and np.array_equal(gd, od), f"after insert {step}"
    assert (gi >= n).any()                      # inserted vectors reach the results
    b.close()
    index.close()
