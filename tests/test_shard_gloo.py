"""The multi-GPU exchange protocol (shard.py) with 2 gloo ranks on CPU.

Each rank owns an LPT share of the lists and computes, on the CPU, exactly
what the device kernels return on a GPU shard: sorted local routing keys,
stage-1 (ADC key, global position) lists restricted to its lists, and the
exact key of every candidate.  The collectives of shard.py then move them and
a NumPy mirror of the device merge forms the result, which must equal the
unsharded oracle search.  A second test runs the phased protocol the same
way (bounds minimum, stage-1 lists to the owners, kappa back to the shards,
each shard's exact top-k of its keys <= kappa to the owners).  A third drops a rank and checks that the
survivor gets an error from the process-group timeout instead of hanging.
"""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
import shard
import synth

NONE = np.uint64(0xFFFFFFFFFFFFFFFF)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _fkey(d, idv):
    return (np.asarray(d, np.float32).view(np.uint32).astype(np.uint64) << np.uint64(32)) | \
        np.asarray(idv, np.uint32).astype(np.uint64)


def _local_route_keys(q, cent, lists, nprobe):
    ids, dd = oracle.route_l2(q, cent[lists], min(nprobe, len(lists)))
    keys = np.full((q.shape[0], nprobe), NONE, np.uint64)
    ok = ids >= 0
    keys[:, :ids.shape[1]][ok] = _fkey(dd[ok], lists[ids[ok]])
    return keys


def _shard_stage1(idx, q, probes, lists, R):
    """stage-1 keys with global positions and the exact key of every candidate."""
    counts = np.zeros_like(idx["counts"])
    counts[lists] = idx["counts"][lists]
    _, _, s1, _ = oracle.pq_search(idx["centroids"], idx["codebook"], idx["codes"], idx["offsets"], counts,
                                   idx["r2o"], q, probes, 1, rerank_n=R, base_u8=idx["base_rr"],
                                   return_stage1=True)
    qu = oracle.make_query_u8(q).astype(np.int64)
    ex = np.full(s1.shape, NONE, np.uint64)
    for i in range(s1.shape[0]):
        for j in range(s1.shape[1]):
            if s1[i, j] == NONE:
                continue
            pos = int(s1[i, j] & np.uint64(0xFFFFFFFF))
            dd = int(((qu[i] - idx["base_rr"][pos].astype(np.int64)) ** 2).sum())
            ex[i, j] = (np.uint64(dd) << np.uint64(32)) | np.uint64(idx["r2o"][pos])
    return s1, ex


def _merge(A, E, R, k):
    """NumPy mirror of the device merge: top-R by ADC key, each position once, top-k by exact key."""
    ids = np.full((A.shape[0], k), -1, np.int32)
    dd = np.full((A.shape[0], k), np.inf, np.float32)
    for i in range(A.shape[0]):
        o = np.argsort(A[i], kind="stable")[:R]
        fin, last = [], None
        for j in o:
            if A[i, j] == NONE:
                continue
            if last is not None and A[i, j] == last:
                continue
            last = A[i, j]
            fin.append(E[i, j])
        fin = sorted(fin)[:k]
        for j, e in enumerate(fin):
            ids[i, j] = int(e & np.uint64(0xFFFFFFFF))
            dd[i, j] = float(int(e >> np.uint64(32)))
    return ids, dd


def _worker(rank, world, port, data, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    idx, q, nprobe, R, k = data["idx"], data["q"], data["nprobe"], data["R"], data["k"]
    owner = shard.lpt_shards(idx["counts"], idx["codes"].shape[1] + q.shape[1], world)
    lists = np.where(owner == rank)[0]
    nq = q.shape[0]
    as_t = lambda a: torch.from_numpy(a.view(np.int64))                      # noqa: E731
    keys_all = torch.empty((world * nq, nprobe), dtype=torch.int64)
    allk = shard.gather_route_keys(dist, as_t(_local_route_keys(q, idx["centroids"], lists, nprobe)), keys_all)
    allk = allk.numpy().view(np.uint64)
    srt = np.sort(allk, axis=1)[:, :nprobe]
    probes = np.where(srt == NONE, -1, (srt & np.uint64(0xFFFFFFFF)).astype(np.int64)).astype(np.int32)
    s1, ex = _shard_stage1(idx, q, probes, lists, R)
    qo = nq // world
    recv = torch.empty((world, qo, R), dtype=torch.int64)
    A = shard.to_owners(dist, world, as_t(s1), recv).numpy().view(np.uint64).copy()
    recv2 = torch.empty((world, qo, R), dtype=torch.int64)
    E = shard.to_owners(dist, world, as_t(ex), recv2).numpy().view(np.uint64).copy()
    ids, dd = _merge(A, E, R, k)
    ids_all = torch.empty((world * qo, k), dtype=torch.int32)
    d_all = torch.empty((world * qo, k), dtype=torch.float32)
    gi, gd = shard.gather_results(dist, torch.from_numpy(ids), torch.from_numpy(dd), ids_all, d_all)
    if rank == 0:
        out.put((probes, gi.numpy(), gd.numpy()))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_exchange_equals_unsharded_oracle():
    n, d, nlist, M = 12000, 32, 24, 16
    base = synth.mixture_u8(n, d, 40, 10.0, seed=81)
    idx = synth.build_pq_index(base, nlist, M, seed=81, kmeans_iters=5, pq_iters=4, train_n=6000)
    q = synth.mixture_u8(40, d, 40, 10.0, seed=81, stream_base=1 << 20).float().numpy()
    data = dict(idx=idx, q=q, nprobe=5, R=64, k=10)
    ctx = mp.get_context("spawn")
    out = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(2, _free_port(), data, out), nprocs=2, join=True, start_method="spawn")
    probes, gi, gd = out.get()
    exp_p, _ = oracle.route_l2(q, idx["centroids"], 5)
    assert np.array_equal(probes, exp_p)
    oi, od = oracle.pq_search(idx["centroids"], idx["codebook"], idx["codes"], idx["offsets"], idx["counts"],
                              idx["r2o"], q, exp_p, 10, rerank_n=64, base_u8=idx["base_rr"])
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)


def _phased_worker(rank, world, port, data, out):
    """the phased protocol: bounds minimum, stage-1 lists to the owners, kappa
    (the R-th key of their union) back to every shard, each shard's exact top-k
    of its keys <= kappa to the owners, owners' merge."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    idx, q, probes, R, k = data["idx"], data["q"], data["probes"], data["R"], data["k"]
    owner = np.arange(len(idx["counts"])) % world
    lists = np.where(owner == rank)[0]
    nq = q.shape[0]
    qo = nq // world
    as_t = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int64))      # noqa: E731
    # bounds: the minimum over ranks of int64 values (no bound = INT64_MAX)
    rng = np.random.default_rng(rank)
    mine = rng.integers(0, 1 << 40, size=nq).astype(np.int64)
    mine[::7] = np.iinfo(np.int64).max
    got = shard.exchange_bounds(dist, torch.from_numpy(mine.copy())).numpy()
    allb = [torch.empty(nq, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(allb, torch.from_numpy(mine))
    assert np.array_equal(got, np.min(np.stack([t.numpy() for t in allb]), axis=0))
    # stage 1 of this shard: R keys per query (global positions), in no particular order
    s1, ex = _shard_stage1(idx, q, probes, lists, R)
    o = np.random.default_rng(7 + rank).permutation(R)
    s1, ex = s1[:, o], ex[:, o]
    recv = torch.empty((world, qo, R), dtype=torch.int64)
    adc_o = shard.to_owners_raw(dist, world, as_t(s1), recv).numpy().view(np.uint64)     # [G][qo][R]
    kap = np.zeros(qo, np.uint64)                           # owner: R-th smallest key of the union
    for i in range(qo):
        allk = np.sort(adc_o[:, i, :].reshape(-1))
        valid = allk[allk != NONE]
        kap[i] = valid[R - 1] if len(valid) > R else NONE - np.uint64(1)
    kap_all = torch.empty((world * qo,), dtype=torch.int64)
    kap_all = shard.kappa_to_shards(dist, torch.from_numpy(kap.view(np.int64)), kap_all).numpy().view(np.uint64)
    # this shard's exact top-k of its distinct stage-1 keys <= kappa
    top = np.full((nq, k), NONE, np.uint64)
    for i in range(nq):
        sel = (s1[i] != NONE) & (s1[i] <= kap_all[i])
        _, first = np.unique(s1[i][sel], return_index=True)
        e = np.sort(ex[i][sel][first])[:k]
        top[i, :len(e)] = e
    recv2 = torch.empty((world, qo, k), dtype=torch.int64)
    top_o = shard.to_owners_raw(dist, world, as_t(top), recv2).numpy().view(np.uint64)     # [G][qo][k]
    ids = np.full((qo, k), -1, np.int32)
    dd = np.full((qo, k), np.inf, np.float32)
    for i in range(qo):
        e = np.sort(top_o[:, i, :].reshape(-1))
        e = e[e != NONE][:k]
        for j, key in enumerate(e):
            ids[i, j] = int(key & np.uint64(0xFFFFFFFF))
            dd[i, j] = float(int(key >> np.uint64(32)))
    # the results travel as one int64 per entry (bench.py's sharded step)
    own = torch.empty((qo, k), dtype=torch.int64)
    allp = torch.empty((world * qo, k), dtype=torch.int64)
    shard.gather_results_packed(dist, torch.from_numpy(ids), torch.from_numpy(dd), own, allp)
    gi, gd = shard.unpack_results(allp.numpy())
    if rank == 0:
        out.put((gi, gd))
    dist.barrier()
    dist.destroy_process_group()


def test_phased_protocol_equals_unsharded_oracle():
    n, d, nlist, M = 12000, 32, 24, 16
    base = synth.mixture_u8(n, d, 40, 10.0, seed=83)
    idx = synth.build_pq_index(base, nlist, M, seed=83, kmeans_iters=5, pq_iters=4, train_n=6000)
    q = synth.mixture_u8(40, d, 40, 10.0, seed=83, stream_base=1 << 20).float().numpy()
    probes, _ = oracle.route_l2(q, idx["centroids"], 5)
    data = dict(idx=idx, q=q, probes=probes, R=48, k=10)
    ctx = mp.get_context("spawn")
    out = ctx.SimpleQueue()
    mp.start_processes(_phased_worker, args=(2, _free_port(), data, out), nprocs=2, join=True, start_method="spawn")
    gi, gd = out.get()
    oi, od = oracle.pq_search(idx["centroids"], idx["codebook"], idx["codes"], idx["offsets"], idx["counts"],
                              idx["r2o"], q, probes, 10, rerank_n=48, base_u8=idx["base_rr"])
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)


def _dropping_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=3))
    if rank == 1:
        return                                # this rank leaves between steps, before the exchange
    t0 = time.time()
    keys_all = torch.empty((world * 4, 2), dtype=torch.int64)
    try:
        shard.gather_route_keys(dist, torch.zeros((4, 2), dtype=torch.int64), keys_all)
        out.put(("no error", time.time() - t0))
    except Exception as e:   # the process-group timeout (or the peer's disconnect) ends the collective
        out.put((type(e).__name__, time.time() - t0))


def test_dropped_rank_is_detected_by_timeout():
    ctx = mp.get_context("spawn")
    out = ctx.SimpleQueue()
    port = _free_port()
    ps = [ctx.Process(target=_dropping_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    assert all(not p.is_alive() for p in ps)
    what, secs = out.get()
    assert what != "no error" and secs < 30


def _build_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench

        src = synth.RowSource("u8", 40000, 32, 40, 10.0, 5, "cpu", chunk=1 << 13)
        kw = dict(kmeans_iters=3, pq_iters=2, train_n=5000, kmeans_sample=4000)
        b = synth.build_pq_shard(src, 48, 8, 5, rank=rank, world=world, dist=dist, **kw)
        b1 = synth.build_pq_shard(src, 48, 8, 5, **kw)
        ok = torch.equal(b["centroids"], b1["centroids"]) and torch.equal(b["codebook"], b1["codebook"])
        for i, l in enumerate(b["my_lists"]):
            s, c, s1 = b["offsets"][i], b["counts"][i], b1["offsets"][l]
            ok &= bool(c == b1["counts"][l])
            ok &= torch.equal(b["codes"][s:s + c], b1["codes"][s1:s1 + c])
            ok &= torch.equal(b["base_rr"][s:s + c], b1["base_rr"][s1:s1 + c])
            ok &= torch.equal(b["r2o"][s:s + c], b1["r2o"][s1:s1 + c])
        needed = np.array([0, 3, 7, 20, 33, 47], np.int64)
        g = bench.gather_lists(b, needed, rank, world, dist, torch.device("cpu"))
        if rank == 0:
            h = bench.host_index(b1)
            for l in range(48):
                c = g["counts"][l]
                if l in needed:
                    s, s1 = g["offsets"][l], h["offsets"][l]
                    ok &= bool(c == h["counts"][l])
                    for key in ("codes", "base_rr", "r2o"):
                        ok &= bool((g[key][s:s + c] == h[key][s1:s1 + c]).all())
                else:
                    ok &= bool(c == 0)
        out[rank] = bool(ok) and len(b["my_lists"]) > 0
    finally:
        dist.destroy_process_group()


def test_shard_local_build_and_list_gather():
    """Two ranks each build only their own lists (rows regenerated from the
    counter-based seeds, assignment split over the ranks): every owned list
    equals the single-rank build's, the lists partition the index, and the
    bench's oracle gather reassembles any set of lists on rank 0."""
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_build_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    assert out.get(0) and out.get(1)
