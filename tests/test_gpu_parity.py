"""GPU parity: every search through the C ABI equals the CPU oracle bit for bit.

Bar: identical ids and distances (int32 for exact uint8; fp32 bits for PQ,
whose sums are written without contraction on both sides, so the 1e-4
relative tolerance of the spec is never needed here).
"""
import json
import os

import numpy as np
import pytest
import torch

import insitu_b200 as ib
import oracle
import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def gpu_exact(e, q_u8, probes, k, route=False, nprobe=None):
    nq = q_u8.shape[0]
    nprobe = nprobe or probes.shape[1]
    index = ib.Index().load_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], e["centroids"])
    b = ib.Batch(max(nq, 1), q_u8.shape[1], nprobe, k, len(e["counts"]))
    b.stage1_prepare(q_u8.astype(np.float32))
    if not route:
        b.set_probes(probes)
    b.u8_search(index, nq, nprobe, k, route=route)
    out = b.get_results_i32(nq, k)
    b.close()
    index.close()
    return out


def gpu_pq(p, q, probes, k, R, delta=None, delta_topk=16, f32=False, delta_mode=None):
    """delta_mode: when given, the mode the library must report for the published delta"""
    nq, nprobe = probes.shape
    index = ib.Index().load_pq(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"],
                               base_u8=None if f32 else p["base_u8"], base_f32=p["base_f32"] if f32 else None)
    if delta is not None:
        index.publish_delta(delta["codes"], delta["ids"], delta["counts"], delta["offsets"],
                            raw_u8=delta.get("raw_u8"), raw_f32=delta.get("raw_f32"))
        if delta_mode is not None:
            assert index.delta_mode() == delta_mode
    b = ib.Batch(nq, q.shape[1], nprobe, k, len(p["counts"]))
    b.stage1_prepare(q)
    b.set_probes(probes)
    b.pq_search(index, nq, nprobe, k, rerank_n=R, overlay=delta is not None, delta_topk=delta_topk, route=False)
    out = b.get_results(nq, k)
    b.close()
    index.close()
    return out


def gpu_stage1(p, q, probes, R, f32=False):
    """stage-1 keys (ADC bits << 32 | position) of every query, sorted, through the shard entry point."""
    nq, nprobe = probes.shape
    index = ib.Index().load_pq(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"],
                               base_u8=None if f32 else p["base_u8"], base_f32=p["base_f32"] if f32 else None)
    b = ib.Batch(nq, q.shape[1], nprobe, 10, len(p["counts"]))
    b.stage1_prepare(q)
    b.set_probes(probes)
    adc = torch.empty((nq, R), dtype=torch.int64, device="cuda")
    ex = torch.empty((nq, R), dtype=torch.int64, device="cuda")
    b.pq_search_shard(index, nq, nprobe, R, 0, adc.data_ptr(), ex.data_ptr())
    b.sync()
    got = np.sort(adc.cpu().numpy().view(np.uint64), axis=1)
    b.close()
    index.close()
    return got


# ---------------------------------------------------------------------------
# golden fixtures
# ---------------------------------------------------------------------------
def test_exact_golden(cuda_ok):
    g = load("exact_small.npz")
    k = int(g["k"])
    gi, gd = gpu_exact(g, g["q_u8"], g["probes"], k)
    oi, od = oracle.exact_u8(g["base_cm"], g["offsets"], g["counts"], g["r2o"], g["q_u8"], g["probes"], k)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)


@pytest.mark.parametrize("case", [c for c in json.load(open(os.path.join(GOLDEN, "kat.json")))
                                  if c["kind"] == "exact"], ids=lambda c: f"k{c['k']}")
def test_exact_kat(cuda_ok, case):
    a = {k: np.array(v) for k, v in case.items() if isinstance(v, list)}
    e = dict(base_cm=a["base_cm"].astype(np.uint8), offsets=a["offsets"], counts=a["counts"], r2o=a["r2o"],
             centroids=a["centroids"].astype(np.float32))
    gi, gd = gpu_exact(e, a["q_u8"].astype(np.uint8), a["probes"], case["k"])
    assert np.array_equal(gi, a["ids"]) and np.array_equal(gd, a["dist"])


@pytest.mark.parametrize("d", [128, 256])
@pytest.mark.parametrize("case", [c for c in json.load(open(os.path.join(GOLDEN, "kat.json")))
                                  if c["kind"] == "exact"], ids=lambda c: f"k{c['k']}")
def test_exact_kat_grouped(cuda_ok, case, d):
    """the known-answer cases with rows and queries zero-padded to d = 128 / 256,
    which leaves every distance unchanged and runs the grouped exact kernel."""
    a = {k: np.array(v) for k, v in case.items() if isinstance(v, list)}
    pad = lambda x: np.pad(x.astype(np.uint8), ((0, 0), (0, d - x.shape[1])))   # noqa: E731
    cent = np.pad(a["centroids"].astype(np.float32), ((0, 0), (0, d - a["centroids"].shape[1])))
    e = dict(base_cm=pad(a["base_cm"]), offsets=a["offsets"], counts=a["counts"], r2o=a["r2o"], centroids=cent)
    gi, gd = gpu_exact(e, pad(a["q_u8"]), a["probes"], case["k"])
    assert np.array_equal(gi, a["ids"]) and np.array_equal(gd, a["dist"])


@pytest.mark.parametrize("d,k", [(128, 1), (128, 10), (128, 16), (128, 17), (256, 10)])
def test_exact_grouped_many_queries(cuda_ok, d, k):
    """more than 64 queries per list (several groups of one list), lists whose
    length is no multiple of the tile, repeated and invalid probe ids; k = 17
    runs the per-pair kernel, the others the grouped one."""
    n, nlist, nq, nprobe = 9000, 24, 700, 6
    base = synth.mixture_u8(n, d, 24, 12.0, seed=61)
    e = synth.build_u8_index(base, nlist, seed=61, iters=5)
    q = synth.mixture_u8(nq, d, 24, 12.0, seed=61, stream_base=1 << 20).numpy()
    probes, _ = oracle.route_l2(q.astype(np.float32), e["centroids"], nprobe)
    probes[::7, 2] = probes[::7, 0]          # a list probed twice
    probes[::11, 3] = -1                     # an invalid probe id
    probes[::13, 4] = nlist + 5
    gi, gd = gpu_exact(e, q, probes, k)
    oi, od = oracle.exact_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], q, probes, k)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)


@pytest.mark.parametrize("d,k,deleted", [(128, 10, False), (128, 16, True), (256, 1, False), (256, 7, True)])
def test_exact_tensor_core_kernel_equals_cuda_core_kernel(cuda_ok, d, k, deleted, monkeypatch):
    """the tcgen05 (kind::i8) grouped exact kernel and the dp4a grouped kernel
    give the oracle's results: lists of several 128-row tiles and ragged
    last tiles, more than 64 queries per list, a list probed twice, invalid
    probe ids, exact distance ties and (optionally) deleted rows."""
    n, nlist, nq, nprobe = 30000, 12, 500, 5
    base = synth.mixture_u8(n, d, 12, 12.0, seed=81)
    e = synth.build_u8_index(base, nlist, seed=81, iters=4)
    e["base_cm"][500:900] = e["base_cm"][499]            # ties, broken by original id
    q = synth.mixture_u8(nq, d, 12, 12.0, seed=81, stream_base=1 << 20).numpy()
    probes, _ = oracle.route_l2(q.astype(np.float32), e["centroids"], nprobe)
    probes[::9, 1] = probes[::9, 0]
    probes[::13, 2] = -1
    dele = synth.delete_mask(e["r2o"], 0.2) if deleted else None
    out = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("INSITU_EXACT_TC", mode)
        index = ib.Index().load_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], e["centroids"])
        if dele is not None:
            index.set_deleted(dele)
        b = ib.Batch(nq, d, nprobe, k, nlist)
        b.stage1_prepare(q.astype(np.float32))
        b.set_probes(probes)
        b.u8_search(index, nq, nprobe, k, route=False)
        out[mode] = b.get_results_i32(nq, k)
        b.close()
        index.close()
    oi, od = oracle.exact_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], q, probes, k, deleted=dele)
    for mode in ("1", "0"):
        gi, gd = out[mode]
        assert np.array_equal(gi, oi) and np.array_equal(gd, od), f"INSITU_EXACT_TC={mode}"


@pytest.mark.parametrize("d", [64, 128])
def test_exact_deletes(cuda_ok, d):
    """deleted positions are not scanned (d = 64: per-pair kernel, d = 128: grouped)."""
    n, nlist, nq, nprobe, k = 6000, 20, 300, 5, 10
    base = synth.mixture_u8(n, d, 20, 12.0, seed=71)
    e = synth.build_u8_index(base, nlist, seed=71, iters=4)
    q = synth.mixture_u8(nq, d, 20, 12.0, seed=71, stream_base=1 << 20).numpy()
    probes, _ = oracle.route_l2(q.astype(np.float32), e["centroids"], nprobe)
    dele = synth.delete_mask(e["r2o"], 0.3)
    index = ib.Index().load_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], e["centroids"])
    index.set_deleted(dele)
    b = ib.Batch(nq, d, nprobe, k, nlist)
    b.stage1_prepare(q.astype(np.float32))
    b.set_probes(probes)
    b.u8_search(index, nq, nprobe, k, route=False)
    gi, gd = b.get_results_i32(nq, k)
    oi, od = oracle.exact_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], q, probes, k, deleted=dele)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)
    index.set_deleted(None)                  # cleared: the plain search again
    b.u8_search(index, nq, nprobe, k, route=False)
    gi, gd = b.get_results_i32(nq, k)
    oi, od = oracle.exact_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], q, probes, k)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)
    b.close()
    index.close()


@pytest.mark.parametrize("f32,overlay", [(False, False), (True, False), (False, True), (True, True)])
def test_pq_deletes(cuda_ok, pq_medium, f32, overlay, monkeypatch):
    """deleted positions keep their stage-1 slots and are not reranked; with a
    published delta, main keys are masked and delta keys are not (f32: the
    delta rows in the combined tile stream, u8: by the direct delta kernel)."""
    monkeypatch.setenv("INSITU_PQ_DELTA", "mix" if f32 else "direct")
    p, q = pq_medium
    nq, nprobe, k, R = q.shape[0], 8, 10, 64
    probes, _ = oracle.route_l2(q, p["centroids"], nprobe)
    dele = synth.delete_mask(p["r2o"], 0.3)
    rr = {"base_f32": p["base_u8"].astype(np.float32)} if f32 else {"base_u8": p["base_u8"]}
    delta = None
    if overlay:
        delta = synth.delta_segment(20000, len(p["counts"]), p["codebook"].shape[0], base_id=p["codes"].shape[0],
                                    d=q.shape[1], seed=5, f32=f32)
    index = ib.Index().load_pq(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"], **rr)
    index.set_deleted(dele)
    if delta is not None:
        index.publish_delta(delta["codes"], delta["ids"], delta["counts"], delta["offsets"],
                            raw_u8=delta.get("raw_u8"), raw_f32=delta.get("raw_f32"))
    b = ib.Batch(nq, q.shape[1], nprobe, k, len(p["counts"]))
    b.stage1_prepare(q)
    b.set_probes(probes)
    b.pq_search(index, nq, nprobe, k, rerank_n=R, overlay=overlay, delta_topk=16, route=False)
    gi, gd = b.get_results(nq, k)
    oi, od = oracle.pq_search(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"], q,
                              probes, k, rerank_n=R, deleted=dele, delta=delta, delta_topk=16, **rr)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)
    b.close()
    index.close()


@pytest.mark.parametrize("name", ["pq_u8_small", "pq_f32_small"])
def test_pq_golden(cuda_ok, name):
    g = load(name + ".npz")
    k, R = int(g["k"]), int(g["R"])
    f32 = "base_f32" in g
    gi, gd = gpu_pq(g, g["q"], g["probes"], k, R, f32=f32)
    oi, od = oracle.pq_search(g["centroids"], g["codebook"], g["codes"], g["offsets"], g["counts"], g["r2o"], g["q"],
                              g["probes"], k, rerank_n=R, base_u8=g.get("base_u8"), base_f32=g.get("base_f32"))
    assert np.array_equal(gi, oi)
    assert np.array_equal(gd, od)


@pytest.mark.parametrize("case", [c for c in json.load(open(os.path.join(GOLDEN, "kat.json")))
                                  if c["kind"] == "pq"], ids=lambda c: f"R{c['R']}k{c['k']}")
def test_pq_kat(cuda_ok, case):
    a = {k: np.array(v) for k, v in case.items() if isinstance(v, list) and k != "dist"}
    p = dict(centroids=a["centroids"].astype(np.float32), codebook=a["codebook"].astype(np.float32),
             codes=a["codes"].astype(np.uint8), offsets=a["offsets"], counts=a["counts"], r2o=a["r2o"],
             base_u8=a["base_u8"].astype(np.uint8))
    gi, gd = gpu_pq(p, a["q"].astype(np.float32), a["probes"], case["k"], case["R"])
    exp = np.array([[np.inf if x == "inf" else x for x in row] for row in case["dist"]], np.float32)
    assert np.array_equal(gi, a["ids"]) and np.array_equal(gd, exp)


# ---------------------------------------------------------------------------
# seeded medium cases, routing, overlay, edge cases
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def pq_medium():
    n, d, nlist, M = 60000, 128, 64, 32
    base = synth.mixture_u8(n, d, 96, 10.0, seed=31)
    p = synth.build_pq_index(base, nlist, M, seed=31, kmeans_iters=8, pq_iters=6, train_n=20000)
    p["base_u8"] = p["base_rr"]
    q = synth.mixture_u8(300, d, 96, 10.0, seed=31, stream_base=1 << 20).float().numpy()
    return p, q


def test_route_matches_oracle(cuda_ok, pq_medium):
    p, q = pq_medium
    nprobe = 12
    index = ib.Index().load_pq(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"],
                               base_u8=p["base_u8"])
    b = ib.Batch(q.shape[0], q.shape[1], nprobe, 10, len(p["counts"]))
    b.stage1_prepare(q)
    b.route(index, q.shape[0], nprobe)
    got = b.get_probes(q.shape[0], nprobe)
    exp, exp_d = oracle.route_l2(q, p["centroids"], nprobe)
    assert np.array_equal(got, exp)
    # the routing distances bit for bit (keys = distance bits << 32 | list id)
    keys = torch.empty((q.shape[0], nprobe), dtype=torch.int64, device="cuda")
    b.stage1_prepare(q)
    b.route_keys(index, q.shape[0], nprobe, keys.data_ptr())
    b.sync()
    k = keys.cpu().numpy().view(np.uint64)
    assert np.array_equal((k & np.uint64(0xFFFFFFFF)).astype(np.int32), exp)
    assert np.array_equal((k >> np.uint64(32)).astype(np.uint32), exp_d.view(np.uint32))


@pytest.mark.parametrize("mode,nprobe", [("0", 8), ("1", 8), ("1", 16), ("2", 12), ("2", 32), ("3", 8),
                                         ("3", 40)])
def test_route_kernels_bit_identical(cuda_ok, mode, nprobe, monkeypatch):
    """every routing kernel (exact CUDA-core, fused tensor-core, tensor-core
    matrix + rescoring) gives the oracle's lists and distance bits; d = 96
    and d = 128 shapes, one with enough lists to split the fused sweep"""
    monkeypatch.setenv("INSITU_ROUTE_TC", mode)
    for d, nlist, seed in ((96, 300, 71), (128, 200, 72), (128, 3000, 73)):
        cent = synth.mixture_f32_unit(nlist, d, 40, 0.05, seed=seed).numpy()
        cent[7] = cent[3]                      # identical centroids: a distance tie broken by id
        cent[11] = 0.0                         # zero norm: never routed
        q = synth.mixture_f32_unit(333, d, 40, 0.05, seed=seed, stream_base=1 << 20).numpy()
        exp, exp_d = oracle.route_l2(q, cent, nprobe)
        counts = np.full(nlist, 1, np.int32)
        offsets = np.arange(nlist, dtype=np.int64)
        rows = np.zeros((nlist, d), np.uint8)
        index = ib.Index().load_u8(rows, offsets, counts, np.arange(nlist, dtype=np.int32), cent)
        b = ib.Batch(q.shape[0], d, nprobe, 10, nlist)
        b.stage1_prepare(q)
        keys = torch.empty((q.shape[0], nprobe), dtype=torch.int64, device="cuda")
        b.route_keys(index, q.shape[0], nprobe, keys.data_ptr())
        b.sync()
        k = keys.cpu().numpy().view(np.uint64)
        b.close()
        index.close()
        assert np.array_equal((k & np.uint64(0xFFFFFFFF)).astype(np.int32), exp)
        assert np.array_equal((k >> np.uint64(32)).astype(np.uint32), exp_d.view(np.uint32))


@pytest.mark.parametrize("R,k", [(512, 10), (100, 7), (33, 33)])
def test_pq_medium_routed(cuda_ok, pq_medium, R, k):
    p, q = pq_medium
    nprobe = 12
    probes, _ = oracle.route_l2(q, p["centroids"], nprobe)
    gi, gd = gpu_pq(p, q, probes, k, R)
    oi, od, s1, _ = oracle.pq_search(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"],
                                     q, probes, k, rerank_n=R, base_u8=p["base_u8"], return_stage1=True)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)
    assert np.array_equal(gpu_stage1(p, q, probes, max(R, k)), np.sort(s1, axis=1))


@pytest.mark.parametrize("mode", ["direct", "mix", "seg"])
def test_pq_overlay(cuda_ok, pq_medium, mode, monkeypatch):
    """main + delta search with the delta rows scanned by their own kernel
    (direct; its rank limit 32 sends delta_topk 48 to seg), in one combined
    tile stream with each list's main rows (mix), or in their own tiles after
    the main rows (seg).  One list has no main rows (delta only), and every
    seventh query probes it twice."""
    monkeypatch.setenv("INSITU_PQ_DELTA", mode)
    p, q = pq_medium
    p = dict(p)
    counts = p["counts"].copy()
    counts[3] = 0
    p["counts"] = counts
    nprobe, k, R = 12, 10, 256
    n = p["codes"].shape[0]
    delta = synth.delta_segment(20000, len(p["counts"]), p["codebook"].shape[0], base_id=n, d=q.shape[1], seed=3)
    probes, _ = oracle.route_l2(q, p["centroids"], nprobe)
    probes[::7, 0] = 3
    for dtk in (16, 5, 48):
        gi, gd = gpu_pq(p, q, probes, k, R, delta=delta, delta_topk=dtk, delta_mode=mode)
        oi, od = oracle.pq_search(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"], q,
                                  probes, k, rerank_n=R, base_u8=p["base_u8"], delta=delta, delta_topk=dtk)
        assert np.array_equal(gi, oi) and np.array_equal(gd, od)


@pytest.mark.parametrize("M", [48, 16, 24])
def test_pq_f32_shapes(cuda_ok, M):
    """fp32 rerank at the c1 shape (d=96, M=48) and other sub-quantizer counts."""
    n, d, nlist = 50000, 96, 32
    base = synth.mixture_f32_unit(n, d, 64, 0.05, seed=61)
    p = synth.build_pq_index(base, nlist, M, seed=61, kmeans_iters=6, pq_iters=5, train_n=20000)
    p["base_f32"] = p["base_rr"]
    q = synth.mixture_f32_unit(200, d, 64, 0.05, seed=61, stream_base=1 << 20).numpy()
    probes, _ = oracle.route_l2(q, p["centroids"], 5)
    gi, gd = gpu_pq(p, q, probes, 10, 512, f32=True)
    oi, od, s1, _ = oracle.pq_search(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"],
                                     q, probes, 10, rerank_n=512, base_f32=p["base_f32"], return_stage1=True)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)
    assert np.array_equal(gpu_stage1(p, q, probes, 512, f32=True), np.sort(s1, axis=1))


def test_pq_edge_probes(cuda_ok, pq_medium):
    """invalid ids, a repeated list, an empty list and k larger than the candidates."""
    p, q = pq_medium
    p = dict(p)
    counts = p["counts"].copy()
    counts[5] = 0                       # an empty list
    p["counts"] = counts
    probes, _ = oracle.route_l2(q[:40], p["centroids"], 6)
    probes[0, :] = 5
    probes[1, 1] = probes[1, 0]
    probes[2, 2] = -1
    probes[3, 3] = 10 ** 6
    gi, gd = gpu_pq(p, q[:40], probes, 16, 20)
    oi, od = oracle.pq_search(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"],
                              q[:40], probes, 16, rerank_n=20, base_u8=p["base_u8"])
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)
    assert (gi[0] == -1).all()


def test_long_lists_span_many_chunks(cuda_ok):
    """lists of ~10k vectors (several scan chunks), duplicated codes (ADC ties)."""
    n, d, nlist, M = 40000, 64, 4, 16
    base = synth.mixture_u8(n, d, 8, 12.0, seed=41)
    p = synth.build_pq_index(base, nlist, M, seed=41, kmeans_iters=5, pq_iters=4, train_n=8000)
    p["codes"][100:3000] = p["codes"][99]      # many identical codes inside one list
    p["base_u8"] = p["base_rr"]
    q = synth.mixture_u8(50, d, 8, 12.0, seed=41, stream_base=1 << 20).float().numpy()
    probes, _ = oracle.route_l2(q, p["centroids"], 3)
    gi, gd = gpu_pq(p, q, probes, 10, 512)
    oi, od = oracle.pq_search(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"], q,
                              probes, 10, rerank_n=512, base_u8=p["base_u8"])
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)
    e = synth.build_u8_index(base, nlist, seed=41, iters=5)
    e["base_cm"][200:2500] = e["base_cm"][199]   # identical vectors: distance ties broken by id
    qu = oracle.make_query_u8(q)
    gi, gd = gpu_exact(e, qu, probes, 10)
    oi, od = oracle.exact_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], qu, probes, 10)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)


@pytest.mark.parametrize("R", [2048, 700])
def test_large_candidate_buffers(cuda_ok, R):
    """long lists and a large rerank_n: with R = 2048 no chunk of the scan ever
    needs a cut (all its keys pass), so a query's buffer holds whole lists
    (beyond the 4096 keys the stage-1 selection keeps in registers); with
    R = 700 chunks are cut to R .. R + R/4 keys."""
    n, d, nlist, M = 40000, 64, 4, 16
    base = synth.mixture_u8(n, d, 8, 12.0, seed=43)
    p = synth.build_pq_index(base, nlist, M, seed=43, kmeans_iters=5, pq_iters=4, train_n=8000)
    p["base_u8"] = p["base_rr"]
    q = synth.mixture_u8(24, d, 8, 12.0, seed=43, stream_base=1 << 20).float().numpy()
    probes, _ = oracle.route_l2(q, p["centroids"], 4)
    gi, gd = gpu_pq(p, q, probes, 10, R)
    oi, od, s1, _ = oracle.pq_search(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"],
                                     q, probes, 10, rerank_n=R, base_u8=p["base_u8"], return_stage1=True)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)
    # the stage-1 keys themselves (the shard entry point returns them unmerged)
    assert np.array_equal(gpu_stage1(p, q, probes, R), np.sort(s1, axis=1))


def test_exact_routed_pipeline(cuda_ok):
    """reference pipeline entry points: stage1_prepare -> stage2_compute -> get_results."""
    n, d, nlist = 30000, 128, 64
    base = synth.mixture_u8(n, d, 64, 12.0, seed=51)
    e = synth.build_u8_index(base, nlist, seed=51, iters=6)
    q = synth.mixture_u8(257, d, 64, 12.0, seed=51, stream_base=1 << 20).float().numpy()
    index = ib.Index().load_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], e["centroids"])
    b = ib.Batch(300, d, 16, 10, nlist)
    b.stage1_prepare(q)
    b.stage2_compute(index, q.shape[0], 16, 10)
    gi, gd = b.get_results(q.shape[0], 10)
    probes, _ = oracle.route_l2(q, e["centroids"], 16)
    oi, od = oracle.exact_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], oracle.make_query_u8(q), probes, 10)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od.astype(np.float32))


def test_coarse_router_handle(cuda_ok, pq_medium):
    p, q = pq_medium
    cent = torch.from_numpy(p["centroids"]).cuda()
    r = ib.CoarseRouter(cent.data_ptr(), cent.shape[0], cent.shape[1])
    got = r.search(q, 9)
    exp, _ = oracle.route_l2(q, p["centroids"], 9)
    assert np.array_equal(got, exp)
    assert r.last_timing().coarse_total_ms > 0
    with pytest.raises(ib.InsituError):
        r.search(q, cent.shape[0] + 1)   # the reference aborts here; this library reports
    r.close()


def test_sharded_merge_equals_unsharded(cuda_ok, pq_medium):
    """lists split over 2 shards (two index contexts on one GPU): local routing keys,
    key merge, per-shard stage 1 + exact scoring, device merge == unsharded result."""
    p, q = pq_medium
    nlist = len(p["counts"])
    nq, nprobe, k, R, dtk = q.shape[0], 12, 10, 256, 16
    n = p["codes"].shape[0]
    delta = synth.delta_segment(9000, nlist, p["codebook"].shape[0], base_id=n, d=q.shape[1], seed=9)
    owner = np.arange(nlist) % 2
    shards = []
    for s in range(2):
        lists = np.where(owner == s)[0]
        rows = np.concatenate([np.arange(p["offsets"][l], p["offsets"][l] + p["counts"][l]) for l in lists])
        cnt = p["counts"][lists]
        off = np.zeros(len(lists), np.int64)
        off[1:] = np.cumsum(cnt)[:-1]
        idx = ib.Index().load_pq(p["centroids"][lists], p["codebook"], p["codes"][rows], off, cnt, p["r2o"][rows],
                                 base_u8=p["base_u8"][rows])
        idx.set_shard(nlist, lists.astype(np.int32), p["offsets"][lists])
        drows = np.concatenate([np.arange(delta["offsets"][l], delta["offsets"][l] + delta["counts"][l])
                                for l in lists])
        dcnt = delta["counts"][lists]
        doff = np.zeros(len(lists), np.int64)
        doff[1:] = np.cumsum(dcnt)[:-1]
        idx.publish_delta(delta["codes"][drows], delta["ids"][drows], dcnt, doff, raw_u8=delta["raw_u8"][drows],
                          key_offsets=delta["offsets"][lists])
        shards.append(idx)
    dev = torch.device("cuda")
    keys = torch.empty((2, nq, nprobe), dtype=torch.int64, device=dev)
    adc = torch.empty((2, nq, R), dtype=torch.int64, device=dev)
    exa = torch.empty((2, nq, R), dtype=torch.int64, device=dev)
    dadc = torch.empty((2, nq, dtk), dtype=torch.int64, device=dev)
    dexa = torch.empty((2, nq, dtk), dtype=torch.int64, device=dev)
    batches = [ib.Batch(nq, q.shape[1], nprobe, k, nlist) for _ in range(2)]
    for s in range(2):
        batches[s].stage1_prepare(q)
        batches[s].route_keys(shards[s], nq, nprobe, keys[s].data_ptr())
    torch.cuda.synchronize()
    for b in batches:
        b.sync()
    allk = keys.permute(1, 0, 2).contiguous()          # [nq, 2 * nprobe]
    for s in range(2):
        # shard 0 merges the transposed keys, shard 1 the all-gather layout [2][nq][nprobe]
        if s == 0:
            batches[s].route_merge(allk.data_ptr(), 2 * nprobe, nq, nprobe)
        else:
            batches[s].route_merge_shards(keys.data_ptr(), 2, nq, nprobe)
        batches[s].pq_search_shard(shards[s], nq, nprobe, R, dtk, adc[s].data_ptr(), exa[s].data_ptr(),
                                   dadc[s].data_ptr(), dexa[s].data_ptr())
    for b in batches:
        b.sync()
    exp_probes, _ = oracle.route_l2(q, p["centroids"], nprobe)
    assert np.array_equal(batches[0].get_probes(nq, nprobe), exp_probes)
    assert np.array_equal(batches[1].get_probes(nq, nprobe), exp_probes)
    cat = lambda t: t.permute(1, 0, 2).contiguous()    # noqa: E731
    A, E, DA, DE = cat(adc), cat(exa), cat(dadc), cat(dexa)
    batches[0].pq_merge_shards(A.data_ptr(), E.data_ptr(), 2 * R, R, DA.data_ptr(), DE.data_ptr(), 2 * dtk, dtk,
                               nq, k, True)
    gi, gd = batches[0].get_results(nq, k)
    oi, od = oracle.pq_search(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"], q,
                              exp_probes, k, rerank_n=R, base_u8=p["base_u8"], delta=delta, delta_topk=dtk)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)
    for o in batches + shards:
        o.close()


@pytest.mark.parametrize("R,k,masked", [(256, 10, False), (40, 32, False), (256, 10, True)])
def test_phased_shard_protocol_equals_unsharded(cuda_ok, pq_medium, R, k, masked):
    """lists split over 3 shards (three index contexts on one GPU), the phased
    protocol with the exchanges done on the host side: nearest-probe scans,
    int64 minimum of the bounds, the other probes, unsorted stage 1 to the
    owners, kappa (R-th key of the union) back, each shard's exact top-k of its
    keys <= kappa, owners' merge == unsharded search.  masked: a delete mask
    (30% of the rows), each shard holding its rows' part of it."""
    p, q = pq_medium
    dele = synth.delete_mask(p["r2o"], 0.3) if masked else None
    nlist = len(p["counts"])
    G, nprobe = 3, 12
    nq = q.shape[0] - q.shape[0] % G
    q = q[:nq]
    qo = nq // G
    owner = np.arange(nlist) % G
    shards = []
    for s in range(G):
        lists = np.where(owner == s)[0]
        rows = np.concatenate([np.arange(p["offsets"][l], p["offsets"][l] + p["counts"][l]) for l in lists])
        cnt = p["counts"][lists]
        off = np.zeros(len(lists), np.int64)
        off[1:] = np.cumsum(cnt)[:-1]
        idx = ib.Index().load_pq(p["centroids"][lists], p["codebook"], p["codes"][rows], off, cnt, p["r2o"][rows],
                                 base_u8=p["base_u8"][rows])
        idx.set_shard(nlist, lists.astype(np.int32), p["offsets"][lists])
        if dele is not None:
            idx.set_deleted(dele[rows])
        shards.append(idx)
    dev = torch.device("cuda")
    exp_probes, _ = oracle.route_l2(q, p["centroids"], nprobe)
    batches = [ib.Batch(nq, q.shape[1], nprobe, k, nlist) for _ in range(G)]
    adc = torch.empty((G, nq, R), dtype=torch.int64, device=dev)
    topk = torch.empty((G, nq, k), dtype=torch.int64, device=dev)
    for s in range(G):
        batches[s].stage1_prepare(q)
        batches[s].set_probes(exp_probes)
        batches[s].pq_shard_scan(shards[s], nq, nprobe, R, 0)
    for b in batches:
        b.sync()

    class Dev:
        def __init__(self, ptr, n):
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i8", "data": (ptr, False), "version": 3}
    bounds = [torch.as_tensor(Dev(b.pq_shard_bounds(), nq), device=dev) for b in batches]
    low = torch.stack(bounds).min(dim=0).values
    for t in bounds:
        t.copy_(low)
    torch.cuda.synchronize()
    for s in range(G):
        batches[s].pq_shard_scan(shards[s], nq, nprobe, R, 1)
        batches[s].pq_shard_select(shards[s], nq, nprobe, R, adc[s].data_ptr())
    for b in batches:
        b.sync()
    # stage 1 to the owners: owner o gets [G][qo][R]
    adc_o = [adc[:, o * qo:(o + 1) * qo, :].contiguous() for o in range(G)]
    kappa_o = [torch.empty((qo,), dtype=torch.int64, device=dev) for _ in range(G)]
    for o in range(G):
        batches[o].pq_shard_kappa(adc_o[o].data_ptr(), G, qo, R, kappa_o[o].data_ptr())
    for b in batches:
        b.sync()
    kappa_all = torch.cat(kappa_o).contiguous()          # [nq], global query order (an all-gather)
    for s in range(G):
        batches[s].pq_shard_rerank(shards[s], nq, R, adc[s].data_ptr(), kappa_all.data_ptr(), k, topk[s].data_ptr())
    for b in batches:
        b.sync()
    gi = np.zeros((nq, k), np.int32)
    gd = np.zeros((nq, k), np.float32)
    for o in range(G):
        tk_o = topk[:, o * qo:(o + 1) * qo, :].contiguous()
        batches[o].pq_shard_final(tk_o.data_ptr(), G, qo, k, True)
        gi[o * qo:(o + 1) * qo], gd[o * qo:(o + 1) * qo] = batches[o].get_results(qo, k)
    oi, od = oracle.pq_search(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"], q,
                              exp_probes, k, rerank_n=R, base_u8=p["base_u8"], deleted=dele)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)
    for o in batches + shards:
        o.close()


def test_errors_are_reported_not_fatal(cuda_ok, pq_medium):
    p, q = pq_medium
    index = ib.Index()
    b = ib.Batch(8, q.shape[1], 4, 4, len(p["counts"]))
    b.stage1_prepare(q[:8])
    with pytest.raises(ib.InsituError):
        b.pq_search(index, 8, 4, 4)            # nothing loaded
    index.load_pq(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], p["r2o"],
                  base_u8=p["base_u8"])
    with pytest.raises(ib.InsituError):
        b.pq_search(index, 9, 4, 4)            # beyond max_n_query
    with pytest.raises(ib.InsituError):
        b.stage2_compute(index, 8, 4, 4, distance_mode=1)   # cosine is out of scope
    b.pq_search(index, 8, 4, 4)                # the context is still usable
    ids, _ = b.get_results(8, 4)
    assert (ids >= 0).all()
    b.close()
    index.close()


def _route_keys(cent, q, nprobe):
    nlist, d = cent.shape
    counts = np.full(nlist, 1, np.int32)
    offsets = np.arange(nlist, dtype=np.int64)
    rows = np.zeros((nlist, d), np.uint8)
    index = ib.Index().load_u8(rows, offsets, counts, np.arange(nlist, dtype=np.int32), cent)
    b = ib.Batch(q.shape[0], d, nprobe, 10, nlist)
    b.stage1_prepare(q)
    keys = torch.empty((q.shape[0], nprobe), dtype=torch.int64, device="cuda")
    b.route_keys(index, q.shape[0], nprobe, keys.data_ptr())
    b.sync()
    b.route(index, q.shape[0], nprobe)
    probes = b.get_probes(q.shape[0], nprobe)
    k = keys.cpu().numpy().view(np.uint64)
    b.close()
    index.close()
    return k, probes


@pytest.mark.parametrize("nlist", [65536, 262144])
def test_route_fused_large_nlist_d128(cuda_ok, nlist):
    """the fused tensor-core routing at the c2 / c3 shapes (d = 128, 65536 and
    262144 lists, the sweep split over many CTAs per query block and merged):
    probe lists and distance bits equal the oracle's exact routing, for
    integer-valued queries (bf16 holds them exactly: two operand parts) and
    for fractional ones (three parts)"""
    g = np.random.default_rng(nlist)
    d = 128
    cent = (32.0 + 192.0 * g.random((nlist, d))).astype(np.float32)
    cent[5] = cent[9]                      # a distance tie broken by list id
    cent[17] = 0.0                         # zero norm: never routed
    comp = g.integers(0, nlist, 300)
    q_int = np.clip(np.round(cent[comp] + 10.0 * g.standard_normal((300, d))), 0, 255).astype(np.float32)
    q_frac = (cent[comp] + 10.0 * g.standard_normal((300, d))).astype(np.float32)
    for q in (q_int, q_frac):
        for nprobe in (1, 8, 16, 32):
            exp, exp_d = oracle.route_l2_par(q, cent, nprobe)
            k, probes = _route_keys(cent, q, nprobe)
            assert np.array_equal(probes, exp)
            assert np.array_equal((k & np.uint64(0xFFFFFFFF)).astype(np.int32), exp)
            assert np.array_equal((k >> np.uint64(32)).astype(np.uint32), exp_d.view(np.uint32))


def test_route_matches_reference_coarse_search(cuda_ok):
    """The library's routing on the GPU against the reference's own
    coarse_search recorded on the same seeded inputs (golden/route_ref.npz,
    cuBLAS SGEMM + warpsort): every query of the c1, c2 and c3-shaped cases;
    probe sets may differ only at rounding-level near-ties
    (oracle.route_disagreement), and the count of differing queries stays
    below 2%."""
    import route_cases

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "route_ref.npz")
    if not os.path.exists(path):
        pytest.skip("route_ref.npz not generated")
    fx = np.load(path)
    for name, case in route_cases.CASES.items():
        cent, q = route_cases.make(name)
        for nprobe in case["nprobes"]:
            ref = fx[f"{name}_nprobe{nprobe}"]
            _, probes = _route_keys(cent, q, nprobe)
            n_diff, worst = oracle.route_disagreement(q, cent, probes, ref)
            print(f"{name} nprobe {nprobe}: {n_diff} of {q.shape[0]} queries differ, worst {worst:.3f}")
            assert worst <= 1.0, (name, nprobe, n_diff, worst)
            assert n_diff <= q.shape[0] // 50, (name, nprobe, n_diff)
