"""Generates the committed golden fixtures of tests/golden/.

Run in the development container (needs oracle/_ref, i.e. the reference tree):
    python tests/golden/make_golden.py

* exact_small.npz / pq_u8_small.npz / pq_f32_small.npz -- seeded inputs plus
  the outputs of the reference's own CPU kernels, compiled unmodified from
  cuda/search/cpu_fine/cpu_fine_kernels_v3_u8.cpp (cpu_fine_kernel_v3_u8_touched)
  and cpu_fine_kernels_pq_resid.cpp (cpu_fine_kernel_pq_resid) into
  oracle/_ref/libref_cpu_fine.so.  They pin the oracle restatement.
* kat.json -- tiny hand-built cases (duplicates, ties at rank k, an empty
  list, k larger than the candidate count, invalid and repeated probe ids)
  with expected results from the brute-force Python loops below, which are
  written independently of oracle/oracle.c.
* MANIFEST.json -- SHA-256 of every fixture.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "insituann-opensource_b200"), os.path.join(ROOT, "oracle")]

import oracle  # noqa: E402
import synth  # noqa: E402


def brute_exact(base_cm, offsets, counts, r2o, q_u8, probes, k):
    """Exact u8 top-k by (dist, original id) with plain Python loops."""
    out_i, out_d = [], []
    for qi in range(q_u8.shape[0]):
        cands = []
        for c in probes[qi]:
            if c < 0 or c >= len(counts):
                continue
            for v in range(counts[c]):
                pos = offsets[c] + v
                diff = q_u8[qi].astype(np.int64) - base_cm[pos].astype(np.int64)
                cands.append((int((diff * diff).sum()), int(r2o[pos])))
        cands.sort()
        cands = cands[:k] + [(2**31 - 1, -1)] * max(0, k - len(cands))
        out_d.append([c[0] for c in cands])
        out_i.append([c[1] for c in cands])
    return np.array(out_i, np.int32), np.array(out_d, np.int32)


def brute_pq(cent, cb, codes, offsets, counts, r2o, base_u8, q, probes, k, R):
    """Residual PQ with integer-valued inputs (every float op exact): stage 1 by
    (ADC, position), dedup, exact u8 rerank, top-k by (dist, id)."""
    M, K, dsub = cb.shape
    out_i, out_d = [], []
    for qi in range(q.shape[0]):
        s1 = []
        for c in probes[qi]:
            if c < 0 or c >= len(counts):
                continue
            r = q[qi].astype(np.float64) - cent[c].astype(np.float64)
            lut = ((r.reshape(M, 1, dsub) - cb.astype(np.float64)) ** 2).sum(-1)
            for v in range(counts[c]):
                pos = offsets[c] + v
                s1.append((float(sum(lut[m, codes[pos, m]] for m in range(M))), int(pos)))
        s1.sort()
        s1 = s1[:R]
        seen, fin = set(), []
        qu = np.clip(np.round(q[qi]), 0, 255).astype(np.int64)
        for _, pos in s1:
            if pos in seen:
                continue
            seen.add(pos)
            diff = qu - base_u8[pos].astype(np.int64)
            fin.append((float((diff * diff).sum()), int(r2o[pos])))
        fin.sort()
        fin = fin[:k] + [(float("inf"), -1)] * max(0, k - len(fin))
        out_d.append([f[0] for f in fin])
        out_i.append([f[1] for f in fin])
    return np.array(out_i, np.int32), np.array(out_d, np.float32)


def kat_cases():
    rng = np.random.default_rng(1234)
    cases = []
    # ---- exact: d=16, 3 lists (one empty), duplicates and ties ----
    d = 16
    base = rng.integers(0, 6, size=(12, d)).astype(np.uint8)
    base[5] = base[2]          # duplicate vectors -> equal distances, tie by id
    base[9] = base[2]
    assign = np.array([0, 0, 0, 0, 2, 2, 0, 2, 2, 0, 2, 2], np.int32)  # list 1 empty
    counts, offsets, r2o = synth.reorder(assign, 3)
    base_cm = base[r2o]
    q = np.stack([base[2], base[4], np.zeros(d, np.uint8), base[11]]).astype(np.uint8)
    probes = np.array([[0, 1, 2], [2, 1, 0], [1, -1, 7], [2, 2, 0]], np.int32)  # empty / invalid / repeated
    cent = np.stack([base[assign == c].mean(0) if (assign == c).any() else np.zeros(d) for c in range(3)]).astype(
        np.float32)
    for k in (3, 10):  # k=10 > candidates of some rows
        ids, dist = brute_exact(base_cm, offsets, counts, r2o, q, probes, k)
        cases.append(dict(kind="exact", k=k, base_cm=base_cm.tolist(), offsets=offsets.tolist(),
                          counts=counts.tolist(), r2o=r2o.tolist(), q_u8=q.tolist(), probes=probes.tolist(),
                          centroids=cent.tolist(), ids=ids.tolist(), dist=dist.tolist()))
    # ---- residual PQ: d=16, M=8, dsub=2, integer codebook -> exact float sums ----
    M, dsub, K = 8, 2, 256
    cb = rng.integers(-3, 4, size=(M, K, dsub)).astype(np.float32)
    n = 20
    codes = rng.integers(0, 4, size=(n, M)).astype(np.uint8)
    codes[7] = codes[3]        # duplicate codes -> equal ADC distances
    codes[8] = codes[3]
    pbase = rng.integers(0, 8, size=(n, d)).astype(np.uint8)
    pbase[8] = pbase[3]        # and equal exact distances
    pass_assign = np.array([0] * 8 + [2] * 12, np.int32)
    pc, po, pr = synth.reorder(pass_assign, 3)
    pcent = np.stack([np.full(d, 2.0), np.full(d, 50.0), np.full(d, 3.0)]).astype(np.float32)
    pq_q = rng.integers(0, 8, size=(3, d)).astype(np.float32)
    pprobes = np.array([[0, 2, 1], [2, -1, 2], [1, 0, 2]], np.int32)
    for R, k in ((4, 3), (64, 10)):
        ids, dist = brute_pq(pcent, cb, codes, po, pc, pr, pbase, pq_q, pprobes, k, R)
        cases.append(dict(kind="pq", k=k, R=R, centroids=pcent.tolist(), codebook=cb.tolist(),
                          codes=codes.tolist(), offsets=po.tolist(), counts=pc.tolist(), r2o=pr.tolist(),
                          base_u8=pbase.tolist(), q=pq_q.tolist(), probes=pprobes.tolist(), ids=ids.tolist(),
                          dist=[[float(x) if np.isfinite(x) else "inf" for x in row] for row in dist]))
    # ---- routing: ties between equal centroids and a zero-norm centroid ----
    rc = np.array([[1, 0], [0, 1], [1, 0], [0, 0], [3, 3]], np.float32)
    rq = np.array([[1, 0], [0.5, 0.5], [0, 0]], np.float32)
    exp = []
    for qq in rq:
        dd = [(float(((qq - c) ** 2).sum()), i) for i, c in enumerate(rc) if np.sqrt((c * c).sum()) >= 1e-6]
        dd.sort()
        exp.append([i for _, i in dd[:3]])
    cases.append(dict(kind="route", centroids=rc.tolist(), q=rq.tolist(), nprobe=3, ids=exp))
    return cases


def seeded_cases():
    out = {}
    # exact
    n, d, nlist, nq, nprobe, k = 4000, 64, 16, 100, 4, 10
    base = synth.mixture_u8(n, d, 24, 10.0, seed=21)
    e = synth.build_u8_index(base, nlist, seed=21, iters=8)
    q = synth.mixture_u8(nq, d, 24, 10.0, seed=21, stream_base=1 << 20).numpy()
    probes, _ = oracle.route_l2(q.astype(np.float32), e["centroids"], nprobe)
    probes[3, 1] = probes[3, 0]   # a repeated probe
    probes[5, 2] = -1             # an invalid probe
    ri, rd = oracle.ref_exact_u8_touched(e["base_cm"], e["offsets"], e["counts"], q, probes, k)
    out["exact_small"] = dict(base_cm=e["base_cm"], offsets=e["offsets"], counts=e["counts"], r2o=e["r2o"],
                              centroids=e["centroids"], q_u8=q, probes=probes, k=np.int32(k),
                              ref_local_idx=ri, ref_dist=rd)
    # residual PQ, uint8 rerank, M = 16 (dsub 4)
    n, d, nlist, M, nq, nprobe, k, R = 4000, 64, 16, 16, 60, 4, 10, 64
    base = synth.mixture_u8(n, d, 24, 10.0, seed=22)
    p = synth.build_pq_index(base, nlist, M, seed=22, kmeans_iters=8, pq_iters=6, train_n=3000)
    q = synth.mixture_u8(nq, d, 24, 10.0, seed=22, stream_base=1 << 20).float().numpy()
    probes, _ = oracle.route_l2(q, p["centroids"], nprobe)
    ri, rd, _, _ = oracle.ref_pq_resid(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], q,
                                       probes, k, rerank_n=R, base_u8=p["base_rr"], q_u8=oracle.make_query_u8(q))
    out["pq_u8_small"] = dict(centroids=p["centroids"], codebook=p["codebook"], codes=p["codes"],
                              offsets=p["offsets"], counts=p["counts"], r2o=p["r2o"], base_u8=p["base_rr"], q=q,
                              probes=probes, k=np.int32(k), R=np.int32(R), ref_local_idx=ri, ref_dist=rd)
    # residual PQ, fp32 rerank, M = 24 (dsub 2)
    n, d, nlist, M, nq, nprobe, k, R = 4000, 48, 16, 24, 60, 4, 10, 64
    base = synth.mixture_f32_unit(n, d, 24, 0.05, seed=23)
    p = synth.build_pq_index(base, nlist, M, seed=23, kmeans_iters=8, pq_iters=6, train_n=3000)
    q = synth.mixture_f32_unit(nq, d, 24, 0.05, seed=23, stream_base=1 << 20).numpy()
    probes, _ = oracle.route_l2(q, p["centroids"], nprobe)
    ri, rd, _, _ = oracle.ref_pq_resid(p["centroids"], p["codebook"], p["codes"], p["offsets"], p["counts"], q,
                                       probes, k, rerank_n=R, base_f32=p["base_rr"])
    out["pq_f32_small"] = dict(centroids=p["centroids"], codebook=p["codebook"], codes=p["codes"],
                               offsets=p["offsets"], counts=p["counts"], r2o=p["r2o"], base_f32=p["base_rr"], q=q,
                               probes=probes, k=np.int32(k), R=np.int32(R), ref_local_idx=ri, ref_dist=rd)
    return out


def main():
    assert oracle.ref_lib() is not None, "build oracle/_ref first: make -C oracle ref"
    manifest = {}
    for name, arrays in seeded_cases().items():
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **arrays)
        manifest[name + ".npz"] = hashlib.sha256(open(path, "rb").read()).hexdigest()
    kat = os.path.join(HERE, "kat.json")
    with open(kat, "w") as f:
        json.dump(kat_cases(), f)
    manifest["kat.json"] = hashlib.sha256(open(kat, "rb").read()).hexdigest()
    with open(os.path.join(HERE, "MANIFEST.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print("wrote", sorted(manifest))


if __name__ == "__main__":
    main()
