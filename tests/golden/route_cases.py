"""Seeded routing inputs shared by tests/golden/make_route_golden.py and the
tests that read route_ref.npz: numpy generators only, so the same bytes come
out on any machine.

* c1: the c1 routing shape -- unit-norm fp32 centroids (d 96, 4096 lists) and
  queries drawn around them (sigma 0.05, renormalised), nprobe 8 and 16;
* c2: the c2 shape -- centroids uniform in [32, 224]^128 (65536 lists),
  integer-valued queries (rounded and clipped draws around a centroid, sigma
  10), nprobe 16;
* c3: the c3 list count (262144) at d 128, the same value ranges, nprobe 16.
"""
from __future__ import annotations

import numpy as np

CASES = {
    "c1": dict(seed=101, nq=2000, nlist=4096, d=96, nprobes=(8, 16), kind="unit"),
    "c2": dict(seed=102, nq=2000, nlist=65536, d=128, nprobes=(16,), kind="u8"),
    "c3": dict(seed=103, nq=1000, nlist=262144, d=128, nprobes=(16,), kind="u8"),
}


def make(name):
    """(centroids [nlist, d] fp32, queries [nq, d] fp32) of one case."""
    c = CASES[name]
    g = np.random.default_rng(c["seed"])
    nq, nlist, d = c["nq"], c["nlist"], c["d"]
    if c["kind"] == "unit":
        cent = g.standard_normal((nlist, d)).astype(np.float32)
        cent /= np.linalg.norm(cent, axis=1, keepdims=True)
        comp = g.integers(0, nlist, nq)
        q = cent[comp] + 0.05 * g.standard_normal((nq, d)).astype(np.float32)
        q = (q / np.linalg.norm(q, axis=1, keepdims=True)).astype(np.float32)
    else:
        cent = (32.0 + 192.0 * g.random((nlist, d))).astype(np.float32)
        comp = g.integers(0, nlist, nq)
        q = np.clip(np.round(cent[comp] + 10.0 * g.standard_normal((nq, d))), 0, 255).astype(np.float32)
    return np.ascontiguousarray(cent), np.ascontiguousarray(q)
