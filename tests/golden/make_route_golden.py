"""Records the reference's own coarse routing on seeded inputs (route_ref.npz).

Needs a GPU and oracle/_ref/libref_coarse.so, the reference's coarse_search
(cuda/search/cpu_fine/ivf_search_cpu_fine.cu:764-1361: cuBLAS SGEMM, norms from
cuda/l2norm/l2norm.cu, fusion_l2_topk_warpsort) compiled unmodified by
`make -C oracle ref-coarse`:
    python tests/golden/make_route_golden.py [out_dir]
The inputs come from tests/golden/route_cases.py (numpy seeds), so the file
holds only the reference's probe lists.  Written to out_dir (default: this
directory, whose MANIFEST.json then gets the file's SHA-256; with another
out_dir, copy the file here and run `python tests/golden/make_route_golden.py
--manifest`).
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)

import route_cases  # noqa: E402


def update_manifest():
    path = os.path.join(HERE, "route_ref.npz")
    man_path = os.path.join(HERE, "MANIFEST.json")
    man = json.load(open(man_path)) if os.path.exists(man_path) else {}
    man["route_ref.npz"] = hashlib.sha256(open(path, "rb").read()).hexdigest()
    json.dump(man, open(man_path, "w"), indent=1, sort_keys=True)


def main(out_dir):
    lib = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_coarse.so"))
    f32 = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
    i32 = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
    lib.ref_coarse_search.argtypes = [f32, C.c_int, C.c_int, f32, C.c_int, C.c_int, i32]
    lib.ref_coarse_search.restype = C.c_int
    out = {}
    for name in route_cases.CASES:
        cent, q = route_cases.make(name)
        for nprobe in route_cases.CASES[name]["nprobes"]:
            ids = np.full((q.shape[0], nprobe), -7, np.int32)
            rc = lib.ref_coarse_search(cent, cent.shape[0], cent.shape[1], q, q.shape[0], nprobe, ids)
            assert rc == 0, rc
            assert (ids >= 0).all() and (ids < cent.shape[0]).all()
            out[f"{name}_nprobe{nprobe}"] = ids
            print(name, nprobe, ids[:2])
    os.makedirs(out_dir, exist_ok=True)
    np.savez_compressed(os.path.join(out_dir, "route_ref.npz"), **out)
    if os.path.abspath(out_dir) == HERE:
        update_manifest()


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "--manifest":
        update_manifest()
    else:
        main(sys.argv[1] if len(sys.argv) > 1 else HERE)
