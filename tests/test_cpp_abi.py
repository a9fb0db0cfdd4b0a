"""The C++ side of the boundary and the reference's file formats.

* The reference's runners are C++ and include cuda/search/cpu_fine/cpu_fine.h,
  cpu_fine_u8.h and cpu_fine_pq_resid.h; tests/cpp/abi_roundtrip.cpp is such a
  runner.  Compiled against the reference's own headers (when the reference
  tree is next to this checkout or REF_ROOT names it) it must link against
  libinsitu_b200.so alone: every C++ symbol it needs is exported here.
* The index files in the reference's layouts (updates/pq_update.cu:46-49,
  scripts/train_ivfpq_residual.py:209-213, 304-307, updates/io.h:183-294)
  written with NumPy read back through the library's readers, and the
  library's writers produce those layouts.
* On a GPU, the runner (compiled against include/cpu_fine_b200.h) reads a
  small index from reference-format files, routes with coarse_search and
  searches with cpu_fine_kernel_pq_resid / cpu_fine_kernel_v3_u8_touched; its
  outputs equal the oracle's.  ivf_pq_load_files loads the same files.
"""
import os
import shutil
import subprocess
import tempfile

import numpy as np
import pytest

import insitu_b200 as ib
import oracle
import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "insituann-opensource_b200")
SRC = os.path.join(ROOT, "tests", "cpp", "abi_roundtrip.cpp")
CUDA = "/usr/local/cuda"


def _ref_root():
    r = os.environ.get("REF_ROOT") or os.path.join(os.path.dirname(ROOT), "reference")
    return r if os.path.isdir(os.path.join(r, "cuda", "search", "cpu_fine")) else None


def _compile(out, ref_headers=None):
    cmd = ["g++", "-std=c++17", "-O1", SRC, "-o", out, "-I" + os.path.join(ROOT, "include"),
           "-I" + os.path.join(CUDA, "include"), "-L" + LIBDIR, "-linsitu_b200", "-L" + os.path.join(CUDA, "lib64"),
           "-lcudart", "-Wl,-rpath," + LIBDIR, "-Wl,-rpath," + os.path.join(CUDA, "lib64")]
    if ref_headers:
        cmd[3:3] = ["-DREF_HEADERS", "-I" + os.path.join(ref_headers, "cuda")]
    return subprocess.run(cmd, capture_output=True, text=True)


@pytest.mark.skipif(shutil.which("g++") is None, reason="no g++")
def test_runner_built_against_reference_headers_links():
    ref = _ref_root()
    if ref is None:
        pytest.skip("the reference tree is not present")
    with tempfile.TemporaryDirectory() as t:
        exe = os.path.join(t, "runner_ref")
        r = _compile(exe, ref_headers=ref)
        assert r.returncode == 0, r.stderr[-2000:]
        und = subprocess.run(["nm", "-u", exe], capture_output=True, text=True).stdout
        need = [ln.split()[-1] for ln in und.splitlines() if "coarse_" in ln or "cpu_fine" in ln]
        have = subprocess.run(["nm", "-D", "--defined-only", os.path.join(LIBDIR, "libinsitu_b200.so")],
                              capture_output=True, text=True).stdout
        assert len(need) >= 6 and all(s in have for s in need), need


def _write_reference_files(dirname, seed=3):
    """a small residual-PQ uint8 index in the reference's file layouts"""
    n, d, nlist, M = 6000, 64, 24, 16
    base = synth.mixture_u8(n, d, 30, 10.0, seed=seed)
    idx = synth.build_pq_index(base, nlist, M, seed=seed, kmeans_iters=5, pq_iters=4, train_n=4000)
    q = synth.mixture_u8(40, d, 30, 10.0, seed=seed, stream_base=1 << 20).numpy()
    ib.write_index_files(os.path.join(dirname, ""), centroids=idx["centroids"], assign=idx["assign"],
                         codebook=idx["codebook"], codes=idx["codes"])
    for name, arr in (("base.u8bin", base.numpy()), ("query.u8bin", q)):
        with open(os.path.join(dirname, name), "wb") as f:
            f.write(np.array(arr.shape, np.int32).tobytes())
            f.write(np.ascontiguousarray(arr).tobytes())
    return idx, base.numpy(), q


def test_reference_file_formats_roundtrip():
    with tempfile.TemporaryDirectory() as t:
        idx, base, q = _write_reference_files(t)
        # the layouts byte by byte, as the reference's readers parse them
        raw = open(os.path.join(t, "centroids.bin"), "rb").read()
        assert np.frombuffer(raw[:8], np.int32).tolist() == list(idx["centroids"].shape)
        raw = open(os.path.join(t, "codes.bin"), "rb").read()
        assert np.frombuffer(raw[:8], np.int64)[0] == idx["codes"].shape[0]
        assert np.frombuffer(raw[8:16], np.int32).tolist() == [idx["codes"].shape[1], 0]
        raw = open(os.path.join(t, "codebook.bin"), "rb").read()
        assert np.frombuffer(raw[:16], np.int32).tolist() == list(idx["codebook"].shape) + [0]
        # and back through the library's readers
        assert np.array_equal(ib.read_centroids(os.path.join(t, "centroids.bin")), idx["centroids"])
        assert np.array_equal(ib.read_assign(os.path.join(t, "assign.bin")), idx["assign"])
        assert np.array_equal(ib.read_codebook(os.path.join(t, "codebook.bin")), idx["codebook"])
        assert np.array_equal(ib.read_codes(os.path.join(t, "codes.bin")), idx["codes"])
        assert np.array_equal(ib.read_bin(os.path.join(t, "base.u8bin")), base)
        # a ground-truth file with the optional trailing distance block
        gt = np.arange(12, dtype=np.int32).reshape(3, 4)
        with open(os.path.join(t, "gt.bin"), "wb") as f:
            f.write(np.array([3, 4], np.int32).tobytes() + gt.tobytes() + np.zeros(12, np.float32).tobytes())
        assert np.array_equal(ib.read_gt(os.path.join(t, "gt.bin")), gt)
        with pytest.raises(ib.InsituError):
            ib.read_centroids(os.path.join(t, "missing.bin"))


@pytest.mark.gpu
def test_cpp_runner_roundtrip_matches_oracle(cuda_ok):
    with tempfile.TemporaryDirectory() as t:
        idx, base, q = _write_reference_files(t, seed=4)
        exe = os.path.join(t, "runner")
        r = _compile(exe)
        assert r.returncode == 0, r.stderr[-2000:]
        run = subprocess.run([exe, t], capture_output=True, text=True, timeout=300)
        assert run.returncode == 0, run.stdout + run.stderr
        nq, nprobe, k, R = q.shape[0], 6, 10, 64
        qf = q.astype(np.float32)
        probes = np.fromfile(os.path.join(t, "out_probes.i32"), np.int32).reshape(nq, nprobe)
        exp_p, _ = oracle.route_l2(qf, idx["centroids"], nprobe)
        assert np.array_equal(probes, exp_p)
        assert np.array_equal(np.fromfile(os.path.join(t, "out_r2o.i32"), np.int32), idx["r2o"])
        pos = np.arange(idx["codes"].shape[0], dtype=np.int32)        # the kernels report cluster-major positions
        oi, od = oracle.pq_search(idx["centroids"], idx["codebook"], idx["codes"], idx["offsets"], idx["counts"],
                                  pos, qf, exp_p, k, rerank_n=R, base_u8=idx["base_rr"])
        assert np.array_equal(np.fromfile(os.path.join(t, "out_pq_ids.i32"), np.int32).reshape(nq, k), oi)
        assert np.array_equal(np.fromfile(os.path.join(t, "out_pq_dist.f32"), np.float32).reshape(nq, k), od)
        ui, ud = oracle.exact_u8(idx["base_rr"], idx["offsets"], idx["counts"], pos, q, exp_p, k)
        assert np.array_equal(np.fromfile(os.path.join(t, "out_u8_ids.i32"), np.int32).reshape(nq, k), ui)
        assert np.array_equal(np.fromfile(os.path.join(t, "out_u8_dist.f32"), np.float32).reshape(nq, k),
                              ud.astype(np.float32))
        # ivf_pq_load_files: the same files, original ids
        index = ib.Index().load_pq_files(*(os.path.join(t, f) for f in ("centroids.bin", "codebook.bin",
                                                                         "codes.bin", "assign.bin", "base.u8bin")))
        b = ib.Batch(nq, q.shape[1], nprobe, k, len(idx["counts"]))
        b.stage1_prepare(qf)
        b.pq_search(index, nq, nprobe, k, rerank_n=R, overlay=False, route=True)
        gi, gd = b.get_results(nq, k)
        oi2, od2 = oracle.pq_search(idx["centroids"], idx["codebook"], idx["codes"], idx["offsets"], idx["counts"],
                                    idx["r2o"], qf, exp_p, k, rerank_n=R, base_u8=idx["base_rr"])
        assert np.array_equal(gi, oi2) and np.array_equal(gd, od2)
        b.close()
        index.close()
