"""The reference's fp32 pipeline on the GPU: ivf_load_dataset (device arrays
whose ownership passes to the index) and the streaming upload
(ivf_init_streaming_upload / ivf_append_cluster_data /
ivf_finalize_streaming_upload, C++ linkage), then
ivf_pipeline_stage2_compute with distance_mode 0 (L2) and 1 (cosine): cosine
routing and an exact scan, equal bit for bit to the oracle's restatement
(oracle.f32_search) -- probe lists, row positions and distances."""
import ctypes as C

import numpy as np
import pytest
import torch

import insitu_b200 as ib
import oracle
import synth

pytestmark = pytest.mark.gpu


def _data(n=12000, d=96, nlist=40, nq=50, seed=17):
    base = synth.mixture_f32_unit(n, d, 30, 0.08, seed=seed)
    cent = synth.kmeans(base, nlist, 5, seed).numpy()
    a = synth.assign(base, torch.from_numpy(cent)).numpy()
    counts, offsets, r2o = synth.reorder(a, nlist)
    rows = base.numpy()[r2o]
    rows[5] = rows[4]                                       # equal rows: ties by position
    q = synth.mixture_f32_unit(nq, d, 30, 0.08, seed=seed, stream_base=1 << 20).numpy()
    q[0] *= 3.0                                             # not unit norm: L2 and cosine rank differently
    return rows.astype(np.float32), counts, offsets, cent.astype(np.float32), q


def _device_copy(L, arr):
    p = C.c_void_p()
    L.cuda_malloc.argtypes = [C.c_void_p, C.c_size_t]
    L.cuda_malloc.restype = C.c_void_p
    L.cuda_malloc(C.byref(p), arr.nbytes)
    assert p.value
    L.cuda_memcpy_h2d.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
    L.cuda_memcpy_h2d(p, arr.ctypes.data, arr.nbytes)
    return p


def _search(idx_h, L, q, nlist, nprobe, k, mode):
    b = ib.Batch(q.shape[0], q.shape[1], nprobe, k, nlist)
    b.stage1_prepare(q)
    b.L.ivf_pipeline_stage2_compute(b.h, idx_h, q.shape[0], nprobe, k, mode)
    assert not b.last_error(), b.last_error()
    ids, dist = b.get_results(q.shape[0], k)
    b.close()
    return ids, dist


@pytest.mark.parametrize("mode", [0, 1])
def test_load_dataset_fp32_search(cuda_ok, mode):
    rows, counts, offsets, cent, q = _data()
    L = ib.load_library(require_device=True)
    nlist, n, d = len(counts), rows.shape[0], rows.shape[1]
    ptrs = [_device_copy(L, np.ascontiguousarray(a)) for a in (counts.astype(np.int32), rows, cent)]
    idx = L.ivf_create_index_context()
    assert L.ivf_load_dataset(idx, ptrs[0], ptrs[1], ptrs[2], nlist, n, d) == 1
    nprobe, k = 7, 10
    ids, dist = _search(idx, L, q, nlist, nprobe, k, mode)
    _, oi, od = oracle.f32_search(rows, offsets, counts, cent, q, nprobe, k, cosine=mode == 1)
    assert np.array_equal(ids, oi) and np.array_equal(dist, od)
    L.ivf_destroy_index_context(idx)          # frees the adopted arrays


def test_streaming_upload_fp32_search(cuda_ok):
    rows, counts, offsets, cent, q = _data(seed=18)
    L = ib.load_library(require_device=True)
    init = getattr(L, "_Z25ivf_init_streaming_uploadPviii")
    append = getattr(L, "_Z23ivf_append_cluster_dataPviPfii")
    fin = getattr(L, "_Z29ivf_finalize_streaming_uploadPvPfi")
    init.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
    append.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int]
    fin.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    for f in (init, append, fin):
        f.restype = None
    nlist, n, d = len(counts), rows.shape[0], rows.shape[1]
    idx = L.ivf_create_index_context()
    init(idx, nlist, n, d)
    for l in range(nlist):                    # clusters in any order, each at its own offset
        l2 = (l * 7) % nlist
        blk = np.ascontiguousarray(rows[offsets[l2]:offsets[l2] + counts[l2]])
        append(idx, l2, blk.ctypes.data if counts[l2] else None, int(counts[l2]), int(offsets[l2]))
    fin(idx, np.ascontiguousarray(cent).ctypes.data, n)
    assert not L.ivf_last_error(idx), L.ivf_last_error(idx)
    for mode in (0, 1):
        ids, dist = _search(idx, L, q, nlist, 5, 8, mode)
        _, oi, od = oracle.f32_search(rows, offsets, counts, cent, q, 5, 8, cosine=mode == 1)
        assert np.array_equal(ids, oi) and np.array_equal(dist, od)
    L.ivf_destroy_index_context(idx)
