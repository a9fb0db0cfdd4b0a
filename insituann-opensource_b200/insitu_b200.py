"""Python binding of libinsitu_b200.so (ctypes over the C ABI in include/insitu_b200.h).

The objects mirror the reference's host API for the IVF query path:
``Index`` is IVFIndexContext, ``Batch`` is IVFQueryBatchContext
(cuda/search/ivf_search_separated.cu:31-93), ``Batch.stage1_prepare`` /
``stage2_compute`` / ``get_results`` are the pipeline stages of
cuda/search/ivf_search.cuh:276-327 and ``CoarseRouter`` wraps the
CoarseHandle / coarse_search routing API of cuda/search/cpu_fine/cpu_fine.h:232-278.

There is no CPU fallback: every search runs in the CUDA library, and the
module raises if the library or a CUDA device is missing.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libinsitu_b200.so")

IVF_OK = 0
ERRORS = {-1: "EINVAL", -2: "ECUDA", -3: "ESTATE", -4: "ENOMEM", -5: "EOVERFLOW", -6: "EUNSUPPORTED"}

# every exported symbol, as declared in include/insitu_b200.h and include/cuda_wrapper.h
EXPORTS = [
    "ivf_create_index_context", "ivf_destroy_index_context", "ivf_load_dataset", "ivf_create_batch_context",
    "ivf_destroy_batch_context", "ivf_pipeline_stage1_prepare", "ivf_pipeline_stage2_compute",
    "ivf_pipeline_get_results", "ivf_pipeline_sync_batch",
    "ivf_create_index_context_wrapper", "ivf_destroy_index_context_wrapper", "ivf_load_dataset_wrapper",
    "ivf_create_batch_context_wrapper", "ivf_destroy_batch_context_wrapper",
    "ivf_pipeline_stage1_prepare_wrapper", "ivf_pipeline_stage2_compute_wrapper",
    "ivf_pipeline_get_results_wrapper", "ivf_pipeline_sync_batch_wrapper", "ivf_check_index_initialized_wrapper",
    "ivf_register_index_instance", "ivf_get_index_instance", "ivf_unregister_index_instance",
    "coarse_handle_init", "coarse_handle_release", "coarse_search", "coarse_get_last_timing",
    "ivf_u8_load", "ivf_pq_load", "ivf_set_shard", "ivf_pq_publish_delta", "ivf_pq_clear_delta",
    "ivf_pq_delta_mode",
    "ivf_route", "ivf_set_probes", "ivf_get_probes", "ivf_u8_search", "ivf_pq_search", "ivf_get_results_i32",
    "ivf_pipeline_stage1_prepare_device", "ivf_get_results_device", "ivf_batch_stream",
    "ivf_route_keys", "ivf_route_merge", "ivf_route_merge_shards", "ivf_set_deleted", "ivf_pq_search_shard", "ivf_pq_merge_shards",
    "ivf_u8_search_shard", "ivf_u8_merge_shards", "ivf_pq_shard_scan", "ivf_pq_shard_bounds",
    "ivf_pq_shard_select", "ivf_pq_shard_kappa", "ivf_pq_shard_rerank", "ivf_pq_shard_final",
    "ivf_last_error", "ivf_global_last_error",
    "ivf_kernel_launches", "ivf_batch_profile", "ivf_batch_stage_ms", "ivf_u8_search_noalloc",
    "ivf_load_centroids", "ivf_assign", "ivf_build_reorder", "ivf_kmeans_update", "ivf_pq_train", "ivf_pq_encode",
    "ivf_read_centroids", "ivf_read_assign", "ivf_read_codebook", "ivf_read_codes", "ivf_read_u8bin",
    "ivf_read_fbin", "ivf_read_gt", "ivf_write_centroids", "ivf_write_assign", "ivf_write_codebook",
    "ivf_write_codes", "ivf_pq_load_files", "ivf_pq_insert",
    "cuda_is_available", "cuda_malloc", "cuda_alloc_pinned", "cuda_free_pinned", "cuda_free", "cuda_memcpy_h2d",
    "cuda_memcpy_d2h", "cuda_memcpy_async_h2d", "cuda_memcpy_async_d2h", "cuda_cleanup_memory",
    "cuda_pipeline_init", "cuda_pipeline_flush", "cuda_pipeline_flush_vectors_only", "cuda_pipeline_free",
    "cuda_device_synchronize", "cuda_get_last_error_string", "cuda_check_last_error",
]

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_longlong

_SIGS = {
    "ivf_create_index_context": ([], vp),
    "ivf_destroy_index_context": ([vp], None),
    "ivf_load_dataset": ([vp, vp, vp, vp, i32, i32, i32], i32),
    "ivf_create_batch_context": ([i32, i32, i32, i32, i32], vp),
    "ivf_destroy_batch_context": ([vp], None),
    "ivf_pipeline_stage1_prepare": ([vp, vp, i32], None),
    "ivf_pipeline_stage2_compute": ([vp, vp, i32, i32, i32, i32], None),
    "ivf_pipeline_get_results": ([vp, vp, vp, i32, i32], None),
    "ivf_pipeline_sync_batch": ([vp], None),
    "ivf_check_index_initialized_wrapper": ([vp], i32),
    "ivf_register_index_instance": ([C.c_uint, vp], None),
    "ivf_get_index_instance": ([C.c_uint], vp),
    "ivf_unregister_index_instance": ([C.c_uint], None),
    "coarse_handle_init": ([vp, vp, i32, i32], None),
    "coarse_handle_release": ([vp], None),
    "coarse_search": ([vp, vp, i32, i32, i32, vp, vp, vp, vp], None),
    "coarse_get_last_timing": ([], vp),
    "ivf_u8_load": ([vp, vp, vp, vp, vp, vp, i32, i64, i32], i32),
    "ivf_pq_load": ([vp, vp, vp, i32, i32, i32, vp, vp, vp, vp, vp, vp, i32, i64, i32], i32),
    "ivf_set_shard": ([vp, i32, vp, vp], i32),
    "ivf_pq_publish_delta": ([vp, vp, vp, vp, vp, vp, vp, vp, i64], i32),
    "ivf_pq_clear_delta": ([vp], i32),
    "ivf_pq_delta_mode": ([vp], i32),
    "ivf_route": ([vp, vp, i32, i32], i32),
    "ivf_set_probes": ([vp, vp, i32, i32], i32),
    "ivf_get_probes": ([vp, vp, i32, i32], i32),
    "ivf_u8_search": ([vp, vp, i32, i32, i32, i32], i32),
    "ivf_pq_search": ([vp, vp, i32, i32, i32, i32, i32, i32, i32], i32),
    "ivf_get_results_i32": ([vp, vp, vp, i32, i32], i32),
    "ivf_pipeline_stage1_prepare_device": ([vp, vp, i32], i32),
    "ivf_get_results_device": ([vp, vp, vp, i32, i32], i32),
    "ivf_batch_stream": ([vp], vp),
    "ivf_route_keys": ([vp, vp, i32, i32, vp], i32),
    "ivf_route_merge": ([vp, vp, i32, i32, i32], i32),
    "ivf_route_merge_shards": ([vp, vp, i32, i32, i32], i32),
    "ivf_set_deleted": ([vp, vp, i64], i32),
    "ivf_pq_search_shard": ([vp, vp, i32, i32, i32, i32, vp, vp, vp, vp], i32),
    "ivf_pq_merge_shards": ([vp, vp, vp, i32, i32, vp, vp, i32, i32, i32, i32, i32], i32),
    "ivf_u8_search_shard": ([vp, vp, i32, i32, i32, vp], i32),
    "ivf_u8_merge_shards": ([vp, vp, i32, i32, i32], i32),
    "ivf_pq_shard_scan": ([vp, vp, i32, i32, i32, i32], i32),
    "ivf_pq_shard_bounds": ([vp], vp),
    "ivf_pq_shard_select": ([vp, vp, i32, i32, i32, vp], i32),
    "ivf_pq_shard_kappa": ([vp, vp, i32, i32, i32, vp], i32),
    "ivf_pq_shard_rerank": ([vp, vp, i32, i32, vp, vp, i32, vp], i32),
    "ivf_pq_shard_final": ([vp, vp, i32, i32, i32, i32], i32),
    "ivf_last_error": ([vp], C.c_char_p),
    "ivf_global_last_error": ([], C.c_char_p),
    "cuda_is_available": ([], C.c_bool),
    "ivf_kernel_launches": ([], C.c_ulonglong),
    "ivf_batch_profile": ([vp, i32], i32),
    "ivf_batch_stage_ms": ([vp, vp, i32], i32),
    "ivf_u8_search_noalloc": ([vp, vp, vp, i32, i32, i32, vp, vp, vp], i32),
    "ivf_load_centroids": ([vp, vp, i32, i32], i32),
    "ivf_assign": ([vp, vp, vp, i32, i64, vp], i32),
    "ivf_build_reorder": ([vp, i64, i32, vp, vp, vp, vp], i32),
    "ivf_kmeans_update": ([vp, i32, i64, i32, vp, i32, vp, vp], i32),
    "ivf_pq_train": ([vp, i32, i64, i32, vp, vp, i32, i32, vp, vp], i32),
    "ivf_pq_encode": ([vp, i32, i64, i32, vp, vp, vp, vp, i32, vp, vp], i32),
    "ivf_read_centroids": ([C.c_char_p, vp, i64, vp, vp], i64),
    "ivf_read_assign": ([C.c_char_p, vp, i64, vp], i64),
    "ivf_read_codebook": ([C.c_char_p, vp, i64, vp, vp, vp], i64),
    "ivf_read_codes": ([C.c_char_p, vp, i64, vp, vp], i64),
    "ivf_read_u8bin": ([C.c_char_p, vp, i64, vp, vp], i64),
    "ivf_read_fbin": ([C.c_char_p, vp, i64, vp, vp], i64),
    "ivf_read_gt": ([C.c_char_p, vp, i64, vp, vp], i64),
    "ivf_write_centroids": ([C.c_char_p, vp, i32, i32], i32),
    "ivf_write_assign": ([C.c_char_p, vp, i64], i32),
    "ivf_write_codebook": ([C.c_char_p, vp, i32, i32, i32], i32),
    "ivf_write_codes": ([C.c_char_p, vp, i64, i32], i32),
    "ivf_pq_load_files": ([vp, C.c_char_p, C.c_char_p, C.c_char_p, C.c_char_p, C.c_char_p], i32),
    "ivf_pq_insert": ([vp, vp, i32, vp, i64], i32),
}

STAGES = ("route", "worklist", "scan", "select", "rerank")

_lib = None


class InsituError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


def library_path() -> str:
    return LIB_PATH


def kernel_launches() -> int:
    """kernels launched by libinsitu_b200 in this process so far"""
    return int(load_library().ivf_kernel_launches())


def load_library(require_device: bool = False):
    """Loads libinsitu_b200.so (raises when it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {HERE}`")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    if require_device and not _lib.cuda_is_available():
        raise RuntimeError("libinsitu_b200 needs a CUDA device; none is visible")
    return _lib


def _p(a) -> Optional[int]:
    """Address of a numpy array or of a torch tensor's data (None passes NULL)."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


_TORCH_DT = {np.uint8: "uint8", np.int32: "int32", np.int64: "int64", np.float32: "float32"}


def _c(a, dt):
    """C-contiguous array of dtype dt; torch tensors (host or device) stay torch tensors."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        import torch

        t = a.to(getattr(torch, _TORCH_DT[dt]))
        return t.contiguous()
    return np.ascontiguousarray(a, dtype=dt)


class Index:
    """Device-resident IVF index (uint8 exact or residual PQ)."""

    def __init__(self):
        self.L = load_library(require_device=True)
        self.h = self.L.ivf_create_index_context()
        if not self.h:
            raise InsituError(-4, self.L.ivf_global_last_error().decode())
        self.kind = None
        self.d = None

    def _check(self, rc):
        if rc != IVF_OK:
            raise InsituError(rc, self.L.ivf_last_error(self.h).decode())

    def load_u8(self, base_u8, offsets, counts, reorder_to_original, centroids):
        base_u8 = _c(base_u8, np.uint8)
        n, d = base_u8.shape
        offsets, counts = _c(offsets, np.int64), _c(counts, np.int32)
        r2o = _c(reorder_to_original, np.int32)
        cent = _c(centroids, np.float32)
        self._check(self.L.ivf_u8_load(self.h, _p(base_u8), _p(offsets), _p(counts), _p(r2o), _p(cent),
                                       counts.shape[0], n, d))
        self.kind, self.d, self.nlist = "u8", d, counts.shape[0]
        return self

    def load_pq(self, centroids, codebook, codes, offsets, counts, reorder_to_original, base_u8=None,
                base_f32=None):
        cent = _c(centroids, np.float32)
        cb = _c(codebook, np.float32)
        M, K, dsub = cb.shape
        codes = _c(codes, np.uint8)
        offsets, counts = _c(offsets, np.int64), _c(counts, np.int32)
        r2o = _c(reorder_to_original, np.int32)
        bu, bf = _c(base_u8, np.uint8), _c(base_f32, np.float32)
        n = codes.shape[0]
        d = cent.shape[1]
        self._check(self.L.ivf_pq_load(self.h, _p(cent), _p(cb), M, K, dsub, _p(codes), _p(offsets), _p(counts),
                                       _p(r2o), _p(bu), _p(bf), counts.shape[0], n, d))
        self.kind, self.d, self.nlist, self.f32 = "pq", d, counts.shape[0], bf is not None
        return self

    def load_pq_files(self, centroids_path, codebook_path, codes_path, assign_path, base_u8bin_path):
        """a residual-PQ index from the reference's files (ivf_pq_load_files)"""
        self._check(self.L.ivf_pq_load_files(self.h, centroids_path.encode(), codebook_path.encode(),
                                             codes_path.encode(), assign_path.encode(), base_u8bin_path.encode()))
        self.kind = "pq"
        return self

    def set_shard(self, nlist_global, local_to_global, key_offsets=None):
        l2g = _c(local_to_global, np.int32)
        ko = _c(key_offsets, np.int64)
        self._check(self.L.ivf_set_shard(self.h, nlist_global, _p(l2g), _p(ko)))
        return self

    def publish_delta(self, codes, ids, counts, offsets, raw_u8=None, raw_f32=None, key_offsets=None):
        codes = _c(codes, np.uint8)
        ids = _c(ids, np.int32)
        counts, offsets = _c(counts, np.int32), _c(offsets, np.int64)
        ko = _c(key_offsets, np.int64)
        ru, rf = _c(raw_u8, np.uint8), _c(raw_f32, np.float32)
        self._check(self.L.ivf_pq_publish_delta(self.h, _p(codes), _p(ids), _p(counts), _p(offsets), _p(ko),
                                                _p(ru), _p(rf), codes.shape[0]))
        return self

    def clear_delta(self):
        self._check(self.L.ivf_pq_clear_delta(self.h))

    def delta_mode(self):
        """how the published delta is searched: None, "direct", "mix" or "seg" (ivf_pq_delta_mode)"""
        r = self.L.ivf_pq_delta_mode(self.h)
        if r < 0:
            self._check(r)
        return [None, "direct", "mix", "seg"][r]

    def insert(self, rows, ids):
        """online insert of device rows (torch uint8 / float32 [n, d]) with ids (int32 [n]) into the delta"""
        import torch

        rows = rows.contiguous()
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        self._check(self.L.ivf_pq_insert(self.h, rows.data_ptr(), 1 if rows.dtype == torch.uint8 else 0, _p(ids),
                                         rows.shape[0]))
        return self

    def set_deleted(self, deleted=None):
        """per-position delete mask (uint8 [n], nonzero = deleted), or None to clear it."""
        m = None if deleted is None else _c(deleted, np.uint8)
        self._check(self.L.ivf_set_deleted(self.h, _p(m), 0 if m is None else m.shape[0]))
        return self

    def close(self):
        if self.h:
            self.L.ivf_destroy_index_context(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Batch:
    """One query batch: a CUDA stream plus scratch (IVFQueryBatchContext)."""

    def __init__(self, max_nq, d, max_nprobe, max_k, nlist):
        self.L = load_library(require_device=True)
        self.h = self.L.ivf_create_batch_context(max_nq, d, max_nprobe, max_k, nlist)
        if not self.h:
            raise InsituError(-4, self.L.ivf_global_last_error().decode())
        self.d = d

    def _check(self, rc):
        if rc != IVF_OK:
            raise InsituError(rc, self.L.ivf_last_error(self.h).decode())

    def last_error(self) -> str:
        return self.L.ivf_last_error(self.h).decode()

    @property
    def stream(self) -> int:
        return self.L.ivf_batch_stream(self.h) or 0

    # ---- reference pipeline ----
    def stage1_prepare(self, q_host):
        """q_host must stay alive until the stream has consumed it (sync or get_results)."""
        self._q_keep = _c(q_host, np.float32)
        self.L.ivf_pipeline_stage1_prepare(self.h, _p(self._q_keep), self._q_keep.shape[0])
        self._raise_if_error()

    def stage1_prepare_ptr(self, host_ptr: int, nq: int):
        self.L.ivf_pipeline_stage1_prepare(self.h, host_ptr, nq)
        self._raise_if_error()

    def stage1_prepare_device(self, d_ptr: int, nq: int):
        self._check(self.L.ivf_pipeline_stage1_prepare_device(self.h, d_ptr, nq))

    def stage2_compute(self, index: Index, nq, nprobe, k, distance_mode=0):
        self.L.ivf_pipeline_stage2_compute(self.h, index.h, nq, nprobe, k, distance_mode)
        self._raise_if_error()

    def get_results(self, nq, k):
        dist = np.empty((nq, k), np.float32)
        ids = np.empty((nq, k), np.int32)
        self.L.ivf_pipeline_get_results(self.h, _p(dist), _p(ids), nq, k)
        self._raise_if_error()
        return ids, dist

    def get_results_into(self, dist_ptr: int, ids_ptr: int, nq, k):
        self.L.ivf_pipeline_get_results(self.h, dist_ptr, ids_ptr, nq, k)
        self._raise_if_error()

    def get_results_i32(self, nq, k):
        dist = np.empty((nq, k), np.int32)
        ids = np.empty((nq, k), np.int32)
        self._check(self.L.ivf_get_results_i32(self.h, _p(ids), _p(dist), nq, k))
        return ids, dist

    def get_results_device(self, d_dist: int, d_ids: int, nq, k):
        self._check(self.L.ivf_get_results_device(self.h, d_dist, d_ids, nq, k))

    def sync(self):
        self.L.ivf_pipeline_sync_batch(self.h)
        self._raise_if_error()

    def _raise_if_error(self):
        msg = self.last_error()
        if msg:
            raise InsituError(-1, msg)

    # ---- observability ----
    def profile(self, enable=True):
        self._check(self.L.ivf_batch_profile(self.h, 1 if enable else 0))

    def stage_ms(self) -> dict:
        out = np.zeros(len(STAGES), np.float64)
        rc = self.L.ivf_batch_stage_ms(self.h, _p(out), len(STAGES))
        if rc < 0:
            self._check(rc)
        return dict(zip(STAGES, out.tolist()))

    # ---- explicit entry points ----
    def route(self, index: Index, nq, nprobe):
        self._check(self.L.ivf_route(self.h, index.h, nq, nprobe))

    def set_probes(self, probes):
        probes = _c(probes, np.int32)
        self._probes_keep = probes
        self._check(self.L.ivf_set_probes(self.h, _p(probes), probes.shape[0], probes.shape[1]))

    def get_probes(self, nq, nprobe):
        out = np.empty((nq, nprobe), np.int32)
        self._check(self.L.ivf_get_probes(self.h, _p(out), nq, nprobe))
        return out

    def u8_search(self, index: Index, nq, nprobe, k, route=True):
        self._check(self.L.ivf_u8_search(self.h, index.h, nq, nprobe, k, 1 if route else 0))

    def pq_search(self, index: Index, nq, nprobe, k, rerank_n=512, overlay=True, delta_topk=16, route=True):
        self._check(self.L.ivf_pq_search(self.h, index.h, nq, nprobe, k, rerank_n, 1 if overlay else 0,
                                         delta_topk, 1 if route else 0))

    # ---- shard exchange (device pointers) ----
    def route_keys(self, index: Index, nq, nprobe, d_keys: int):
        self._check(self.L.ivf_route_keys(self.h, index.h, nq, nprobe, d_keys))

    def route_merge(self, d_keys: int, n_in, nq, nprobe):
        self._check(self.L.ivf_route_merge(self.h, d_keys, n_in, nq, nprobe))

    def route_merge_shards(self, d_keys: int, n_shards, nq, nprobe):
        """d_keys: the shards' sorted routing keys as all-gathered, [n_shards][nq][nprobe]."""
        self._check(self.L.ivf_route_merge_shards(self.h, d_keys, n_shards, nq, nprobe))

    def pq_search_shard(self, index: Index, nq, nprobe, rerank_n, delta_topk, d_adc, d_exact, d_dadc=None,
                        d_dexact=None):
        self._check(self.L.ivf_pq_search_shard(self.h, index.h, nq, nprobe, rerank_n, delta_topk, d_adc, d_exact,
                                               d_dadc, d_dexact))

    def pq_merge_shards(self, d_adc, d_exact, n_main, rerank_n, d_dadc, d_dexact, n_delta, delta_topk, nq, k,
                        exact_is_int):
        self._check(self.L.ivf_pq_merge_shards(self.h, d_adc, d_exact, n_main, rerank_n, d_dadc, d_dexact, n_delta,
                                               delta_topk, nq, k, 1 if exact_is_int else 0))

    # phased sharded PQ search (see the header): device pointers as ints
    def pq_shard_scan(self, index: Index, nq, nprobe, rerank_n, pass_):
        self._check(self.L.ivf_pq_shard_scan(self.h, index.h, nq, nprobe, rerank_n, pass_))

    def pq_shard_bounds(self) -> int:
        """device address of the [nq] int64 rank-R bounds"""
        return int(self.L.ivf_pq_shard_bounds(self.h) or 0)

    def pq_shard_select(self, index: Index, nq, nprobe, rerank_n, d_adc):
        self._check(self.L.ivf_pq_shard_select(self.h, index.h, nq, nprobe, rerank_n, d_adc))

    def pq_shard_kappa(self, d_adc_all, n_shards, n_owned, rerank_n, d_kappa):
        """owner: d_adc_all [n_shards][n_owned][R] -> d_kappa [n_owned], the R-th smallest key of the union"""
        self._check(self.L.ivf_pq_shard_kappa(self.h, d_adc_all, n_shards, n_owned, rerank_n, d_kappa))

    def pq_shard_rerank(self, index: Index, nq, rerank_n, d_adc, d_kappa, k, d_topk):
        """this shard's exact top-k [nq, k] (keys) of its stage-1 keys <= d_kappa[q]"""
        self._check(self.L.ivf_pq_shard_rerank(self.h, index.h, nq, rerank_n, d_adc, d_kappa, k, d_topk))

    def pq_shard_final(self, d_topk_all, n_shards, n_owned, k, exact_is_int):
        """owner: d_topk_all [n_shards][n_owned][k] -> the batch results of its n_owned queries"""
        self._check(self.L.ivf_pq_shard_final(self.h, d_topk_all, n_shards, n_owned, k, 1 if exact_is_int else 0))

    def u8_search_shard(self, index: Index, nq, nprobe, k, d_keys):
        self._check(self.L.ivf_u8_search_shard(self.h, index.h, nq, nprobe, k, d_keys))

    def u8_merge_shards(self, d_keys, n_in, nq, k):
        self._check(self.L.ivf_u8_merge_shards(self.h, d_keys, n_in, nq, k))

    def close(self):
        if self.h:
            self.L.ivf_destroy_batch_context(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- the reference's index file formats (host code, no device needed) ----
def _err(L):
    return L.ivf_global_last_error().decode()


def read_centroids(path):
    L = load_library()
    nl, d = C.c_int(0), C.c_int(0)
    if L.ivf_read_centroids(path.encode(), None, 0, C.byref(nl), C.byref(d)) < 0:
        raise InsituError(-1, _err(L))
    out = np.empty((nl.value, d.value), np.float32)
    if L.ivf_read_centroids(path.encode(), _p(out), out.size, C.byref(nl), C.byref(d)) < 0:
        raise InsituError(-1, _err(L))
    return out


def read_assign(path):
    L = load_library()
    n = C.c_longlong(0)
    if L.ivf_read_assign(path.encode(), None, 0, C.byref(n)) < 0:
        raise InsituError(-1, _err(L))
    out = np.empty(n.value, np.int32)
    if L.ivf_read_assign(path.encode(), _p(out), out.size, C.byref(n)) < 0:
        raise InsituError(-1, _err(L))
    return out


def read_codebook(path):
    L = load_library()
    M, K, ds = C.c_int(0), C.c_int(0), C.c_int(0)
    if L.ivf_read_codebook(path.encode(), None, 0, C.byref(M), C.byref(K), C.byref(ds)) < 0:
        raise InsituError(-1, _err(L))
    out = np.empty((M.value, K.value, ds.value), np.float32)
    if L.ivf_read_codebook(path.encode(), _p(out), out.size, C.byref(M), C.byref(K), C.byref(ds)) < 0:
        raise InsituError(-1, _err(L))
    return out


def read_codes(path):
    L = load_library()
    n, M = C.c_longlong(0), C.c_int(0)
    if L.ivf_read_codes(path.encode(), None, 0, C.byref(n), C.byref(M)) < 0:
        raise InsituError(-1, _err(L))
    out = np.empty((n.value, M.value), np.uint8)
    if L.ivf_read_codes(path.encode(), _p(out), out.size, C.byref(n), C.byref(M)) < 0:
        raise InsituError(-1, _err(L))
    return out


def read_bin(path, dtype=np.uint8):
    """DiskANN u8bin (dtype uint8) or fbin (float32) [n, d]"""
    L = load_library()
    n, d = C.c_longlong(0), C.c_int(0)
    fn = L.ivf_read_u8bin if dtype == np.uint8 else L.ivf_read_fbin
    if fn(path.encode(), None, 0, C.byref(n), C.byref(d)) < 0:
        raise InsituError(-1, _err(L))
    out = np.empty((n.value, d.value), dtype)
    if fn(path.encode(), _p(out), out.size, C.byref(n), C.byref(d)) < 0:
        raise InsituError(-1, _err(L))
    return out


def read_gt(path):
    L = load_library()
    n, k = C.c_longlong(0), C.c_int(0)
    if L.ivf_read_gt(path.encode(), None, 0, C.byref(n), C.byref(k)) < 0:
        raise InsituError(-1, _err(L))
    out = np.empty((n.value, k.value), np.int32)
    if L.ivf_read_gt(path.encode(), _p(out), out.size, C.byref(n), C.byref(k)) < 0:
        raise InsituError(-1, _err(L))
    return out


def write_index_files(prefix, centroids=None, assign=None, codebook=None, codes=None):
    """writes the given arrays in the reference formats as prefix + {centroids,assign,codebook,codes}.bin"""
    L = load_library()
    rc = 0
    if centroids is not None:
        c = _c(centroids, np.float32)
        rc |= L.ivf_write_centroids((prefix + "centroids.bin").encode(), _p(c), c.shape[0], c.shape[1])
    if assign is not None:
        a = _c(assign, np.int32)
        rc |= L.ivf_write_assign((prefix + "assign.bin").encode(), _p(a), a.shape[0])
    if codebook is not None:
        cb = _c(codebook, np.float32)
        rc |= L.ivf_write_codebook((prefix + "codebook.bin").encode(), _p(cb), *cb.shape)
    if codes is not None:
        cd = _c(codes, np.uint8)
        rc |= L.ivf_write_codes((prefix + "codes.bin").encode(), _p(cd), cd.shape[0], cd.shape[1])
    if rc:
        raise InsituError(-1, _err(L))


class Builder:
    """GPU index build through the C ABI (device tensors in and out).

    ``assign`` is the exact routing with n_probes = 1; ``kmeans`` runs Lloyd
    iterations of assign + ivf_kmeans_update; ``reorder``, ``pq_train`` and
    ``pq_encode`` wrap the other build entry points.  Work runs on the current
    torch stream of the tensors' device."""

    def __init__(self, d: int, batch_rows: int = 65536):
        self.L = load_library(require_device=True)
        self.d = d
        self.batch_rows = batch_rows

    def _stream(self):
        import torch

        return torch.cuda.current_stream().cuda_stream

    def _check(self, rc, ctx=None):
        if rc != IVF_OK:
            msg = (self.L.ivf_last_error(ctx) if ctx else self.L.ivf_global_last_error()).decode()
            raise InsituError(rc, msg)

    def assign(self, x, centroids):
        """nearest centroid (int32 [n]) of the rows of x (uint8 or fp32 device tensor)."""
        import torch

        n = x.shape[0]
        nlist = centroids.shape[0]
        out = torch.empty(n, dtype=torch.int32, device=x.device)
        idx = self.L.ivf_create_index_context()
        b = self.L.ivf_create_batch_context(min(self.batch_rows, max(n, 1)), self.d, 1, 1, nlist)
        try:
            c = centroids.float().contiguous()
            self._check(self.L.ivf_load_centroids(idx, c.data_ptr(), nlist, self.d), idx)
            torch.cuda.current_stream().synchronize()
            self._check(self.L.ivf_assign(b, idx, x.contiguous().data_ptr(), 1 if x.dtype == torch.uint8 else 0,
                                          n, out.data_ptr()), b)
            self.L.ivf_pipeline_sync_batch(b)
        finally:
            self.L.ivf_destroy_batch_context(b)
            self.L.ivf_destroy_index_context(idx)
        return out

    def kmeans_update(self, x, assign, centroids):
        import torch

        self._check(self.L.ivf_kmeans_update(x.contiguous().data_ptr(), 1 if x.dtype == torch.uint8 else 0,
                                             x.shape[0], self.d, assign.data_ptr(), centroids.shape[0],
                                             centroids.data_ptr(), self._stream()))
        return centroids

    def kmeans(self, x, init_centroids, iters):
        """Lloyd k-means from init_centroids (fp32 [nlist, d], updated copy returned)."""
        cent = init_centroids.float().clone().contiguous()
        for _ in range(iters):
            a = self.assign(x, cent)
            self.kmeans_update(x, a, cent)
        return cent

    def reorder(self, assign, nlist):
        """(counts int32 [nlist], offsets int64 [nlist], order int32 [n]) as device tensors."""
        import torch

        n = assign.shape[0]
        counts = torch.empty(nlist, dtype=torch.int32, device=assign.device)
        offsets = torch.empty(nlist, dtype=torch.int64, device=assign.device)
        order = torch.empty(max(n, 1), dtype=torch.int32, device=assign.device)
        self._check(self.L.ivf_build_reorder(assign.data_ptr(), n, nlist, counts.data_ptr(), offsets.data_ptr(),
                                             order.data_ptr(), self._stream()))
        return counts, offsets, order[:n]

    def pq_train(self, x, centroids, assign, codebook, iters):
        import torch

        M = codebook.shape[0]
        self._check(self.L.ivf_pq_train(x.contiguous().data_ptr(), 1 if x.dtype == torch.uint8 else 0, x.shape[0],
                                        self.d, centroids.data_ptr(), assign.data_ptr(), M, iters,
                                        codebook.data_ptr(), self._stream()))
        return codebook

    def pq_encode(self, x, centroids, assign, codebook, rows=None):
        import torch

        M = codebook.shape[0]
        n = rows.shape[0] if rows is not None else x.shape[0]
        codes = torch.empty((n, M), dtype=torch.uint8, device=x.device)
        self._check(self.L.ivf_pq_encode(x.contiguous().data_ptr(), 1 if x.dtype == torch.uint8 else 0, n, self.d,
                                         None if rows is None else rows.data_ptr(), centroids.data_ptr(),
                                         assign.data_ptr(), codebook.data_ptr(), M, codes.data_ptr(),
                                         self._stream()))
        return codes


class CoarseTiming(C.Structure):
    _fields_ = [(n, C.c_double) for n in ("query_h2d_ms", "seq_init_ms", "query_norm_ms", "gemm_ms", "topk_ms",
                                          "cluster_d2h_ms", "coarse_compute_ms", "coarse_total_ms")]


class _CoarseHandle(C.Structure):
    _fields_ = [("d_centers", vp), ("d_centers_norm", vp), ("cublas_handle", vp), ("n_total_clusters", i32),
                ("dim", i32), ("distance_mode_cached", i32)]


class CoarseRouter:
    """CoarseHandle + coarse_search (cpu_fine.h:232-278): host queries in, host probe ids out."""

    def __init__(self, d_centers_ptr: int, nlist: int, dim: int):
        self.L = load_library(require_device=True)
        self.h = _CoarseHandle()
        self.L.coarse_handle_init(C.byref(self.h), d_centers_ptr, nlist, dim)
        if not self.h.cublas_handle:
            raise InsituError(-1, self.L.ivf_global_last_error().decode())

    def search(self, q, nprobe):
        q = _c(q, np.float32)
        out = np.full((q.shape[0], nprobe), -7, np.int32)
        t = [C.c_double(0), C.c_double(0), C.c_double(0)]
        self.L.coarse_search(C.byref(self.h), _p(q), q.shape[0], nprobe, 0, _p(out), C.byref(t[0]),
                             C.byref(t[1]), C.byref(t[2]))
        err = self.L.ivf_global_last_error().decode()
        if (out == -7).any() and err:
            raise InsituError(-1, err)
        return out

    def last_timing(self) -> CoarseTiming:
        return CoarseTiming.from_address(self.L.coarse_get_last_timing())

    def close(self):
        if self.h.cublas_handle:
            self.L.coarse_handle_release(C.byref(self.h))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
