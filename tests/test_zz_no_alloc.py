"""The allocation-free exact search entry point (ivf_u8_search_noalloc).

It serves callers that cannot allocate device memory while they answer
queries -- e.g. a database worker with a fixed device-memory budget, or a
latency-critical service that keeps the allocator (and its implicit
synchronisation) off the request path.  The test calls it through the C ABI
twice in a row and checks that both calls return exactly what the ordinary
entry point (ivf_u8_search on the same probe table) returns; integer
distances, so the tolerance is exact equality.  The file is named so that
pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

import insitu_b200 as ib
import oracle
import synth

pytestmark = pytest.mark.gpu


def _reference_search(e, q_u8, probes, k):
    nq, nprobe = probes.shape
    index = ib.Index().load_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], e["centroids"])
    b = ib.Batch(nq, q_u8.shape[1], nprobe, k, len(e["counts"]))
    b.stage1_prepare(q_u8.astype(np.float32))
    b.set_probes(probes)
    b.u8_search(index, nq, nprobe, k, route=False)
    out = b.get_results_i32(nq, k)
    b.close()
    index.close()
    return out


def test_noalloc_matches_ivf_u8_search_twice(cuda_ok):
    n, d, nlist = 40000, 128, 64
    base = synth.mixture_u8(n, d, 64, 12.0, seed=71)
    e = synth.build_u8_index(base, nlist, seed=71, iters=6)
    e["base_cm"][300:1400] = e["base_cm"][299]   # distance ties, broken by original id
    L = ib.load_library(require_device=True)
    index = ib.Index().load_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], e["centroids"])
    stream = torch.cuda.Stream()
    # two calls in a row at k = 10 (the grouped kernel: d = 128, k <= 16), then one at
    # k = 20 (the per-pair kernel); each must equal ivf_u8_search on the same probes
    for call, (nq, nprobe, seed, k) in enumerate([(200, 8, 72, 10), (97, 13, 73, 10), (64, 8, 75, 20)]):
        q = synth.mixture_u8(nq, d, 64, 12.0, seed=71, stream_base=(1 << 20) + seed).numpy()
        probes, _ = oracle.route_l2(q.astype(np.float32), e["centroids"], nprobe)
        exp_ids, exp_dist = _reference_search(e, q, probes, k)
        dq = torch.from_numpy(q).cuda()
        dp = torch.from_numpy(probes).cuda()
        ids = torch.full((nq, k), -7, dtype=torch.int32, device="cuda")
        dist = torch.full((nq, k), -7, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        rc = L.ivf_u8_search_noalloc(index.h, dq.data_ptr(), dp.data_ptr(), nq, nprobe, k, ids.data_ptr(),
                                     dist.data_ptr(), ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, L.ivf_global_last_error().decode()
        assert torch.cuda.current_device() == 0          # the caller's device is left as it was
        stream.synchronize()
        assert np.array_equal(ids.cpu().numpy(), exp_ids), f"call {call}: ids differ"
        assert np.array_equal(dist.cpu().numpy(), exp_dist), f"call {call}: distances differ"
    index.close()


def test_noalloc_rejects_batches_beyond_its_scratch(cuda_ok):
    n, d, nlist = 20000, 64, 16
    base = synth.mixture_u8(n, d, 16, 12.0, seed=74)
    e = synth.build_u8_index(base, nlist, seed=74, iters=4)
    L = ib.load_library(require_device=True)
    index = ib.Index().load_u8(e["base_cm"], e["offsets"], e["counts"], e["r2o"], e["centroids"])
    nq, nprobe, k = 8192, 16, 64      # ~8192 * 16 * 2 chunks * 64 keys * 8 B >> 16 MiB
    dq = torch.zeros((nq, d), dtype=torch.uint8, device="cuda")
    dp = torch.zeros((nq, nprobe), dtype=torch.int32, device="cuda")
    ids = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    dist = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    rc = L.ivf_u8_search_noalloc(index.h, dq.data_ptr(), dp.data_ptr(), nq, nprobe, k, ids.data_ptr(),
                                 dist.data_ptr(), None)
    assert rc == -1 and "scratch" in L.ivf_global_last_error().decode()
    index.close()
