"""Cluster-sharded multi-GPU exchange for the IVF query path.

The reference searches on one GPU only (updates/pq_update.cu:676); this module
is the host side of the sharded path: inverted lists are placed on ranks by
bytes (LPT), and one query batch moves through three collectives:

  1. every rank's local routing keys (distance bits << 32 | global list id,
     [nq, nprobe], sorted) are all-gathered, so every rank can form the
     global top-nprobe (ivf_route_merge_shards reads the all-gather layout);
  2. every rank's per-query stage-1 lists (ADC key, exact key) are sent to the
     rank that owns the query (block partition of the batch) with one
     all-to-all, and the owner merges them (ivf_pq_merge_shards);
  3. the owners' top-k are all-gathered, one int64 per result
     ((distance bits << 32) | id, gather_results_packed).

The phased protocol (ivf_pq_shard_* entry points) replaces step 2 by:

  2a. after every shard has scanned each query's nearest probe, the per-query
      rank-R bounds are reduced with an int64 minimum (exchange_bounds) and
      every shard scans the other probes with the global bound;
  2b. the stage-1 lists go to the owners (to_owners_raw); each owner computes
      kappa, the R-th smallest key of the union, and the owners' kappas are
      all-gathered (kappa_to_shards);
  2c. each shard reranks its keys <= kappa and sends its exact top-k to the
      owners (to_owners_raw), which merge them.

The functions take torch tensors and a process group, so the same code runs
over NCCL with device tensors (bench.py) and over gloo with CPU tensors
(tests/test_shard_gloo.py).
"""
from __future__ import annotations

import numpy as np


def lpt_shards(counts: np.ndarray, row_bytes: int, n_shards: int) -> np.ndarray:
    """Owner rank of every list: longest-processing-time placement by bytes."""
    order = np.argsort(-(np.asarray(counts, np.int64) * row_bytes), kind="stable")
    load = np.zeros(n_shards, np.int64)
    owner = np.empty(len(counts), np.int32)
    for l in order:
        s = int(np.argmin(load))
        owner[l] = s
        load[s] += int(counts[l]) * row_bytes
    return owner


def shard_rows(offsets: np.ndarray, counts: np.ndarray, lists: np.ndarray):
    """Rows (cluster-major positions) of the given lists and their local offsets."""
    rows = np.concatenate([np.arange(offsets[l], offsets[l] + counts[l], dtype=np.int64) for l in lists]) \
        if len(lists) else np.zeros(0, np.int64)
    cnt = np.asarray(counts)[lists].astype(np.int32)
    off = np.zeros(len(lists), np.int64)
    if len(lists):
        off[1:] = np.cumsum(cnt, dtype=np.int64)[:-1]
    return rows, off, cnt


def gather_route_keys(dist, keys_local, keys_all):
    """keys_local [nq, nprobe] -> [nq, world * nprobe] (contiguous), via all-gather.

    keys_all is the receive buffer, [world * nq, nprobe] (ranks concatenated)."""
    nq, nprobe = keys_local.shape
    dist.all_gather_into_tensor(keys_all, keys_local)
    return keys_all.reshape(-1, nq, nprobe).permute(1, 0, 2).contiguous().reshape(nq, -1)


def to_owners(dist, world, per_query, recv):
    """per_query [nq, R] (nq = world * qo, block-partitioned) -> owners' [qo, world * R]."""
    nq, R = per_query.shape
    qo = nq // world
    dist.all_to_all_single(recv, per_query.reshape(world, qo, R))  # recv [world (source), qo, R]
    return recv.permute(1, 0, 2).contiguous().reshape(qo, world * R)


def gather_results(dist, ids_local, dist_local, ids_all, dist_all):
    """owners' [qo, k] results -> [world * qo, k] on every rank (buffers [world * qo, k])."""
    dist.all_gather_into_tensor(ids_all, ids_local)
    dist.all_gather_into_tensor(dist_all, dist_local)
    return ids_all.reshape(-1, ids_local.shape[1]), dist_all.reshape(-1, dist_local.shape[1])


def gather_results_packed(dist, ids_local, dist_local, packed_local, packed_all):
    """owners' [qo, k] results -> [world * qo, k] on every rank with one
    all-gather: each result travels as (distance bits << 32) | id (int64)."""
    import torch

    packed_local.copy_((dist_local.view(torch.int32).to(torch.int64) << 32) |
                       (ids_local.to(torch.int64) & 0xFFFFFFFF))
    dist.all_gather_into_tensor(packed_all, packed_local)
    return packed_all


def unpack_results(packed):
    """int64 (distance bits << 32) | id -> (ids int32, distances float32), NumPy"""
    p = np.asarray(packed, np.int64)
    ids = (p & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
    dd = ((p >> 32) & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return ids, dd


def exchange_bounds(dist, bounds):
    """bounds [nq] int64 (no bound: INT64_MAX) -> elementwise minimum over ranks, in place."""
    dist.all_reduce(bounds, op=dist.ReduceOp.MIN)
    return bounds


def to_owners_raw(dist, world, per_query, recv):
    """per_query [nq, R] (nq = world * qo, block-partitioned) -> recv [world (source), qo, R]."""
    nq, R = per_query.shape
    dist.all_to_all_single(recv, per_query.reshape(world, nq // world, R))
    return recv


def kappa_to_shards(dist, kappa_owned, kappa_all):
    """each owner's key limits [qo] (int64) -> every shard's [world * qo] in global query order."""
    dist.all_gather_into_tensor(kappa_all, kappa_owned)
    return kappa_all
