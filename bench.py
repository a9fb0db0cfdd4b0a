#!/usr/bin/env python3
"""Benchmark of the IVF residual-PQ query hot path (BASELINE.json configs[2] by default).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c0|c1|c2|...]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...

Workload c2 (the largest single-GPU config of BASELINE.json): 100M x 128 uint8
vectors from a seeded 65536-component Gaussian mixture (centers U[32,224],
sigma 10), nlist 65536, residual PQ M=32 x 8 bit trained on a 500k sample, 10k
queries from the same mixture, k=10, rerank_n=512 with uint8 rerank.  A step
is one pass of the hot path over the 10k-query batch: routing, probe
inversion, ADC scan, top-R selection, exact rerank, top-k.

Index build (not timed): every rank generates the seeded rows itself
(counter-based generators), rank 0 runs k-means and trains the codebook, the
assignment is split over the ranks, and each rank keeps and encodes only the
lists it owns (LPT by bytes), so nothing of the index is broadcast.

N>1: inverted lists are sharded over the ranks; every rank routes over its own
centroids, the local routing keys are all-gathered and merged, each rank scans
its own lists (nearest probe first, then the others under the exchanged
bounds), the stage-1 lists go to the owners of the queries, the owners find
the rank-R key limit, each shard reranks its keys below it and the owners
merge the shards' exact top-k (the phased protocol in include/insitu_b200.h).
Total work is fixed, so "scaling" is "strong".

--impl reference times the reference's own CPU kernel
(cuda/search/cpu_fine/cpu_fine_kernels_pq_resid.cpp, compiled unmodified into
oracle/_ref) on the host cores, on samples of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(ROOT, "insituann-opensource_b200"), os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "QPS @ recall@10≥0.9 vs nprobe; scanned GB/s vs 8 TB/s HBM; at 1/2/4/8 B200"

CONFIGS = {
    # the exact uint8 path (ivf_u8_search); one GPU
    "c0": dict(kind="u8", n=1_000_000, d=128, ncomp=1024, sigma=12.0, nlist=1024, nq=10_000, k=10, nprobe=32,
               seed=20260600, train_n=0, M=0, rerank_n=0, sweep=(32,),
               desc="c0: exact IVF, 1M x 128 uint8 (1024-comp mixture, centers U[32,224], sigma 12), nlist 1024, "
                    "10k queries, nprobe 32, k=10, exact int32 L2"),
    # BASELINE.json configs[1]
    # nprobe: the smallest sweep point whose recall@10 is >= 0.9 on this data (0.99998 measured at 8)
    "c1": dict(kind="f32", n=10_000_000, d=96, ncomp=4096, sigma=0.05, nlist=4096, M=48, train_n=500_000,
               nq=10_000, k=10, rerank_n=512, nprobe=8, sweep=(8, 16, 32, 64, 128), seed=20260601,
               desc="c1: residual-PQ IVF, 10M x 96 fp32 unit-norm (4096-comp mixture, sigma 0.05), nlist 4096, "
                    "M=48 x 8b, 10k queries, k=10, rerank_n=512 (fp32 rerank)"),
    # BASELINE.json configs[2] on one GPU: 100M x 128 uint8, residual PQ M=32 (dsub 4), uint8 rerank
    "c2": dict(kind="pq_u8", n=100_000_000, d=128, ncomp=65536, sigma=10.0, nlist=65536, M=32, train_n=500_000,
               nq=10_000, k=10, rerank_n=512, nprobe=16, sweep=(16, 32, 64, 128, 256), seed=20260602,
               desc="c2: residual-PQ IVF, 100M x 128 uint8 (65536-comp mixture, centers U[32,224], sigma 10), "
                    "nlist 65536, M=32 x 8b, 10k queries, k=10, rerank_n=512 (uint8 rerank)"),
    # 1B x 128 uint8 with Zipf(1.1) component weights, nlist 262144, sharded
    # over the GPUs (run it with --gpus 8); k-means on a 4.2M-row sample, 10 iterations
    "c3": dict(kind="pq_u8", n=1_000_000_000, d=128, ncomp=262144, sigma=10.0, zipf=1.1, nlist=262144, M=32,
               train_n=500_000, nq=10_000, k=10, rerank_n=512, nprobe=32, sweep=(32, 64, 128), seed=20260603,
               kmeans_iters=10, kmeans_sample=16 * 262144,
               desc="c3: residual-PQ IVF, 1B x 128 uint8 (262144-comp mixture, Zipf(1.1) weights, sigma 10), "
                    "nlist 262144, M=32 x 8b, 10k queries, k=10, rerank_n=512 (uint8 rerank), lists sharded",
               # Zipf-skewed lists (the largest about 10x the mean after k-means) need larger
               # candidate buffers for a whole 10k-query batch in one sub-batch
               scratch_mb=65536),
    # c3's shapes (Zipf(1.1) weights, nlist 262144, nprobe 32) at 100M rows: a 2-GPU check of c3's path
    "c3-small": dict(kind="pq_u8", n=100_000_000, d=128, ncomp=262144, sigma=10.0, zipf=1.1, nlist=262144, M=32,
                     train_n=500_000, nq=10_000, k=10, rerank_n=512, nprobe=32, sweep=(32,), seed=20260603,
                     kmeans_iters=6, kmeans_sample=8 * 262144, scratch_mb=49152,
                     desc="c3 shapes at 100M rows (Zipf(1.1), nlist 262144)"),
    # c2 at a tenth of the rows (the c2 list count and shapes): a quick check of the c2 path
    "c2-small": dict(kind="pq_u8", n=10_000_000, d=128, ncomp=65536, sigma=10.0, nlist=65536, M=32,
                     train_n=500_000, nq=10_000, k=10, rerank_n=512, nprobe=16, sweep=(16,), seed=20260602,
                     kmeans_iters=6, kmeans_sample=16 * 65536,
                     desc="c2 shapes at 10M rows (quick checks)"),
    # c2-shaped lists (about 1526 vectors each, 2.4 probing queries per list at nprobe 16) at a
    # tenth of the rows and queries: the scan's per-group work equals c2's (profiling case)
    "c2-mid": dict(kind="pq_u8", n=10_000_000, d=128, ncomp=6554, sigma=10.0, nlist=6554, M=32,
                   train_n=500_000, nq=1000, k=10, rerank_n=512, nprobe=16, sweep=(16,), seed=17,
                   desc="c2-shaped lists at 10M rows, 1k queries (profiling case)"),
    # the c2 routing shape (10k queries, 65536 centroids, d 128, nprobe 16) over 1M rows:
    # the routing kernels' work equals c2's (profiling case for the routing kernels)
    "c2-route": dict(kind="pq_u8", n=1_000_000, d=128, ncomp=65536, sigma=10.0, nlist=65536, M=32,
                     train_n=200_000, nq=10_000, k=10, rerank_n=512, nprobe=16, sweep=(16,), seed=19,
                     kmeans_iters=4, kmeans_sample=16 * 65536,
                     desc="c2 routing shape over 1M rows (profiling case)"),
    # c1-shaped lists (about 2440 vectors each) at a size small enough for a full ncu capture
    "c1-mid": dict(kind="f32", n=1_000_000, d=96, ncomp=410, sigma=0.05, nlist=410, M=48, train_n=200_000,
                   nq=2000, k=10, rerank_n=512, nprobe=32, sweep=(32,), seed=11,
                   desc="c1-shaped lists at 1M vectors (profiling case)"),
    # the c1 routing shape (10k queries, 4096 centroids, d 96, nprobe 8) over 1M
    # vectors: the routing kernels' work equals c1's, the device holds ~1.5 GB
    # (profiling case for the routing kernels)
    "c1-route": dict(kind="f32", n=1_000_000, d=96, ncomp=4096, sigma=0.05, nlist=4096, M=48, train_n=200_000,
                     nq=10_000, k=10, rerank_n=512, nprobe=8, sweep=(8,), seed=13,
                     desc="c1 routing shape over 1M vectors (profiling case)"),
    # reduced copy for quick checks of the harness itself (not a bench line)
    "c1-small": dict(kind="f32", n=400_000, d=96, ncomp=512, sigma=0.05, nlist=512, M=48, train_n=100_000,
                     nq=2000, k=10, rerank_n=512, nprobe=16, sweep=(8, 16, 32), seed=7,
                     desc="reduced c1 for harness checks"),
}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        j = json.load(open(path))
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """8-bit dense tensor peak: twice the measured dense bf16 burst rate."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        j = json.load(open(path))
        return 2.0 * float(j["bf16_tflops"]), "measured bf16 burst x 2 (kind::i8 rate)"
    return 2.0 * 1590.0, "fallback bf16 x 2 (kind::i8 rate)"


class Clocks:
    """nvidia-smi sampling during the timed region (SM clock and throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "samples": len(rows), "reasons": reasons}


def clock_soak(step, sync, seconds=1.0, dist=None, dev=None):
    """Untimed steps of the same work, run under the clock sampler right before
    the timed region: nvidia-smi samples every 100 ms, so a timed region of a
    few hundred ms alone would give it one or two samples.  Every rank runs the
    same number of steps (the maximum over ranks), since a step may hold
    collectives."""
    sync()
    t0 = time.perf_counter()
    step()
    sync()
    dt = time.perf_counter() - t0
    n = min(200, max(0, int(seconds / max(dt, 1e-4)) + 1))
    if dist is not None:
        import torch

        t = torch.tensor([n], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        n = int(t.item())
    for _ in range(n):
        step()
    sync()


# ----------------------------------------------------------------------------
# workload
# ----------------------------------------------------------------------------
def pq_build(cfg, dev, rank=0, world=1, dist=None):
    """Seeded data, this rank's lists of the residual-PQ index, and the exact
    ground truth over all ranks' rows (all outside any timed region)."""
    import torch

    import synth

    t0 = time.time()
    kind = "u8" if cfg["kind"] == "pq_u8" else "f32"
    src = synth.RowSource(kind, cfg["n"], cfg["d"], cfg["ncomp"], cfg["sigma"], cfg["seed"], dev,
                          zipf=cfg.get("zipf"))
    qsrc = synth.RowSource(kind, cfg["nq"], cfg["d"], cfg["ncomp"], cfg["sigma"], cfg["seed"], dev,
                           zipf=cfg.get("zipf"), stream_base=1 << 30)
    q = qsrc.rows(0, cfg["nq"]).float()

    def say(what):
        if rank == 0:
            log(f"[bench] {what} {time.time() - t0:.1f}s")
    builder = None
    if dev.type == "cuda":
        import insitu_b200 as ib

        builder = ib.Builder(cfg["d"], batch_rows=65536)     # the library's GPU index build
    b = synth.build_pq_shard(src, cfg["nlist"], cfg["M"], cfg["seed"], rank, world, dist,
                             kmeans_iters=cfg.get("kmeans_iters", 20), pq_iters=12, train_n=cfg["train_n"],
                             kmeans_sample=cfg.get("kmeans_sample", 64 * cfg["nlist"]), log=say, builder=builder)
    keys = synth.gt_keys(b["base_rr"], q, cfg["k"], ids=b["r2o"])
    if world > 1:
        allk = torch.empty(world * keys.numel(), dtype=keys.dtype, device=dev)
        dist.all_gather_into_tensor(allk, keys.reshape(-1))
        keys = allk.reshape((world,) + tuple(keys.shape))
    b["gt"] = synth.merge_gt_keys(keys, cfg["k"])
    say("ground truth")
    b["q"] = q
    b["q_np"] = q.cpu().numpy()
    torch.cuda.empty_cache()
    return b


def host_index(b):
    """Host copy of a whole index (one rank owns every list) for the CPU oracle and baselines."""
    return dict(centroids=b["centroids"].cpu().numpy(), codebook=b["codebook"].cpu().numpy(),
                codes=b["codes"].cpu().numpy(), offsets=b["offsets_global"], counts=b["counts_global"],
                r2o=b["r2o"].cpu().numpy(), base_rr=b["base_rr"].cpu().numpy())


def gather_lists(b, needed, rank, world, dist, dev):
    """Rank 0 receives the codes, rerank rows and ids of the lists `needed`
    (sorted global ids) from the ranks that own them and returns a host index
    that holds those lists alone, in increasing global order (so cluster-major
    positions keep their relative order and ties break as in the whole index);
    the other lists are empty.  Other ranks return None."""
    import torch

    my = b["my_lists"]
    pos = np.searchsorted(my, needed)
    own = (pos < len(my)) & (my[np.minimum(pos, max(len(my) - 1, 0))] == needed) if len(my) else \
        np.zeros(len(needed), bool)
    loc = pos[own]
    rows = (np.concatenate([np.arange(b["offsets"][l], b["offsets"][l] + b["counts"][l], dtype=np.int64)
                            for l in loc]) if len(loc) else np.zeros(0, np.int64))
    it = torch.from_numpy(rows).to(dev)
    part = [torch.from_numpy(needed[own].astype(np.int32)).to(dev), b["codes"][it].contiguous(),
            b["base_rr"][it].contiguous(), b["r2o"][it].contiguous()]
    sz = torch.tensor([int(own.sum()), len(rows)], dtype=torch.int64, device=dev)
    allsz = torch.empty(world * 2, dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(allsz, sz)
    allsz = allsz.reshape(world, 2).cpu().numpy()
    parts = [part] if rank == 0 else None
    for r in range(1, world):
        nl, nr = int(allsz[r, 0]), int(allsz[r, 1])
        if nl == 0:
            continue
        if rank == r:
            for t in part:
                dist.send(t, dst=0)
        elif rank == 0:
            recv = [torch.empty(nl, dtype=torch.int32, device=dev),
                    torch.empty((nr,) + tuple(part[1].shape[1:]), dtype=part[1].dtype, device=dev),
                    torch.empty((nr,) + tuple(part[2].shape[1:]), dtype=part[2].dtype, device=dev),
                    torch.empty(nr, dtype=torch.int32, device=dev)]
            for t in recv:
                dist.recv(t, src=r)
            parts.append(recv)
    if rank != 0:
        return None
    lists = np.concatenate([p[0].cpu().numpy() for p in parts])
    codes = torch.cat([p[1] for p in parts]).cpu().numpy()
    rr = torch.cat([p[2] for p in parts]).cpu().numpy()
    r2o = torch.cat([p[3] for p in parts]).cpu().numpy()
    cnt_g = b["counts_global"]
    src_off = np.zeros(len(lists), np.int64)
    src_off[1:] = np.cumsum(cnt_g[lists], dtype=np.int64)[:-1]
    order = np.argsort(lists, kind="stable")
    idx = (np.concatenate([np.arange(src_off[i], src_off[i] + cnt_g[lists[i]], dtype=np.int64) for i in order])
           if len(order) else np.zeros(0, np.int64))
    counts = np.zeros(len(cnt_g), np.int32)
    counts[lists] = cnt_g[lists]
    offsets = np.zeros(len(cnt_g), np.int64)
    offsets[1:] = np.cumsum(counts, dtype=np.int64)[:-1]
    return dict(centroids=b["centroids"].cpu().numpy(), codebook=b["codebook"].cpu().numpy(), codes=codes[idx],
                offsets=offsets, counts=counts, r2o=r2o[idx], base_rr=rr[idx])


def rr_kw(rows):
    """rerank rows as the loaders and the oracle take them: uint8 or fp32 by dtype."""
    return {"base_u8": rows} if rows.dtype == np.uint8 else {"base_f32": rows}


def algorithmic_bytes(probes, counts, M):
    """codes bytes scanned: sum over (query, probed list) of count * M, the code bytes every probe must read."""
    p = probes[(probes >= 0)]
    return int(counts[p].astype(np.int64).sum()) * M


# ----------------------------------------------------------------------------
# reference arm / CPU baseline
# ----------------------------------------------------------------------------
def time_reference(idx, q, probes, cfg, target_s, max_queries, stock=True):
    """Times oracle/_ref (the reference's cpu_fine_kernel_pq_resid) on a query sample.

    The sample (at most max_queries queries, with their probe lists) is searched
    repeatedly until about target_s seconds of CPU work have been timed.
    stock: the reference's own compiler flags (else the build that pins the oracle)."""
    import oracle

    L = oracle.ref_lib(stock)
    if L is None:
        return None
    threads = os.cpu_count() or 1
    kw = dict(rerank_n=cfg["rerank_n"], threads=threads, stock=stock, **rr_kw(idx["base_rr"]))
    args = (idx["centroids"], idx["codebook"], idx["codes"], idx["offsets"], idx["counts"])
    S = min(max_queries, q.shape[0])
    if idx["base_rr"].dtype == np.uint8:
        kw["q_u8"] = oracle.make_query_u8(q[:S])
    kw64 = dict(kw, q_u8=kw["q_u8"][:min(S, 64)]) if "q_u8" in kw else kw
    oracle.ref_pq_resid(*args, q[:min(S, 64)], probes[:min(S, 64)], cfg["k"], **kw64)   # warm-up
    done, dt, ids = 0, 0.0, None
    while dt < target_s:
        t = time.perf_counter()
        ids, _, _, _ = oracle.ref_pq_resid(*args, q[:S], probes[:S], cfg["k"], **kw)
        dt += time.perf_counter() - t
        done += S
    return dict(qps=done / dt, seconds=dt, sample=done, distinct=S, threads=threads,
                lib=os.path.basename(L.library_path), local_ids=ids)


def build_workload_u8(cfg, device):
    """c0: seeded uint8 data, exact index, exact ground truth (outside any timed region)."""
    import torch

    import synth

    t0 = time.time()
    base = synth.mixture_u8(cfg["n"], cfg["d"], cfg["ncomp"], cfg["sigma"], cfg["seed"], device=device)
    q = synth.mixture_u8(cfg["nq"], cfg["d"], cfg["ncomp"], cfg["sigma"], cfg["seed"], device=device,
                         stream_base=1 << 30)
    idx = synth.build_u8_index(base, cfg["nlist"], cfg["seed"], iters=20, kmeans_sample=64 * cfg["nlist"])
    log(f"[bench] c0 data + index {time.time() - t0:.1f}s")
    gt = synth.brute_force_gt(base, q, cfg["k"], batch_rows=1 << 16)
    del base
    torch.cuda.empty_cache()
    return idx, q.float().cpu().numpy(), gt


def time_reference_u8(idx, q, probes, cfg, target_s, stock=True):
    """Times oracle/_ref's cpu_fine_kernel_v3_u8_touched (all threads) on the batch, repeated to ~target_s."""
    import oracle

    L = oracle.ref_lib(stock)
    if L is None:
        return None
    threads = os.cpu_count() or 1
    qu = oracle.make_query_u8(q)
    oracle.ref_exact_u8_touched(idx["base_cm"], idx["offsets"], idx["counts"], qu[:64], probes[:64], cfg["k"],
                                threads=threads, stock=stock)
    done, dt, ids = 0, 0.0, None
    while dt < target_s:
        t = time.perf_counter()
        ids, _ = oracle.ref_exact_u8_touched(idx["base_cm"], idx["offsets"], idx["counts"], qu, probes, cfg["k"],
                                             threads=threads, stock=stock)
        dt += time.perf_counter() - t
        done += q.shape[0]
    return dict(qps=done / dt, seconds=dt, sample=done, threads=threads, lib=os.path.basename(L.library_path),
                local_ids=ids)


def run_exact(args, cfg):
    """c0 on one GPU: ivf_u8_search (routing, probe inversion, exact scan, top-k) over a resident batch."""
    import torch

    import insitu_b200 as ib
    import oracle
    import synth

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"metric": METRIC, "unavailable": "config c0 is a single-GPU bench line"}))
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    nq, d, k, nlist = cfg["nq"], cfg["d"], cfg["k"], cfg["nlist"]
    nprobe = args.nprobe or cfg["nprobe"]
    idx, q_np, gt = build_workload_u8(cfg, dev)
    index = ib.Index().load_u8(idx["base_cm"], idx["offsets"], idx["counts"], idx["r2o"], idx["centroids"])
    batch = ib.Batch(nq, d, nprobe, k, nlist)
    ext = torch.cuda.ExternalStream(batch.stream, device=dev)
    q_dev = torch.from_numpy(q_np).to(dev)

    def step():
        batch.stage1_prepare_device(q_dev.data_ptr(), nq)
        batch.u8_search(index, nq, nprobe, k, route=True)

    step()
    batch.sync()
    ids_g, dist_g = batch.get_results(nq, k)
    probes = batch.get_probes(nq, nprobe)
    P = min(args.parity_queries, nq)
    exp_p, _ = oracle.route_l2_par(q_np[:P], idx["centroids"], nprobe)
    oi, od = oracle.exact_u8(idx["base_cm"], idx["offsets"], idx["counts"], idx["r2o"],
                             oracle.make_query_u8(q_np[:P]), exp_p, k)
    parity = bool(np.array_equal(probes[:P], exp_p) and np.array_equal(ids_g[:P], oi)
                  and np.array_equal(dist_g[:P], od.astype(np.float32)))
    recall = synth.recall_at_k(ids_g, gt, k)
    log(f"[bench] c0 parity({P} queries vs oracle)={parity} recall@10={recall:.4f}")
    for _ in range(args.warmup):
        step()
    batch.sync()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(0) as clk:
        clock_soak(step, batch.sync)
        batch.profile(True)
        launches0 = ib.kernel_launches()
        torch.cuda.synchronize()
        ev0.record(ext)
        for _ in range(args.steps):
            step()
        ev1.record(ext)
        torch.cuda.synchronize()
    launches = ib.kernel_launches() - launches0
    stage = batch.stage_ms()
    batch.profile(False)
    ms_step = ev0.elapsed_time(ev1) / args.steps
    value = nq / (ms_step / 1000.0)
    # e2e: pinned host queries in, host results out, through the C ABI
    hq = torch.from_numpy(q_np).pin_memory()
    h_ids = torch.empty((nq, k), dtype=torch.int32).pin_memory()
    h_dist = torch.empty((nq, k), dtype=torch.float32).pin_memory()

    def e2e_step():
        batch.stage1_prepare_ptr(hq.data_ptr(), nq)
        batch.u8_search(index, nq, nprobe, k, route=True)
        batch.get_results_into(h_dist.data_ptr(), h_ids.data_ptr(), nq, k)

    for _ in range(args.warmup):
        e2e_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e_ms = (time.perf_counter() - t0) * 1000.0 / args.steps
    e2e = {"value": nq / (e_ms / 1000.0), "unit": "queries/s", "h2d_bytes_per_step": int(nq * d * 4),
           "d2h_bytes_per_step": int(nq * k * 8)}
    # roofline of the exact scan: sum over (query, probed list) of count * d
    p = probes[probes >= 0]
    bytes_search = int(idx["counts"][p].astype(np.int64).sum()) * d
    scan_ms = stage["scan"] / args.steps
    # the exact kernel multiplies query tiles by row tiles on the tensor cores (kind::i8):
    # its roofline is the 8-bit tensor rate, 2 ops per byte of a scanned row (one
    # multiply-add with the query's byte); the measured dense bf16 rate doubled is
    # that rate's peak (kind::i8 issues twice the MACs of kind::f16 per cycle)
    tpeak, tpeak_kind = tensor_peak()
    achieved = 2.0 * bytes_search / (scan_ms / 1000.0) / 1e12
    traffic = None
    # the grouped exact search runs on the tensor cores unless INSITU_EXACT_TC=0
    kname = "exact_group_kernel" if os.environ.get("INSITU_EXACT_TC", "1").startswith("0") else "exact_tc_kernel"
    prof_path = os.path.join(ROOT, "profiles", f"{kname}_c0_nprobe{nprobe}.md")
    if os.path.exists(prof_path):
        for line in open(prof_path):
            if line.startswith("dram_bytes_per_search:"):
                traffic = int(line.split(":")[1].strip())
    if kname == "exact_group_kernel":      # CUDA cores (dp4a): rows streamed per query group
        peak, peak_kind = peaks()
        gbs = bytes_search / (scan_ms / 1000.0) / 1e9
        roofline = {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                    "traffic": traffic, "kernel": f"{kname} (d = 128; 2 launches per search)",
                    "peak_source": peak_kind, "algorithmic_bytes_per_launch": bytes_search,
                    "kernel_ms_per_launch": scan_ms}
    else:
        roofline = {"bound": "tensor", "achieved": achieved, "peak": tpeak, "unit": "TFLOP/s",
                    "frac": achieved / tpeak, "traffic": traffic,
                    "kernel": f"{kname} (d = 128; 2 launches per search; u8 multiply-add = 2 ops)",
                    "peak_source": tpeak_kind, "algorithmic_ops_per_launch": 2 * bytes_search,
                    "algorithmic_bytes_per_launch": bytes_search, "kernel_ms_per_launch": scan_ms,
                    "scanned_gbs": bytes_search / (scan_ms / 1000.0) / 1e9}
    cpu = None
    if not args.no_cpu_baseline:
        S = 2048
        r = time_reference_u8(idx, q_np[:S], probes[:S], cfg, target_s=12.0)
        r2 = time_reference_u8(idx, q_np[:S], probes[:S], cfg, target_s=4.0, stock=False)
        if r is not None:
            cpu = {"value": r["qps"], "unit": "queries/s", "cores": r["threads"], "kind": "reference",
                   "sample": f"{r['sample']} query searches ({S} distinct queries of the batch, repeated) with "
                             f"reference cpu_fine_kernel_v3_u8_touched ({r['lib']}: the reference's flags -O3 "
                             f"-ffast-math -funroll-loops, AVX-512), probe lists given, {r['seconds']:.1f}s",
                   "without_fast_math": None if r2 is None else {"value": r2["qps"], "lib": r2["lib"]}}
    out = {
        "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": cfg["desc"], "n_base": cfg["n"], "d": d, "nlist": nlist, "nq": nq,
                   "nprobe": nprobe, "k": k, "recall@10": recall, "recall_target_met": bool(recall >= 0.9),
                   "parity_vs_oracle": parity, "parity_queries": P, "inputs_exceed_l2": True,
                   "l2_note": "the 128 MB of vectors are probed 320k times per step (40 GB logical)",
                   "parallelism": "single GPU"},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches),
        "clocks": clk.summary(), "stages_ms_per_step": {s_: v / args.steps for s_, v in stage.items()},
        "sweep": [],
    }
    print(json.dumps(out), flush=True)
    batch.close()
    index.close()


def run_reference_arm(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    import oracle

    if oracle.ref_lib() is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref was not built (needs the reference tree)"}))
        return
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    if cfg["kind"] == "u8":                    # c0: the reference's exact CPU kernel on the whole batch
        import synth

        idx, q, gt = build_workload_u8(cfg, dev)
        nprobe = args.nprobe or cfg["nprobe"]
        probes, _ = oracle.route_l2(q, idx["centroids"], nprobe)
        times, samples = [], []
        for step in range(args.warmup + args.steps):
            r = time_reference_u8(idx, q, probes, cfg, target_s=4.0)
            if step >= args.warmup:
                times.append(r["seconds"])
                samples.append(r["sample"])
        qps = sum(samples) / sum(times)
        rec = synth.recall_at_k(idx["r2o"][r["local_ids"]], gt, cfg["k"])
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": {"workload": cfg["desc"], "nprobe": nprobe, "k": cfg["k"], "recall@10": rec,
                       "routing": "not timed (probe lists from the exact fp32 router)"},
            "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": r["threads"], "kind": "reference",
                             "sample": f"{samples[-1]} query searches per step (the {cfg['nq']}-query batch, "
                                       f"repeated), cpu_fine_kernel_v3_u8_touched ({r['lib']})"},
            "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return
    b = pq_build(cfg, dev)
    idx, q, gt = host_index(b), b["q_np"], b["gt"]
    del b
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    nprobe = args.nprobe or cfg["nprobe"]
    probes, _ = oracle.route_l2_par(q, idx["centroids"], nprobe)
    times, samples = [], []
    for step in range(args.warmup + args.steps):
        r = time_reference(idx, q, probes, cfg, target_s=4.0, max_queries=cfg["nq"])
        if step >= args.warmup:
            times.append(r["seconds"])
            samples.append(r["sample"])
    qps = sum(samples) / sum(times)
    ids = idx["r2o"][r["local_ids"]]
    import synth

    rec = synth.recall_at_k(ids, gt[:ids.shape[0]], cfg["k"])
    out = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sum(times) / len(times),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg["desc"], "nprobe": nprobe, "k": cfg["k"], "rerank_n": cfg["rerank_n"],
                   "recall@10": rec, "routing": "not timed (probe lists from the exact fp32 router)"},
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": r["threads"], "kind": "reference",
                         "sample": f"{samples[-1]} query searches per step ({r['distinct']} distinct queries of "
                                   f"the {cfg['nq']}-query batch), cpu_fine_kernel_pq_resid stage 1 + fp32 "
                                   f"rerank ({r['lib']})"},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--parity-queries", type=int, default=1000,
                    help="queries of the batch checked against the CPU oracle (ids, distances and probes)")
    ap.add_argument("--nprobe", type=int, default=0)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--overlay", default="auto",
                    help="also time the search with published delta segments of these sizes, e.g. "
                         "1000000,5000000,10000000 (BASELINE configs[4]; 1 GPU); 'auto' (default): "
                         "those three on c2 at N=1, none otherwise; 'none' for none")
    ap.add_argument("--overlay-nprobe", default="64",
                    help="nprobe values of the overlay runs (BASELINE configs[4]: 64)")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference_arm(args, cfg)
    if cfg["kind"] == "u8":
        return run_exact(args, cfg)

    import torch
    import torch.distributed as dist

    import insitu_b200 as ib
    import oracle
    import shard
    import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    N = world
    if N > 1:
        # the phased sharded search keeps a whole 10k-query batch in one
        # sub-batch; at c2 its candidate buffers pass the 6 GB default scratch
        os.environ.setdefault("INSITU_SCRATCH_MB", str(cfg.get("scratch_mb", 24576)))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if N > 1:
        from datetime import timedelta

        # NCCL logs to stdout by default; rank 0's stdout must be the JSON line alone
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    nq, d, k, R, M = cfg["nq"], cfg["d"], cfg["k"], cfg["rerank_n"], cfg["M"]
    nlist = cfg["nlist"]
    nprobe = args.nprobe or cfg["nprobe"]

    # ---- workload: every rank builds its own lists (nothing of the index is broadcast) ----
    W = pq_build(cfg, dev, rank, N, dist if N > 1 else None)
    my_lists, gt, q_np = W["my_lists"], W["gt"], W["q_np"]
    counts, offsets = W["counts_global"], W["offsets_global"]
    q_dev = W["q"].contiguous()
    rr_u8 = W["base_rr"].dtype == torch.uint8
    rr_bytes = W["base_rr"].element_size()

    # ---- load this rank's lists (device tensors are copied device to device) ----
    R, k = cfg["rerank_n"], cfg["k"]
    index = ib.Index()
    cent_np = W["centroids"].cpu().numpy()
    cb_np = W["codebook"].cpu().numpy()
    rr_arg = {"base_u8": W["base_rr"]} if rr_u8 else {"base_f32": W["base_rr"]}
    index.load_pq(cent_np[my_lists], cb_np, W["codes"], W["offsets"], W["counts"], W["r2o"], **rr_arg)
    if N > 1:
        index.set_shard(nlist, my_lists, offsets[my_lists])
    # the oracle's view: the whole index on rank 0 when one GPU holds it
    idx = host_index(W) if (N == 1 and rank == 0) else None
    codes_mb = W["codes"].numel() / 1e6 * N
    rr_gb = W["base_rr"].numel() * rr_bytes / 1e9 * N
    del rr_arg
    if N == 1:
        del W["codes"], W["base_rr"]      # sharded runs keep them until the oracle check gathered its lists
    torch.cuda.empty_cache()
    batch = ib.Batch(nq, d, max(nprobe, max(cfg["sweep"])), k, nlist)
    ext = torch.cuda.ExternalStream(batch.stream, device=dev)

    # ---- one step of the hot path ----
    if N > 1:
        assert nq % N == 0, "nq must divide by the GPU count"
        qo = nq // N
        keys_l = torch.empty((nq, nprobe), dtype=torch.int64, device=dev)
        keys_all = torch.empty((N * nq, nprobe), dtype=torch.int64, device=dev)
        adc = torch.empty((nq, R), dtype=torch.int64, device=dev)
        topk = torch.empty((nq, k), dtype=torch.int64, device=dev)
        adc_r = torch.empty((N, qo, R), dtype=torch.int64, device=dev)
        topk_r = torch.empty((N, qo, k), dtype=torch.int64, device=dev)
        kappa_o = torch.empty((qo,), dtype=torch.int64, device=dev)
        kappa_all = torch.empty((nq,), dtype=torch.int64, device=dev)

        class _DevArray:              # a library-owned device array seen as a torch tensor (no copy)
            def __init__(self, ptr, n):
                self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i8", "data": (ptr, False),
                                                 "version": 3}
        out_ids = torch.empty((qo, k), dtype=torch.int32, device=dev)
        out_dist = torch.empty((qo, k), dtype=torch.float32, device=dev)
        own_packed = torch.empty((qo, k), dtype=torch.int64, device=dev)
        all_packed = torch.empty((N * qo, k), dtype=torch.int64, device=dev)

    def step(np_=nprobe, marks=None):
        batch.stage1_prepare_device(q_dev.data_ptr(), nq)
        if N == 1:
            batch.pq_search(index, nq, np_, k, rerank_n=R, overlay=False, route=True)
            return

        def mark(name):               # CUDA events between the phases of one step (diagnostics)
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(ext)
                marks.append((name, ev))
        with torch.cuda.stream(ext):
            mark("start")
            batch.route_keys(index, nq, np_, keys_l.data_ptr())
            mark("route")
            dist.all_gather_into_tensor(keys_all, keys_l)
            mark("gather keys")
            batch.route_merge_shards(keys_all.data_ptr(), N, nq, np_)
            mark("route merge")
            # nearest probes, global bounds, the other probes
            batch.pq_shard_scan(index, nq, np_, R, 0)
            mark("scan nearest")
            bounds = torch.as_tensor(_DevArray(batch.pq_shard_bounds(), nq), device=dev)
            shard.exchange_bounds(dist, bounds)
            mark("exchange bounds")
            batch.pq_shard_scan(index, nq, np_, R, 1)
            mark("scan rest")
            batch.pq_shard_select(index, nq, np_, R, adc.data_ptr())
            mark("select")
            shard.to_owners_raw(dist, N, adc, adc_r)
            mark("stage 1 to owners")
            batch.pq_shard_kappa(adc_r.data_ptr(), N, qo, R, kappa_o.data_ptr())
            shard.kappa_to_shards(dist, kappa_o, kappa_all)
            mark("kappa")
            batch.pq_shard_rerank(index, nq, R, adc.data_ptr(), kappa_all.data_ptr(), k, topk.data_ptr())
            mark("rerank")
            shard.to_owners_raw(dist, N, topk, topk_r)
            mark("top-k to owners")
            batch.pq_shard_final(topk_r.data_ptr(), N, qo, k, rr_u8)    # uint8 rerank: int32 distances
            batch.get_results_device(out_dist.data_ptr(), out_ids.data_ptr(), qo, k)
            mark("final")
            shard.gather_results_packed(dist, out_ids, out_dist, own_packed, all_packed)
            mark("gather results")

    def results():
        if N == 1:
            return batch.get_results(nq, k)
        torch.cuda.synchronize()
        return shard.unpack_results(all_packed.reshape(nq, k).cpu().numpy())

    def barrier():
        torch.cuda.synchronize()
        batch.sync()
        if N > 1:
            dist.barrier()

    # ---- per-phase times of one sharded step (INSITU_BENCH_PHASES=1, stderr) ----
    if N > 1 and os.environ.get("INSITU_BENCH_PHASES") == "1":
        for _ in range(3):
            step()
        marks = []
        step(marks=marks)
        torch.cuda.synchronize()
        log(f"[bench] rank {rank} phases (ms): " + ", ".join(
            f"{marks[i][0]} {marks[i - 1][1].elapsed_time(marks[i][1]):.3f}" for i in range(1, len(marks))))

    # ---- recall sweep over nprobe (untimed) ----
    sweep = []
    if not args.no_sweep:
        for np_ in cfg["sweep"]:
            if N > 1 and np_ != nprobe:
                continue  # the sharded step keeps buffers for the headline nprobe only
            step(np_)
            ids, _ = results()
            rec = synth.recall_at_k(ids, gt, k) if rank == 0 else None
            step(np_)                 # buffers for this nprobe are in place after the first step
            barrier()
            reps = 5
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(ext)
            for _ in range(reps):
                step(np_)
            s1.record(ext)
            barrier()
            ms = s0.elapsed_time(s1)
            if N > 1:
                t = torch.tensor([ms], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            dt = ms / 1000.0 / reps
            sweep.append({"nprobe": np_, "recall@10": rec, "qps": nq / dt})
            if rank == 0:
                log(f"[bench] nprobe {np_}: recall@10 {rec} qps {nq / dt:.0f}")

    # ---- parity against the CPU oracle on the first P queries of the batch (untimed):
    # probe lists, result ids and distances, and (one GPU) the stage-1 keys ----
    step()
    ids_g, dist_g = results()
    probes_g = batch.get_probes(nq, nprobe)
    barrier()
    P = min(args.parity_queries, nq)
    s1_g = None
    if N == 1:
        adc_d = torch.empty((P, R), dtype=torch.int64, device=dev)
        exa_d = torch.empty((P, R), dtype=torch.int64, device=dev)
        batch.pq_search_shard(index, P, nprobe, R, 0, adc_d.data_ptr(), exa_d.data_ptr())
        batch.sync()
        s1_g = adc_d.cpu().numpy().view(np.uint64)
        del adc_d, exa_d
    needed = [None]
    probes_o = None
    t_par = time.time()
    if rank == 0:
        probes_o, _ = oracle.route_l2_par(q_np[:P], cent_np, nprobe)
        needed = [np.unique(probes_o[probes_o >= 0]).astype(np.int64)]
    if N > 1:
        dist.broadcast_object_list(needed, src=0)
    oidx = idx if N == 1 else gather_lists(W, needed[0], rank, N, dist, dev)
    parity, parity_detail = None, None
    if rank == 0:
        oi, od, s1_o, _ = oracle.pq_search_par(oidx["centroids"], oidx["codebook"], oidx["codes"], oidx["offsets"],
                                               oidx["counts"], oidx["r2o"], q_np[:P], probes_o, k, rerank_n=R,
                                               return_stage1=True, **rr_kw(oidx["base_rr"]))
        ok_p = bool(np.array_equal(probes_g[:P], probes_o))
        ok_i = bool(np.array_equal(oi, ids_g[:P]))
        ok_d = bool(np.array_equal(od, dist_g[:P]))
        ok_s = None if s1_g is None else bool(np.array_equal(np.sort(s1_g, axis=1), np.sort(s1_o, axis=1)))
        bad = ~((oi == ids_g[:P]).all(1) & (od == dist_g[:P]).all(1))
        parity = ok_p and ok_i and ok_d and (ok_s is not False)
        parity_detail = {"queries": P, "probes_equal": ok_p, "ids_equal": ok_i, "distances_equal": ok_d,
                         "stage1_keys_equal": ok_s, "queries_differing": int(bad.sum())}
        log(f"[bench] parity({P} queries vs oracle)={parity} {parity_detail} "
            f"recall@10={synth.recall_at_k(ids_g, gt, k):.4f} ({time.time() - t_par:.1f}s)")
    # ---- routing against the reference's own coarse_search (cuBLAS SGEMM, norm expansion) on
    # the same P queries, when that build is present: how many probe sets differ, and the
    # recall@10 of the search run on the reference's probe lists instead of this library's ----
    route_vs_ref = None
    if N == 1 and rank == 0 and oracle.ref_coarse_lib() is not None:
        rp = oracle.ref_coarse_search(cent_np, q_np[:P], nprobe)
        diff = ~(np.sort(rp, axis=1) == np.sort(probes_g[:P], axis=1)).all(1)
        batch.stage1_prepare_device(q_dev.data_ptr(), P)
        batch.set_probes(rp)
        batch.pq_search(index, P, nprobe, k, rerank_n=R, overlay=False, route=False)
        ids_r, _ = batch.get_results(P, k)
        rec_own = synth.recall_at_k(ids_g[:P], gt[:P], k)
        rec_ref = synth.recall_at_k(ids_r, gt[:P], k)
        route_vs_ref = {"queries": P, "probe_sets_differing": int(diff.sum()),
                        "recall@10_own_probes": rec_own, "recall@10_reference_probes": rec_ref,
                        "recall_delta": rec_own - rec_ref}
        log(f"[bench] routing vs reference coarse_search: {route_vs_ref}")
    del oidx
    if N > 1:
        del W["codes"], W["base_rr"]
        torch.cuda.empty_cache()
    barrier()

    # ---- timed region ----
    for _ in range(args.warmup):
        step()
    barrier()
    probes_all = batch.get_probes(nq, nprobe) if N == 1 else None
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        clock_soak(step, barrier, dist=dist if N > 1 else None, dev=dev)
        batch.profile(True)
        launches0 = ib.kernel_launches()
        barrier()
        ev0.record(ext)
        for _ in range(args.steps):
            step()
        ev1.record(ext)
        barrier()
    launches = ib.kernel_launches() - launches0
    stage = batch.stage_ms()
    batch.profile(False)
    ms_total = ev0.elapsed_time(ev1)
    if N > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps
    value = nq / (ms_step / 1000.0)
    clocks = clk.summary()

    # ---- e2e through the public C ABI with host buffers ----
    e2e = None
    hq = torch.from_numpy(q_np).pin_memory()
    h_ids = torch.empty((nq, k), dtype=torch.int32).pin_memory()
    h_dist = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    h_packed = torch.empty((nq, k), dtype=torch.int64).pin_memory() if N > 1 else None

    # N = 1: two batch contexts in flight, as the reference's pipeline API is
    # meant to be driven -- while the host waits for one batch's results
    # (ivf_pipeline_get_results copies them and synchronises that batch's
    # stream), the next batch's upload and search are already queued on the
    # other context's stream.  Every step still uploads its queries from pinned
    # host memory and reads its results back to the host.
    batches = [batch, ib.Batch(nq, d, max(nprobe, max(cfg["sweep"])), k, nlist)] if N == 1 else [batch]

    def e2e_issue(b):
        b.stage1_prepare_ptr(hq.data_ptr(), nq)
        b.pq_search(index, nq, nprobe, k, rerank_n=R, overlay=False, route=True)

    def e2e_run(n):
        if N == 1:
            e2e_issue(batches[0])
            for i in range(n):
                if i + 1 < n:
                    e2e_issue(batches[(i + 1) % 2])
                batches[i % 2].get_results_into(h_dist.data_ptr(), h_ids.data_ptr(), nq, k)
            return
        for _ in range(n):
            with torch.cuda.stream(ext):
                q_dev.copy_(hq, non_blocking=True)
            step()
            if rank == 0:
                with torch.cuda.stream(ext):
                    h_packed.copy_(all_packed.reshape(nq, k), non_blocking=True)
            ext.synchronize()

    e2e_run(args.warmup)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    e2e_run(args.steps)
    e1.record(ext)
    barrier()
    e_ms = e0.elapsed_time(e1)
    if N == 1:
        # both contexts searched the same queries: their results must agree
        ids_b, _ = batches[1].get_results(nq, k)
        if not np.array_equal(ids_b, h_ids.numpy()):
            raise RuntimeError("the two batch contexts of the e2e pipeline returned different results")
        batches[1].close()
    if N > 1:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e = {"value": nq / (e_ms / args.steps / 1000.0), "unit": "queries/s",
           "h2d_bytes_per_step": int(nq * d * 4 * N), "d2h_bytes_per_step": int(nq * k * 8)}

    # ---- update overlay (BASELINE configs[4] style): a published delta segment of
    # seeded uniform codes (the reference's generators), ids after the base, scanned in
    # the same launches as the main lists; QPS with and without it ----
    overlay = None
    ov_arg = str(args.overlay)
    if ov_arg == "auto":
        ov_arg = "1000000,5000000,10000000" if args.config == "c2" else ""
    sizes = [int(x) for x in ov_arg.split(",") if x and x != "none" and int(x) > 0]
    if sizes and N == 1:
        def ostep(np_, ov):
            batch.stage1_prepare_device(q_dev.data_ptr(), nq)
            batch.pq_search(index, nq, np_, k, rerank_n=R, overlay=ov, delta_topk=16, route=True)

        def timed(np_, ov):
            for _ in range(args.warmup):
                ostep(np_, ov)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            batch.profile(True)
            e0.record(ext)
            for _ in range(args.steps):
                ostep(np_, ov)
            e1.record(ext)
            torch.cuda.synchronize()
            st = {s_: round(v / args.steps, 4) for s_, v in batch.stage_ms().items()}
            batch.profile(False)
            return nq / (e0.elapsed_time(e1) / args.steps / 1000.0), st

        onp = sorted({int(x) for x in str(args.overlay_nprobe).split(",") if x})
        base = {np_: timed(np_, False) for np_ in onp}
        base_qps = {np_: v[0] for np_, v in base.items()}
        runs = []
        for nd in sizes:
            t_g = time.time()
            dseg = synth.delta_segment(nd, nlist, M, base_id=cfg["n"], d=d, seed=cfg["seed"] + 1,
                                       f32=idx["base_rr"].dtype != np.uint8)
            raw = {"raw_f32": dseg["raw_f32"]} if "raw_f32" in dseg else {"raw_u8": dseg["raw_u8"]}
            index.publish_delta(dseg["codes"], dseg["ids"], dseg["counts"], dseg["offsets"], **raw)
            log(f"[bench] delta segment of {nd} vectors published in {time.time() - t_g:.1f}s")
            ostep(64, True)
            batch.sync()
            oid, odd = batch.get_results(nq, k)
            Po = min(P, nq, 500)
            po, _ = oracle.route_l2_par(q_np[:Po], idx["centroids"], 64)
            ei, ed = oracle.pq_search_par(idx["centroids"], idx["codebook"], idx["codes"], offsets, counts,
                                          idx["r2o"], q_np[:Po], po, k, rerank_n=R, delta=dseg, delta_topk=16,
                                          **rr_kw(idx["base_rr"]))
            o_par = bool(np.array_equal(ei, oid[:Po]) and np.array_equal(ed, odd[:Po]))
            for np_ in onp:
                qw, st_w = timed(np_, True)
                # the delta's share of the scanned bytes: delta rows over all rows of the probed lists
                pr = batch.get_probes(nq, np_)
                dsum = float(dseg["counts"][pr].sum())
                share = dsum / (dsum + float(counts[pr].sum()))
                mode = index.delta_mode()          # how the library searches this delta
                runs.append({"delta_vectors": nd, "nprobe": np_, "delta_search": mode,
                             "qps_without": base_qps[np_], "qps_with": qw,
                             "overhead": 1.0 - qw / base_qps[np_], "delta_share_of_scanned": share,
                             "overhead_within_share_plus_5pct": bool(1.0 - qw / base_qps[np_] <= share + 0.05),
                             "stages_ms_without": base[np_][1], "stages_ms_with": st_w,
                             "parity_vs_oracle": o_par, "parity_queries": Po})
                log(f"[bench] overlay {nd}: nprobe {np_}: {base_qps[np_]:.0f} -> {qw:.0f} qps "
                    f"(delta share {share:.3f}), parity {o_par}; stages {base[np_][1]} -> {st_w}")
            index.clear_delta()
            del dseg, raw
        overlay = {"delta_topk": 16, "runs": runs}

    # ---- roofline of the ADC scan kernel (this rank) ----
    if probes_all is None:
        probes_all = batch.get_probes(nq, nprobe)
    mine = np.zeros(nlist, bool)
    mine[my_lists] = True
    p = probes_all.copy()
    p[(p >= 0) & ~mine[np.clip(p, 0, nlist - 1)]] = -1
    bytes_per_launch = algorithmic_bytes(p, counts, M)
    bytes_total = algorithmic_bytes(probes_all, counts, M)
    scan_ms = stage["scan"] / args.steps
    peak, peak_kind = peaks()
    achieved = bytes_per_launch / (scan_ms / 1000.0) / 1e9
    traffic = None
    prof_path = os.path.join(ROOT, "profiles", f"pq_stagger_kernel_{args.config}_nprobe{nprobe}.md")
    if os.path.exists(prof_path) and N == 1:
        for line in open(prof_path):
            if line.startswith("dram_bytes_per_search:"):
                traffic = int(line.split(":")[1].strip())
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": traffic, "kernel": f"pq_stagger_kernel<{M},{d // M}> (2 launches per search)",
                "peak_source": peak_kind,
                "algorithmic_bytes_per_launch": bytes_per_launch, "kernel_ms_per_launch": scan_ms}

    cpu = None
    if rank == 0 and N == 1 and not args.no_cpu_baseline:
        probes_o, _ = oracle.route_l2_par(q_np[:4096], idx["centroids"], nprobe)
        r = time_reference(idx, q_np[:4096], probes_o, cfg, target_s=12.0, max_queries=4096)
        r2 = time_reference(idx, q_np[:4096], probes_o, cfg, target_s=4.0, max_queries=4096, stock=False)
        if r is not None:
            cpu = {"value": r["qps"], "unit": "queries/s", "cores": r["threads"], "kind": "reference",
                   "sample": f"{r['sample']} query searches ({r['distinct']} distinct queries of the batch, "
                             f"repeated) with reference cpu_fine_kernel_pq_resid (stage 1 + "
                             f"{'uint8' if idx['base_rr'].dtype == np.uint8 else 'fp32'} rerank, "
                             f"{r['lib']}: the reference's flags -O3 -ffast-math -funroll-loops, AVX-512), "
                             f"probe lists given, {r['seconds']:.1f}s",
                   "without_fast_math": None if r2 is None else {"value": r2["qps"], "lib": r2["lib"]}}

    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": N, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfg["desc"], "n_base": cfg["n"], "d": d, "nlist": nlist, "M": M,
                       "nq": nq, "nprobe": nprobe, "k": k, "rerank_n": R,
                       "recall@10": synth.recall_at_k(ids_g, gt, k), "recall_target_met": bool(
                           synth.recall_at_k(ids_g, gt, k) >= 0.9), "parity_vs_oracle": parity,
                       "parity_detail": parity_detail, "routing_vs_reference": route_vs_ref,
                       "inputs_exceed_l2": True,
                       "l2_note": f"{codes_mb:.0f} MB of codes and {rr_gb:.2f} GB of rerank rows per step",
                       "parallelism": "single GPU" if N == 1 else f"lists sharded x{N} (LPT by bytes), NCCL"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches),
            "clocks": clocks, "stages_ms_per_step": {s: v / args.steps for s, v in stage.items()},
            "gbs_scanned_logical": bytes_total / (ms_step / 1000.0) / 1e9,
            "sweep": sweep,
            "overlay": overlay,
        }
        print(json.dumps(out), flush=True)
    torch.cuda.synchronize()
    if N > 1:
        # tensors that took part in collectives on the batch stream keep references to it
        # until the interpreter frees them, so that stream must outlive them: the batch
        # context is left to process exit
        dist.barrier()
        dist.destroy_process_group()
        return
    batch.close()
    index.close()


if __name__ == "__main__":
    main()
