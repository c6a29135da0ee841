#!/usr/bin/env python3
"""bench.py -- build throughput of the B200-native bucketed kNN / CAGRA graph build.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2] [--n N]

Metric: kNN-graph build Mpts/s (points whose final degree-K graph row is built,
per second, whole job).  One step = one full build of the configured synthetic
dataset: k-means on the sample, top-2 bucket assignment, per-bucket all-pairs
tensor-core distances with fused top-M, merge, sanitize, CAGRA detour prune
and reverse-edge merge.  The dataset is resident in HBM when timing starts.

Multi-GPU (torchrun): one global build over all ranks (gta/dist.py).  Each rank
holds N rows of the configured size (rank r: shard r, a mixture of the configured
shape with its own centres) and the bucket count grows with the rank count, so the
per-GPU problem stays the configured one (weak scaling).  k-means sums are
all-reduced, points go to their buckets' owners and lists come back by
all-to-all, and the id tables are all-gathered for the prune (NCCL).  The
job's time is the max over ranks.

--impl reference times the reference's CPU implementation of the path on this
host's cores (the oracle's C restatement of the kNN stages plus the
reference's own compiled prune / reverse-edge code from oracle/_ref), on a
bounded sample of the same workload, extrapolated per stage to the full size.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "gpu-talored-ann_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "kNN-graph build Mpts/s"
UNIT = "Mpts/s"


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _compute_dtype(cfg) -> str:
    """Operand type of the bucket distance kernel: u8 rows with lists of at most 64 run on
    kind::i8 MMAs (int32 accumulation), other 8-bit rows on bf16, f32 rows on a tf32 screen
    with an exact fp32 rerank."""
    if cfg.dtype == "uint8" and cfg.knn_degree <= 64:
        return "u8"
    return "bf16" if cfg.dtype in ("uint8", "int8") else "tf32"


# DRAM bytes (read + write) per algorithmic unit of a kernel, from one ncu capture of each
# kernel on the C2 distribution (bucket distance kernel, u8 operands: N = 600 000; prune:
# N = 400 000), scaled to a launch by its units (the traffic grows with the rows processed)
TRAFFIC_PER_UNIT = {"dist_topk_bucket": 430.70e6 / 3.3754e12, "prune": 139.38e6 / 6.7069e9}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown," \
             "clocks_event_reasons.sw_power_cap"

    def __init__(self, index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(index), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = []
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), float(parts[2]), parts[3:7]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        loaded = [r[0] for r in rows if r[2] > 150.0] or [r[0] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------- CPU pipeline (reference arm / cpu_baseline)
def cpu_pipeline_sample(X: np.ndarray, cfg, seed: int = 42, budget_buckets: int = 2):
    """Times the reference's CPU implementation of every stage on a bounded sample of the
    workload, using all host threads, and extrapolates each stage to the full job.

    k-means / top-2 / per-bucket kNN: the reference's Python CPU path (torch matmul + topk,
    oracle/cpu_port.py); merge: the C restatement of the reference's merge rule (oracle);
    prune + reverse edges: the reference's own C++ code (oracle/_ref) when it was built.
    Returns (seconds for the full job, per-stage detail, sample description)."""
    import torch

    from oracle import cpu_port
    from oracle import oracle as orc

    N, d = X.shape
    B, M, K = cfg.n_buckets, cfg.knn_degree, cfg.graph_degree
    rng = np.random.default_rng(seed)
    threads = torch.get_num_threads()
    detail = {}
    Xt = torch.from_numpy(X.astype(np.float32))
    # k-means: one Lloyd iteration on the k-means sample, times the iteration count
    n_s = cfg.kmeans_sample or orc.default_sample_size(N)
    Xs = Xt[torch.from_numpy(orc.kmeans_sample_ids(N, n_s, seed))]
    C = Xs[:B].clone()
    t = time.perf_counter()
    C = cpu_port.lloyd_step(Xs, C)
    detail["kmeans_s"] = (time.perf_counter() - t) * cfg.kmeans_iters
    # top-2 assignment of every point (measured in full)
    t = time.perf_counter()
    top2, _ = cpu_port.topk_from_A_to_B(Xt, C, 2)
    detail["top2_s"] = time.perf_counter() - t
    sizes = np.bincount(top2.numpy().reshape(-1), minlength=B).astype(np.float64)
    full_cost = float((sizes ** 2).sum())
    # per-bucket kNN on `budget_buckets` median-size buckets, extrapolated by sum(n_b^2)
    order = np.argsort(-sizes)
    pick = order[len(order) // 2: len(order) // 2 + budget_buckets]
    t_knn, cost = 0.0, 0.0
    t2 = top2.numpy()
    for b in pick:
        mem = np.nonzero((t2 == b).any(axis=1))[0]
        if mem.size < 2:
            continue
        Xb = Xt[torch.from_numpy(mem)]
        t = time.perf_counter()
        cpu_port.bucket_knn(Xb, M)
        t_knn += time.perf_counter() - t
        cost += float(mem.size) ** 2
    detail["bucket_knn_s"] = t_knn * full_cost / max(cost, 1.0)
    # merge of each point's two lists (synthetic sorted lists of the real shape)
    nm = min(N, 200_000)
    da = np.sort(rng.random((nm, M), dtype=np.float32), axis=1)
    db = np.sort(rng.random((nm, M), dtype=np.float32), axis=1)
    ia = rng.integers(0, N, (nm, M)).astype(np.int32)
    ib = rng.integers(0, N, (nm, M)).astype(np.int32)
    t = time.perf_counter()
    orc.merge_lists(ia, da, ib, db)
    detail["merge_s"] = (time.perf_counter() - t) * N / nm
    # CAGRA prune + reverse edges on a distance-sorted graph of the real shape
    ng = min(N, 200_000)
    Xg = X[:ng].astype(np.float32)
    base = np.arange(ng)[:, None] + rng.integers(-2000, 2000, (ng, M))
    knn = orc.sort_rows_l2(Xg, np.clip(base, 0, ng - 1).astype(np.int32))
    san, _ = orc.sanitize(knn)
    R = orc.ref_lib()
    out = np.empty((ng, K), np.uint32)
    t = time.perf_counter()
    if R is not None:
        assert R.ref_optimize(orc._p(san), ng, M, K, orc._p(out)) == 0
        kind = "reference"
    else:
        out = orc.optimize(san, K)
        kind = "port"
    detail["prune_reverse_s"] = (time.perf_counter() - t) * N / ng
    detail["prune_impl"] = kind
    total = sum(v for k, v in detail.items() if k.endswith("_s"))
    detail["threads"] = threads
    sample = (f"k-means: 1 of {cfg.kmeans_iters} Lloyd iterations on the {n_s}-point sample (x{cfg.kmeans_iters}); "
              f"top-2 of all {N} points; per-bucket kNN: {len(pick)} median-size buckets, scaled by sum(n_b^2); "
              f"merge: {nm} lists (x{N / nm:g}); prune+reverse ({kind} code): {ng}-row graph (x{N / ng:g})")
    return total, detail, sample


# ---------------------------------------------------------------- main
SEARCH_QUERIES = 2000
SEARCH_SAMPLES = 16384


def exact_knn(Xall, Xq, k: int, exclude=None) -> np.ndarray:
    """Exact k nearest rows of ``Xall`` (device) for each row of ``Xq``, fp64 on the GPU;
    ``exclude[i]`` (a row index of Xall) is left out of query i's answer."""
    import torch

    Xq = Xq.double()
    best = []
    for c0 in range(0, Xall.shape[0], 1 << 18):
        Xc = Xall[c0:c0 + (1 << 18)].double()
        dd = (Xq * Xq).sum(1, keepdim=True) + (Xc * Xc).sum(1)[None, :] - 2.0 * Xq @ Xc.T
        if exclude is not None:
            idx = torch.arange(c0, c0 + Xc.shape[0], device="cuda")
            dd[exclude[:, None] == idx[None, :]] = float("inf")
        v, i = torch.topk(dd, k, dim=1, largest=False)
        best.append((v, i + c0))
    v = torch.cat([b[0] for b in best], 1)
    i = torch.cat([b[1] for b in best], 1)
    return torch.gather(i, 1, torch.topk(v, k, dim=1, largest=False).indices).cpu().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2")
    ap.add_argument("--n", type=int, default=0, help="override N (smaller case, e.g. for profiling)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the graph-search and reference-bucketing measurements (large configs)")
    args = ap.parse_args()

    import gta

    cfg = gta.CONFIGS[args.config]
    if args.n:
        cfg = gta.scaled(cfg, args.n)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    workload = (f"{cfg.name}: N={cfg.n} per GPU x d={cfg.d} {cfg.dtype}, {cfg.n_clusters}-Gaussian mixture, "
                f"B={cfg.n_buckets} buckets per GPU (2-way), M={cfg.knn_degree}, K={cfg.graph_degree}, "
                f"{cfg.kmeans_iters} Lloyd iterations")
    n_buckets_job = cfg.n_buckets * world
    config = {"workload": workload, "n_per_rank": cfg.n, "n_total": cfg.n * world, "d": cfg.d, "dtype": cfg.dtype,
              "n_buckets": n_buckets_job,
              "knn_degree": cfg.knn_degree, "graph_degree": cfg.graph_degree, "kmeans_iters": cfg.kmeans_iters,
              "kmeans_sample": cfg.kmeans_sample or None,
              "l2": "inputs and intermediates larger than L2 (no flush needed)",
              "parallelism": (f"{world} ranks, buckets sharded (NCCL all-reduce / all-to-all / all-gather)"
                              if world > 1 else "1 GPU"),
              "shards": "rank r holds shard r: the configured mixture with its own centres (weak scaling)"}

    if args.impl == "reference":
        if rank != 0:
            return 0
        X = gta.generate(cfg, seed=42)
        per = []
        detail = sample = None
        for s in range(args.warmup + args.steps):
            t, detail, sample = cpu_pipeline_sample(X, cfg)
            if s >= args.warmup:
                per.append(t)
        sec = statistics.mean(per)
        # the CPU pipeline's cost is linear in N at a fixed bucket size, so the whole job's
        # throughput on the host equals that of one shard: value = points / second of CPU work
        value = cfg.n / sec / 1e6
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config, "impl": "reference",
                "cpu_baseline": {"value": value, "unit": UNIT, "cores": detail["threads"],
                                 "kind": "port", "sample": sample, "prune_reverse_code": detail["prune_impl"],
                                 "stages_s": {k: v for k, v in detail.items() if k.endswith("_s")}},
                "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return 0

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    X = gta.generate_shard(cfg, rank, seed=42)
    Xd = torch.from_numpy(X).cuda()
    torch.cuda.synchronize()
    import gta.dist as gd

    prm = gd.ShardParams(n_buckets=n_buckets_job, knn_degree=cfg.knn_degree, graph_degree=cfg.graph_degree,
                         kmeans_iters=cfg.kmeans_iters, kmeans_sample=cfg.kmeans_sample, seed=42)
    last = {}

    def step(Xin=Xd):
        if world == 1:
            return gta.build_cagra(Xin, cfg.n_buckets, cfg.knn_degree, cfg.graph_degree, cfg.kmeans_iters,
                                   cfg.kmeans_sample, 42)
        res = gd.build_sharded(Xin, prm)
        last["res"] = res
        return res.graph

    for _ in range(args.warmup):
        g = step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches0 = gta._lib.launch_count()
    sampler = ClockSampler(local_rank)
    gta._lib.profile_enable(True)
    st = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(st)
    for _ in range(args.steps):
        g = step()
    ev1.record(st)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    launches = gta._lib.launch_count() - launches0
    ms = ev0.elapsed_time(ev1) / args.steps
    recs = gta._lib.profile_records()
    gta._lib.profile_enable(False)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = cfg.n * world / (ms / 1e3) / 1e6

    # per-stage device time inside the timed steps
    stages = {}
    for name, t_ms, units, cnt in recs:
        s = stages.setdefault(name, {"ms": 0.0, "units": 0.0, "launches": 0, "counters": [0.0] * 8})
        s["ms"] += t_ms
        s["units"] += units
        s["launches"] += 1
        s["counters"] = [a + b for a, b in zip(s["counters"], cnt)]
    hbm, tflops, peak_src = _peaks()
    # the bucket distance kernel runs as one launch per phase (lower-bucket rows, then the seeded
    # higher-bucket rows): one kernel for the roofline
    roof = {}
    for k, v in stages.items():
        r = roof.setdefault("dist_topk_bucket" if k.startswith("dist_topk_bucket") else k,
                            {"ms": 0.0, "units": 0.0, "launches": 0})
        r["ms"] += v["ms"]
        r["units"] += v["units"]
        r["launches"] += v["launches"]
    kernels = [k for k in roof if not k.endswith("_total") and roof[k]["units"] > 0]
    dom = max(kernels, key=lambda k: roof[k]["ms"]) if kernels else None
    roofline = None
    if dom:
        s = roof[dom]
        per_launch_units = s["units"] / s["launches"]
        per_launch_s = s["ms"] / s["launches"] / 1e3
        if dom.startswith("dist_topk"):
            achieved = per_launch_units / per_launch_s / 1e12
            roofline = {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": tflops, "unit": "TFLOP/s",
                        "frac": achieved / tflops, "peak_source": f"{peak_src} bf16 burst"}
            if _compute_dtype(cfg) == "u8":
                roofline["note"] = ("kind::i8 MMAs: operations per second against the measured bf16 burst "
                                    "(no measured i8 peak; the nominal dense i8 rate is twice bf16)")
        else:
            achieved = per_launch_units / per_launch_s / 1e9
            roofline = {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                        "frac": achieved / hbm, "peak_source": f"{peak_src} HBM copy"}
        tpu = TRAFFIC_PER_UNIT.get(dom)
        roofline["traffic"] = tpu * per_launch_units if tpu else None
    step_ms_sum = sum(s["ms"] for k, s in stages.items() if not k.endswith("_total")) / args.steps
    stage_summary = {k: {"ms_per_step": v["ms"] / args.steps, "launches_per_step": v["launches"] / args.steps,
                         "share": v["ms"] / args.steps / ms} for k, v in sorted(stages.items(), key=lambda kv: -kv[1]["ms"])}
    for k, v in stages.items():
        if k.startswith("dist_topk"):
            stage_summary[k]["tflops"] = v["units"] / (v["ms"] / 1e3) / 1e12
            rows = max(v["counters"][2], 1.0)
            stage_summary[k]["list_passes_per_row"] = v["counters"][0] / rows
            stage_summary[k]["list_merges_per_row_group"] = v["counters"][1] * 32.0 / rows
            c = v["counters"]
            if c[5] > 0:
                stage_summary[k]["epilogue_share_waiting_acc"] = c[3] / c[5]
                stage_summary[k]["epilogue_share_merging"] = c[4] / c[5]
                stage_summary[k]["epilogue_cycles_per_warp"] = c[5] / (rows / 32.0)
                stage_summary[k]["mma_wait_acc_vs_epilogue"] = c[6] / c[5] * 4.0
                stage_summary[k]["mma_wait_full_vs_epilogue"] = c[7] / c[5] * 4.0
        elif v["units"] > 0:
            stage_summary[k]["gbs"] = v["units"] / (v["ms"] / 1e3) / 1e9

    # bucket balance (k-means leaves buckets skewed; the bucket stage costs sum n_b^2) and, on
    # several GPUs, the device time of each phase of one more (untimed) build
    skew = phases = None
    if world == 1:
        _, _, _, t2 = gta.build_bucket(Xd, cfg.n_buckets, cfg.knn_degree, cfg.kmeans_iters, cfg.kmeans_sample, 42,
                                       with_extras=True)
        sizes = torch.bincount(t2.reshape(-1).long(), minlength=cfg.n_buckets).double()
    else:
        res = gd.build_sharded(Xd, prm, timing=True)
        sizes = torch.tensor(res.sizes, dtype=torch.float64)
        phases = {k: round(v, 3) for k, v in res.phase_ms.items()}
        t = torch.tensor([phases[k] for k in phases], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        phases = {k: round(float(v), 3) for k, v in zip(phases, t.tolist())}
    skew = {"max_bucket": int(sizes.max()), "sum_sq_over_balanced": float((sizes * sizes).sum() * sizes.numel()
                                                                         / sizes.sum() ** 2)}

    # quality: recall@32 of the pre-prune kNN graph on 1000 sampled points of rank 0's rows
    # (exact GT over the whole job's dataset in fp64 on the GPU)
    recall = None
    if world == 1:
        ids, _ = gta.build_bucket(Xd, cfg.n_buckets, cfg.knn_degree, cfg.kmeans_iters, cfg.kmeans_sample, 42)
        Xall = Xd
    else:
        ids = last["res"].knn_ids
        Xall = torch.empty((cfg.n * world, cfg.d), dtype=Xd.dtype, device="cuda")
        dist.all_gather_into_tensor(Xall, Xd)
    if world > 1:
        g_all = torch.empty((cfg.n * world, cfg.graph_degree), dtype=g.dtype, device="cuda")
        dist.all_gather_into_tensor(g_all, g.contiguous())
    else:
        g_all = g
    search_q = None
    if rank == 0:
        q = torch.from_numpy(np.random.default_rng(0).choice(cfg.n, 1000, replace=False)).cuda()
        gt = exact_knn(Xall, Xall[q], 32, exclude=q)
        approx = ids[q].cpu().numpy()[:, :32]
        recall = float(np.mean([len(np.intersect1d(approx[r], gt[r])) / 32.0 for r in range(1000)]))
    if rank == 0 and not args.no_extras:
        # graph search over the final graph with the reference search's defaults
        # (topk 10, ef 200, 4 random entry points, seed 42) on held-out queries
        Q = torch.from_numpy(gta.generate_queries(cfg, SEARCH_QUERIES)).cuda()
        gt10 = exact_knn(Xall, Q, 10)
        search_q = {"queries": int(Q.shape[0]), "topk": 10, "ef": 200, "num_entry": 4,
                    "queries_from": "held-out rows of the same mixture"}
        # (1) the reference's entry rule: 4 uniform random rows per query; (2) the 4 nearest of
        # SEARCH_SAMPLES seeded random rows (random-sampling seeding).  The synthetic mixture's
        # clusters are far apart, so the graph has one component per cluster and (1) only
        # finds the query's cluster when an entry happens to fall in it.
        ent_ref = gta.search_entries(Xall.shape[0], Q.shape[0], 4, 42)
        samp = torch.from_numpy(np.random.default_rng(7).choice(Xall.shape[0], SEARCH_SAMPLES, replace=False)).cuda()
        ent_smp = samp[torch.from_numpy(exact_knn(Xall[samp], Q, 4)).cuda()].int().cpu().numpy()
        for tag, ent in (("reference_entries", ent_ref), ("sampled_entries", ent_smp)):
            gta.search(Xall, g_all, Q, 10, 200, entries=ent)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            sid, _ = gta.search(Xall, g_all, Q, 10, 200, entries=ent)
            e1.record()
            torch.cuda.synchronize()
            sid = sid.cpu().numpy()
            search_q[tag] = {"recall_at_10": float(np.mean([len(np.intersect1d(sid[r], gt10[r])) / 10.0
                                                            for r in range(Q.shape[0])])),
                             "qps": Q.shape[0] / (e0.elapsed_time(e1) / 1e3)}
        search_q["sampled_entries"]["samples"] = SEARCH_SAMPLES
    # the reference tool's own bucketing (KMeans||, balanced 1-way, own + nprobe pools) on the same
    # data: device time of one build and recall@32 of its lists on the same sampled points
    ref_bucketing = None
    if world == 1 and rank == 0 and not args.no_extras:
        gta.build_bucket2(Xd, cfg.knn_degree, 32, 0.01, 42)  # warm-up
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        rids, _ = gta.build_bucket2(Xd, cfg.knn_degree, 32, 0.01, 42)
        e1.record()
        torch.cuda.synchronize()
        rms = e0.elapsed_time(e1)
        approx = rids[q].cpu().numpy()[:, :32]
        ref_bucketing = {"centroid_ratio": 0.01, "nprobe": 32, "ms": rms, "value": cfg.n / (rms / 1e3) / 1e6,
                         "unit": UNIT, "recall_at_32": float(np.mean([len(np.intersect1d(approx[r], gt[r])) / 32.0
                                                                      for r in range(1000)])),
                         "stage": "kNN lists only (no CAGRA optimize)"}
    del Xall, g_all

    # end to end with host buffers (pinned), copies inside the timed region: through the C ABI
    # (gta_build_cagra) on one GPU, through the sharded build on several
    e2e = None
    if not args.no_e2e:
        Xh = torch.from_numpy(X).pin_memory()
        gh_t = torch.empty((cfg.n, cfg.graph_degree), dtype=torch.int32).pin_memory()
        gh = gh_t.numpy().view(np.uint32)
        from gta import _lib as L
        import ctypes

        def step_host():
            if world > 1:
                g = step(Xh.to("cuda", non_blocking=True))
                gh_t.copy_(g, non_blocking=True)
                torch.cuda.current_stream().synchronize()
                return
            Xn = Xh.numpy()
            ds = L.gta_dataset(data=Xn.ctypes.data_as(ctypes.c_void_p), n=cfg.n, d=cfg.d,
                               dtype=L.GTA_U8 if cfg.dtype == "uint8" else L.GTA_F32, metric=0, on_device=0)
            bp = L.gta_bucket_params(n_buckets=cfg.n_buckets, kmeans_iters=cfg.kmeans_iters, knn_degree=cfg.knn_degree,
                                     rounds=1, kmeans_sample=cfg.kmeans_sample, seed=42, init_centroids=None,
                                     init_on_device=0, out_on_device=0, centroids_out=None, top2_out=None)
            p = L.gta_cagra_params(bucket=bp, graph_degree=cfg.graph_degree, reserved0=0)
            L.check(L.lib().gta_build_cagra(ctypes.byref(ds), ctypes.byref(p), gh.ctypes.data_as(ctypes.c_void_p), None))

        step_host()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step_host()
        torch.cuda.synchronize()
        e2e_s = (time.perf_counter() - t0) / args.steps
        if world > 1:
            t = torch.tensor([e2e_s], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        e2e = {"value": cfg.n * world / e2e_s / 1e6, "unit": UNIT, "ms_per_step": e2e_s * 1e3,
               "h2d_bytes_per_step": int(X.nbytes), "d2h_bytes_per_step": int(gh.nbytes),
               "path": "gta_build_cagra (C ABI, host buffers)" if world == 1 else "gta.dist.build_sharded"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        sec, detail, sample = cpu_pipeline_sample(X, cfg)
        cpu = {"value": cfg.n / sec / 1e6, "unit": UNIT, "cores": detail["threads"], "kind": "port",
               "sample": sample, "stages_s": {k: round(v, 4) for k, v in detail.items() if k.endswith("_s")},
               "prune_reverse_code": detail["prune_impl"]}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": _compute_dtype(cfg),
                "data": "synthetic (seeded Gaussian mixture)", "config": config, "roofline": roofline,
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
                "clocks": clocks, "recall_at_32": recall, "search": search_q, "reference_bucketing": ref_bucketing, "bucket_skew": skew, "phases_ms_max_over_ranks": phases,
                "stages": stage_summary,
                "instrumented_ms_per_step": step_ms_sum}
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
