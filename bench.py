#!/usr/bin/env python3
"""bench.py -- build throughput of the B200-native bucketed kNN / CAGRA graph build.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c3] [--n N]

Metric: kNN-graph build Mpts/s (points whose final degree-K graph row is built,
per second, whole job).  One step = one full build of the configured synthetic
dataset: k-means on the sample, top-2 bucket assignment, per-bucket all-pairs
tensor-core distances with fused top-M, merge, sanitize, CAGRA detour prune
and reverse-edge merge.  The dataset is resident in HBM when timing starts.

Multi-GPU (torchrun): one global build over all ranks (gta/dist.py) of the same
configured dataset (one seeded mixture, N rows, B buckets): rank r holds its
contiguous block of about N/W rows (strong scaling: the job is fixed, W grows).
k-means sums are all-reduced, buckets are placed on ranks by their cost n_b^2,
points go to their buckets' owners and lists come back by all-to-all, and the id
tables are all-gathered for the prune (NCCL).  The job's time is the max over
ranks; value = N / that time.

Default workload: C3 (1M x 960 f32, B=256, M=128 -> K=64), the largest single-GPU
configuration and the one dominated by the distance contraction: its bucket stage
runs the tensor-core screen (fp16 hi/lo parts, kind::f16) and the exact fp32
rerank.  After the timed steps (outside them) the line carries a parity block: the
build's own kNN lists of 500 sampled points against the oracle pipeline's lists at
full size (a checker, never timed).

--impl reference times the reference's CPU implementation of the path on this
host's cores: torch-CPU restatements of build_bucket.py's k-means++, Lloyd, top-2
and per-bucket kNN, the oracle's C merge, the reference's own compiled CAGRA prune
/ reverse-edge code from oracle/_ref, and prune.py's Python occlusion prune
(reported beside them, a different rule).  Each stage runs on a bounded sample
scaled to the whole job (the scaled stages listed in `extrapolated`); --full runs
every stage whole (C1 / C2 sizes).
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
    """(HBM GB/s, bf16 burst TFLOP/s, bf16 sustained TFLOP/s, source)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return (float(p["hbm_gbs"]), float(p["bf16_tflops"]),
                float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def _compute_dtype(cfg) -> str:
    """Operand type of the bucket distance kernel: u8 rows with lists of at most 64 run on
    kind::i8 MMAs (int32 accumulation), other exact 8-bit rows on bf16, float rows on the
    fp16 screen with an exact fp32 rerank: one fp16 part per element for d >= 256 ("f16"; a wave
    falls back to the hi/lo split when it rescans too many rows), the hi/lo split (three kind::f16
    products per element, "f16x3") below."""
    if cfg.dtype == "uint8" and cfg.knn_degree <= 64 and cfg.d <= 129:
        return "u8"
    if cfg.dtype in ("uint8", "int8") and cfg.d <= 129:
        return "bf16"
    return "f16" if cfg.d >= 256 else "f16x3"


# DRAM bytes (read + write) per launch of the dominant stage's kernel, averaged over the launches
# of one build, from the committed one-pass ncu launch list of the same command and workload
# (`dram__bytes_read.sum + dram__bytes_write.sum`, profiles/launches_*.md):
# {(stage, config, N, unseeded rows on the split screen): (bytes per launch, source)}.
TRAFFIC_PER_LAUNCH = {
    ("dist_topk_bucket", "c3", 1000000, False): (2.104e10, "profiles/launches_c3_bench.md"),
}


def _unseeded_split() -> bool:
    """The library's screen option for rows without a seed (on unless GTA_SCREEN_UNSEEDED_SPLIT=0)."""
    return not os.environ.get("GTA_SCREEN_UNSEEDED_SPLIT", "").startswith("0")


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
def cpu_info() -> dict:
    import torch

    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count(), "torch_threads": torch.get_num_threads(),
            "omp_num_threads": os.environ.get("OMP_NUM_THREADS")}


def cpu_reference(X: np.ndarray, cfg, seed: int = 42, full: bool = False):
    """Times the reference's CPU implementation of every stage on this host's cores (all threads)
    and returns per-stage seconds for the WHOLE job.  full=True runs every stage on the whole
    workload (C1 / C2 sizes); otherwise each stage runs on a bounded sample (a few seconds in
    all) and is scaled to the whole job, the scaled stages listed in `extrapolated`.

      k-means++      cpu_port.kmeans_pp_centers  (build_bucket.py:189, whole pool of min(N, 20 B))
      Lloyd          cpu_port.lloyd_step x iters (build_bucket.py:232, on the k-means sample)
      top-2          cpu_port.topk_from_A_to_B(X, C, 2) (build_bucket.py:96)
      bucket kNN     cpu_port.bucket_knn per bucket (build_bucket.py:602-628), cost ~ sum n_b^2
      merge          the oracle's C restatement of the resident merge (bucket.cu:5025)
      CAGRA prune + reverse edges: the reference's own C++ (prune_windowed_core.hpp +
                     edge_chunk_accumulator.hpp via oracle/_ref), else the oracle's restatement
      occlusion prune: cpu_port.prune_graph (prune.py:8, the reference's Python prune -- a
                     different rule, reported beside the CAGRA total, not inside it)
    """
    import torch

    from oracle import cpu_port
    from oracle import oracle as orc

    N, d = X.shape
    B, M, K = cfg.n_buckets, cfg.knn_degree, cfg.graph_degree
    rng = np.random.default_rng(seed)
    st, share = {}, {}
    Xt = torch.from_numpy(np.ascontiguousarray(X, dtype=np.float32))

    def timed(fn):
        t = time.perf_counter()
        out = fn()
        return out, time.perf_counter() - t

    (_, C), st["kmeans_pp_s"] = timed(lambda: cpu_port.kmeans_pp_centers(Xt, B, seed))
    share["kmeans_pp_s"] = 1.0
    n_s = cfg.kmeans_sample or orc.default_sample_size(N)
    Xs = Xt[torch.from_numpy(orc.kmeans_sample_ids(N, n_s, seed).astype(np.int64))]
    runs = cfg.kmeans_iters if full else min(1, cfg.kmeans_iters)
    t0 = time.perf_counter()
    for _ in range(runs):
        C = cpu_port.lloyd_step(Xs, C)
    st["lloyd_s"] = (time.perf_counter() - t0) * (cfg.kmeans_iters / max(runs, 1))
    share["lloyd_s"] = runs / max(cfg.kmeans_iters, 1)
    if runs < cfg.kmeans_iters:
        # untimed: the remaining iterations on a tenth of the sample, so that the bucket sizes
        # (which scale the bucket-kNN stage) come from converged centroids
        sub = Xs[: max(B * 4, Xs.shape[0] // 10)]
        for _ in range(cfg.kmeans_iters - runs):
            C = cpu_port.lloyd_step(sub, C)
    # top-2 of every point (full) or of a row sample sized to about 2e10 flops
    n_t = N if full else min(N, max(20000, int(2e10 / (2.0 * B * d))))
    (t2, _), t = timed(lambda: cpu_port.topk_from_A_to_B(Xt[:n_t], C, 2))
    st["top2_s"] = t * N / n_t
    share["top2_s"] = n_t / N
    sizes = np.bincount(t2.numpy().reshape(-1), minlength=B).astype(np.float64) * (N / n_t)
    sum_sq = float((sizes ** 2).sum())
    # per-bucket kNN: every bucket (full), else the median-size bucket scaled by sum n_b^2
    if full:
        t2n = t2.numpy()
        t_knn = 0.0
        for b in range(B):
            mem = np.nonzero((t2n == b).any(axis=1))[0]
            if mem.size >= 2:
                _, t = timed(lambda: cpu_port.bucket_knn(Xt[torch.from_numpy(mem)], M))
                t_knn += t
        st["bucket_knn_s"] = t_knn
        share["bucket_knn_s"] = 1.0
    else:
        n_med = int(max(M + 2, np.median(sizes[sizes > 0])))
        rows = torch.from_numpy(rng.choice(N, min(N, n_med), replace=False))
        _, t = timed(lambda: cpu_port.bucket_knn(Xt[rows], M))
        st["bucket_knn_s"] = t * sum_sq / float(n_med) ** 2
        share["bucket_knn_s"] = float(n_med) ** 2 / sum_sq
    # merge of each point's two lists (sorted lists of the real shape)
    nm = N if full else min(N, 200_000)
    da = np.sort(rng.random((nm, M), dtype=np.float32), axis=1)
    db = np.sort(rng.random((nm, M), dtype=np.float32), axis=1)
    ia = rng.integers(0, N, (nm, M)).astype(np.int32)
    ib = rng.integers(0, N, (nm, M)).astype(np.int32)
    _, t = timed(lambda: orc.merge_lists(ia, da, ib, db))
    st["merge_s"] = t * N / nm
    share["merge_s"] = nm / N
    # CAGRA prune + reverse edges on a distance-sorted graph of the real shape
    ng = N if full else min(N, 100_000)
    Xg = np.ascontiguousarray(X[:ng], dtype=np.float32)
    base = np.arange(ng)[:, None] + rng.integers(-2000, 2000, (ng, M))
    knn = orc.sort_rows_l2(Xg, np.clip(base, 0, ng - 1).astype(np.int32))
    san, _ = orc.sanitize(knn)
    R = orc.ref_lib()
    out = np.empty((ng, K), np.uint32)
    t0 = time.perf_counter()
    if R is not None:
        assert R.ref_optimize(orc._p(san), ng, M, K, orc._p(out)) == 0
        kind = "reference"
    else:
        orc.optimize(san, K)
        kind = "port"
    st["cagra_prune_reverse_s"] = (time.perf_counter() - t0) * N / ng
    share["cagra_prune_reverse_s"] = ng / N
    # the reference's Python occlusion prune on sampled rows of the same graph
    n_o = min(ng, 400 if full else max(8, int(2.0e9 / (M * M * d))))
    rows_o = rng.choice(ng, n_o, replace=False)
    _, t = timed(lambda: cpu_port.prune_graph(Xg, knn, K, rows=rows_o))
    occlusion_s = t * N / n_o
    build = sum(st[k] for k in ("kmeans_pp_s", "lloyd_s", "top2_s", "bucket_knn_s", "merge_s"))
    total = build + st["cagra_prune_reverse_s"]
    detail = {"stages_s": {k: round(v, 4) for k, v in st.items()},
              "measured_share": {k: round(v, 6) for k, v in share.items()},
              "extrapolated": sorted(k for k, v in share.items() if v < 1.0),
              "occlusion_prune_s": round(occlusion_s, 3), "occlusion_rows_timed": int(n_o),
              "occlusion_extrapolated": bool(n_o < N),
              "total_with_occlusion_prune_s": round(build + occlusion_s, 3),
              "prune_reverse_code": kind, "sum_nb2_over_balanced": sum_sq * B / float(sizes.sum()) ** 2,
              **cpu_info()}
    sample = ("whole job" if full else
              f"k-means++ whole pool; Lloyd {runs} of {cfg.kmeans_iters} iterations on the {n_s}-point sample; "
              f"top-2 on {n_t} rows; bucket kNN on one median-size bucket scaled by sum(n_b^2); merge {nm} lists; "
              f"CAGRA prune+reverse ({kind} code) on a {ng}-row graph; occlusion prune on {n_o} rows")
    return total, detail, sample


def parity_sample(X: np.ndarray, top2: np.ndarray, ids: np.ndarray, dists: np.ndarray, M: int, gt, q: np.ndarray):
    """CHECKER (outside every timed region): the oracle pipeline's merged kNN lists of the
    sampled points ``q`` (their exact top-M within each of their two buckets, merged by the
    resident merge rule: oracle.point_lists) against the build's own lists at full size."""
    from oracle import oracle as orc

    Xf = np.ascontiguousarray(X, dtype=np.float32)
    oi, od = orc.point_lists(Xf, top2, q, M)
    gi, gd = ids[q], dists[q]
    same = gi == oi
    r, c = np.nonzero(~same)
    ties_ok = True
    max_tie = 0.0
    if len(r):
        valid = (gi[r, c] >= 0) & (oi[r, c] >= 0)
        own = orc.pair_l2(Xf, q[r[valid]], gi[r, c][valid]) if valid.any() else np.zeros(0, np.float32)
        rel = np.abs(own.astype(np.float64) - od[r, c][valid]) / np.maximum(np.abs(od[r, c][valid]), 1e-30)
        max_tie = float(rel.max()) if rel.size else 0.0
        ties_ok = bool(valid.all() and (rel <= 1e-5).all() and (gd[r, c][valid] == own).all())
    dd = np.abs(gd[same].astype(np.float64) - od[same]) / np.maximum(np.abs(od[same]), 1e-30)
    dd = dd[np.isfinite(dd)]
    k = min(32, M)
    rec = lambda L: float(np.mean([len(np.intersect1d(L[i, :k], gt[i, :k])) / k for i in range(len(q))]))
    return {"points": int(len(q)), "m": M, "ids_equal_frac": float(same.mean()),
            "rows_identical_frac": float(same.all(axis=1).mean()), "differing_positions": int(len(r)),
            "differing_ids_are_ties_within_1e-5": ties_ok, "max_rel_tie_gap": max_tie,
            "max_rel_dist_diff_same_ids": float(dd.max()) if dd.size else 0.0,
            f"recall_at_{k}_build": rec(gi), f"recall_at_{k}_oracle": rec(oi),
            "checker": "oracle.point_lists (per-bucket exact top-M + resident merge), untimed"}


# ---------------------------------------------------------------- main
SEARCH_QUERIES = 2000
SEARCH_SAMPLES = 16384


def exact_knn(Xall, Xq, k: int, exclude=None, q_chunk: int = 2048, col_chunk: int = 1 << 18) -> np.ndarray:
    """Exact k nearest rows of ``Xall`` for each row of ``Xq`` (fp64, on the tensors' device);
    ``exclude[i]`` (a row index of Xall) is left out of query i's answer.  Queries run in blocks
    of ``q_chunk`` against column blocks of ``col_chunk`` rows (bounded scratch)."""
    import torch

    out = []
    for q0 in range(0, Xq.shape[0], q_chunk):
        xq = Xq[q0:q0 + q_chunk].double()
        ex = None if exclude is None else exclude[q0:q0 + q_chunk]
        vals, idxs = [], []
        for c0 in range(0, Xall.shape[0], col_chunk):
            Xc = Xall[c0:c0 + col_chunk].double()
            dd = (xq * xq).sum(1, keepdim=True) + (Xc * Xc).sum(1)[None, :] - 2.0 * xq @ Xc.T
            if ex is not None:
                idx = torch.arange(c0, c0 + Xc.shape[0], device=Xc.device)
                dd[ex[:, None] == idx[None, :]] = float("inf")
            v, i = torch.topk(dd, min(k, Xc.shape[0]), dim=1, largest=False)
            vals.append(v)
            idxs.append(i + c0)
        v = torch.cat(vals, 1)
        i = torch.cat(idxs, 1)
        out.append(torch.gather(i, 1, torch.topk(v, k, dim=1, largest=False).indices).cpu().numpy())
    return np.concatenate(out) if out else np.empty((0, k), np.int64)


DEFAULT_CONFIG = "c3"
# recall@32 of the kNN lists is measured on this many sampled points (exact ground truth for those)
RECALL_POINTS = 10000
# stage names whose work unit is flops (the rest count bytes; "search" counts queries)
FLOP_STAGES = ("dist_topk", "assign_exact", "screen_pilot")


def stage_rate_key(name: str) -> str:
    if name.startswith(FLOP_STAGES):
        return "tflops"
    return "queries_per_s" if name == "search" else "gbs"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=DEFAULT_CONFIG)
    ap.add_argument("--n", type=int, default=0, help="override N (smaller case, e.g. for profiling)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the sampled-point oracle parity check")
    ap.add_argument("--full", action="store_true",
                    help="--impl reference: time every CPU stage on the whole workload (C1 / C2 sizes)")
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
    workload = (f"{cfg.name}: N={cfg.n} x d={cfg.d} {cfg.dtype}, {cfg.n_clusters}-Gaussian mixture, "
                f"B={cfg.n_buckets} buckets (2-way), M={cfg.knn_degree}, K={cfg.graph_degree}, "
                f"{cfg.kmeans_iters} Lloyd iterations")
    # one dataset for the whole job at every N: rank r holds row block r (strong scaling)
    n_buckets_job = cfg.n_buckets
    row_lo = cfg.n * rank // world
    row_hi = cfg.n * (rank + 1) // world
    config = {"workload": workload, "n_per_rank": row_hi - row_lo, "n_total": cfg.n, "d": cfg.d, "dtype": cfg.dtype,
              "n_buckets": n_buckets_job,
              "knn_degree": cfg.knn_degree, "graph_degree": cfg.graph_degree, "kmeans_iters": cfg.kmeans_iters,
              "kmeans_sample": cfg.kmeans_sample or None,
              "l2": "inputs and intermediates larger than L2 (no flush needed)",
              "parallelism": (f"{world} ranks, buckets sharded, a bucket above a rank's share of n_b^2 cut into "
                              "row ranges on several ranks (NCCL all-reduce / all-to-all / all-gather)"
                              if world > 1 else "1 GPU"),
              "shards": "one seeded mixture; rank r holds its contiguous block of N/W rows (strong scaling)"}
    if not _unseeded_split():
        config["screen_unseeded_split"] = False  # the library option is off for this run

    if args.impl == "reference":
        if rank != 0:
            return 0
        X = gta.generate(cfg, seed=42)
        per, walls = [], []
        detail = sample = None
        for s_ in range(args.warmup + args.steps):
            w0 = time.perf_counter()
            t, detail, sample = cpu_reference(X, cfg, full=args.full)
            if s_ >= args.warmup:
                per.append(t)
                walls.append(time.perf_counter() - w0)
        sec = statistics.mean(per)
        # whole-job throughput of the reference's CPU path on this host (extrapolated stages marked)
        value = cfg.n / sec / 1e6
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": statistics.mean(walls) * 1e3,
                "job_ms_cpu": sec * 1e3, "extrapolated": bool(detail["extrapolated"]),
                "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Gaussian mixture)", "config": config,
                "impl": "reference",
                "cpu_baseline": {"value": value, "unit": UNIT, "cores": detail["torch_threads"],
                                 "kind": "reference" if detail["prune_reverse_code"] == "reference" else "port",
                                 "sample": sample, **detail},
                "note": ("ms_per_step is the wall time of one timed step (the bounded sample that ran); "
                         "value is the whole job's throughput from job_ms_cpu, the per-stage times scaled to the "
                         "whole job where `extrapolated` lists them"),
                "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return 0

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    X_all = gta.generate(cfg, seed=42)
    X = np.ascontiguousarray(X_all[row_lo:row_hi]) if world > 1 else X_all
    del X_all
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
    value = cfg.n / (ms / 1e3) / 1e6

    # per-stage device time inside the timed steps
    stages = {}
    for name, t_ms, units, cnt in recs:
        s = stages.setdefault(name, {"ms": 0.0, "units": 0.0, "launches": 0, "counters": [0.0] * 8})
        s["ms"] += t_ms
        s["units"] += units
        s["launches"] += 1
        s["counters"] = [a + b for a, b in zip(s["counters"], cnt)]
    hbm, tflops_burst, tflops, peak_src = _peaks()
    # the bucket distance kernel runs as one launch per phase (lower-bucket rows, then the seeded
    # higher-bucket rows): one kernel for the roofline
    roof = {}
    for k, v in stages.items():
        r = roof.setdefault("dist_topk_bucket" if k.startswith("dist_topk_bucket") else k,
                            {"ms": 0.0, "units": 0.0, "launches": 0, "rows": 0.0, "issued": 0.0})
        r["ms"] += v["ms"]
        r["units"] += v["units"]
        # the float screen's split waves issue three fp16 products per element, the others one
        r["issued"] += v["units"] * (3.0 if k.endswith("_split") else 1.0)
        r["launches"] += v["launches"]
        r["rows"] += v["counters"][2] if k.startswith("dist_topk") else 0.0
    kernels = [k for k in roof if not k.endswith("_total") and roof[k]["units"] > 0]
    dom = max(kernels, key=lambda k: roof[k]["ms"]) if kernels else None
    roofline = None
    if dom:
        s = roof[dom]
        per_launch_units = s["units"] / s["launches"]
        per_launch_s = s["ms"] / s["launches"] / 1e3
        if dom.startswith("dist_topk"):
            achieved = per_launch_units / per_launch_s / 1e12
            cd = _compute_dtype(cfg)
            # the stage runs inside a multi-second build under the power cap: the sustained figure
            roofline = {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": tflops, "unit": "TFLOP/s",
                        "frac": achieved / tflops, "peak_source": f"{peak_src} bf16 sustained",
                        "frac_of_burst": achieved / tflops_burst}
            if cd == "u8":
                roofline["frac_i8_nominal"] = achieved / (2.0 * tflops)
                roofline["note"] = ("kind::i8 MMAs: algorithmic operations per second against the measured bf16 "
                                    "sustained rate; frac_i8_nominal divides by twice that (the nominal dense i8 "
                                    "rate is twice bf16)")
            elif cd in ("f16", "f16x3"):
                issued = s["issued"] / s["units"] if s["units"] > 0 else 1.0
                roofline["kernel_detail"] = ("screen_kernel: kind::f16 on scaled fp16 rows, one product per element "
                                             "(hi.hi) in the seeded chunk waves, three (hi/lo split) for unseeded rows "
                                             "and in the waves that fall back to the split")
                roofline["mma_issued_per_algorithmic"] = issued
                roofline["frac_issued"] = issued * achieved / tflops
                roofline["note"] = ("algorithmic flops (sum 2 n_b^2 d, once) per second of the screen launches; "
                                    "frac_issued: the tensor pipe's issued rate (split waves count three products "
                                    "per element) against the measured bf16 sustained rate, fp16 runs at the "
                                    "bf16 rate")
        else:
            achieved = per_launch_units / per_launch_s / 1e9
            roofline = {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                        "frac": achieved / hbm, "peak_source": f"{peak_src} HBM copy"}
        # DRAM bytes of one launch, from the committed capture of this workload and screen
        # configuration (None elsewhere)
        tpl = TRAFFIC_PER_LAUNCH.get((dom, args.config, cfg.n, _unseeded_split()))
        roofline["traffic"] = tpl[0] if tpl else None
        if tpl:
            roofline["traffic_source"] = tpl[1]
        elif any(k[:3] == (dom, args.config, cfg.n) for k in TRAFFIC_PER_LAUNCH):
            roofline["traffic_note"] = ("the committed capture of this workload ran the unseeded rows on the one-part "
                                        "screen (GTA_SCREEN_UNSEEDED_SPLIT=0); none yet of this configuration")
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
            key = stage_rate_key(k)
            scale = 1e12 if key == "tflops" else (1.0 if key == "queries_per_s" else 1e9)
            stage_summary[k][key] = v["units"] / (v["ms"] / 1e3) / scale
        if k in ("rerank",) and v["counters"][2] > 0:
            stage_summary[k]["exact_candidates_per_row"] = v["counters"][0] / v["counters"][2]
            stage_summary[k]["rows_rescanned"] = v["counters"][1] / args.steps

    # bucket balance (k-means leaves buckets skewed; the bucket stage costs sum n_b^2) and, on
    # several GPUs, the device time of each phase of one more (untimed) build
    skew = phases = None
    knn_h = None
    if world == 1:
        ids_b, d_b, _, t2 = gta.build_bucket(Xd, cfg.n_buckets, cfg.knn_degree, cfg.kmeans_iters, cfg.kmeans_sample,
                                             42, with_extras=True)
        sizes = torch.bincount(t2.reshape(-1).long(), minlength=cfg.n_buckets).double()
        knn_h = (ids_b.cpu().numpy(), d_b.cpu().numpy(), t2.cpu().numpy())
    else:
        res = gd.build_sharded(Xd, prm, timing=True)
        sizes = torch.tensor(res.sizes, dtype=torch.float64)
        phases = {k: round(v, 3) for k, v in res.phase_ms.items()}
        n_pieces = {}
        for b, _, _, _ in res.pieces:
            n_pieces[b] = n_pieces.get(b, 0) + 1
        split = {b: c for b, c in n_pieces.items() if c > 1}
        t = torch.tensor([phases[k] for k in phases], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        phases = {k: round(float(v), 3) for k, v in zip(phases, t.tolist())}
    skew = {"max_bucket": int(sizes.max()), "sum_sq_over_balanced": float((sizes * sizes).sum() * sizes.numel()
                                                                         / sizes.sum() ** 2)}
    if world > 1:
        skew["split_buckets"] = {str(b): c for b, c in sorted(split.items())}  # bucket -> ranks sharing it

    # quality: recall@32 of the pre-prune kNN graph on RECALL_POINTS sampled points of rank 0's rows
    # (exact GT over the whole job's dataset in fp64 on the GPU)
    recall = None
    if world == 1:
        ids = ids_b
        Xall = Xd
    else:
        ids = last["res"].knn_ids
        counts = [cfg.n * (r + 1) // world - cfg.n * r // world for r in range(world)]
        Xall = gd._all_gather_rows(Xd, counts)
    if world > 1:
        g_all = gd._all_gather_rows(g.contiguous(), counts)
    else:
        g_all = g
    search_q = None
    if rank == 0:
        # points of rank 0's row block (global ids 0 .. its rows - 1)
        n_q = min(RECALL_POINTS, X.shape[0])
        q = torch.from_numpy(np.random.default_rng(0).choice(X.shape[0], n_q, replace=False)).cuda()
        gt = exact_knn(Xall, Xall[q], 32, exclude=q)
        approx = ids[q].cpu().numpy()[:, :32]
        recall = float(np.mean([len(np.intersect1d(approx[r], gt[r])) / 32.0 for r in range(n_q)]))
    parity = None
    if rank == 0 and world == 1 and not args.no_parity:
        # the build's own lists at full size against the oracle pipeline on 500 of the sampled points
        qn = q.cpu().numpy()[:500].astype(np.int64)
        parity = parity_sample(X, knn_h[2], knn_h[0], knn_h[1], cfg.knn_degree, gt[:500], qn)
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
    if world == 1 and rank == 0 and not args.no_extras and _compute_dtype(cfg) != "f16x3":
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
                                                                      for r in range(n_q)])),
                         "stage": "kNN lists only (no CAGRA optimize)"}
    del Xall, g_all

    # end to end with host buffers (pinned), copies inside the timed region: through the C ABI
    # (gta_build_cagra) on one GPU, through the sharded build on several
    e2e = None
    if not args.no_e2e:
        Xh = torch.from_numpy(X).pin_memory()
        gh_t = torch.empty((X.shape[0], cfg.graph_degree), dtype=torch.int32).pin_memory()
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
        e2e = {"value": cfg.n / e2e_s / 1e6, "unit": UNIT, "ms_per_step": e2e_s * 1e3,
               "h2d_bytes_per_step": int(X.nbytes), "d2h_bytes_per_step": int(gh.nbytes),
               "path": "gta_build_cagra (C ABI, host buffers)" if world == 1 else "gta.dist.build_sharded"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        sec, detail, sample = cpu_reference(X, cfg)
        cpu = {"value": cfg.n / sec / 1e6, "unit": UNIT, "cores": detail["torch_threads"],
               "kind": "reference" if detail["prune_reverse_code"] == "reference" else "port",
               "sample": sample, "job_ms_cpu": sec * 1e3, **detail}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": _compute_dtype(cfg),
                "data": "synthetic (seeded Gaussian mixture)", "config": config, "roofline": roofline,
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
                "clocks": clocks, "recall_at_32": recall,
                "recall_points": n_q if rank == 0 else None, "parity": parity, "search": search_q, "reference_bucketing": ref_bucketing, "bucket_skew": skew, "phases_ms_max_over_ranks": phases,
                "stages": stage_summary,
                "instrumented_ms_per_step": step_ms_sum}
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
