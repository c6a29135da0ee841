"""Seeded synthetic stand-ins for the benchmark datasets (SIFT / msTuring are not shipped).

The five workload configurations of this build (N points, d dims, element
type, Gaussian-mixture shape, bucket count B, intermediate degree M, graph
degree K).  Generator: numpy default_rng(seed); mixture centres first, then
labels uniform over the clusters, then the noise.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Config:
    name: str
    n: int
    d: int
    dtype: str          # "float32" or "uint8"
    n_clusters: int
    sigma: float
    centre_lo: float
    centre_hi: float
    n_buckets: int
    knn_degree: int
    graph_degree: int
    kmeans_iters: int = 10
    kmeans_sample: int = 0      # 0: min(0.1, 1e7/N) of N
    metric: str = "l2"
    transform: str = ""         # "abs" | "normalize"


CONFIGS = {
    "c1": Config("c1", 10_000, 128, "float32", 64, 0.1, -1.0, 1.0, 16, 64, 32, kmeans_sample=10_000),
    "c2": Config("c2", 1_000_000, 128, "uint8", 1000, 20.0, 0.0, 255.0, 256, 64, 32),
    "c3": Config("c3", 1_000_000, 960, "float32", 500, 0.05, 0.0, 0.2, 256, 128, 64, transform="abs"),
    "c4": Config("c4", 10_000_000, 96, "float32", 10_000, 0.15, -1.0, 1.0, 1024, 64, 32, metric="ip",
                 transform="normalize"),
    "c5": Config("c5", 100_000_000, 128, "uint8", 100_000, 16.0, 0.0, 255.0, 8192, 64, 32),
}


def scaled(cfg: Config, n: int, n_buckets: int | None = None) -> Config:
    """The same distribution at a smaller N (bucket count scaled to keep the bucket size)."""
    b = n_buckets if n_buckets is not None else max(2, int(round(cfg.n_buckets * n / cfg.n)))
    return Config(**{**cfg.__dict__, "n": n, "n_buckets": b, "kmeans_sample": min(cfg.kmeans_sample, n) if
                     cfg.kmeans_sample else 0, "n_clusters": max(2, min(cfg.n_clusters, n // 10))})


def _centres(cfg: Config, rng) -> np.ndarray:
    centres = rng.uniform(cfg.centre_lo, cfg.centre_hi, size=(cfg.n_clusters, cfg.d)).astype(np.float32)
    if cfg.transform == "normalize":
        centres /= np.linalg.norm(centres, axis=1, keepdims=True)
    return centres


def _rows(cfg: Config, centres: np.ndarray, rng, chunk: int) -> np.ndarray:
    labels = rng.integers(0, cfg.n_clusters, size=cfg.n)
    out = np.empty((cfg.n, cfg.d), dtype=cfg.dtype)
    for s in range(0, cfg.n, chunk):
        e = min(cfg.n, s + chunk)
        x = centres[labels[s:e]] + rng.normal(0.0, cfg.sigma, size=(e - s, cfg.d)).astype(np.float32)
        if cfg.transform == "abs":
            x = np.abs(x)
        elif cfg.transform == "normalize":
            x /= np.linalg.norm(x, axis=1, keepdims=True)
        if cfg.dtype == "uint8":
            x = np.clip(np.rint(x), 0, 255)
        out[s:e] = x.astype(cfg.dtype)
    return out


def generate(cfg: Config, seed: int = 42, chunk: int = 1 << 20) -> np.ndarray:
    rng = np.random.default_rng(seed)
    centres = _centres(cfg, rng)
    return _rows(cfg, centres, rng, chunk)


def generate_shard(cfg: Config, shard: int, seed: int = 42, chunk: int = 1 << 20) -> np.ndarray:
    """cfg.n rows of shard ``shard`` of a weak-scaling dataset: every shard is a
    mixture of the configured shape with its own centres, labels and noise, so a
    W-shard dataset is W independent copies of the configured problem (the bucket
    count grows with W).  Shard 0 is generate(cfg, seed) itself."""
    if shard == 0:
        return generate(cfg, seed, chunk)
    rng = np.random.default_rng([seed, shard])
    centres = _centres(cfg, rng)
    return _rows(cfg, centres, rng, chunk)


def generate_queries(cfg: Config, nq: int, shard: int = 0, seed: int = 42) -> np.ndarray:
    """``nq`` held-out rows drawn from the same mixture as ``generate_shard(cfg, shard, seed)``
    (same centres, an independent row stream), for graph-search recall."""
    rng = np.random.default_rng(seed if shard == 0 else [seed, shard])
    centres = _centres(cfg, rng)
    qcfg = Config(**{**cfg.__dict__, "n": nq})
    return _rows(qcfg, centres, np.random.default_rng([seed, shard, 0x5EA4C4]), 1 << 20)
