"""Python host layer over the libgta C ABI.

Mirrors the reference's build-path interface (paths relative to the reference
project root):

  build_bucket      bucket2 Steps 2-6 / GpuResidentKnn::run_round (bucketDemo/buildBucket/src/bucket.cu:8523, :5310)
  optimize          cuvs cagra::helpers::optimize (bucketDemo/buildBucket/src/optimize.cu:396)
  build_cagra       bucket2 --fused-optimize-degree (bucket.cu:8434 fused_optimize_translate)
  kmeans_init       kmeans_pp_centers (bucketDemo/build_bucket.py:189)
  kmeans_fit        refine_centers_kmeans (bucketDemo/build_bucket.py:232)
  assign_topk       topk_from_A_to_B(X, C, k) (bucketDemo/build_bucket.py:96)
  merge_lists       resident_merge_kernel (bucket.cu:5025)
  sanitize          sanitize_to_uint32_inplace (optimize.cu:95)
  prune / reverse_merge   prune_windowed_core.hpp:190-263 / edge_chunk_accumulator.hpp:386-494
  search            graph_search_single (bucketDemo/search.py:20-93)

Device arrays are torch CUDA tensors (torch supplies device memory and the
current stream only; every computation runs in libgta's own kernels).  Host
arrays are numpy arrays.  Errors raise ``GtaError`` carrying the C status code.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _lib as L

_DT = {"float32": L.GTA_F32, "uint8": L.GTA_U8, "int8": L.GTA_I8}


def _torch():
    import torch

    return torch


def _is_dev(x) -> bool:
    return hasattr(x, "is_cuda") and x.is_cuda


def _ptr(x) -> ctypes.c_void_p:
    if x is None:
        return ctypes.c_void_p(0)
    if _is_dev(x):
        if not x.is_contiguous():
            raise L.GtaError(L.GTA_EINVAL, "device arrays must be contiguous")
        return ctypes.c_void_p(x.data_ptr())
    if not (isinstance(x, np.ndarray) and x.flags["C_CONTIGUOUS"]):
        raise L.GtaError(L.GTA_EINVAL, "host arrays must be C-contiguous numpy arrays")
    return x.ctypes.data_as(ctypes.c_void_p)


def _dev(*xs) -> None:
    """Stage entry points read and write device memory only: every array argument (None skipped)
    must be a CUDA tensor, checked before anything is allocated or launched."""
    for x in xs:
        if x is not None and not _is_dev(x):
            raise L.GtaError(L.GTA_EINVAL, "stage entry points take torch CUDA tensors")


def _same_side(dev: bool, *xs) -> None:
    """Arguments of one call all on the device or all on the host (None skipped)."""
    for x in xs:
        if x is not None and _is_dev(x) != dev:
            raise L.GtaError(L.GTA_EINVAL, "arguments must be all torch CUDA tensors or all numpy arrays")


def _stream():
    torch = _torch()
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dtype_code(x) -> int:
    name = str(x.dtype).replace("torch.", "")
    if name not in _DT:
        raise L.GtaError(L.GTA_EINVAL, f"unsupported dataset dtype {x.dtype}")
    return _DT[name]


def _empty(shape, dtype, like_dev: bool):
    if like_dev:
        torch = _torch()
        return torch.empty(shape, dtype=getattr(torch, dtype), device="cuda")
    return np.empty(shape, dtype=dtype)


def _dataset(X, metric: str = "l2", host_resident: bool = False) -> L.gta_dataset:
    if host_resident and (_is_dev(X) or not X.flags["C_CONTIGUOUS"]):
        raise L.GtaError(L.GTA_EINVAL, "host_resident needs a C-contiguous host array")
    return L.gta_dataset(data=_ptr(X), n=X.shape[0], d=X.shape[1], dtype=_dtype_code(X),
                         metric=L.GTA_IP if metric == "ip" else L.GTA_L2,
                         on_device=2 if host_resident else (1 if _is_dev(X) else 0))


def _bucket_params(n_buckets, knn_degree, kmeans_iters, kmeans_sample, seed, init_centroids, dev, cent_out, top2_out,
                   rounds=1, device_budget=0):
    return L.gta_bucket_params(
        device_budget=device_budget,
        n_buckets=n_buckets, kmeans_iters=kmeans_iters, knn_degree=knn_degree, rounds=rounds,
        kmeans_sample=kmeans_sample, seed=seed, init_centroids=_ptr(init_centroids),
        init_on_device=1 if (init_centroids is not None and _is_dev(init_centroids)) else 0,
        out_on_device=1 if dev else 0, centroids_out=_ptr(cent_out), top2_out=_ptr(top2_out))


# ---------------------------------------------------------------- pipeline
def build_bucket(X, n_buckets: int, knn_degree: int = 64, kmeans_iters: int = 10, kmeans_sample: int = 0,
                 seed: int = 42, init_centroids=None, metric: str = "l2", with_extras: bool = False,
                 rounds: int = 1, device_budget: int = 0, host_resident: bool = False):
    """Bucketed kNN graph of X (N x d, float32 / uint8 / int8; torch CUDA tensor or numpy).

    Returns (ids[N, M] int32, dists[N, M] float32) on X's side (device or host);
    with ``with_extras`` also the final centroids (B x d) and top-2 buckets (N x 2).
    ``rounds`` > 1 repeats the build with seeds seed+1, ... and merges each round's
    lists into the running ones (bucket2 ``-t``).  ``device_budget`` (bytes, 0 = 80% of free
    device memory) bounds the bucket kNN stage; buckets beyond it run in batches, same result.
    ``host_resident`` (numpy X): the build reads X in place from host memory (registered for the
    call) and never copies it whole to the device -- datasets larger than the device's memory.
    """
    dev = _is_dev(X)
    N, d = X.shape
    ids = _empty((N, knn_degree), "int32", dev)
    dists = _empty((N, knn_degree), "float32", dev)
    cent = _empty((n_buckets, d), "float32", dev) if with_extras else None
    top2 = _empty((N, 2), "int32", dev) if with_extras else None
    ds = _dataset(X, metric, host_resident)
    p = _bucket_params(n_buckets, knn_degree, kmeans_iters, kmeans_sample, seed, init_centroids, dev, cent, top2,
                       rounds, device_budget)
    L.check(L.lib().gta_build_bucket(ctypes.byref(ds), ctypes.byref(p), _ptr(ids), _ptr(dists),
                                     _stream() if dev else ctypes.c_void_p(0)))
    if with_extras:
        return ids, dists, cent, top2
    return ids, dists


def build_bucket2(X, knn_degree: int = 64, nprobe: int = 0, centroid_ratio: float = 0.01, seed: int = 42,
                  rounds: int = 1, knn_k: int = 0, with_extras: bool = False, assign_rule: str = "default"):
    """kNN graph with the reference's own bucketing (its bucket2 tool): KMeans|| data-point
    centroids (max(2, N * centroid_ratio) requested), balanced 1-way buckets, every bucket's
    points searched in the pool of their bucket and its ``nprobe`` nearest buckets (0: knn_k,
    0: 32), ``rounds`` builds merged.  ``assign_rule``: "default" (the second centroid when its
    bucket is below 0.8 x the first's) or "diskjoin" (the tool's BUCKET2_ASSIGN_RULE=diskjoin).
    Returns (ids[N, M], dists[N, M]); with ``with_extras`` also the bucket of every point (N,)
    and the centroids' point ids."""
    rules = {"default": 0, "diskjoin": 1}
    if assign_rule not in rules:
        raise L.GtaError(L.GTA_EINVAL, f"build_bucket2: assign_rule must be one of {sorted(rules)}")
    dev = _is_dev(X)
    N = X.shape[0]
    ids = _empty((N, knn_degree), "int32", dev)
    dists = _empty((N, knn_degree), "float32", dev)
    n_req = max(2, int(float(N) * (float(np.float32(centroid_ratio)) if centroid_ratio > 0 else 0.01)))
    assign = _empty((N,), "int32", dev) if with_extras else None
    cid = _empty((n_req,), "int32", dev) if with_extras else None
    nb = ctypes.c_int32(0)
    p = L.gta_bucket2_params(knn_degree=knn_degree, nprobe=nprobe, knn_k=knn_k, rounds=rounds,
                             centroid_ratio=centroid_ratio, assign_rule=rules[assign_rule], seed=seed,
                             out_on_device=1 if dev else 0,
                             reserved1=0, assign_out=_ptr(assign), centroid_ids_out=_ptr(cid),
                             n_buckets_out=ctypes.pointer(nb))
    ds = _dataset(X)
    L.check(L.lib().gta_build_bucket2(ctypes.byref(ds), ctypes.byref(p), _ptr(ids), _ptr(dists),
                                      _stream() if dev else ctypes.c_void_p(0)))
    if with_extras:
        return ids, dists, assign, cid[: nb.value]
    return ids, dists


def build_cagra(X, n_buckets: int, knn_degree: int = 64, graph_degree: int = 32, kmeans_iters: int = 10,
                kmeans_sample: int = 0, seed: int = 42, init_centroids=None, metric: str = "l2", rounds: int = 1,
                device_budget: int = 0, host_resident: bool = False):
    """Whole build: bucketed kNN (degree M), sanitize, CAGRA optimize -> graph[N, K] uint32.
    ``host_resident``: as for build_bucket."""
    dev = _is_dev(X)
    N = X.shape[0]
    graph = _empty((N, graph_degree), "uint32" if not dev else "int32", dev)
    ds = _dataset(X, metric, host_resident)
    bp = _bucket_params(n_buckets, knn_degree, kmeans_iters, kmeans_sample, seed, init_centroids, dev, None, None,
                        rounds, device_budget)
    p = L.gta_cagra_params(bucket=bp, graph_degree=graph_degree, reserved0=0)
    L.check(L.lib().gta_build_cagra(ctypes.byref(ds), ctypes.byref(p), _ptr(graph),
                                    _stream() if dev else ctypes.c_void_p(0)))
    return graph


def optimize(knn, graph_degree: int):
    """CAGRA optimize (prune + reverse edges) of a distance-sorted, sanitized uint32 graph (N x M)."""
    dev = _is_dev(knn)
    N, M = knn.shape
    out = _empty((N, graph_degree), "int32" if dev else "uint32", dev)
    L.check(L.lib().gta_optimize(_ptr(knn), N, M, graph_degree, _ptr(out), 1 if dev else 0,
                                 _stream() if dev else ctypes.c_void_p(0)))
    return out


def optimize_knn(knn, graph_degree: int, X=None):
    """The optimize tool (optimize.cu main): sanitize an int32 kNN graph (-1 padding), sort each
    row by exact L2 to its point when ``X`` is given (else the rows must already be ascending:
    ``--skip-sort``), prune + reverse edges -> graph[N, K] uint32 (int32 view on the device)."""
    dev = _is_dev(knn)
    N, M = knn.shape
    out = _empty((N, graph_degree), "int32" if dev else "uint32", dev)
    ds = _dataset(X) if X is not None else None
    L.check(L.lib().gta_optimize_knn(ctypes.byref(ds) if ds is not None else None, _ptr(knn), N, M, graph_degree,
                                     _ptr(out), 1 if dev else 0, _stream() if dev else ctypes.c_void_p(0)))
    return out


# ---------------------------------------------------------------- graph search
def search_entries(n: int, nq: int, num_entry: int = 4, seed: int = 42) -> np.ndarray:
    """Entry points of the reference's search (bucketDemo/search.py:40-41 with the
    generator of :163, called per query at :170-172): one numpy default_rng(seed) shared
    by the queries in order,
    ``np.unique(rng.integers(0, n, num_entry))`` per query; -1 pads a row."""
    rng = np.random.default_rng(seed)
    k = max(1, num_entry)
    out = np.full((nq, k), -1, np.int32)
    for i in range(nq):
        u = np.unique(rng.integers(0, n, size=k, endpoint=False))
        out[i, :u.size] = u
    return out


def search(base, graph, queries, topk: int = 10, ef: int = 200, num_entry: int = 4, seed: int = 42, entries=None):
    """Best-first graph search of ``queries`` over ``graph`` (N x K ids) with the rule of
    bucketDemo/search.py graph_search_single (its defaults: topk 10, ef 200, 4 random
    entry points, seed 42).  ``base`` / ``queries`` / ``graph`` all on the device (torch)
    or all on the host (numpy).  Returns (ids[nq, topk], dists[nq, topk])."""
    dev = _is_dev(base)
    _same_side(dev, queries, graph)
    n, d = base.shape
    nq = queries.shape[0]
    ef = max(ef, topk)
    if entries is None:
        entries = search_entries(n, nq, num_entry, seed)
    if dev:
        torch = _torch()
        entries = torch.as_tensor(np.ascontiguousarray(entries, np.int32)).cuda()
        graph = graph.contiguous()
    else:
        entries = np.ascontiguousarray(entries, np.int32)
        graph = np.ascontiguousarray(graph).view(np.uint32) if graph.dtype.itemsize == 4 else \
            np.ascontiguousarray(graph, np.uint32)
    ids = _empty((nq, topk), "int32", dev)
    dists = _empty((nq, topk), "float32", dev)
    ds = _dataset(base)
    L.check(L.lib().gta_search(ctypes.byref(ds), _ptr(queries), nq, _ptr(graph), graph.shape[1], _ptr(entries),
                               entries.shape[1], topk, ef, _ptr(ids), _ptr(dists),
                               _stream() if dev else ctypes.c_void_p(0)))
    return ids, dists


# ---------------------------------------------------------------- stages (device tensors)
def kmeans_init(X, pool_n: int, n_buckets: int, seed: int = 42):
    _dev(X)
    C = _empty((n_buckets, X.shape[1]), "float32", True)
    L.check(L.lib().gta_kmeans_init(_ptr(X), pool_n, X.shape[1], n_buckets, seed, _ptr(C), _stream()))
    return C


def kmeans_fit(X, C0, iters: int):
    _dev(X, C0)
    C = C0.clone().contiguous()
    assign = _empty((X.shape[0],), "int32", True)
    L.check(L.lib().gta_kmeans_fit(_ptr(X), X.shape[0], X.shape[1], _ptr(C), C.shape[0], iters, _ptr(assign),
                                   _stream()))
    return C, assign


def assign_topk(X, C, k: int):
    _dev(X, C)
    ids = _empty((X.shape[0], k), "int32", True)
    dists = _empty((X.shape[0], k), "float32", True)
    L.check(L.lib().gta_assign_topk(_ptr(X), X.shape[0], X.shape[1], _ptr(C), C.shape[0], k, _ptr(ids), _ptr(dists),
                                    _stream()))
    return ids, dists


def build_memberships(top2, n_buckets: int):
    _dev(top2)
    torch = _torch()
    N = top2.shape[0]
    members = torch.empty(2 * N, dtype=torch.int32, device="cuda")
    offsets = torch.empty(n_buckets + 1, dtype=torch.int64, device="cuda")
    mem_row = torch.empty((N, 2), dtype=torch.int64, device="cuda")
    L.check(L.lib().gta_build_memberships(_ptr(top2), N, n_buckets, _ptr(members), _ptr(offsets), _ptr(mem_row),
                                          _stream()))
    return offsets, members, mem_row


def bucket_knn(X, members, offsets, knn_degree: int):
    _dev(X, members, offsets)
    n_mem = members.shape[0]
    ids = _empty((n_mem, knn_degree), "int32", True)
    dists = _empty((n_mem, knn_degree), "float32", True)
    L.check(L.lib().gta_bucket_knn(_ptr(X), _dtype_code(X), X.shape[0], X.shape[1], _ptr(members), _ptr(offsets),
                                   offsets.shape[0] - 1, knn_degree, _ptr(ids), _ptr(dists), _stream()))
    return ids, dists


def merge_memberships(list_ids, list_dists, mem_row):
    _dev(list_ids, list_dists, mem_row)
    N, M = mem_row.shape[0], list_ids.shape[1]
    ids = _empty((N, M), "int32", True)
    dists = _empty((N, M), "float32", True)
    L.check(L.lib().gta_merge_memberships(_ptr(list_ids), _ptr(list_dists), _ptr(mem_row), N, M, _ptr(ids),
                                          _ptr(dists), _stream()))
    return ids, dists


def merge_lists(run_ids, run_dists, new_ids, new_dists):
    _dev(run_ids, run_dists, new_ids, new_dists)
    N, M = run_ids.shape
    ids = _empty((N, M), "int32", True)
    dists = _empty((N, M), "float32", True)
    L.check(L.lib().gta_merge_lists(_ptr(run_ids), _ptr(run_dists), _ptr(new_ids), _ptr(new_dists), N, M, _ptr(ids),
                                    _ptr(dists), _stream()))
    return ids, dists


def sanitize(knn):
    _dev(knn)
    out = _empty(tuple(knn.shape), "int32", True)
    L.check(L.lib().gta_sanitize(_ptr(knn), knn.shape[0], knn.shape[1], _ptr(out), _stream()))
    return out


def sort_rows(X, knn):
    _dev(X, knn)
    out = _empty(tuple(knn.shape), "int32", True)
    L.check(L.lib().gta_sort_rows(_ptr(X), X.shape[0], X.shape[1], _ptr(knn), knn.shape[1], _ptr(out), _stream()))
    return out


def prune(knn, graph_degree: int):
    _dev(knn)
    out = _empty((knn.shape[0], graph_degree), "int32", True)
    L.check(L.lib().gta_prune(_ptr(knn), knn.shape[0], knn.shape[1], graph_degree, _ptr(out), _stream()))
    return out


def reverse_merge(pruned):
    _dev(pruned)
    out = _empty(tuple(pruned.shape), "int32", True)
    L.check(L.lib().gta_reverse_merge(_ptr(pruned), pruned.shape[0], pruned.shape[1], _ptr(out), _stream()))
    return out


# ---------------------------------------------------------------- bucket-contiguous renumbering
def _side(x):
    dev = _is_dev(x)
    return dev, (_stream() if dev else ctypes.c_void_p(0))


def bucket_order(centroids, k: int = 32, window: int = 0):
    """Processing order of the buckets (bucket2 Step 3 + bucket_order.hpp): exact kNN graph of
    the centroids (k columns, self excluded) and the greedy windowed order over it.
    Returns (order[B] int32, centroid_knn[B, k] int32) on the centroids' side."""
    dev, st = _side(centroids)
    B, d = centroids.shape
    order = _empty((B,), "int32", dev)
    knn = _empty((B, k), "int32", dev)
    L.check(L.lib().gta_bucket_order(_ptr(centroids), B, d, k, window, _ptr(order), _ptr(knn), 1 if dev else 0, st))
    return order, knn


def bucket_reorder(assign, n_buckets: int, order=None):
    """compute_bucket_reorder: new ids bucket by bucket in ``order`` (default 0..B-1), ascending
    old id inside a bucket.  ``assign`` is (N,) or an (N, 2) top-2 table (column 0 is used).
    Returns (inverse_perm[N] uint32 (int32 view on the device), offsets[B+1] int64)."""
    dev, st = _side(assign)
    _same_side(dev, order)
    n = assign.shape[0]
    stride = 1 if assign.ndim == 1 else assign.shape[1]
    inv = _empty((n,), "int32" if dev else "uint32", dev)
    off = _empty((n_buckets + 1,), "int64", dev)
    L.check(L.lib().gta_bucket_reorder(_ptr(assign), n, stride, n_buckets, _ptr(order), _ptr(inv), _ptr(off),
                                       1 if dev else 0, st))
    return inv, off


def permute_rows(X, inverse_perm):
    """Row i of the result = row inverse_perm[i] of X (the reordered dataset)."""
    dev, st = _side(X)
    _same_side(dev, inverse_perm)
    if dev:
        torch = _torch()
        out = torch.empty_like(X)
    else:
        out = np.empty_like(X)
    row_bytes = X[0].numel() * X.element_size() if dev else X[0].nbytes
    L.check(L.lib().gta_permute_rows(_ptr(X), X.shape[0], row_bytes, _ptr(inverse_perm), _ptr(out), 1 if dev else 0, st))
    return out


def permute_graph(g, inverse_perm, to_original: bool = True, keep_padding: bool = False):
    """translate_ids (to_original) or the renumbering into the reordered id space of an
    N x M id table; -1 padding kept when ``keep_padding``."""
    dev, st = _side(g)
    _same_side(dev, inverse_perm)
    if not dev:
        g = np.ascontiguousarray(g)
        g = g.view(np.int32) if g.dtype.itemsize == 4 else g.astype(np.int32)
    out = _empty(tuple(g.shape), "int32", dev)
    L.check(L.lib().gta_permute_graph(_ptr(g), g.shape[0], g.shape[1], _ptr(inverse_perm), int(to_original),
                                      int(keep_padding), _ptr(out), 1 if dev else 0, st))
    return out


# ---------------------------------------------------------------- files (host)
def read_dataset(path: str, row0: int = 0, nrows: Optional[int] = None) -> np.ndarray:
    n, d, dt = ctypes.c_int64(), ctypes.c_int32(), ctypes.c_int32()
    L.check(L.lib().gta_read_dataset_header(path.encode(), ctypes.byref(n), ctypes.byref(d), ctypes.byref(dt)))
    nrows = n.value - row0 if nrows is None else nrows
    out = np.empty((nrows, d.value), dtype={0: np.float32, 1: np.uint8, 2: np.int8}[dt.value])
    L.check(L.lib().gta_read_dataset(path.encode(), row0, nrows, _ptr(out)))
    return out


def write_dataset(path: str, X: np.ndarray) -> None:
    X = np.ascontiguousarray(X)
    L.check(L.lib().gta_write_dataset(path.encode(), _ptr(X), X.shape[0], X.shape[1], _dtype_code(X)))


def write_knn(path: str, ids: np.ndarray) -> None:
    ids = np.ascontiguousarray(ids, np.int32)
    L.check(L.lib().gta_write_knn(path.encode(), _ptr(ids), ids.shape[0], ids.shape[1]))


def write_knn_dists(path: str, dists: np.ndarray) -> None:
    dists = np.ascontiguousarray(dists, np.float32)
    L.check(L.lib().gta_write_knn_dists(path.encode(), _ptr(dists), dists.shape[0], dists.shape[1]))


def read_knn(path: str) -> np.ndarray:
    n, m = ctypes.c_int64(), ctypes.c_int32()
    L.check(L.lib().gta_read_knn_header(path.encode(), ctypes.byref(n), ctypes.byref(m)))
    out = np.empty((n.value, m.value), np.int32)
    L.check(L.lib().gta_read_knn(path.encode(), _ptr(out)))
    return out


def write_graph(path: str, graph: np.ndarray) -> None:
    graph = np.ascontiguousarray(graph, np.uint32)
    L.check(L.lib().gta_write_graph(path.encode(), _ptr(graph), graph.shape[0], graph.shape[1]))


def read_graph(path: str) -> np.ndarray:
    n, k = ctypes.c_int64(), ctypes.c_int32()
    L.check(L.lib().gta_read_graph_header(path.encode(), ctypes.byref(n), ctypes.byref(k)))
    out = np.empty((n.value, k.value), np.uint32)
    L.check(L.lib().gta_read_graph(path.encode(), _ptr(out)))
    return out


def read_npy_i64(path: str) -> np.ndarray:
    """An int64 (N, M) .npy narrowed to int32 by the library's reader (-1 padding kept)."""
    n, m = ctypes.c_int64(), ctypes.c_int32()
    L.check(L.lib().gta_read_npy_i64_header(path.encode(), ctypes.byref(n), ctypes.byref(m)))
    out = np.empty((n.value, m.value), np.int32)
    L.check(L.lib().gta_read_npy_i64(path.encode(), _ptr(out)))
    return out


def write_u32(path: str, v: np.ndarray) -> None:
    v = np.ascontiguousarray(v, np.uint32)
    L.check(L.lib().gta_write_u32(path.encode(), _ptr(v), v.size))


def read_u32(path: str) -> np.ndarray:
    n = ctypes.c_int64()
    L.check(L.lib().gta_read_u32_count(path.encode(), ctypes.byref(n)))
    out = np.empty(n.value, np.uint32)
    L.check(L.lib().gta_read_u32(path.encode(), _ptr(out)))
    return out


def write_npy(path: str, ids: np.ndarray) -> None:
    ids = np.ascontiguousarray(ids, np.int32)
    L.check(L.lib().gta_write_npy_i64(path.encode(), _ptr(ids), ids.shape[0], ids.shape[1]))
