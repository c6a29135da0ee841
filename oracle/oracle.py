"""TEST INFRASTRUCTURE ONLY: the CPU oracle for the bucketed kNN-graph build.

Loads ``oracle/_build/liboracle.so`` (the C restatement in gta_oracle.c) and
composes the reference's pipeline stages on the CPU.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline / reference arm
import this module; the product library never does.

Stage map (reference file:line, paths relative to the reference project root):
  kmeans_update        bucketDemo/build_bucket.py:232-262  refine_centers_kmeans (one Lloyd step)
  topk_assign          bucketDemo/build_bucket.py:96-159   topk_from_A_to_B(X, C, k); ties -> smaller id
                       (bucketDemo/buildBucket/src/bucket.cu:1225-1228)
  build_csr            bucketDemo/build_bucket.py:444-446  bucket membership lists (2-way here)
  bucket_knn           bucketDemo/build_bucket.py:602-628  per-bucket top-M with the self filter
  merge_memberships    bucketDemo/buildBucket/src/bucket.cu:5025-5059 resident_merge_kernel
  sanitize             bucketDemo/buildBucket/src/optimize.cu:95-133
  optimize             cuvs cagra::helpers::optimize (bucketDemo/buildBucket/src/optimize.cu:396),
                       restated as prune_windowed_core.hpp:190-263 + edge_chunk_accumulator.hpp:386-494
  exact_knn            bucketDemo/build_knn.py:98-149 build_exact_knn
  knn_recall           .claude/skills/optimize-bucket2/scripts/knn_similarity.py (|approx ∩ exact| / k)
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
_REF_PATH = os.path.join(HERE, "_ref", "libgta_ref.so")

_lib = None
_ref = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32


def build() -> None:
    """Compile the oracle (and the reference bridge when the reference tree exists)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_topk_assign.argtypes = [_P, _I64, _I32, _P, _I32, _I32, _P, _P]
        L.orc_lloyd_update.argtypes = [_P, _I64, _I32, _P, _P, _I32, _P]
        L.orc_bucket_knn.argtypes = [_P, _I64, _I32, _P, _P, _I32, _I32, _P, _P]
        L.orc_exact_knn.argtypes = [_P, _I64, _I32, _P, _I64, _I32, _P, _P]
        L.orc_merge_lists.argtypes = [_P, _P, _P, _P, _P, _P, _I64, _I32]
        L.orc_merge_memberships.argtypes = [_P, _P, _P, _I64, _I32, _P, _P]
        L.orc_sanitize.argtypes = [_P, _I64, _I32, _P]
        L.orc_sanitize.restype = _I64
        L.orc_sort_rows_l2.argtypes = [_P, _I32, _P, _I64, _I32, _P]
        L.orc_detour_counts.argtypes = [_P, _I64, _I32, _I64, _P]
        L.orc_prune.argtypes = [_P, _I64, _I32, _I32, _P]
        L.orc_graph_search.argtypes = [_P, _I64, _I32, _P, _I32, _P, _I64, _P, _I32, _I32, _I32, _P, _P]
        L.orc_graph_search.restype = None
        L.orc_reverse_merge.argtypes = [_P, _I64, _I32]
        L.orc_optimize.argtypes = [_P, _I64, _I32, _I32, _P]
        L.orc_merge_rev_row.argtypes = [_P, _P, ctypes.c_uint32, ctypes.c_uint32]
        L.orc_exact_l2.argtypes = [_P, _P, _I32]
        L.orc_exact_l2.restype = ctypes.c_float
        L.orc_pair_l2.argtypes = [_P, _I32, _P, _P, _I64, _P]
        L.orc_pair_l2.restype = None
        L.orc_num_threads.restype = ctypes.c_int
        L.orc_bucket_reorder.argtypes = [_P, _I64, _I32, _I32, _P, _P, _P]
        L.orc_bucket_reorder.restype = _I64
        L.orc_permute_graph.argtypes = [_P, _I64, _I32, _P, _I32, _I32, _P]
        L.orc_permute_graph.restype = _I64
        L.orc_bucket_order.argtypes = [_P, _I32, _I32, _I32, _P]
        L.orc_bucket_order.restype = None
        L.orc_kmeans_parallel.argtypes = [_P, _I64, _I32, _I64, ctypes.c_uint64, _P]
        L.orc_kmeans_parallel.restype = _I64
        L.orc_balanced_assign.argtypes = [_P, _P, _I64, _I32, _P, _I32, _P]
        L.orc_balanced_assign.restype = _I64
        L.orc_pool_tables.argtypes = [_P, _I64, _I32, _P, _I32, _P, _P, _P, _P, _P]
        L.orc_pool_tables.restype = None
        L.orc_pool_knn.argtypes = [_P, _I64, _I32, _P, _I32, _P, _I32, _I32, _P, _P]
        L.orc_pool_knn.restype = None
        _lib = L
    return _lib


def ref_lib():
    """The reference's own prune / reverse-edge code (oracle/_ref), or None."""
    global _ref
    if _ref is None:
        if not os.path.exists(_REF_PATH):
            return None
        R = ctypes.CDLL(_REF_PATH)
        R.ref_detour_counts.argtypes = [_P, _I64, _I32, _I64, _P]
        R.ref_select_pruned_row.argtypes = [_P, _I32, _P, _I32, _P]
        R.ref_sort_row_by_l2.argtypes = [_P, _I32, _P, _I64, _I32, _I64, _P]
        R.ref_optimize.argtypes = [_P, _I64, _I32, _I32, _P]
        R.ref_rank_ordered_csr.argtypes = [_P, _P, _P, _I64, ctypes.c_uint32, ctypes.c_uint32, _P, _P]
        R.ref_merge_rank_ordered_into_row.argtypes = [_P, _P, ctypes.c_uint32, ctypes.c_uint32]
        R.ref_bucket_order.argtypes = [_P, _I64, _I32, _I32, _P]
        R.ref_translate_graph.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p]
        R.ref_translate_npy.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p]
        _ref = R
    return _ref


_REF_ASSIGN_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libgta_ref_assign.so")
_ref_assign = None


def ref_assign_lib():
    """The reference's own balanced-choice loop and pool tables (oracle/_ref), or None."""
    global _ref_assign
    if _ref_assign is None:
        if not os.path.exists(_REF_ASSIGN_PATH):
            return None
        R = ctypes.CDLL(_REF_ASSIGN_PATH)
        R.ref_balanced_assign.argtypes = [_P, _P, _I64, _I32, _P, _I32, _I64, _P]
        R.ref_balanced_assign.restype = None
        R.ref_pool_tables.argtypes = [_P, _I64, _I64, _P, ctypes.c_uint32, _P, _P, _P, _P, _P]
        R.ref_pool_tables.restype = None
        _ref_assign = R
    return _ref_assign


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(X) -> np.ndarray:
    return np.ascontiguousarray(X, dtype=np.float32)


# --------------------------------------------------------------------------
# sampling rules shared (by specification, not by code) with the CUDA library
# --------------------------------------------------------------------------
MASK64 = (1 << 64) - 1


def splitmix64(x: np.ndarray) -> np.ndarray:
    """splitmix64 finaliser over uint64 arrays (Steele et al., 2014)."""
    z = (np.asarray(x, dtype=np.uint64) + np.uint64(0x9E3779B97F4A7C15)) & np.uint64(MASK64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def kmeans_sample_ids(N: int, n_s: int, seed: int) -> np.ndarray:
    """Jittered stratified sample: one point from each of n_s equal strata of [0, N)."""
    if n_s >= N:
        return np.arange(N, dtype=np.int64)
    j = np.arange(n_s, dtype=np.int64)
    lo = (j * N) // n_s
    hi = ((j + 1) * N) // n_s
    h = splitmix64(np.uint64(seed) * np.uint64(0x100000001B3) ^ j.astype(np.uint64))
    return lo + (h % (hi - lo).astype(np.uint64)).astype(np.int64)


def default_sample_size(N: int) -> int:
    """min(0.1, 1e7/N) of N (the reference harness's k-means training fraction,
    .claude/skills/optimize-bucket2/scripts/dataset_env.py:8-20)."""
    frac = min(0.1, 1e7 / max(N, 1))
    return max(1, int(round(frac * N)))


# --------------------------------------------------------------------------
# stages
# --------------------------------------------------------------------------
def pair_l2(X, a, b) -> np.ndarray:
    """Exact fp32 squared distances of the row pairs (X[a[i]], X[b[i]]): the ascending-dimension
    fmaf chain of the reference's exact rerank (bucket.cu:4350-4363 s6_dot_rows)."""
    X = _f32(X)
    a = np.ascontiguousarray(a, dtype=np.int32).reshape(-1)
    b = np.ascontiguousarray(b, dtype=np.int32).reshape(-1)
    out = np.empty(a.shape[0], np.float32)
    lib().orc_pair_l2(_p(X), X.shape[1], _p(a), _p(b), a.shape[0], _p(out))
    return out


def topk_assign(X, C, k: int):
    X = _f32(X); C = _f32(C)
    N, d = X.shape
    B = C.shape[0]
    ids = np.empty((N, k), np.int32)
    dist = np.empty((N, k), np.float32)
    lib().orc_topk_assign(_p(X), N, d, _p(C), B, k, _p(ids), _p(dist))
    return ids, dist


def kmeans_update(X, assign, C):
    X = _f32(X); C = _f32(C)
    a = np.ascontiguousarray(assign, dtype=np.int32)
    out = np.empty_like(C)
    lib().orc_lloyd_update(_p(X), X.shape[0], X.shape[1], _p(a), _p(C), C.shape[0], _p(out))
    return out


def kmeans(X, C0, iters: int):
    """Lloyd iterations from given initial centroids (refine_centers_kmeans)."""
    C = _f32(C0).copy()
    assign = None
    for _ in range(iters):
        ids, _ = topk_assign(X, C, 1)
        assign = ids[:, 0]
        C = kmeans_update(X, assign, C)
    return C, assign


def build_csr(top2: np.ndarray, B: int):
    """Memberships (point, bucket) sorted by (bucket, the point's other bucket, point):
    offsets[B+1], members[2N] (point ids) and mem_row[N, 2] = membership rows of each
    point, column 0 = lower bucket id (the merge's running side).  The secondary key
    groups a bucket's members by boundary region; it changes row positions only, not
    any list content."""
    top2 = np.asarray(top2, dtype=np.int64)
    N, W = top2.shape
    pts = np.repeat(np.arange(N, dtype=np.int64), W)
    bk = top2.reshape(-1)
    other = top2[:, ::-1].reshape(-1)
    order = np.lexsort((pts, other, bk))
    members = pts[order].astype(np.int32)
    bsorted = bk[order]
    offsets = np.zeros(B + 1, np.int64)
    np.add.at(offsets, bsorted + 1, 1)
    offsets = np.cumsum(offsets)
    mem_row = np.empty((N, W), np.int64)
    rows = np.arange(N * W, dtype=np.int64)
    # rank of this membership among the point's buckets (ascending bucket id)
    lo_b = top2.min(axis=1)
    way = (bsorted != lo_b[members]).astype(np.int64)
    mem_row[members.astype(np.int64), way] = rows
    return offsets, members, mem_row


def bucket_knn(X, offsets, members, M: int):
    X = _f32(X)
    offsets = np.ascontiguousarray(offsets, dtype=np.int64)
    members = np.ascontiguousarray(members, dtype=np.int32)
    n = members.shape[0]
    ids = np.empty((n, M), np.int32)
    dist = np.empty((n, M), np.float32)
    lib().orc_bucket_knn(_p(X), X.shape[0], X.shape[1], _p(offsets), _p(members), offsets.shape[0] - 1, M,
                         _p(ids), _p(dist))
    return ids, dist


def point_lists(X, top2, points, M: int):
    """The oracle pipeline's merged kNN list of each of ``points`` (a sample), without building
    every bucket: the point's exact top-M within each of its two buckets (fp32 chain, ties by id,
    itself excluded: bucket_knn's rule), merged with the lower bucket's list as the running side
    (merge_memberships' rule, bucket.cu:5025-5059).  Returns (ids, dists) [len(points) x M]."""
    X = _f32(X)
    top2 = np.asarray(top2, dtype=np.int64)
    points = np.asarray(points, dtype=np.int64)
    flat = top2.reshape(-1)
    order = np.argsort(flat, kind="stable")
    starts = np.searchsorted(flat[order], np.arange(flat.max() + 2))
    P = len(points)
    lists = [(np.full((P, M), -1, np.int32), np.full((P, M), np.inf, np.float32)) for _ in range(2)]
    for i, p in enumerate(points):
        bs = np.sort(top2[p])
        for way, b in enumerate(bs):
            mem = (order[starts[b]:starts[b + 1]] // top2.shape[1]).astype(np.int64)
            mem = mem[mem != p]
            dist = pair_l2(X, np.full(mem.shape[0], p), mem)
            sel = np.lexsort((mem, dist))[:M]
            lists[way][0][i, :sel.size] = mem[sel]
            lists[way][1][i, :sel.size] = dist[sel]
    return merge_lists(lists[0][0], lists[0][1], lists[1][0], lists[1][1])


def merge_lists(run_n, run_d, new_n, new_d):
    run_n = np.ascontiguousarray(run_n, np.int32); run_d = np.ascontiguousarray(run_d, np.float32)
    new_n = np.ascontiguousarray(new_n, np.int32); new_d = np.ascontiguousarray(new_d, np.float32)
    N, M = run_n.shape
    on = np.empty_like(run_n); od = np.empty_like(run_d)
    lib().orc_merge_lists(_p(run_n), _p(run_d), _p(new_n), _p(new_d), _p(on), _p(od), N, M)
    return on, od


def merge_memberships(list_n, list_d, mem_row):
    list_n = np.ascontiguousarray(list_n, np.int32); list_d = np.ascontiguousarray(list_d, np.float32)
    mem_row = np.ascontiguousarray(mem_row, np.int64)
    N = mem_row.shape[0]
    M = list_n.shape[1]
    on = np.empty((N, M), np.int32); od = np.empty((N, M), np.float32)
    lib().orc_merge_memberships(_p(list_n), _p(list_d), _p(mem_row), N, M, _p(on), _p(od))
    return on, od


def sanitize(knn):
    knn = np.ascontiguousarray(knn, np.int32)
    N, M = knn.shape
    out = np.empty((N, M), np.uint32)
    n_pad = lib().orc_sanitize(_p(knn), N, M, _p(out))
    return out, int(n_pad)


def sort_rows_l2(X, knn):
    X = _f32(X); knn = np.ascontiguousarray(knn, np.int32)
    out = np.empty_like(knn)
    lib().orc_sort_rows_l2(_p(X), X.shape[1], _p(knn), knn.shape[0], knn.shape[1], _p(out))
    return out


def detour_counts(g, a: int):
    g = np.ascontiguousarray(g, np.uint32)
    out = np.empty(g.shape[1], np.uint32)
    lib().orc_detour_counts(_p(g), g.shape[0], g.shape[1], int(a), _p(out))
    return out


def prune(g, K: int):
    g = np.ascontiguousarray(g, np.uint32)
    out = np.empty((g.shape[0], K), np.uint32)
    lib().orc_prune(_p(g), g.shape[0], g.shape[1], K, _p(out))
    return out


def reverse_merge(pruned):
    out = np.ascontiguousarray(pruned, np.uint32).copy()
    rc = lib().orc_reverse_merge(_p(out), out.shape[0], out.shape[1])
    assert rc == 0
    return out


def optimize(knn_u32, K: int):
    g = np.ascontiguousarray(knn_u32, np.uint32)
    out = np.empty((g.shape[0], K), np.uint32)
    rc = lib().orc_optimize(_p(g), g.shape[0], g.shape[1], K, _p(out))
    if rc != 0:
        raise ValueError(f"orc_optimize failed ({rc})")
    return out


def graph_search(base, graph, queries, entries, topk: int, ef: int):
    """search.py:20-93 graph_search_single for every query, with the given entry
    points (nq x ne, ascending, -1 unused): ids / distances (nq x topk)."""
    base = _f32(base)
    q = _f32(queries)
    g = np.ascontiguousarray(graph, np.uint32)
    e = np.ascontiguousarray(entries, np.int32)
    nq = q.shape[0]
    ids = np.empty((nq, topk), np.int32)
    dist = np.empty((nq, topk), np.float32)
    lib().orc_graph_search(_p(base), base.shape[0], base.shape[1], _p(g), g.shape[1], _p(q), nq, _p(e), e.shape[1],
                           topk, ef, _p(ids), _p(dist))
    return ids, dist


def search_entries(n: int, nq: int, num_entry: int, seed: int = 42) -> np.ndarray:
    """The entry points search.py draws (:40-41 with the generator of :163, called per query at :170-172): one
    default_rng(seed) shared by the queries in order, np.unique per query; padded with -1."""
    rng = np.random.default_rng(seed)
    k = max(1, num_entry)
    out = np.full((nq, k), -1, np.int32)
    for i in range(nq):
        u = np.unique(rng.integers(0, n, size=k, endpoint=False))
        out[i, :u.size] = u
    return out


def bucket_reorder(assign, B: int, order=None, stride: int = 1):
    """compute_bucket_reorder (bucket.cu:8356-8417): (inverse_perm uint32[placed], offsets int64[B+1])."""
    a = np.ascontiguousarray(assign, np.int32)
    n = a.size // stride
    inv = np.zeros(n, np.uint32)
    off = np.zeros(B + 1, np.int64)
    o = None if order is None else np.ascontiguousarray(order, np.int32)
    placed = lib().orc_bucket_reorder(_p(a), n, stride, B, _p(o) if o is not None else None, _p(inv), _p(off))
    return inv[:placed], off


def permute_graph(g, inv, to_original: bool, keep_padding: bool):
    """translate_graph_ids.hpp:75-200 (to_original) and its inverse; returns (out, bad) with
    bad = -1 when inv is not a permutation."""
    g = np.ascontiguousarray(g).view(np.int32) if np.asarray(g).dtype.itemsize == 4 else np.ascontiguousarray(g, np.int32)
    inv = np.ascontiguousarray(inv, np.uint32)
    out = np.empty_like(g)
    bad = lib().orc_permute_graph(_p(g), g.shape[0], g.shape[1], _p(inv), int(to_original), int(keep_padding), _p(out))
    return out, int(bad)


def bucket_order(adj, window: int):
    """compute_bucket_processing_order (bucket_order.hpp:143-200) over a flat (B, K) bucket graph."""
    adj = np.ascontiguousarray(adj, np.int32)
    B, K = adj.shape
    out = np.empty(B, np.int32)
    lib().orc_bucket_order(_p(adj), B, K, window, _p(out))
    return out


def bucket2_requested(N: int, ratio: float) -> int:
    """max(2, floor(N * r)) with r the ratio as a C float widened to double (0 means 0.01)."""
    r = float(np.float32(ratio)) if ratio > 0 else 0.01
    return max(2, int(float(N) * r))


def kmeans_parallel(X, n_req: int, seed: int) -> np.ndarray:
    """KMeans|| data-point centroids (bucket.cu:2919-3172 restated): their point ids."""
    X = _f32(X)
    out = np.empty(n_req, np.int32)
    n = lib().orc_kmeans_parallel(_p(X), X.shape[0], X.shape[1], n_req, ctypes.c_uint64(seed & (2**64 - 1)), _p(out))
    return out[:n].copy()


def balanced_assign(top2, B: int, cid, top2_d=None, rule: int = 0) -> np.ndarray:
    """The balanced 1-way choice (bucket.cu:1655-1660, :2276-2301), each point against the sizes
    left by the earlier ones; rule 1 = BUCKET2_ASSIGN_RULE=diskjoin (needs top2_d)."""
    top2 = np.ascontiguousarray(top2, np.int32)
    cid = np.ascontiguousarray(cid, np.int32)
    td = None if top2_d is None else np.ascontiguousarray(top2_d, np.float32)
    assert rule == 0 or td is not None
    out = np.full(top2.shape[0], -1, np.int32)
    bad = lib().orc_balanced_assign(_p(top2), None if td is None else _p(td), top2.shape[0], B, _p(cid), rule,
                                    _p(out))
    assert bad == 0
    return out


def pool_tables(assign, B: int, adj):
    """The resident round's pool tables (bucket.cu:5317-5346 restated): (offsets[B+1], members[N],
    seg_bucket[B, P+1], seg_ofs[B, P+1], pool_size[B])."""
    assign = np.ascontiguousarray(assign, np.int32)
    adj = np.ascontiguousarray(adj, np.int32).reshape(B, -1)
    P = adj.shape[1]
    N = assign.shape[0]
    off = np.empty(B + 1, np.int64)
    mem = np.empty(max(N, 1), np.int32)
    seg_b = np.empty((B, P + 1), np.int32)
    seg_o = np.empty((B, P + 1), np.int64)
    pool = np.empty(B, np.int64)
    lib().orc_pool_tables(_p(assign), N, B, _p(adj), P, _p(off), _p(mem), _p(seg_b), _p(seg_o), _p(pool))
    return off, mem[:N], seg_b, seg_o, pool


def pool_knn(X, assign, B: int, adj, M: int):
    """Own + neighbour-bucket pool kNN of every point (bucket.cu:5310-5365 restated)."""
    X = _f32(X)
    assign = np.ascontiguousarray(assign, np.int32)
    adj = np.ascontiguousarray(adj, np.int32).reshape(B, -1)
    P = adj.shape[1]
    ids = np.empty((X.shape[0], M), np.int32)
    dist = np.empty((X.shape[0], M), np.float32)
    lib().orc_pool_knn(_p(X), X.shape[0], X.shape[1], _p(assign), B, _p(adj), P, M, _p(ids), _p(dist))
    return ids, dist


def build_bucket2(X, M: int, nprobe: int = 0, centroid_ratio: float = 0.01, seed: int = 42, rounds: int = 1,
                  knn_k: int = 0, assign_rule: int = 0):
    """The reference-bucketing build restated: (ids, dists, assign, centroid ids) of the last round,
    rounds merged with the resident merge rule."""
    Xf = _f32(X)
    N = Xf.shape[0]
    n_req = bucket2_requested(N, centroid_ratio)
    run = None
    for r in range(max(1, rounds)):
        cid = kmeans_parallel(Xf, n_req, seed + r)
        B = cid.size
        C = Xf[cid]
        P = nprobe if nprobe > 0 else (knn_k if knn_k > 0 else 32)
        P = min(P, B - 1)
        adj = np.zeros((B, max(P, 0)), np.int32)
        if P > 0:
            ki, _ = topk_assign(C, C, P + 1)
            for b in range(B):
                row = list(ki[b])
                row.remove(b) if b in row else row.pop()
                adj[b] = row[:P]
        top2, t2d = topk_assign(Xf, C, 2)
        assign = balanced_assign(top2, B, cid, t2d, assign_rule)
        ids, dist = pool_knn(Xf, assign, B, adj, M)
        run = (ids, dist) if run is None else merge_lists(run[0], run[1], ids, dist)
    return run[0], run[1], assign, cid


def exact_knn(X, queries, k: int):
    X = _f32(X)
    q = np.ascontiguousarray(queries, np.int64)
    ids = np.empty((q.shape[0], k), np.int32)
    dist = np.empty((q.shape[0], k), np.float32)
    lib().orc_exact_knn(_p(X), X.shape[0], X.shape[1], _p(q), q.shape[0], k, _p(ids), _p(dist))
    return ids, dist


def knn_recall(approx_ids, gt_ids, k: int) -> float:
    """|approx top-k ∩ exact top-k| / k averaged over rows (knn_similarity.py rule)."""
    a = np.asarray(approx_ids)[:, :k]
    g = np.asarray(gt_ids)[:, :k]
    hit = 0
    for i in range(a.shape[0]):
        hit += len(np.intersect1d(a[i][a[i] >= 0], g[i]))
    return hit / float(a.shape[0] * k)


def build_knn_graph(X, C0, B: int, M: int, kmeans_iters: int, sample_ids=None):
    """Whole oracle pipeline up to the per-point kNN lists (given initial centroids)."""
    X = _f32(X)
    Xs = X if sample_ids is None else X[sample_ids]
    C, _ = kmeans(Xs, C0, kmeans_iters)
    top2, _ = topk_assign(X, C, 2)
    offsets, members, mem_row = build_csr(top2, B)
    ln, ld = bucket_knn(X, offsets, members, M)
    kn, kd = merge_memberships(ln, ld, mem_row)
    return dict(centroids=C, top2=top2, offsets=offsets, members=members, mem_row=mem_row,
                list_ids=ln, list_dists=ld, knn_ids=kn, knn_dists=kd)
