"""Multi-GPU bucketed kNN / CAGRA build: one process per GPU, torch.distributed
(NCCL) for the exchanges, libgta kernels for every computation.

This follows the multi-GPU plan of the reference's build (bucketDemo/buildBucket/src/
bucket.cu: row-sharded k-means with all-reduced sums, buckets placed on owner GPUs,
points and lists exchanged, then a merge on the point's owner), with one
difference of layout: every rank keeps the original row order, so the reference's
inverse permutation is the identity.

A rank holds global rows [row0, row0 + n_local) of an N-row dataset (rank r's rows
come before rank r+1's).  The steps and their exchanges:

  1. k-means.  The k-means++ pool is drawn over all N ids (identical on every
     rank), each rank fills the rows it holds and an all-reduce completes it; the
     initial centroids are then computed identically everywhere.  Lloyd runs on the
     rank's part of the global sample: local assignment, local fp64 sums and counts,
     an all-reduce of both, new means.
  2. Top-2 buckets of the local rows.
  3. Bucket placement: global bucket sizes (all-reduce), then longest-processing-
     time placement on the cost n_b^2, the same on every rank.  A bucket that costs
     more than a rank's share of the whole is cut into row ranges (pieces) placed on
     distinct ranks, each of which holds all the bucket's rows as columns.
  4. Points to every rank holding a piece of their bucket (all-to-all of rows and
     (id, bucket, other) triples), grouped by (bucket, other) in arrival order: the
     membership order of the single-GPU build, the same on every holder.
  5. Per-bucket all-pairs top-M on the holders, each for its row range, in two
     passes: the rows whose bucket is the lower of their point's two, then (after an
     all-reduce (min) of each point's lower-list M-th distance by global id) the
     other rows, bounded by that distance and skipping the points of the lower
     bucket; the merged lists are unchanged.
  6. The lists of each rank's row ranges back to the points' owners (all-to-all),
     merged per point.
  7. CAGRA: sanitize the local rows, all-gather the id table, prune the local rows,
     all-gather the pruned graph, merge reverse edges into the local rows.

For integer data (u8 / i8) every value the single-GPU build computes is
reproduced exactly: the centroid sums are sums of integers in fp64, and every
other stage sees the same inputs in the same order.  For f32 data the centroid
sums are added in a different order, so centroids may differ in the last bit.

``Stages`` is the per-rank compute interface; ``CudaStages`` binds libgta (the packing of
every exchange included: gta_shard_pack_memberships / gta_shard_pack_lists).  The driver
itself only places buckets (host arithmetic on B sizes) and runs the collectives.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib as L

_ELEM = {torch.float32: L.GTA_F32, torch.uint8: L.GTA_U8, torch.int8: L.GTA_I8}


@dataclass
class ShardParams:
    """Parameters of the build; the same meaning as gta_bucket_params / gta_cagra_params."""

    n_buckets: int
    knn_degree: int = 64
    graph_degree: int = 0  # 0: stop after the kNN lists
    kmeans_iters: int = 10
    kmeans_sample: int = 0
    seed: int = 42
    # a bucket whose cost n_b^2 exceeds split_share x (sum n_b^2 / ranks) runs as row ranges on
    # several ranks (inf: whole buckets only)
    split_share: float = 1.0


@dataclass
class ShardResult:
    row0: int
    n_total: int
    knn_ids: torch.Tensor  # n_local x M int32, global ids
    knn_dists: torch.Tensor  # n_local x M float32
    centroids: torch.Tensor  # B x d float32
    top2: torch.Tensor  # n_local x 2 int32
    graph: Optional[torch.Tensor] = None  # n_local x K (int32 view of uint32 ids)
    owner: Optional[list] = None  # bucket -> rank (of its first piece)
    pieces: Optional[list] = None  # (bucket, rank, row_lo, row_hi) per piece, by (bucket, row_lo)
    sizes: Optional[list] = None  # memberships per bucket (whole job)
    comm_bytes: int = 0  # bytes this rank sent
    phase_ms: Optional[dict] = None  # device time per phase when timing was requested


# ---------------------------------------------------------------- libgta stages
def _p(t: Optional[torch.Tensor]) -> ctypes.c_void_p:
    if t is None:
        return ctypes.c_void_p(0)
    if not t.is_contiguous():
        raise L.GtaError(L.GTA_EINVAL, "libgta stages take contiguous tensors")
    return ctypes.c_void_p(t.data_ptr())


class CudaStages:
    """The per-rank computations, each one libgta call on the current CUDA stream."""

    def __init__(self):
        self.L = L.lib()

    @staticmethod
    def _st():
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def kmeans_sizes(self, n, prm: ShardParams):
        bp = L.gta_bucket_params(n_buckets=prm.n_buckets, kmeans_iters=prm.kmeans_iters, knn_degree=prm.knn_degree,
                                 kmeans_sample=prm.kmeans_sample, seed=prm.seed)
        n_s, pool_n, pseed = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_uint64()
        L.check(self.L.gta_kmeans_sizes(n, ctypes.byref(bp), ctypes.byref(n_s), ctypes.byref(pool_n),
                                        ctypes.byref(pseed)))
        return n_s.value, pool_n.value, pseed.value

    def sample_ids(self, n, n_s, seed, device):
        out = torch.empty(n_s, dtype=torch.int32, device=device)
        L.check(self.L.gta_sample_ids(n, n_s, seed, _p(out), self._st()))
        return out

    def gather_rows(self, X, row0, ids):
        out = torch.empty((ids.numel(), X.shape[1]), dtype=torch.float32, device=X.device)
        L.check(self.L.gta_gather_rows(_p(X), _ELEM[X.dtype], X.shape[0], X.shape[1], row0, _p(ids), ids.numel(),
                                       _p(out), self._st()))
        return out

    def kmeans_init(self, pool, B, seed):
        C = torch.empty((B, pool.shape[1]), dtype=torch.float32, device=pool.device)
        L.check(self.L.gta_kmeans_init(_p(pool), pool.shape[0], pool.shape[1], B, seed, _p(C), self._st()))
        return C

    def assign_topk(self, Xf, C, k, integer_rows=False):
        n = Xf.shape[0]
        ids = torch.empty((n, k), dtype=torch.int32, device=Xf.device)
        dd = torch.empty((n, k), dtype=torch.float32, device=Xf.device)
        if n:
            L.check(self.L.gta_assign_topk_ex(_p(Xf), n, Xf.shape[1], _p(C), C.shape[0], k, _p(ids), _p(dd),
                                              L.GTA_ROWS_INTEGER if integer_rows else 0, self._st()))
        return ids

    def centroid_sums(self, Xf, assign, B):
        d = Xf.shape[1]
        sums = torch.empty((B, d), dtype=torch.float64, device=Xf.device)
        counts = torch.empty(B, dtype=torch.int64, device=Xf.device)
        L.check(self.L.gta_centroid_sums(_p(Xf), Xf.shape[0], d, _p(assign), B, _p(sums), _p(counts), self._st()))
        return sums, counts

    def centroid_means(self, sums, counts, C):
        C = C.clone()
        L.check(self.L.gta_centroid_means(_p(sums), _p(counts), C.shape[0], C.shape[1], _p(C), self._st()))
        return C

    def group_memberships(self, bucket, other, B):
        n = bucket.numel()
        order = torch.empty(n, dtype=torch.int32, device=bucket.device)
        offsets = torch.empty(B + 1, dtype=torch.int64, device=bucket.device)
        L.check(self.L.gta_group_memberships(_p(bucket), _p(other), n, B, _p(order), _p(offsets), self._st()))
        return order, offsets

    def bucket_knn_rows(self, R, order, gid, offsets, M):
        n = R.shape[0]
        ids = torch.empty((n, M), dtype=torch.int32, device=R.device)
        dd = torch.empty((n, M), dtype=torch.float32, device=R.device)
        L.check(self.L.gta_bucket_knn_rows(_p(R), _ELEM[R.dtype], n, R.shape[1], _p(order), _p(gid), _p(offsets),
                                           offsets.numel() - 1, M, _p(ids), _p(dd), self._st()))
        return ids, dd

    def bucket_knn_rows_phased(self, R, order, gid, offsets, partner, M, phase, seed, lid, ldist):
        """Rows of one phase into lid / ldist (see gta_bucket_knn_rows_phased)."""
        n = R.shape[0]
        L.check(self.L.gta_bucket_knn_rows_phased(_p(R), _ELEM[R.dtype], n, R.shape[1], _p(order), _p(gid),
                                                  _p(offsets), _p(partner), offsets.numel() - 1, M, phase, _p(seed),
                                                  _p(lid), _p(ldist), self._st()))

    def bucket_knn_rows_ranged(self, R, order, gid, offsets, partner, M, phase, seed, row_lo, row_hi, lid, ldist):
        """Rows of one phase and of each bucket's range [row_lo[b], row_hi[b]) (host int64 tensors)
        into lid / ldist (see gta_bucket_knn_rows_ranged)."""
        n = R.shape[0]
        rlo = row_lo.to(torch.int64).contiguous()
        rhi = row_hi.to(torch.int64).contiguous()
        L.check(self.L.gta_bucket_knn_rows_ranged(_p(R), _ELEM[R.dtype], n, R.shape[1], _p(order), _p(gid),
                                                  _p(offsets), _p(partner), offsets.numel() - 1, M, phase, _p(seed),
                                                  ctypes.c_void_p(rlo.data_ptr()), ctypes.c_void_p(rhi.data_ptr()),
                                                  _p(lid), _p(ldist), self._st()))

    def pack_memberships(self, X_local, row0, top2, holders, world):
        """Every local membership to the holders of its bucket, packed by destination rank:
        (rows [k x d] of X's dtype, meta [k x 3] int32, per-rank counts)."""
        n, d = X_local.shape
        cnt = (ctypes.c_int64 * world)()
        h = holders.to(device=X_local.device, dtype=torch.int64).contiguous()
        args = (_p(X_local), _ELEM[X_local.dtype], n, d, row0, _p(top2), h.numel(), _p(h), world, cnt)
        L.check(self.L.gta_shard_pack_memberships(*args, None, None, 0, self._st()))
        k = sum(cnt)
        rows = torch.empty((k, d), dtype=X_local.dtype, device=X_local.device)
        meta = torch.empty((k, 3), dtype=torch.int32, device=X_local.device)
        L.check(self.L.gta_shard_pack_memberships(*args, _p(rows), _p(meta), k, self._st()))
        return rows, meta, list(cnt)

    def pack_lists(self, lid, ldist, order, gid, offsets, row_lo, row_hi, starts, world):
        """The lists of this rank's row ranges to their points' owners, packed by destination:
        (ids [k x M], dists [k x M], meta [k x 2] = (global id, bucket), per-rank counts)."""
        n, M = lid.shape
        cnt = (ctypes.c_int64 * world)()
        lo = row_lo.to(torch.int64).contiguous()
        hi = row_hi.to(torch.int64).contiguous()
        stt = torch.tensor(starts, dtype=torch.int64)
        args = (_p(lid), _p(ldist), n, M, _p(order), _p(gid), _p(offsets), offsets.numel() - 1,
                ctypes.c_void_p(lo.data_ptr()), ctypes.c_void_p(hi.data_ptr()), ctypes.c_void_p(stt.data_ptr()),
                world, cnt)
        L.check(self.L.gta_shard_pack_lists(*args, None, None, None, 0, self._st()))
        k = sum(cnt)
        ids = torch.empty((k, M), dtype=torch.int32, device=lid.device)
        dd = torch.empty((k, M), dtype=torch.float32, device=lid.device)
        meta = torch.empty((k, 2), dtype=torch.int32, device=lid.device)
        L.check(self.L.gta_shard_pack_lists(*args, _p(ids), _p(dd), _p(meta), k, self._st()))
        return ids, dd, meta, list(cnt)

    def member_rows(self, meta, row0, n_local, top2):
        mem_row = torch.empty((n_local, 2), dtype=torch.int64, device=top2.device)
        L.check(self.L.gta_shard_member_rows(_p(meta), meta.shape[0], row0, n_local, _p(top2), _p(mem_row),
                                             self._st()))
        return mem_row

    def lower_seeds(self, ldist, order, gid, offsets, partner, row_lo, row_hi, N):
        seed = torch.empty((N,), dtype=torch.float32, device=ldist.device)
        lo = row_lo.to(torch.int64).contiguous()
        hi = row_hi.to(torch.int64).contiguous()
        L.check(self.L.gta_shard_lower_seeds(_p(ldist), ldist.shape[1], ldist.shape[0], _p(order), _p(gid),
                                             _p(offsets), _p(partner), offsets.numel() - 1,
                                             ctypes.c_void_p(lo.data_ptr()), ctypes.c_void_p(hi.data_ptr()), N,
                                             _p(seed), self._st()))
        return seed

    def merge_memberships(self, lid, ldist, mem_row):
        n, M = mem_row.shape[0], lid.shape[1]
        ids = torch.empty((n, M), dtype=torch.int32, device=lid.device)
        dd = torch.empty((n, M), dtype=torch.float32, device=lid.device)
        if n:
            L.check(self.L.gta_merge_memberships(_p(lid), _p(ldist), _p(mem_row), n, M, _p(ids), _p(dd), self._st()))
        return ids, dd

    def sanitize_rows(self, knn, row0, n_total):
        out = torch.empty(knn.shape, dtype=torch.int32, device=knn.device)
        L.check(self.L.gta_sanitize_rows(_p(knn), knn.shape[0], row0, n_total, knn.shape[1], _p(out), self._st()))
        return out

    def prune_rows(self, g_full, K, row0, n_rows, top2, B):
        out = torch.empty((n_rows, K), dtype=torch.int32, device=g_full.device)
        L.check(self.L.gta_prune_rows(_p(g_full), g_full.shape[0], g_full.shape[1], K, row0, n_rows, _p(top2), B,
                                      _p(out), self._st()))
        return out

    def reverse_merge_rows(self, pruned_full, row0, n_rows):
        K = pruned_full.shape[1]
        out = torch.empty((n_rows, K), dtype=torch.int32, device=pruned_full.device)
        L.check(self.L.gta_reverse_merge_rows(_p(pruned_full), pruned_full.shape[0], K, row0, n_rows, _p(out),
                                              self._st()))
        return out


# ---------------------------------------------------------------- host logic
def place_buckets(sizes, world: int) -> list:
    """Longest-processing-time placement of whole buckets on ranks by cost n_b^2.

    Largest cost first (ties: lower bucket id), each to the least-loaded rank
    (ties: lower rank).  Deterministic, so every rank computes the same owners.
    """
    return [p[1] for p in place_pieces(sizes, world, float("inf"))]


def place_pieces(sizes, world: int, split_share: float = 1.0, align: int = 128) -> list:
    """Row ranges of buckets placed on ranks: [(bucket, rank, row_lo, row_hi)] by (bucket, row_lo).

    A bucket of n rows costs n^2 (all pairs).  One whose cost exceeds split_share x the
    mean cost per rank is cut into s = min(ranks, ceil(cost / that), n // align) pieces of
    about n / s rows (cuts at multiples of ``align``), each costing its rows x n; every
    other bucket is one piece [0, n).  Pieces are placed longest-processing-time: largest
    cost first (ties: bucket, then row_lo), each on the least-loaded rank (ties: lower rank)
    that holds no other piece of its bucket.  Deterministic, so every rank computes the
    same placement.
    """
    sizes = [int(x) for x in sizes]
    share = split_share * sum(x * x for x in sizes) / max(world, 1)
    items = []
    for b, n in enumerate(sizes):
        s = 1
        if world > 1 and n > 0 and n * n > share:
            s = max(1, min(world, -(-(n * n) // max(int(share), 1)), n // align))
        cuts = [(i * n // s) // align * align for i in range(s)] + [n]
        for i in range(s):
            items.append(((cuts[i + 1] - cuts[i]) * n, b, cuts[i], cuts[i + 1]))
    items.sort(key=lambda it: (-it[0], it[1], it[2]))
    load = [0] * world
    held = [set() for _ in range(world)]
    out = []
    for cost, b, lo, hi in items:
        r = min((q for q in range(world) if b not in held[q]), key=lambda q: (load[q], q))
        load[r] += cost
        held[r].add(b)
        out.append((b, r, lo, hi))
    out.sort(key=lambda p: (p[0], p[2]))
    return out


def _exchange(send: torch.Tensor, send_counts: torch.Tensor, recv_counts: torch.Tensor, group=None) -> torch.Tensor:
    """all_to_all_single of row-blocks with per-rank row counts."""
    row_shape = tuple(send.shape[1:])
    out = torch.empty((int(recv_counts.sum()),) + row_shape, dtype=send.dtype, device=send.device)
    dist.all_to_all_single(out, send.contiguous(), recv_counts.tolist(), send_counts.tolist(), group=group)
    return out


def _all_gather_rows(local: torch.Tensor, counts: list, group=None) -> torch.Tensor:
    """Concatenation of every rank's rows (rank order), for uneven row counts."""
    world = len(counts)
    mx = max(counts)
    if all(c == mx for c in counts):
        out = torch.empty((mx * world,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    pad = torch.zeros((mx,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    buf = torch.empty((mx * world,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, pad, group=group)
    return torch.cat([buf[r * mx: r * mx + counts[r]] for r in range(world)])


class _Phases:
    """CUDA-event marks between the driver's phases (when timing is on)."""

    def __init__(self, on: bool):
        self.on = on and torch.cuda.is_available()
        self.marks = []

    def mark(self, name: str):
        if self.on:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.marks.append((name, ev))

    def result(self):
        if not self.on or len(self.marks) < 2:
            return None
        torch.cuda.synchronize()
        return {n: self.marks[i - 1][1].elapsed_time(e) for i, (n, e) in enumerate(self.marks) if i > 0}


def build_sharded(X_local: torch.Tensor, prm: ShardParams, stages=None, init_centroids: Optional[torch.Tensor] = None,
                  group=None, timing: bool = False) -> ShardResult:
    """One rank's part of the multi-GPU build.  X_local: this rank's rows (contiguous
    global row block, rank order), on the rank's device.  Collective: every rank of
    ``group`` calls it with the same ``prm``.  With ``timing`` the result carries the
    device time of each phase (kernels and collectives) on this rank."""
    st = stages if stages is not None else CudaStages()
    ph = _Phases(timing)
    ph.mark("start")
    dev = X_local.device
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n_local, d = X_local.shape
    int_rows = X_local.dtype in (torch.uint8, torch.int8)  # exact in tf32: the split assignment screen
    B, M = prm.n_buckets, prm.knn_degree
    sent = 0

    # ---- row ranges
    cnt = torch.tensor([n_local], dtype=torch.int64, device=dev)
    counts_t = torch.empty(world, dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(counts_t, cnt, group=group)
    counts = counts_t.tolist()
    starts = [0] * (world + 1)
    for r in range(world):
        starts[r + 1] = starts[r] + counts[r]
    N, row0 = starts[world], starts[rank]
    if not (2 <= B <= N):
        raise L.GtaError(L.GTA_EINVAL, "build_sharded: need 2 <= n_buckets <= N")

    # ---- 1. k-means
    n_s, pool_n, pool_seed = st.kmeans_sizes(N, prm)
    if init_centroids is not None:
        C = init_centroids.to(device=dev, dtype=torch.float32).contiguous()
    else:
        pool_ids = st.sample_ids(N, pool_n, pool_seed, dev)
        pool = st.gather_rows(X_local, row0, pool_ids)
        dist.all_reduce(pool, group=group)
        C = st.kmeans_init(pool, B, prm.seed)
        del pool
    ph.mark("kmeans_init")
    sid = st.sample_ids(N, n_s, prm.seed, dev)
    mine = sid[(sid >= row0) & (sid < row0 + n_local)].contiguous()
    Xs = st.gather_rows(X_local, row0, mine)
    for _ in range(prm.kmeans_iters):
        a = st.assign_topk(Xs, C, 1, int_rows).reshape(-1).contiguous()
        sums, cts = st.centroid_sums(Xs, a, B)
        dist.all_reduce(sums, group=group)
        dist.all_reduce(cts, group=group)
        C = st.centroid_means(sums, cts, C)
    del Xs
    ph.mark("lloyd")

    # ---- 2. top-2 buckets of the local rows
    gid_local = torch.arange(row0, row0 + n_local, dtype=torch.int32, device=dev)
    Xf = st.gather_rows(X_local, row0, gid_local)
    top2 = st.assign_topk(Xf, C, 2, int_rows).contiguous()
    del Xf

    # ---- 3. placement.  The count of memberships without a valid bucket (a non-finite row) rides
    # on the sizes' all-reduce, so every rank raises together rather than one rank leaving the
    # others waiting in the next collective.
    flat = top2.reshape(-1).long()
    ok = (flat >= 0) & (flat < B)
    sizes = torch.cat([torch.bincount(flat[ok], minlength=B).to(torch.int64),
                       (~ok).sum().reshape(1).to(torch.int64)])
    dist.all_reduce(sizes, group=group)
    sizes_l = sizes.tolist()
    if sizes_l.pop() > 0:
        raise L.GtaError(L.GTA_EDATA, "build_sharded: a row has no valid bucket (non-finite input?)")
    pieces = place_pieces(sizes_l, world, prm.split_share)
    holders = [0] * B
    row_lo, row_hi = [0] * B, [0] * B
    owner = [-1] * B
    for b, r, lo, hi in pieces:
        holders[b] |= 1 << r
        if owner[b] < 0:
            owner[b] = r
        if r == rank:
            row_lo[b], row_hi[b] = lo, hi
    # the holder masks as int64 bit patterns (bit 63 is rank 63)
    holders_t = torch.tensor([h - (1 << 64) if h >= 1 << 63 else h for h in holders], dtype=torch.int64)
    rlo_h = torch.tensor(row_lo, dtype=torch.int64)
    rhi_h = torch.tensor(row_hi, dtype=torch.int64)
    ph.mark("top2_placement")

    # ---- 4. memberships to every holder of their bucket (slot s of point p is membership 2p+s),
    # packed by destination in membership order
    rows, meta, send_l = st.pack_memberships(X_local, row0, top2, holders_t, world)
    send_counts = torch.tensor(send_l, dtype=torch.int64, device=dev)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    elem = rows.element_size()
    R = _exchange(rows.reshape(rows.shape[0], -1).view(torch.uint8), send_counts, recv_counts, group)
    R = R.view(X_local.dtype).reshape(-1, d)
    meta_r = _exchange(meta, send_counts, recv_counts, group)
    sent += rows.numel() * elem + meta.numel() * 4
    del rows, meta
    ph.mark("exchange_points")

    # ---- 5. per-bucket top-M for this rank's row range of each bucket it holds: first the rows
    # whose bucket is the lower of their point's two, then the others, bounded by the point's
    # lower-bucket list (its M-th distance, gathered by global id over the ranks) and skipping the
    # points of that lower bucket
    gid_r = meta_r[:, 0].contiguous()
    order, offsets = st.group_memberships(meta_r[:, 1].contiguous(), meta_r[:, 2].contiguous(), B)
    n_r = R.shape[0]
    partner_s = meta_r[:, 2][order.long()].contiguous()
    lid = torch.full((n_r, M), -1, dtype=torch.int32, device=dev)
    ldist = torch.full((n_r, M), float("inf"), dtype=torch.float32, device=dev)
    st.bucket_knn_rows_ranged(R, order, gid_r, offsets, partner_s, M, 1, None, rlo_h, rhi_h, lid, ldist)
    seed = st.lower_seeds(ldist, order, gid_r, offsets, partner_s, rlo_h, rhi_h, N)
    dist.all_reduce(seed, op=dist.ReduceOp.MIN, group=group)
    st.bucket_knn_rows_ranged(R, order, gid_r, offsets, partner_s, M, 2, seed, rlo_h, rhi_h, lid, ldist)
    del R, seed
    ph.mark("bucket_knn")

    # ---- 6. the ranges' lists back to the points' owners, merged per point
    ids_s, dists_s, meta2, send2_l = st.pack_lists(lid, ldist, order, gid_r, offsets, rlo_h, rhi_h, starts, world)
    send2 = torch.tensor(send2_l, dtype=torch.int64, device=dev)
    recv2 = torch.empty_like(send2)
    dist.all_to_all_single(recv2, send2, group=group)
    lid_b = _exchange(ids_s, send2, recv2, group)
    ldist_b = _exchange(dists_s, send2, recv2, group)
    meta_b = _exchange(meta2, send2, recv2, group)
    sent += ids_s.numel() * 8 + meta2.numel() * 4
    del lid, ldist, ids_s, dists_s, meta2
    ph.mark("exchange_lists")
    mem_row = st.member_rows(meta_b, row0, n_local, top2)
    knn_ids, knn_dists = st.merge_memberships(lid_b.contiguous(), ldist_b.contiguous(), mem_row)
    del lid_b, ldist_b
    ph.mark("merge")

    res = ShardResult(row0=row0, n_total=N, knn_ids=knn_ids, knn_dists=knn_dists, centroids=C, top2=top2,
                      owner=owner, pieces=pieces, sizes=sizes_l)
    # ---- 7. CAGRA
    if prm.graph_degree > 0:
        K = prm.graph_degree
        g_local = st.sanitize_rows(knn_ids, row0, N)
        g_full = _all_gather_rows(g_local, counts, group)
        sent += g_local.numel() * 4 * (world - 1)
        ph.mark("gather_graph")
        pruned = st.prune_rows(g_full, K, row0, n_local, top2, B)
        del g_full
        ph.mark("prune")
        p_full = _all_gather_rows(pruned, counts, group)
        sent += pruned.numel() * 4 * (world - 1)
        ph.mark("gather_pruned")
        res.graph = st.reverse_merge_rows(p_full, row0, n_local)
        ph.mark("reverse")
    res.comm_bytes = sent
    res.phase_ms = ph.result()
    return res
