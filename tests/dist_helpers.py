"""Helpers for the multi-process tests of the sharded build (gta/dist.py).

``OracleStages`` runs every per-rank computation of the sharded build with the
CPU oracle (test infrastructure), so the driver's own logic -- row ranges, bucket
placement, the all-to-all exchanges, the grouping of received memberships, the
per-point merge rows and the gathers of the id tables -- can be checked on CPU
ranks (gloo) against the single-process oracle pipeline.  ``gloo_worker`` and
``nccl_worker`` are the per-rank entry points the tests spawn.
"""
from __future__ import annotations

import os

import numpy as np
import torch
import torch.distributed as dist

from oracle import oracle as orc


def _np(t):
    return t.detach().cpu().numpy()


def _t(a, dtype=None):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    t = torch.from_numpy(a.copy())
    return t if dtype is None else t.to(dtype)


class OracleStages:
    """The per-rank computations of gta.dist.build_sharded, done by the CPU oracle."""

    def kmeans_sizes(self, n, prm):
        n_s = min(prm.kmeans_sample, n) if prm.kmeans_sample > 0 else orc.default_sample_size(n)
        n_s = max(n_s, prm.n_buckets)
        return n_s, min(n_s, 20 * prm.n_buckets), 0

    def sample_ids(self, n, n_s, seed, device):
        return _t(orc.kmeans_sample_ids(n, n_s, seed), torch.int32)

    def gather_rows(self, X, row0, ids):
        x, i = _np(X), _np(ids).astype(np.int64) - row0
        out = np.zeros((i.shape[0], x.shape[1]), np.float32)
        ok = (i >= 0) & (i < x.shape[0])
        out[ok] = x[i[ok]].astype(np.float32)
        return _t(out)

    def kmeans_init(self, pool, B, seed):
        raise NotImplementedError("the oracle has no k-means++: pass init_centroids")

    def assign_topk(self, Xf, C, k, integer_rows=False):  # the oracle is exact whatever the rows
        if Xf.shape[0] == 0:
            return torch.empty((0, k), dtype=torch.int32)
        return _t(orc.topk_assign(_np(Xf), _np(C), k)[0], torch.int32)

    def centroid_sums(self, Xf, assign, B):
        x, a = _np(Xf).astype(np.float64), _np(assign).astype(np.int64)
        sums = np.zeros((B, x.shape[1]), np.float64)
        np.add.at(sums, a, x)
        return _t(sums), _t(np.bincount(a, minlength=B).astype(np.int64))

    def centroid_means(self, sums, counts, C):
        s, c, old = _np(sums), _np(counts), _np(C)
        out = old.copy()
        ne = c > 0
        out[ne] = (s[ne] / c[ne, None].astype(np.float64)).astype(np.float32)
        return _t(out)

    def group_memberships(self, bucket, other, B):
        b, o = _np(bucket).astype(np.int64), _np(other).astype(np.int64)
        order = np.argsort(b * B + o, kind="stable")
        offsets = np.zeros(B + 1, np.int64)
        offsets[1:] = np.cumsum(np.bincount(b, minlength=B))
        return _t(order.astype(np.int32)), _t(offsets)

    def bucket_knn_rows(self, R, order, gid, offsets, M):
        ids, dd = orc.bucket_knn(_np(R), _np(offsets), _np(order), M)
        g = _np(gid)
        out = np.where(ids >= 0, g[np.maximum(ids, 0)], -1).astype(np.int32)
        return _t(out), _t(dd)

    def bucket_knn_rows_phased(self, R, order, gid, offsets, partner, M, phase, seed, lid, ldist):
        """Phase 1: the oracle's lists of the rows whose partner is above their bucket.  Phase 2:
        the other rows restricted as the library restricts them (columns of the row's partner
        bucket dropped, distance at most the point's seed, ties by received row as the oracle
        breaks them), so the merged lists check the seeding argument too."""
        Rn, o, g, off, part = _np(R), _np(order).astype(np.int64), _np(gid), _np(offsets), _np(partner)
        n = o.shape[0]
        if n == 0:
            return
        B = off.shape[0] - 1
        bucket = np.repeat(np.arange(B), np.diff(off))
        lower = part > bucket
        if phase == 1:
            ids, dd = orc.bucket_knn(Rn, off, o.astype(np.int32), M)
            out = np.where(ids >= 0, g[np.maximum(ids, 0)], -1).astype(np.int32)
            rows = torch.from_numpy(np.nonzero(lower)[0])
            lid[rows] = torch.from_numpy(out[lower])
            ldist[rows] = torch.from_numpy(dd[lower])
            return
        sd = _np(seed)
        X = Rn.astype(np.float64)
        for j in np.nonzero(~lower)[0]:
            b = bucket[j]
            cols = np.arange(off[b], off[b + 1])
            cols = cols[(cols != j) & (part[cols] != part[j])]
            dv = ((X[o[cols]] - X[o[j]]) ** 2).sum(1)
            keep = dv <= sd[g[o[j]]]
            cols, dv = cols[keep], dv[keep]
            srt = np.lexsort((o[cols], dv))[:M]
            row_i = np.full(M, -1, np.int32)
            row_d = np.full(M, np.inf, np.float32)
            row_i[:len(srt)] = g[o[cols[srt]]]
            row_d[:len(srt)] = dv[srt]
            lid[int(j)] = torch.from_numpy(row_i)
            ldist[int(j)] = torch.from_numpy(row_d)

    def bucket_knn_rows_ranged(self, R, order, gid, offsets, partner, M, phase, seed, row_lo, row_hi, lid, ldist):
        """bucket_knn_rows_phased, then only the rows of each bucket's range kept."""
        tl, td = lid.clone(), ldist.clone()
        self.bucket_knn_rows_phased(R, order, gid, offsets, partner, M, phase, seed, tl, td)
        off = _np(offsets)
        for b in range(off.shape[0] - 1):
            lo, hi = off[b] + int(row_lo[b]), off[b] + int(row_hi[b])
            lid[lo:hi] = tl[lo:hi]
            ldist[lo:hi] = td[lo:hi]

    def pack_memberships(self, X_local, row0, top2, holders, world):
        """Membership m = 2p + s to every holder of its bucket, rank by rank, in membership order."""
        t2 = _np(top2).reshape(-1)
        h = _np(holders).astype(np.int64).view(np.uint64)
        X = _np(X_local)
        items = [[m for m in range(t2.size) if (int(h[t2[m]]) >> r) & 1] for r in range(world)]
        flat = np.array([m for it in items for m in it], np.int64)
        rows = X[flat // 2] if flat.size else np.zeros((0, X.shape[1]), X.dtype)
        meta = np.stack([row0 + flat // 2, t2[flat], t2[flat ^ 1]], 1).astype(np.int32) if flat.size else \
            np.zeros((0, 3), np.int32)
        return torch.from_numpy(np.ascontiguousarray(rows)), _t(meta), [len(it) for it in items]

    def pack_lists(self, lid, ldist, order, gid, offsets, row_lo, row_hi, starts, world):
        """Grouped rows inside this rank's ranges to their points' owners, rank by rank, in row order."""
        o, g, off = _np(order).astype(np.int64), _np(gid), _np(offsets)
        lo, hi = _np(row_lo), _np(row_hi)
        n = o.shape[0]
        bucket = np.repeat(np.arange(off.shape[0] - 1), np.diff(off))
        rel = np.arange(n) - off[bucket]
        mine = (rel >= lo[bucket]) & (rel < hi[bucket])
        owner = np.searchsorted(np.asarray(starts[1:world]), g[o], side="right")
        items = [np.nonzero(mine & (owner == r))[0] for r in range(world)]
        flat = np.concatenate(items) if items else np.zeros(0, np.int64)
        li, ld = _np(lid), _np(ldist)
        meta = np.stack([g[o[flat]], bucket[flat]], 1).astype(np.int32)
        return _t(li[flat]), _t(ld[flat]), _t(meta), [len(it) for it in items]

    def member_rows(self, meta, row0, n_local, top2):
        m, t2 = _np(meta), _np(top2)
        mem_row = np.full((n_local, 2), -1, np.int64)
        for i in range(m.shape[0]):
            p = int(m[i, 0]) - row0
            mem_row[p, 0 if m[i, 1] == t2[p].min() else 1] = i
        return _t(mem_row)

    def lower_seeds(self, ldist, order, gid, offsets, partner, row_lo, row_hi, N):
        o, g, off, part = _np(order).astype(np.int64), _np(gid), _np(offsets), _np(partner)
        lo, hi, ld = _np(row_lo), _np(row_hi), _np(ldist)
        n = o.shape[0]
        bucket = np.repeat(np.arange(off.shape[0] - 1), np.diff(off))
        rel = np.arange(n) - off[bucket]
        sel = (rel >= lo[bucket]) & (rel < hi[bucket]) & (part > bucket)
        seed = np.full(N, np.inf, np.float32)
        seed[g[o[sel]]] = ld[sel, -1]
        return _t(seed)

    def merge_memberships(self, lid, ldist, mem_row):
        ids, dd = orc.merge_memberships(_np(lid), _np(ldist), _np(mem_row))
        return _t(ids), _t(dd)

    def sanitize_rows(self, knn, row0, n_total):
        k = _np(knn)
        full = np.full((n_total, k.shape[1]), -1, np.int32)
        full[row0:row0 + k.shape[0]] = k
        return _t(orc.sanitize(full)[0][row0:row0 + k.shape[0]])

    def prune_rows(self, g_full, K, row0, n_rows, top2, B):
        return _t(orc.prune(_np(g_full).view(np.uint32), K)[row0:row0 + n_rows])

    def reverse_merge_rows(self, pruned_full, row0, n_rows):
        return _t(orc.reverse_merge(_np(pruned_full).view(np.uint32))[row0:row0 + n_rows])


def _init(rank, world, port, backend):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=120))


def gloo_worker(rank, world, port, X, counts, C0, prm_kw, out_dir):
    """One CPU rank: build_sharded with OracleStages on its row block; saves its results."""
    import gta.dist as gd

    _init(rank, world, port, "gloo")
    try:
        row0 = int(sum(counts[:rank]))
        Xl = torch.from_numpy(np.ascontiguousarray(X[row0:row0 + counts[rank]]))
        prm = gd.ShardParams(**prm_kw)
        res = gd.build_sharded(Xl, prm, stages=OracleStages(), init_centroids=torch.from_numpy(C0))
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), row0=res.row0, ids=_np(res.knn_ids),
                 dists=_np(res.knn_dists), C=_np(res.centroids), top2=_np(res.top2),
                 graph=_np(res.graph) if res.graph is not None else np.zeros(0), owner=np.array(res.owner),
                 pieces=np.array(res.pieces, dtype=np.int64))
    finally:
        dist.destroy_process_group()


class _BadBucketStages(OracleStages):
    """OracleStages whose top-2 pass leaves one membership of its first row without a bucket (what
    a non-finite row gives): a data fault made on the host, on one rank only."""

    def assign_topk(self, Xf, C, k, integer_rows=False):
        out = super().assign_topk(Xf, C, k, integer_rows)
        if k == 2 and out.shape[0]:
            out[0, 1] = -1
        return out


def gloo_fault_worker(rank, world, port, X, counts, C0, prm_kw, bad_rank, out_dir):
    """One CPU rank of a build where rank ``bad_rank`` meets a row without a bucket: records the
    status each rank's build_sharded raised (every rank must raise, none may wait in a collective)."""
    import gta.dist as gd
    from gta import _lib as L

    _init(rank, world, port, "gloo")
    try:
        row0 = int(sum(counts[:rank]))
        Xl = torch.from_numpy(np.ascontiguousarray(X[row0:row0 + counts[rank]]))
        stages = _BadBucketStages() if rank == bad_rank else OracleStages()
        status = 0
        try:
            gd.build_sharded(Xl, gd.ShardParams(**prm_kw), stages=stages, init_centroids=torch.from_numpy(C0))
        except L.GtaError as e:
            status = e.code
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.array([status]))
    finally:
        dist.destroy_process_group()


def nccl_worker(rank, world, port, X, prm_kw, out_dir):
    """One GPU rank: build_sharded with the libgta stages; saves its results."""
    import gta.dist as gd

    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl")
    try:
        n = X.shape[0]
        bounds = [(n * r) // world for r in range(world + 1)]
        Xl = torch.from_numpy(np.ascontiguousarray(X[bounds[rank]:bounds[rank + 1]])).cuda()
        prm = gd.ShardParams(**prm_kw)
        res = gd.build_sharded(Xl, prm)
        torch.cuda.synchronize()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), row0=res.row0, ids=_np(res.knn_ids),
                 dists=_np(res.knn_dists), C=_np(res.centroids), top2=_np(res.top2),
                 graph=_np(res.graph) if res.graph is not None else np.zeros(0))
    finally:
        dist.destroy_process_group()
