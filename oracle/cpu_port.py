"""TEST INFRASTRUCTURE ONLY: the reference's CPU build path restated with torch on the host cores.

Used only to TIME the reference's CPU implementation (bench.py's cpu_baseline leg
and --impl reference).  Exactness checks use oracle.py / gta_oracle.c instead.
Each function follows the reference's Python code path on the CPU branch
(device=cpu, prec=float32), paths relative to the reference project root:

  dist_one_to_all     bucketDemo/build_bucket.py:164-186 _dist_one_to_all
  kmeans_pp_centers   bucketDemo/build_bucket.py:189-229 (D^2 sampling on a pool of min(N, 20 B), torch RNG)
  assign_nearest      bucketDemo/build_bucket.py:48-92   pairwise_l2_min_assign
  lloyd_step          bucketDemo/build_bucket.py:249-261 refine_centers_kmeans (one iteration)
  topk_from_A_to_B    bucketDemo/build_bucket.py:96-159
  bucket_knn          bucketDemo/build_bucket.py:602-628 (top m+1 within the pool, self removed)
  prune_graph         bucketDemo/prune.py:8-83 (the reference's Python occlusion prune: a different
                      rule from the CAGRA detour-count prune, timed and labelled as such)
"""
from __future__ import annotations

import numpy as np
import torch


@torch.inference_mode()
def dist_one_to_all(c: torch.Tensor, X: torch.Tensor, batch: int = 65536) -> torch.Tensor:
    """Squared L2 from one centre c (1 x D) to every row of X, clamped at 0 (CPU branch)."""
    N = X.shape[0]
    out = torch.empty(N)
    cn2 = (c.float() ** 2).sum()
    for s in range(0, N, batch):
        xb = X[s:s + batch]
        xb2 = (xb.float() ** 2).sum(dim=1)
        dots = (xb @ c.T).float().squeeze(1)
        out[s:s + batch] = (xb2 + cn2 - 2.0 * dots).clamp(min=0.0)
    return out


@torch.inference_mode()
def kmeans_pp_centers(X: torch.Tensor, B: int, seed: int, pool_ratio: int = 20):
    """k-means++ on a random pool of min(N, pool_ratio * B) rows: the first centre uniform, each
    next one drawn with probability proportional to its squared distance to the nearest chosen
    centre.  The same torch RNG calls in the same order as the reference, so the same torch build
    draws the same centres.  Returns (centre row ids, centres)."""
    torch.manual_seed(seed)
    N = X.shape[0]
    pool_n = min(N, pool_ratio * B)
    pool_ids = torch.randperm(N)[:pool_n]
    Xp = X[pool_ids]
    chosen = [int(torch.randint(pool_n, (1,)).item())]
    min_d2 = torch.full((pool_n,), float("inf"))
    for _ in range(1, B):
        d2 = dist_one_to_all(Xp[chosen[-1]].unsqueeze(0), Xp)
        torch.minimum(min_d2, d2, out=min_d2)
        probs = min_d2.clamp(min=0.0)
        total = probs.sum()
        if total > 0:
            nxt = int(torch.multinomial(probs / total, 1).item())
        else:
            nxt = int(torch.randint(pool_n, (1,)).item())
        chosen.append(nxt)
    ids = pool_ids[torch.tensor(chosen, dtype=torch.long)]
    return ids, X[ids].clone()


def prune_graph(X: np.ndarray, neighbors: np.ndarray, max_degree: int | None = None, rows=None) -> np.ndarray:
    """The reference's Python occlusion prune, row by row: a row's valid neighbours (not -1, not
    itself, < N) sorted by distance; neighbour z is dropped when an earlier kept neighbour u is
    closer to z than the row's point is (d(u, z) < d(v, z)); the first max_degree kept, -1 after.
    ``rows`` restricts the work to those rows (the others stay -1), for a timed sample."""
    X = np.asarray(X, dtype=np.float32)
    N = X.shape[0]
    nb = np.asarray(neighbors)
    M = nb.shape[1]
    pruned = -np.ones((N, M), dtype=np.int64)
    for v in (range(N) if rows is None else rows):
        nbrs = nb[v]
        nbrs = nbrs[(nbrs >= 0) & (nbrs < N) & (nbrs != v)]
        if nbrs.size == 0:
            continue
        diff = X[nbrs] - X[v]
        dist_v = np.einsum("ij,ij->i", diff, diff)
        order = np.argsort(dist_v)
        nbrs, dist_v = nbrs[order], dist_v[order]
        k = nbrs.size
        removed = np.zeros(k, dtype=bool)
        for i in range(k):
            if removed[i]:
                continue
            x_u = X[int(nbrs[i])]
            for j in range(i + 1, k):
                if removed[j]:
                    continue
                dz = x_u - X[int(nbrs[j])]
                if float(dz.dot(dz)) < dist_v[j]:
                    removed[j] = True
        kept = nbrs[~removed]
        if max_degree is not None and max_degree > 0:
            kept = kept[:max_degree]
        pruned[v, :kept.size] = kept
    return pruned


@torch.inference_mode()
def assign_nearest(X: torch.Tensor, C: torch.Tensor, batch: int = 65536) -> torch.Tensor:
    N = X.shape[0]
    Cn = (C * C).sum(dim=1)
    out = torch.empty(N, dtype=torch.long)
    for s in range(0, N, batch):
        xb = X[s:s + batch]
        dist = (xb * xb).sum(dim=1, keepdim=True) + Cn.unsqueeze(0) - 2.0 * (xb @ C.T)
        out[s:s + batch] = torch.argmin(dist, dim=1)
    return out


@torch.inference_mode()
def lloyd_step(X: torch.Tensor, C: torch.Tensor) -> torch.Tensor:
    B, D = C.shape
    assign = assign_nearest(X, C)
    new = torch.zeros(B, D, dtype=torch.float32)
    new.scatter_add_(0, assign.unsqueeze(1).expand(-1, D), X)
    counts = torch.bincount(assign, minlength=B)
    nz = counts > 0
    new[nz] /= counts[nz].unsqueeze(1).float()
    new[~nz] = C[~nz]
    return new


@torch.inference_mode()
def topk_from_A_to_B(A: torch.Tensor, B: torch.Tensor, k: int, query_chunk: int = 32768, base_chunk: int = 262144):
    NA = A.shape[0]
    Bn = (B * B).sum(dim=1)
    out_i = torch.empty(NA, k, dtype=torch.long)
    out_d = torch.empty(NA, k, dtype=torch.float32)
    for s in range(0, NA, query_chunk):
        q = A[s:s + query_chunk]
        q2 = (q * q).sum(dim=1, keepdim=True)
        best_d = best_i = None
        for b0 in range(0, B.shape[0], base_chunk):
            Bb = B[b0:b0 + base_chunk]
            dist = q2 + Bn[b0:b0 + base_chunk].unsqueeze(0) - 2.0 * (q @ Bb.T)
            kk = min(k, Bb.shape[0])
            d, i = torch.topk(dist, k=kk, dim=1, largest=False)
            i = i + b0
            if best_d is None:
                best_d, best_i = d, i
            else:
                md, sel = torch.topk(torch.cat([best_d, d], 1), k=k, dim=1, largest=False)
                best_i = torch.gather(torch.cat([best_i, i], 1), 1, sel)
                best_d = md
        out_i[s:s + query_chunk] = best_i
        out_d[s:s + query_chunk] = best_d
    return out_i, out_d


@torch.inference_mode()
def bucket_knn(Xb: torch.Tensor, m: int):
    """Top-m within one bucket's members, self removed (vectorised form of the reference's row loop)."""
    n = Xb.shape[0]
    idx, dist = topk_from_A_to_B(Xb, Xb, min(m + 1, n))
    keep = idx != torch.arange(n).unsqueeze(1)
    order = torch.argsort((~keep).to(torch.int8), dim=1, stable=True)[:, :m]
    return torch.gather(idx, 1, order), torch.gather(dist, 1, order)
