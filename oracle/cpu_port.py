"""TEST INFRASTRUCTURE ONLY: the reference's CPU build path restated with torch on the host cores.

Used only to TIME the reference's CPU implementation (bench.py's cpu_baseline leg
and --impl reference).  Exactness checks use oracle.py / gta_oracle.c instead.
Each function follows the reference's Python code path on the CPU branch
(device=cpu, prec=float32), paths relative to the reference project root:

  assign_nearest      bucketDemo/build_bucket.py:48-92   pairwise_l2_min_assign
  lloyd_step          bucketDemo/build_bucket.py:249-261 refine_centers_kmeans (one iteration)
  topk_from_A_to_B    bucketDemo/build_bucket.py:96-159
  bucket_knn          bucketDemo/build_bucket.py:602-628 (top m+1 within the pool, self removed)
"""
from __future__ import annotations

import torch


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
