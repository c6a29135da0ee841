"""Evaluation command line, the reference's ``search.py`` front end (bucketDemo/search.py:270-323)
with the graph search on the GPU:

    python -m gta.eval search --base base.u8bin --query query.u8bin --index neighbors.npy --gt gt.ibin \
        [--topk 10] [--ef 200] [--num-entry 4] [--normalize]
    python -m gta.eval compare --index1 a.npy --index2 b.npy [--k_cmp K] [--save_csv out.csv]

``search`` runs ``gta.search`` (one warp per query, the rule of graph_search_single, entry
points from the same numpy generator as search_graph_recall, search.py:163-172) and prints
recall_vs_gt's three figures (search.py:95-127).  ``--index`` may be a ``.npy`` (N, M)
integer matrix (-1 padding) or a CAGRA ``.bin`` graph (int64 N, int32 K header).
``compare`` is compare_indices_setwise (search.py:196-265): set overlap of two indices.
Dataset rows are read by the library's BIGANN reader; an ``.i8bin`` file is read as signed
bytes (the reference's loader reads it as unsigned, load.py:34-40).
"""
import argparse
import os
import sys
from typing import Optional, Tuple

import numpy as np

from . import api


def load_ibin(path: str) -> np.ndarray:
    """Ground truth .ibin: int32 N, int32 D, then N*D int32 (load.py:43-58)."""
    with open(path, "rb") as f:
        head = np.fromfile(f, dtype=np.int32, count=2)
        if head.size < 2:
            raise ValueError(f"File too small: {path}")
        n, d = int(head[0]), int(head[1])
        g = np.fromfile(f, dtype=np.int32, count=n * d)
    if g.size != n * d:
        raise ValueError("Size mismatch for ibin")
    return g.reshape(n, d)


def load_index(path: str) -> np.ndarray:
    """A neighbour matrix as int64 (N, M), -1 padding: ``.npy`` (load.py:60-90) or a CAGRA ``.bin``."""
    if path.endswith(".npy"):
        idx = np.load(path)
        if idx.ndim != 2:
            raise ValueError(f"Expected 2D neighbors matrix, got shape={idx.shape}")
        if not np.issubdtype(idx.dtype, np.integer):
            raise ValueError(f"neighbors must be integer dtype, got {idx.dtype}")
        return idx.astype(np.int64, copy=False)
    return api.read_graph(path).astype(np.int64)


def recall_vs_gt(pred: np.ndarray, gt: np.ndarray, topk: int) -> Tuple[float, float, float]:
    """search.py:95-127: hit of GT[:,0] in pred, any overlap with GT, and the mean
    set overlap of pred[:, :k] with GT[:, :k] (k = min(topk, widths), -1 ignored) / k."""
    nq = pred.shape[0]
    if nq == 0:
        return 0.0, 0.0, 0.0
    hit_first = sum(int(gt[i, 0] in pred[i]) for i in range(nq))
    hit_any = sum(int(np.intersect1d(pred[i], gt[i]).size > 0) for i in range(nq))
    k = min(topk, pred.shape[1], gt.shape[1])
    total = 0.0
    for i in range(nq):
        a = pred[i, :k]
        b = gt[i, :k]
        total += len(set(a[a >= 0].tolist()) & set(b[b >= 0].tolist())) / float(k)
    return hit_first / nq, hit_any / nq, total / nq


def search_graph_recall(base_path: str, query_path: str, index_path: str, gt_path: str, topk: int, ef: int,
                        num_entry: int, normalize: bool = False, seed: int = 42):
    """search.py:134-180 with the per-query loop replaced by one device search."""
    import torch

    base = api.read_dataset(base_path)
    Q = api.read_dataset(query_path)
    if Q.shape[1] != base.shape[1]:
        raise ValueError(f"Dim mismatch: base D={base.shape[1]}, query D={Q.shape[1]}")
    neighbors = load_index(index_path)
    if neighbors.shape[0] != base.shape[0]:
        raise ValueError("Index N mismatch with base")
    GT = load_ibin(gt_path)
    if GT.shape[0] != Q.shape[0]:
        raise ValueError("GT nq mismatch with query")
    if normalize:
        print("[eval] L2-normalizing base & queries")
        base = base.astype(np.float32)
        Q = Q.astype(np.float32)
        base /= np.linalg.norm(base, axis=1, keepdims=True) + 1e-12
        Q /= np.linalg.norm(Q, axis=1, keepdims=True) + 1e-12
    ef = max(ef, topk)
    # ids outside [0, N) (the -1 padding) become 0xFFFFFFFF, which the search skips like the reference
    g = np.where((neighbors >= 0) & (neighbors < base.shape[0]), neighbors, -1).astype(np.int32)
    print("[eval] start searching ...")
    ids, _ = api.search(torch.from_numpy(np.ascontiguousarray(base)).cuda(), torch.from_numpy(g).cuda(),
                        torch.from_numpy(np.ascontiguousarray(Q)).cuda(), topk, ef, num_entry, seed)
    preds = ids.cpu().numpy().astype(np.int64)
    r_first, r_any, recall = recall_vs_gt(preds, GT, topk)
    print("\n======== Recall vs GT ========")
    print(f"Recall@{topk} (hit GT[:,0])         : {r_first:.6f}")
    print(f"Recall@{topk} (hit any of GT[:,:]) : {r_any:.6f}")
    print(f"Recall@{topk} (recall mean overlap): {recall:.6f}")
    return preds, (r_first, r_any, recall)


def compare_indices_setwise(index_a_path: str, index_b_path: str, k_cmp: Optional[int] = None,
                            save_csv: Optional[str] = None):
    """search.py:196-265: per node |A_k ∩ B_k| / k over the first k columns (-1 ignored)."""
    A = load_index(index_a_path)
    B = load_index(index_b_path)
    if A.shape[0] != B.shape[0]:
        raise ValueError(f"N mismatch: A={A.shape[0]}, B={B.shape[0]}")
    N, Ma, Mb = A.shape[0], A.shape[1], B.shape[1]
    k = min(Ma, Mb) if k_cmp is None else min(int(k_cmp), Ma, Mb)
    if k <= 0:
        raise ValueError("k_cmp must be > 0")
    overlaps = np.empty(N, dtype=np.float32)
    hits_any = set_equal = 0
    rows = []
    for i in range(N):
        a = A[i, :k]
        b = B[i, :k]
        SA, SB = set(a[a >= 0].tolist()), set(b[b >= 0].tolist())
        inter = len(SA & SB)
        overlaps[i] = inter / float(k)
        hits_any += inter >= 1
        set_equal += len(SA) == len(SB) == k and inter == k
        if save_csv is not None:
            rows.append((i, inter, len(SA), len(SB), overlaps[i]))
    mean_overlap = float(overlaps.mean()) if N else 0.0
    print("\n======= Index Comparison (set-wise) =======")
    print(f"N={N}, k={k} (A:{Ma}, B:{Mb})")
    print(f"MeanOverlap@{k} (|A∩B|/k) : {mean_overlap:.6f}")
    print(f"HitsAny@{k}               : {hits_any / float(N) if N else 0.0:.6f}")
    print(f"SetEqual@{k}              : {set_equal / float(N) if N else 0.0:.6f}")
    if save_csv is not None:
        os.makedirs(os.path.dirname(save_csv) or ".", exist_ok=True)
        with open(save_csv, "w") as f:
            f.write("node,intersect_size,deg_A,deg_B,overlap\n")
            for (i, inter, la, lb, ov) in rows:
                f.write(f"{i},{inter},{la},{lb},{ov:.6f}\n")
        print(f"[compare] per-node stats saved to: {save_csv}")
    return mean_overlap


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m gta.eval")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("search", help="Run graph search (GPU)")
    s.add_argument("--base", required=True, help="base vectors (.fbin/.bin/.u8bin/.i8bin)")
    s.add_argument("--query", required=True, help="query vectors (.fbin/.bin/.u8bin/.i8bin)")
    s.add_argument("--index", required=True, help="neighbors .npy (N, M) or CAGRA graph .bin")
    s.add_argument("--gt", required=True, help="groundtruth .ibin (nq, k_gt)")
    s.add_argument("--topk", type=int, default=10)
    s.add_argument("--ef", type=int, default=200)
    s.add_argument("--num-entry", type=int, default=4)
    s.add_argument("--normalize", action="store_true")
    c = sub.add_parser("compare", help="Compare two indices (set-wise)")
    c.add_argument("--index1", required=True)
    c.add_argument("--index2", required=True)
    c.add_argument("--k_cmp", type=int, default=None)
    c.add_argument("--save_csv", default=None)
    a = ap.parse_args(argv)
    if a.cmd == "search":
        search_graph_recall(a.base, a.query, a.index, a.gt, a.topk, a.ef, a.num_entry, a.normalize)
    else:
        compare_indices_setwise(a.index1, a.index2, a.k_cmp, a.save_csv)
    return 0


if __name__ == "__main__":
    sys.exit(main())
