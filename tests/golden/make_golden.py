"""Regenerate the golden fixtures in tests/golden/ from the REFERENCE's own code.

Run where the reference tree is present, with its project root in the
GTA_REFERENCE environment variable (required).  The fixtures are small .npz files committed to
the repository, so the tests themselves never read the reference tree.

  * The reference's Python functions (bucketDemo/build_bucket.py,
    bucketDemo/build_knn.py) are imported and run on seeded synthetic data.
  * The reference's header-only C++ prune / reverse-edge code
    (prune_windowed_core.hpp, edge_chunk_accumulator.hpp) runs through
    oracle/_ref/libgta_ref.so, compiled in place by oracle/Makefile.
  * The reference's balanced-choice loop and pool tables (bucket.cu lines
    streamed by oracle/Makefile into oracle/ref_assign_bridge.cpp) run through
    oracle/_ref/libgta_ref_assign.so.

    GTA_REFERENCE=<reference root> python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("GTA_REFERENCE", "")
if not REF or not os.path.isdir(os.path.join(REF, "bucketDemo")):
    sys.exit("make_golden.py: set GTA_REFERENCE to the reference project root (the directory holding bucketDemo/)")
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(REF, "bucketDemo"))

import torch  # noqa: E402

from oracle import oracle as orc  # noqa: E402


def _mixture(rng, n, d, n_clusters, sigma, lo, hi):
    centres = rng.uniform(lo, hi, size=(n_clusters, d)).astype(np.float32)
    labels = rng.integers(0, n_clusters, size=n)
    return (centres[labels] + rng.normal(0.0, sigma, size=(n, d))).astype(np.float32)


def _as_int32_rows(ids):
    return np.ascontiguousarray(np.asarray(ids, dtype=np.int64).astype(np.int32))


def make_python_fixtures():
    import build_bucket as bb  # the reference's module
    import build_knn as bk

    cpu = torch.device("cpu")
    f32 = torch.float32
    rng = np.random.default_rng(7)

    # --- k-means++ init + Lloyd + top-2 (build_bucket.py:189-262, :96-159)
    X = _mixture(rng, 3000, 16, 24, 0.08, -1.0, 1.0)
    Xt = torch.from_numpy(X)
    B = 12
    _, C0 = bb.kmeans_pp_centers(Xt, B, cpu, f32, 65536, 262144, seed=42)
    C, assign = bb.refine_centers_kmeans(Xt, C0.clone(), 5, 65536, 262144, cpu, f32)
    top2_idx, top2_dist = bb.topk_from_A_to_B(Xt, C, 2, cpu, f32, 65536, 262144)
    np.savez_compressed(os.path.join(HERE, "kmeans_top2.npz"), X=X, C0=C0.numpy(), C=C.numpy(),
                        assign=assign.numpy().astype(np.int32), top2_idx=top2_idx.numpy().astype(np.int32),
                        top2_dist=top2_dist.numpy(), iters=np.int32(5))

    # --- per-bucket kNN with the self filter (build_bucket.py:602-628)
    Xb = _mixture(rng, 700, 24, 6, 0.2, 0.0, 2.0)
    M = 16
    q_idx = np.arange(Xb.shape[0])
    idx, dist = bb.topk_from_A_to_B(torch.from_numpy(Xb), torch.from_numpy(Xb), M + 1, cpu, f32, 32768, 262144)
    keep_i = np.full((Xb.shape[0], M), -1, np.int64)
    keep_d = np.full((Xb.shape[0], M), np.inf, np.float32)
    for i in range(Xb.shape[0]):  # the reference's row filter, restated
        ri = idx[i].numpy(); rd = dist[i].numpy()
        m = ri != q_idx[i]
        fi, fd = ri[m][:M], rd[m][:M]
        keep_i[i, :fi.size] = fi
        keep_d[i, :fd.size] = fd
    np.savez_compressed(os.path.join(HERE, "bucket_knn.npz"), X=Xb, M=np.int32(M), ids=_as_int32_rows(keep_i),
                        dists=keep_d)

    # --- multi-list dedupe merge (build_bucket.py:640-671)
    N, M2 = 400, 12
    a_d = np.sort(rng.uniform(0, 10, (N, M2)).astype(np.float32), axis=1)
    b_d = np.sort(rng.uniform(0, 10, (N, M2)).astype(np.float32), axis=1)
    a_i = np.stack([rng.choice(60, M2, replace=False) for _ in range(N)]).astype(np.int64)
    b_i = np.stack([rng.choice(60, M2, replace=False) for _ in range(N)]).astype(np.int64)
    # an id present in both lists carries the same distance in both (one pair, one distance)
    for r in range(N):
        for j in range(M2):
            hit = np.nonzero(a_i[r] == b_i[r, j])[0]
            if hit.size:
                b_d[r, j] = a_d[r, hit[0]]
        o = np.argsort(b_d[r], kind="stable")
        b_d[r], b_i[r] = b_d[r][o], b_i[r][o]
    b_i[::7, -3:] = -1
    b_d[::7, -3:] = np.inf
    fi, fd = bb._merge_dedup_neighbors(torch.from_numpy(np.concatenate([a_i, b_i], 1)),
                                       torch.from_numpy(np.concatenate([a_d, b_d], 1)), M2)
    np.savez_compressed(os.path.join(HERE, "merge.npz"), a_i=_as_int32_rows(a_i), a_d=a_d, b_i=_as_int32_rows(b_i),
                        b_d=b_d, out_i=_as_int32_rows(fi.numpy()), out_d=fd.numpy())

    # --- exact kNN ground truth (build_knn.py:98-149), through its own .fbin reader
    Xg = _mixture(rng, 1500, 20, 10, 0.3, -1.0, 1.0)
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "base.fbin")
        with open(path, "wb") as f:
            np.array([Xg.shape[0], Xg.shape[1]], np.int32).tofile(f)
            Xg.tofile(f)
        ip, dp = bk.build_exact_knn(path, 10, td, query_chunk=512, base_chunk=600)
        gi, gd = np.load(ip), np.load(dp)
    np.savez_compressed(os.path.join(HERE, "exact_knn.npz"), X=Xg, k=np.int32(10), ids=_as_int32_rows(gi), dists=gd)


def make_search_fixture():
    """search.py:20-93 graph_search_single on 8-bit data (exact float32 distances) over an
    exact kNN graph, with the reference's own generator drawing the entry points."""
    import search as rs  # the reference's module

    rng = np.random.default_rng(11)
    X = np.clip(np.rint(_mixture(rng, 3060, 24, 16, 18.0, 0.0, 255.0)), 0, 255).astype(np.uint8)
    base, Q = X[:3000], X[3000:]
    ids, _ = orc.exact_knn(base, np.arange(base.shape[0]), 13)
    graph = np.ascontiguousarray(ids[:, 1:].astype(np.uint32))  # drop self (column 0)
    topk, ef, ne = 10, 32, 4
    r = np.random.default_rng(42)
    out_i = np.full((Q.shape[0], topk), -1, np.int32)
    out_d = np.full((Q.shape[0], topk), np.inf, np.float32)
    bf, qf = base.astype(np.float32), Q.astype(np.float32)
    for i in range(Q.shape[0]):
        idx, dst = rs.graph_search_single(qf[i], bf, graph.astype(np.int64), topk, ef, r, num_entry=ne)
        out_i[i, :idx.size] = idx
        out_d[i, :dst.size] = dst
    np.savez_compressed(os.path.join(HERE, "search.npz"), base=base, graph=graph, queries=Q,
                        entries=orc.search_entries(base.shape[0], Q.shape[0], ne, 42), topk=np.int32(topk),
                        ef=np.int32(ef), ids=out_i, dists=out_d)


def make_eval_fixture():
    """search.py:95-127 recall_vs_gt on random predictions with -1 padding, duplicates
    and partial hits, for the evaluation front end's recall figures."""
    import search as rs  # the reference's module

    rng = np.random.default_rng(5)
    nq, topk, k_gt = 200, 10, 100
    gt = np.stack([rng.choice(1000, k_gt, replace=False) for _ in range(nq)]).astype(np.int32)
    pred = np.where(rng.random((nq, topk)) < 0.6, gt[:, :topk], rng.integers(0, 1000, (nq, topk))).astype(np.int64)
    pred[rng.random((nq, topk)) < 0.05] = -1
    pred[::17, 3] = pred[::17, 2]  # duplicate ids in a row
    out = {"pred": pred, "gt": gt, "topk": np.int32(topk)}
    out["recall"] = np.array(rs.recall_vs_gt(pred, gt, topk), np.float64)
    out["recall_k5"] = np.array(rs.recall_vs_gt(pred, gt, 5), np.float64)
    np.savez_compressed(os.path.join(HERE, "eval_recall.npz"), **out)


def make_occlusion_fixture():
    """prune.py:8-83 prune_graph (the reference's Python occlusion prune) on an exact kNN graph
    with -1 padding, self entries and out-of-range ids mixed in, with and without a degree cap."""
    import prune as rp  # the reference's module

    rng = np.random.default_rng(31)
    X = _mixture(rng, 600, 12, 8, 0.3, -1.0, 1.0)
    ids, _ = orc.exact_knn(X, np.arange(600), 20)
    nb = ids.astype(np.int64)
    nb[rng.random(nb.shape) < 0.05] = -1
    nb[::11, 4] = np.arange(0, 600, 11)      # the row's own id
    nb[::13, 7] = 600 + 5                    # beyond N
    out = {"X": X, "neighbors": nb}
    out["pruned"] = rp.prune_graph(X, nb, None)
    out["pruned_k8"] = rp.prune_graph(X, nb, 8)
    np.savez_compressed(os.path.join(HERE, "occlusion.npz"), **out)


def make_reorder_fixture():
    """The reference's own bucket_order.hpp (processing order of a bucket graph) and
    translate_graph_ids.hpp (graph .bin and .npy back to the original id order), compiled
    in place into oracle/_ref, on seeded random inputs."""
    R = orc.ref_lib()
    if R is None:
        raise SystemExit("oracle/_ref/libgta_ref.so missing: run `make -C oracle` with the reference tree present")
    p = orc._p
    rng = np.random.default_rng(23)
    out = {}
    cases = [(40, 6, 8), (100, 10, 16), (256, 32, 128), (64, 8, 1), (50, 4, 200)]
    for c, (B, K, w) in enumerate(cases):
        adj = rng.integers(0, B, (B, K)).astype(np.uint32)
        adj[rng.random((B, K)) < 0.05] = B + 3  # entries the adjacency drops
        order = np.empty(B, np.int32)
        assert R.ref_bucket_order(p(adj), B, K, w, p(order)) == 0
        out[f"order_adj_{c}"] = adj
        out[f"order_window_{c}"] = np.int32(w)
        out[f"order_{c}"] = order
    N, K = 3000, 12
    inv = rng.permutation(N).astype(np.uint32)
    g = rng.integers(0, N, (N, K)).astype(np.uint32)
    gp = g.astype(np.int64)
    gp[rng.random((N, K)) < 0.1] = -1
    with tempfile.TemporaryDirectory() as td:
        gpath, ipath, opath = (os.path.join(td, f) for f in ("g.bin", "inv.bin", "o.bin"))
        with open(gpath, "wb") as f:
            np.array([N], np.int64).tofile(f)
            np.array([K], np.int32).tofile(f)
            g.tofile(f)
        inv.tofile(ipath)
        assert R.ref_translate_graph(gpath.encode(), ipath.encode(), opath.encode()) == 0
        out["translate_bin"] = np.fromfile(opath, dtype=np.uint32, offset=12).reshape(N, K)
        npath, nopath = os.path.join(td, "g.npy"), os.path.join(td, "o.npy")
        np.save(npath, gp)
        assert R.ref_translate_npy(npath.encode(), ipath.encode(), nopath.encode()) == 0
        out["translate_npy"] = np.load(nopath)
    out["translate_inv"] = inv
    out["translate_g"] = g
    out["translate_g_pad"] = gp
    np.savez_compressed(os.path.join(HERE, "reorder.npz"), **out)


def make_assign_fixture():
    """The reference's own balanced-choice loop (bucket.cu:2277-2302, one thread) and pool tables
    (bucket.cu:5317-5347), compiled from their lines into oracle/_ref, on seeded inputs: top-2
    centroids of mixture points (both rules) and random top-2 pairs over few buckets."""
    R = orc.ref_assign_lib()
    if R is None:
        raise SystemExit("oracle/_ref/libgta_ref_assign.so missing: run `make -C oracle` with the reference tree present")
    p = orc._p
    rng = np.random.default_rng(31)
    out = {}
    cases = []
    X = _mixture(rng, 6000, 8, 30, 0.15, -1.0, 1.0)
    cid = rng.choice(6000, 60, replace=False).astype(np.int32)
    t2, t2d = orc.topk_assign(X, X[cid], 2)
    cases.append(("mix", t2.astype(np.int32), t2d.astype(np.float32), cid))
    N, B = 4000, 5
    c1 = rng.integers(0, B, N)
    c2 = (c1 + rng.integers(1, B, N)) % B
    d1 = rng.uniform(0.5, 2.0, N).astype(np.float32)
    d2 = (d1 * rng.uniform(1.0, 1.4, N)).astype(np.float32)
    cases.append(("few", np.stack([c1, c2], 1).astype(np.int32), np.stack([d1, d2], 1),
                  rng.choice(N, B, replace=False).astype(np.int32)))
    for name, t2, t2d, cid in cases:
        t2, t2d = np.ascontiguousarray(t2), np.ascontiguousarray(t2d, np.float32)
        B = cid.size
        for rule in (0, 1):
            res = []
            for batch in (1024, 333, t2.shape[0]):  # one thread: the batch size does not matter
                a = np.full(t2.shape[0], -1, np.int32)
                R.ref_balanced_assign(p(t2), p(t2d), t2.shape[0], B, p(cid), rule, batch, p(a))
                res.append(a)
            assert all((r == res[0]).all() for r in res)
            out[f"assign_{name}_rule{rule}"] = res[0]
        out[f"top2_{name}"] = t2
        out[f"top2d_{name}"] = t2d
        out[f"cid_{name}"] = cid
    # pool tables of the mixture's default-rule buckets over each bucket's 8 nearest buckets
    # (some entries past the last bucket: the reference drops them)
    assign = out["assign_mix_rule0"]
    cid = out["cid_mix"]
    B, P = cid.size, 8
    ki, _ = orc.topk_assign(X[cid], X[cid], P + 1)
    adj = ki[:, 1:].astype(np.uint32)
    adj[rng.random(adj.shape) < 0.05] = B + 2
    off = np.empty(B + 1, np.int64)
    mem = np.empty(assign.size, np.int32)
    sb = np.empty((B, P + 1), np.int32)
    so = np.empty((B, P + 1), np.int32)
    ps = np.empty(B, np.int64)
    R.ref_pool_tables(p(assign), assign.size, B, p(adj), P, p(off), p(mem), p(sb), p(so), p(ps))
    out.update(pool_assign=assign, pool_adj=adj, pool_off=off, pool_members=mem, pool_seg_bucket=sb,
               pool_seg_ofs=so, pool_size=ps)
    np.savez_compressed(os.path.join(HERE, "bucket2_assign.npz"), **out)


def _random_graph(rng, N, M):
    """M distinct non-self candidates per row (the reference test's generator shape)."""
    g = np.empty((N, M), np.uint32)
    for i in range(N):
        pool = np.delete(np.arange(N), i)
        g[i] = rng.choice(pool, M, replace=False)
    return g


def make_cpp_fixtures():
    R = orc.ref_lib()
    if R is None:
        raise SystemExit("oracle/_ref/libgta_ref.so missing: run `make -C oracle` with the reference tree present")
    p = orc._p
    rng = np.random.default_rng(11)
    out = {}
    # detour counts on random graphs (test_prune_windowed_core.cpp:127-148 shapes: N=40 M=6, N=60 M=8)
    for N, M in ((40, 6), (60, 8), (300, 24)):
        g = _random_graph(rng, N, M)
        cnt = np.empty((N, M), np.uint32)
        for a in range(N):
            assert R.ref_detour_counts(p(g.view(np.int32)), N, M, a, p(cnt[a])) == 0
        out[f"g_{N}_{M}"] = g
        out[f"cnt_{N}_{M}"] = cnt
    # optimize on distance-sorted graphs: exact kNN (with some far candidates mixed in) of random points
    for name, (N, d, M, K, pad) in {"opt_a": (2000, 16, 32, 16, False), "opt_b": (1500, 8, 24, 12, True),
                                     "opt_c": (1200, 12, 64, 32, False)}.items():
        X = _mixture(rng, N, d, 12, 0.25, -1.0, 1.0)
        ids, _ = orc.exact_knn(X, np.arange(N), M)
        knn = ids.astype(np.int32)
        # replace a few candidates by random far points, then re-sort each row by distance
        rep = rng.random((N, M)) < 0.1
        knn[rep] = rng.integers(0, N, rep.sum())
        if pad:
            knn[::5, -5:] = -1  # padding that sanitize turns into duplicates of the first valid id
        knn = orc.sort_rows_l2(X, knn)
        san, _ = orc.sanitize(knn)
        g = np.empty((N, K), np.uint32)
        assert R.ref_optimize(p(san), N, M, K, p(g)) == 0
        out[f"{name}_X"] = X
        out[f"{name}_knn"] = knn
        out[f"{name}_san"] = san
        out[f"{name}_graph"] = g
        # the reference's own row sort on the same rows (stable, column order on ties)
        srt = np.empty((N, M), np.int32)
        for a in range(N):
            assert R.ref_sort_row_by_l2(p(X), d, p(knn), N, M, a, p(srt[a])) == 0
        out[f"{name}_sorted"] = srt
    np.savez_compressed(os.path.join(HERE, "prune_ref.npz"), **out)


if __name__ == "__main__":
    # `python make_golden.py [python] [cpp] [search] [eval] [reorder] [occlusion] [assign]`: the named
    # fixture groups (default all)
    want = set(sys.argv[1:]) or {"python", "cpp", "search", "eval", "reorder", "occlusion", "assign"}
    orc.build()
    if "python" in want:
        make_python_fixtures()
    if "cpp" in want:
        make_cpp_fixtures()
    if "search" in want:
        make_search_fixture()
    if "eval" in want:
        make_eval_fixture()
    if "reorder" in want:
        make_reorder_fixture()
    if "occlusion" in want:
        make_occlusion_fixture()
    if "assign" in want:
        make_assign_fixture()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")
