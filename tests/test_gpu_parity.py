"""GPU parity: every stage of libgta, called through its C ABI, against the CPU
oracle and the fixtures made from the reference's own code.

Bars (from the build's contract):
  * prune / reverse edges / sanitize / sort / merge: bit-exact;
  * 8-bit data: kNN lists bit-exact (distances are exact integers);
  * float32 data: kNN ids identical except ties within 1e-5 relative distance,
    distances bit-identical for identical ids (both sides use the same fp32
    fmaf chain);
  * k-means: centroids bit-identical per Lloyd step, assignments identical.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import gta  # noqa: E402
from oracle import oracle as orc  # noqa: E402

pytestmark = pytest.mark.gpu

REL_TIE = 1e-5


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def mixture(rng, n, d, k, sigma, lo=-1.0, hi=1.0):
    c = rng.uniform(lo, hi, (k, d)).astype(np.float32)
    return (c[rng.integers(0, k, n)] + rng.normal(0, sigma, (n, d))).astype(np.float32)


def assert_lists_match(ids, dists, ref_ids, ref_dists, exact: bool, X=None, qrows=None):
    """Row-wise: identical lists, or (float data) identical up to near-ties.

    Float data: at every position where the ids differ, the build's id must be a real tie of the
    reference's entry there -- its own exact fp32 distance to the query (recomputed with the
    oracle's ascending-dimension fmaf chain) must equal the distance the build reports, bit for
    bit, and lie within REL_TIE (relative) of the reference's distance at that position.  No
    fraction of differing ids is waived.  ``X`` is the dataset, ``qrows[r]`` the dataset row of
    list r (default: r itself)."""
    if exact:
        np.testing.assert_array_equal(ids, ref_ids)
        np.testing.assert_array_equal(dists, ref_dists)
        return
    same = ids == ref_ids
    np.testing.assert_array_equal(dists[same], ref_dists[same])
    if same.all():
        return
    assert X is not None, "a float-data list differs from the oracle: the check needs the dataset"
    r, c = np.nonzero(~same)
    got, want = ids[r, c], ref_ids[r, c]
    assert (got >= 0).all() and (want >= 0).all(), "a padding entry differs from the oracle"
    q = r if qrows is None else np.asarray(qrows)[r]
    own = orc.pair_l2(X, q, got)
    np.testing.assert_array_equal(dists[r, c], own)          # the build reports the id's exact distance
    rel = np.abs(own.astype(np.float64) - ref_dists[r, c]) / np.maximum(np.abs(ref_dists[r, c]), 1e-30)
    assert (rel <= REL_TIE).all(), f"{int((rel > REL_TIE).sum())} differing ids are not ties within {REL_TIE}"
    for row in np.unique(r):                                  # a tie swap never duplicates an id
        v = ids[row][ids[row] >= 0]
        assert len(np.unique(v)) == len(v), f"row {row} repeats an id"


# ---------------------------------------------------------------- CAGRA optimize
@pytest.mark.parametrize("name", ["opt_a", "opt_b", "opt_c"])
def test_optimize_bit_exact_vs_reference_code(golden, name):
    f = golden("prune_ref.npz")
    san = f[f"{name}_san"]
    K = f[f"{name}_graph"].shape[1]
    g = host(gta.optimize(dev(san.view(np.int32)), K)).view(np.uint32)
    np.testing.assert_array_equal(g, f[f"{name}_graph"])
    # host-buffer entry point gives the same graph
    np.testing.assert_array_equal(gta.optimize(np.ascontiguousarray(san), K), f[f"{name}_graph"])


@pytest.mark.parametrize("N,M,K", [(3000, 64, 32), (1500, 128, 64), (800, 24, 12), (500, 33, 7)])
def test_prune_and_reverse_vs_oracle(N, M, K):
    rng = np.random.default_rng(N + M)
    X = mixture(rng, N, 16, 8, 0.3)
    ids, _ = orc.exact_knn(X, np.arange(N), M)
    ids[rng.random(ids.shape) < 0.05] = -1           # padding -> duplicates after sanitize
    san, _ = orc.sanitize(ids)
    pr = host(gta.prune(dev(san.view(np.int32)), K)).view(np.uint32)
    np.testing.assert_array_equal(pr, orc.prune(san, K))
    rv = host(gta.reverse_merge(dev(pr.view(np.int32)))).view(np.uint32)
    np.testing.assert_array_equal(rv, orc.reverse_merge(pr))


def test_reverse_merge_hub_with_large_indegree():
    # every row points at node 0 first: in-degree N-1 (> the 512-key fast path)
    N, K = 2000, 8
    rng = np.random.default_rng(3)
    g = np.empty((N, K), np.uint32)
    for i in range(N):
        others = rng.choice(np.delete(np.arange(N), [i, 0]), K - 1, replace=False)
        g[i] = np.concatenate([[0 if i != 0 else 1], others])
    np.testing.assert_array_equal(host(gta.reverse_merge(dev(g.view(np.int32)))).view(np.uint32),
                                  orc.reverse_merge(g))


def test_sanitize_vs_oracle():
    rng = np.random.default_rng(5)
    N, M = 4000, 40
    knn = rng.integers(-3, N + 5, (N, M)).astype(np.int32)
    knn[7] = -1
    knn[np.arange(N), rng.integers(0, M, N)] = np.arange(N)  # self loops
    ref, _ = orc.sanitize(knn)
    np.testing.assert_array_equal(host(gta.sanitize(dev(knn))).view(np.uint32), ref)


@pytest.mark.parametrize("name", ["opt_a", "opt_b", "opt_c"])
def test_sort_rows_vs_reference_code(golden, name):
    f = golden("prune_ref.npz")
    got = host(gta.sort_rows(dev(f[f"{name}_X"]), dev(f[f"{name}_knn"])))
    np.testing.assert_array_equal(got, f[f"{name}_sorted"])


# ---------------------------------------------------------------- merge
def test_merge_vs_reference_python_fixture(golden):
    f = golden("merge.npz")
    on, od = gta.merge_lists(dev(f["a_i"]), dev(f["a_d"]), dev(f["b_i"]), dev(f["b_d"]))
    np.testing.assert_array_equal(host(on), f["out_i"])
    np.testing.assert_array_equal(host(od), f["out_d"])


@pytest.mark.parametrize("M", [1, 16, 64, 100, 128])
def test_merge_lists_vs_oracle_with_ties_and_dups(M):
    rng = np.random.default_rng(M)
    N = 3000
    # integer distances: many exact ties; shared ids carry the same distance on both sides
    pool_d = rng.integers(0, 20, (N, 300)).astype(np.float32)
    a_cols = np.stack([rng.choice(300, M, replace=False) for _ in range(N)])
    b_cols = np.stack([rng.choice(300, M, replace=False) for _ in range(N)])
    def lists(cols):
        d = np.take_along_axis(pool_d, cols, 1)
        o = np.lexsort((cols, d), axis=1) if False else np.argsort(d * 1000 + cols, axis=1, kind="stable")
        return np.take_along_axis(cols, o, 1).astype(np.int32), np.take_along_axis(d, o, 1)
    ai, ad = lists(a_cols)
    bi, bd = lists(b_cols)
    ai[::5, M // 2:] = -1; ad[::5, M // 2:] = np.inf
    bi[::3, M // 3:] = -1; bd[::3, M // 3:] = np.inf
    ri, rd = orc.merge_lists(ai, ad, bi, bd)
    gi, gd = gta.merge_lists(dev(ai), dev(ad), dev(bi), dev(bd))
    np.testing.assert_array_equal(host(gi), ri)
    np.testing.assert_array_equal(host(gd), rd)


# ---------------------------------------------------------------- assignment / k-means
@pytest.mark.parametrize("N,d,B,k", [(5000, 128, 16, 2), (4097, 96, 300, 2), (2000, 960, 64, 1), (3000, 20, 7, 3)])
def test_assign_topk_vs_oracle(N, d, B, k):
    rng = np.random.default_rng(d + B)
    X = mixture(rng, N, d, 12, 0.2)
    C = X[rng.choice(N, B, replace=False)] + rng.normal(0, 0.01, (B, d)).astype(np.float32)
    gi, gd = gta.assign_topk(dev(X), dev(C), k)
    ri, rd = orc.topk_assign(X, C, k)
    gi, gd = host(gi), host(gd)
    np.testing.assert_array_equal(gd, rd)     # same fp32 chain, bit-identical
    np.testing.assert_array_equal(gi, ri)     # ties resolved to the smaller centroid id on both sides


def test_assign_topk_u8_values():
    rng = np.random.default_rng(2)
    X = rng.integers(0, 256, (3000, 128)).astype(np.float32)
    C = rng.uniform(0, 255, (256, 128)).astype(np.float32)
    gi, gd = gta.assign_topk(dev(X), dev(C), 2)
    ri, rd = orc.topk_assign(X, C, 2)
    np.testing.assert_array_equal(host(gi), ri)
    np.testing.assert_array_equal(host(gd), rd)


def test_kmeans_lloyd_steps_vs_oracle():
    rng = np.random.default_rng(9)
    X = mixture(rng, 20000, 64, 40, 0.15)
    C = X[:32].copy()
    for _ in range(3):  # one Lloyd step at a time from identical centroids
        gC, ga = gta.kmeans_fit(dev(X), dev(C), 1)
        gC, ga = host(gC), host(ga)
        ids, _ = orc.topk_assign(X, C, 1)
        rC = orc.kmeans_update(X, ids[:, 0], C)
        np.testing.assert_array_equal(gC, rC)
        ri, _ = orc.topk_assign(X, rC, 1)
        np.testing.assert_array_equal(ga, ri[:, 0])
        C = rC


@pytest.mark.parametrize("d", [32, 960])
def test_kmeans_init_is_deterministic_and_picks_data_points(d):
    # d = 960 (C3) takes the layout without resident pool rows (they exceed shared memory)
    rng = np.random.default_rng(4)
    X = mixture(rng, 5000, d, 20, 0.1)
    a = host(gta.kmeans_init(dev(X), 2000, 40, seed=7))
    b = host(gta.kmeans_init(dev(X), 2000, 40, seed=7))
    np.testing.assert_array_equal(a, b)
    pool = X[:2000]
    for c in a:
        assert (np.abs(pool - c).max(axis=1) == 0).any()
    assert len({tuple(r) for r in a}) >= 38


# ---------------------------------------------------------------- memberships and per-bucket kNN
def test_memberships_vs_oracle():
    rng = np.random.default_rng(6)
    N, B = 10000, 37
    t0 = rng.integers(0, B, N)
    t1 = (t0 + rng.integers(1, B, N)) % B
    top2 = np.stack([t0, t1], 1).astype(np.int32)
    off, mem, mrow = gta.build_memberships(dev(top2), B)
    roff, rmem, rrow = orc.build_csr(top2, B)
    np.testing.assert_array_equal(host(off), roff)
    np.testing.assert_array_equal(host(mem), rmem)
    np.testing.assert_array_equal(host(mrow), rrow)


def _csr_for(X, B, rng):
    C = X[rng.choice(X.shape[0], B, replace=False)]
    top2, _ = orc.topk_assign(X, C, 2)
    return orc.build_csr(top2, B)


# u8 rows with M <= 64 run on kind::i8 operands, int8 rows and longer lists on bf16 operands
@pytest.mark.parametrize("N,d,B,M,dtype", [(6000, 128, 8, 64, np.uint8), (3000, 128, 3, 16, np.uint8),
                                           (2500, 100, 5, 128, np.uint8), (3000, 128, 4, 64, np.int8),
                                           (2000, 40, 3, 32, np.uint8),
                                           # d > 129: 8-bit rows no longer exact in bf16 -> float screen + rerank
                                           (3000, 200, 4, 32, np.uint8)])
def test_bucket_knn_8bit_bit_exact(N, d, B, M, dtype):
    rng = np.random.default_rng(N)
    X = np.clip(np.rint(mixture(rng, N, d, 15, 20.0, 0, 255)), 0, 255)
    X = (X - 128 if dtype == np.int8 else X).astype(dtype)
    X[100:130] = X[99]  # exact duplicates: distance-0 ties broken by id
    off, mem, mrow = _csr_for(X.astype(np.float32), B, rng)
    gi, gd = gta.bucket_knn(dev(X), dev(mem), dev(off), M)
    ri, rd = orc.bucket_knn(X.astype(np.float32), off, mem, M)
    np.testing.assert_array_equal(host(gi), ri)
    np.testing.assert_array_equal(host(gd), rd)
    mi, md = gta.merge_memberships(gi, gd, dev(mrow))
    ki, kd = orc.merge_memberships(ri, rd, mrow)
    np.testing.assert_array_equal(host(mi), ki)
    np.testing.assert_array_equal(host(md), kd)


@pytest.mark.parametrize("N,d,B,M", [(6000, 128, 8, 64), (3000, 96, 6, 64), (1500, 960, 4, 128)])
def test_bucket_knn_f32_vs_oracle(N, d, B, M):
    rng = np.random.default_rng(N + d)
    X = mixture(rng, N, d, 12, 0.1)
    off, mem, _ = _csr_for(X, B, rng)
    gi, gd = gta.bucket_knn(dev(X), dev(mem), dev(off), M)
    ri, rd = orc.bucket_knn(X, off, mem, M)
    assert_lists_match(host(gi), host(gd), ri, rd, exact=False, X=X, qrows=mem)


@pytest.mark.parametrize("N,d,M,edges,dup", [
    (70000, 8, 16, [65535, 65536, 65537], False),               # 65 536-column chunks: two waves
    (70000, 960, 128, [32767, 32768, 32769, 65535, 65536], False),  # long rows, one-part screen: three waves
    (70000, 512, 64, [65535, 65536, 65537], True),              # near-duplicates: rescans, split screen after wave 0
])
def test_bucket_knn_f32_long_segment_column_chunks(N, d, M, edges, dup):
    """A long float segment runs as column chunks (sized for the L2 with the operand bytes a row
    tile reads) whose exact lists are merged wave by wave: sampled rows (chunk edges included)
    against the oracle's exact top-M over the whole segment.  dup: groups of near-identical rows,
    so the one-part screen's margin holds more columns than a list and rows are rescanned (the
    later waves run the split screen)."""
    rng = np.random.default_rng(70)
    X = mixture(rng, N, d, 40, 0.2)
    if dup:
        base = X[rng.integers(0, N, 200)]
        idx = rng.choice(N, N // 2, replace=False)
        X[idx] = base[rng.integers(0, 200, idx.size)] + rng.normal(0, 1e-4, (idx.size, d)).astype(np.float32)
    mem = np.arange(N, dtype=np.int32)
    off = np.array([0, N], np.int64)
    from gta import _lib as GL
    GL.profile_enable(True)
    gi, gd = gta.bucket_knn(dev(X), dev(mem), dev(off), M)
    torch.cuda.synchronize()
    stages = {rec[0] for rec in GL.profile_records()}
    GL.profile_enable(False)
    if dup:  # half the rows rescanned in wave 0: wave 1 ran the split screen
        assert "dist_topk_bucket_split" in stages
    gi, gd = host(gi), host(gd)
    rows = np.concatenate([rng.choice(N, 200, replace=False), [0, 1, N - 1] + edges])
    ri = np.empty((len(rows), M), np.int32)
    rd = np.empty((len(rows), M), np.float32)
    allc = np.arange(N)
    for k, r in enumerate(rows):
        dd = orc.pair_l2(X, np.full(N, r), allc)
        dd[r] = np.inf
        sel = np.lexsort((allc, dd))[:M]
        ri[k], rd[k] = sel, dd[sel]
    assert_lists_match(gi[rows], gd[rows], ri, rd, exact=False, X=X, qrows=rows)


def test_bucket_knn_f32_overflow_rescan():
    # 400 identical points in one bucket: the screen list overflows and the rows are rescanned exactly
    rng = np.random.default_rng(8)
    X = mixture(rng, 2000, 32, 4, 0.3)
    X[:400] = X[0]
    off = np.array([0, 2000], np.int64)
    mem = np.arange(2000, dtype=np.int32)
    gi, gd = gta.bucket_knn(dev(X), dev(mem), dev(off), 64)
    ri, rd = orc.bucket_knn(X, off, mem, 64)
    np.testing.assert_array_equal(host(gi), ri)
    np.testing.assert_array_equal(host(gd), rd)


@pytest.mark.parametrize("lo,hi", [(0, 40), (150, 151), (260, 300)])
def test_rescan_of_few_rows_in_column_slices(lo, hi):
    """A row range of a bucket whose rows all need the whole-segment rescan (300 identical points:
    more columns within the bound than a list holds): so few rows that each is spread over several
    CTAs in column slices whose lists are merged by key.  Exact top-M against the oracle; rows
    outside the range untouched."""
    import gta.dist as gd

    rng = np.random.default_rng(12)
    n, d, M = 2500, 32, 16
    X = mixture(rng, n, d, 6, 0.3)
    X[:300] = X[0]
    order = torch.arange(n, dtype=torch.int32, device="cuda")
    offsets = dev(np.array([0, n], np.int64))
    partner = torch.ones(n, dtype=torch.int32, device="cuda")
    lid = torch.full((n, M), -1, dtype=torch.int32, device="cuda")
    ldist = torch.full((n, M), float("inf"), dtype=torch.float32, device="cuda")
    gd.CudaStages().bucket_knn_rows_ranged(dev(X), order, order.clone(), offsets, partner, M, 1, None,
                                           torch.tensor([lo]), torch.tensor([hi]), lid, ldist)
    gi, gdist = host(lid), host(ldist)
    allc = np.arange(n)
    for r in range(lo, hi):
        dd = orc.pair_l2(X, np.full(n, r), allc)
        dd[r] = np.inf
        sel = np.lexsort((allc, dd))[:M]
        np.testing.assert_array_equal(gi[r], sel)
        np.testing.assert_array_equal(gdist[r], dd[sel])
    outside = np.ones(n, bool)
    outside[lo:hi] = False
    assert (gi[outside] == -1).all()


def test_bucket_knn_tiny_and_ragged_buckets():
    rng = np.random.default_rng(10)
    X = rng.integers(0, 256, (700, 64)).astype(np.uint8)
    # bucket sizes 1, 2, 129, 568 (ragged tiles, a singleton with an empty list)
    mem = np.arange(700, dtype=np.int32)
    off = np.array([0, 1, 3, 132, 700], np.int64)
    gi, gd = gta.bucket_knn(dev(X), dev(mem), dev(off), 64)
    ri, rd = orc.bucket_knn(X.astype(np.float32), off, mem, 64)
    np.testing.assert_array_equal(host(gi), ri)
    np.testing.assert_array_equal(host(gd), rd)
    assert (host(gi)[0] == -1).all()


# ---------------------------------------------------------------- pipelines
def _sample_rows(N, n_s, seed):
    return orc.kmeans_sample_ids(N, n_s, seed)


@pytest.mark.parametrize("cfg_name,n,n_buckets,dtype_exact", [
    ("c1", 10000, None, False), ("c2", 40000, None, True),
    ("c3", 8000, 8, False),     # d = 960 f32, M = 128 lists
    ("c4", 20000, 16, False)])  # d = 96, unit rows (inner product served as L2)
def test_build_bucket_pipeline_vs_oracle(cfg_name, n, n_buckets, dtype_exact):
    cfg = gta.scaled(gta.CONFIGS[cfg_name], n, n_buckets)
    X = gta.generate(cfg, seed=3)
    Xf = X.astype(np.float32)
    n_s = cfg.kmeans_sample or orc.default_sample_size(n)
    sid = _sample_rows(n, n_s, 42)
    C0 = Xf[sid[: cfg.n_buckets]].copy()
    ids, dists, cent, top2 = gta.build_bucket(dev(X), cfg.n_buckets, cfg.knn_degree, cfg.kmeans_iters, n_s, 42,
                                              init_centroids=dev(C0), with_extras=True)
    ids, dists, cent, top2 = host(ids), host(dists), host(cent), host(top2)
    rC, _ = orc.kmeans(Xf[sid], C0, cfg.kmeans_iters)
    if dtype_exact:  # 8-bit rows: exact integer sums, centroids bit-identical per Lloyd step
        np.testing.assert_array_equal(cent, rC)
    else:
        np.testing.assert_allclose(cent, rC, rtol=1e-6, atol=1e-6)
    rt2, rt2d = orc.topk_assign(Xf, cent, 2)
    np.testing.assert_array_equal(top2, rt2)
    offs, mem, mrow = orc.build_csr(top2, cfg.n_buckets)
    li, ld = orc.bucket_knn(Xf, offs, mem, cfg.knn_degree)
    ki, kd = orc.merge_memberships(li, ld, mrow)
    assert_lists_match(ids, dists, ki, kd, exact=dtype_exact, X=Xf)
    # recall of the kNN graph vs exact kNN on sampled points (knn_similarity.py rule)
    q = np.random.default_rng(0).choice(n, 300, replace=False)
    gt, _ = orc.exact_knn(Xf, q, 32)
    rec, rec_ref = orc.knn_recall(ids[q], gt, 32), orc.knn_recall(ki[q], gt, 32)
    assert abs(rec - rec_ref) <= 1e-3
    if cfg_name in ("c1", "c2"):   # clustered data; c4's unit rows at 16 buckets reach ~0.5 in both builds
        assert rec > 0.8
    # the CAGRA graph of those lists (K of the configuration)
    g = gta.optimize_knn(ids, cfg.graph_degree)
    np.testing.assert_array_equal(g, orc.optimize(orc.sanitize(ids)[0], cfg.graph_degree))


def test_build_cagra_matches_oracle_optimize():
    cfg = gta.scaled(gta.CONFIGS["c2"], 20000)
    X = gta.generate(cfg, seed=1)
    ids, dists = gta.build_bucket(dev(X), cfg.n_buckets, 64, 5, 0, 9)
    g = host(gta.build_cagra(dev(X), cfg.n_buckets, 64, 32, 5, 0, 9)).view(np.uint32)
    san, _ = orc.sanitize(host(ids))
    np.testing.assert_array_equal(g, orc.optimize(san, 32))
    # host-buffer entry point (H2D / D2H inside the call) gives the same graph
    g2 = gta.build_cagra(X, cfg.n_buckets, 64, 32, 5, 0, 9)
    np.testing.assert_array_equal(g2, g)


def test_invalid_arguments_are_rejected():
    X = dev(np.zeros((100, 8), np.float32))
    with pytest.raises(gta.GtaError) as e:
        gta.build_bucket(X, 1, 8)            # 2-way membership needs B >= 2
    assert e.value.code == 1
    with pytest.raises(gta.GtaError) as e:
        gta.optimize(dev(np.zeros((10, 4), np.int32)), 8)   # K > M
    assert e.value.code == 1


def test_prune_refuses_out_of_range_neighbours():
    """A neighbour id outside [0, N) is a data error (status 5), never an out-of-range read."""
    rng = np.random.default_rng(9)
    g = np.stack([rng.choice(np.delete(np.arange(50), i), 8, replace=False) for i in range(50)]).astype(np.uint32)
    g[7, 3] = 50 + 11          # a neighbour row that does not exist
    g[9, 5] = 0xFFFFFFFF       # all ones
    with pytest.raises(gta.GtaError) as e:
        gta.prune(dev(g.view(np.int32)), 4)
    assert e.value.code == 5


def test_reverse_merge_refuses_out_of_range_neighbours():
    """The reverse-edge merge reports an id outside [0, N) (status 5) instead of dropping the edge,
    through the whole-graph and the row-range entry points alike."""
    import ctypes

    from gta import _lib as L

    rng = np.random.default_rng(10)
    g = np.stack([rng.choice(np.delete(np.arange(60), i), 8, replace=False) for i in range(60)]).astype(np.uint32)
    g[5, 2] = 60               # one past the last row
    with pytest.raises(gta.GtaError) as e:
        gta.reverse_merge(dev(g.view(np.int32)))
    assert e.value.code == 5
    gd = dev(g.view(np.int32))
    out = torch.empty((30, 8), dtype=torch.int32, device="cuda")
    rc = L.lib().gta_reverse_merge_rows(ctypes.c_void_p(gd.data_ptr()), 60, 8, 30, 30, ctypes.c_void_p(out.data_ptr()),
                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 5
    g[5, 2] = 0xFFFFFFFF       # all ones
    with pytest.raises(gta.GtaError) as e:
        gta.reverse_merge(dev(g.view(np.int32)))
    assert e.value.code == 5


def test_bucket_knn_refuses_a_bad_membership_csr():
    """A membership id outside [0, n) or offsets that decrease are a data error (status 5), found
    before any kernel reads a row through them."""
    rng = np.random.default_rng(11)
    X = rng.normal(size=(300, 16)).astype(np.float32)
    mem = np.arange(300, dtype=np.int32)
    off = np.array([0, 100, 300], np.int64)
    gi, _ = gta.bucket_knn(dev(X), dev(mem), dev(off), 8)   # the valid CSR runs
    assert (host(gi) >= 0).all()
    bad = mem.copy()
    bad[150] = 300                                          # one past the last row
    with pytest.raises(gta.GtaError) as e:
        gta.bucket_knn(dev(X), dev(bad), dev(off), 8)
    assert e.value.code == 5
    with pytest.raises(gta.GtaError) as e:
        gta.bucket_knn(dev(X), dev(mem), dev(np.array([0, 200, 100], np.int64)), 8)
    assert e.value.code == 5


@pytest.mark.parametrize("N,K,hubs", [(4000, 32, 3), (3000, 64, 2), (2000, 100, 2), (5000, 1, 1), (900, 5, 4)])
def test_reverse_merge_random_graphs_with_repeats_vs_oracle(N, K, hubs):
    """Random pruned-graph-shaped inputs with repeated ids inside rows (sanitized padding) and hub
    destinations of in-degree well above K: every register path (K <= 32, <= 64, <= 128) and the
    multi-chunk selection, bit-exact vs the oracle's serial rule."""
    rng = np.random.default_rng(N + K)
    g = rng.integers(0, N, (N, K)).astype(np.uint32)
    hub_ids = rng.choice(N, hubs, replace=False)
    rows = rng.random(N) < 0.4
    g[rows, rng.integers(0, K, rows.sum())] = hub_ids[rng.integers(0, hubs, rows.sum())]
    dup = rng.random((N, K)) < 0.1                      # repeats of the row's first entry
    g[dup] = np.repeat(g[:, :1], K, axis=1)[dup]
    rv = host(gta.reverse_merge(dev(g.view(np.int32)))).view(np.uint32)
    np.testing.assert_array_equal(rv, orc.reverse_merge(g))


@pytest.mark.parametrize("cfg_name,n,budget", [("c2", 30000, 1 << 20), ("c2", 30000, 6 << 20), ("c1", 10000, 1 << 20)])
def test_budgeted_bucket_batches_equal_one_pass(cfg_name, n, budget):
    """A device budget far below the memberships' pool + lists runs the buckets in batches;
    the lists and the final graph are the one-pass build's, bit for bit."""
    cfg = gta.scaled(gta.CONFIGS[cfg_name], n)
    X = dev(gta.generate(cfg, seed=5))
    a_ids, a_d = gta.build_bucket(X, cfg.n_buckets, cfg.knn_degree, 3, 0, 9)
    b_ids, b_d = gta.build_bucket(X, cfg.n_buckets, cfg.knn_degree, 3, 0, 9, device_budget=budget)
    np.testing.assert_array_equal(host(b_ids), host(a_ids))
    np.testing.assert_array_equal(host(b_d), host(a_d))
    ga = gta.build_cagra(X, cfg.n_buckets, cfg.knn_degree, cfg.graph_degree, 3, 0, 9)
    gb = gta.build_cagra(X, cfg.n_buckets, cfg.knn_degree, cfg.graph_degree, 3, 0, 9, device_budget=budget)
    np.testing.assert_array_equal(host(gb), host(ga))


def test_build_bucket_many_buckets_u8_split_screen():
    """More than 384 buckets on 8-bit data: the Lloyd steps and the top-2 pass run the tensor-core
    screen on split operands ([x | x] against [hi | lo] centroids) with the exact rerank; centroids,
    top-2 and lists must equal the oracle's."""
    cfg = gta.scaled(gta.CONFIGS["c2"], 60000, n_buckets=500)
    X = gta.generate(cfg, seed=8)
    Xf = X.astype(np.float32)
    n_s = 20000
    sid = _sample_rows(60000, n_s, 42)
    C0 = Xf[sid[:500]].copy()
    ids, dists, cent, top2 = gta.build_bucket(dev(X), 500, 32, 3, n_s, 42, init_centroids=dev(C0), with_extras=True)
    ids, dists, cent, top2 = host(ids), host(dists), host(cent), host(top2)
    rC, _ = orc.kmeans(Xf[sid], C0, 3)
    np.testing.assert_array_equal(cent, rC)
    rt2, _ = orc.topk_assign(Xf, cent, 2)
    np.testing.assert_array_equal(top2, rt2)
    offs, mem, mrow = orc.build_csr(top2, 500)
    li, ld = orc.bucket_knn(Xf, offs, mem, 32)
    ki, kd = orc.merge_memberships(li, ld, mrow)
    np.testing.assert_array_equal(ids, ki)
    np.testing.assert_array_equal(dists, kd)


@pytest.mark.parametrize("B,k", [(600, 1), (1000, 2)])
def test_assign_topk_integer_rows_split_screen(B, k):
    """gta_assign_topk_ex with GTA_ROWS_INTEGER (8-bit rows as f32) equals the exact oracle."""
    rng = np.random.default_rng(B)
    X = rng.integers(0, 256, (20000, 96)).astype(np.float32)
    C = (rng.integers(0, 256, (B, 96)) + rng.random((B, 96))).astype(np.float32)
    ids = torch.empty((20000, k), dtype=torch.int32, device="cuda")
    dd = torch.empty((20000, k), dtype=torch.float32, device="cuda")
    from gta import _lib as L
    Xd, Cd = dev(X), dev(C)
    L.check(L.lib().gta_assign_topk_ex(Xd.data_ptr(), 20000, 96, Cd.data_ptr(), B, k, ids.data_ptr(), dd.data_ptr(),
                                       L.GTA_ROWS_INTEGER, torch.cuda.current_stream().cuda_stream))
    ri, rd = orc.topk_assign(X, C, k)
    np.testing.assert_array_equal(host(ids), ri)
    np.testing.assert_array_equal(host(dd), rd)


@pytest.mark.parametrize("kind", ["u8", "f32"])
def test_host_resident_dataset_matches_device_copy(kind):
    """gta_dataset.on_device == 2: the build reads the rows in place from host memory (registered
    and mapped for the call, never copied whole to the device); with a small device budget the
    bucket stage runs in batches.  The graph and lists equal those of the ordinary build."""
    rng = np.random.default_rng(21)
    if kind == "u8":
        cfg = gta.scaled(gta.CONFIGS["c2"], 30000)
        X = gta.generate(cfg, seed=5)
        B, M, K = 24, 32, 16
    else:
        X = mixture(rng, 20000, 300, 30, 0.3)
        B, M, K = 12, 32, 16
    ids0, d0 = gta.build_bucket(X, B, M, 3)
    ids1, d1 = gta.build_bucket(X, B, M, 3, host_resident=True, device_budget=8 << 20)
    np.testing.assert_array_equal(ids1, ids0)
    np.testing.assert_array_equal(d1, d0)
    g0 = gta.build_cagra(X, B, M, K, 3)
    g1 = gta.build_cagra(X, B, M, K, 3, host_resident=True, device_budget=8 << 20)
    np.testing.assert_array_equal(g1, g0)
    # a device tensor cannot be host-resident; the other entry points take host (0) or device (1)
    with pytest.raises(gta.GtaError):
        gta.build_bucket(torch.from_numpy(X).cuda(), B, M, 3, host_resident=True)
