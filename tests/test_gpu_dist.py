"""The sharded (multi-GPU) build on GPUs: the row-range stage entry points against
their whole-graph versions, and gta.dist.build_sharded over NCCL ranks against
the single-GPU build of the same data (u8, so bit-exact: the fp64 centroid sums
are sums of integers and every other stage sees the same inputs in the same
order).  The two-rank case needs two GPUs and is skipped on one."""
import socket
import tempfile

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402

import gta  # noqa: E402
import gta.dist as gd  # noqa: E402
from gta import _lib as L  # noqa: E402
import dist_helpers  # noqa: E402

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data(n, d=64, seed=3):
    cfg = gta.scaled(gta.CONFIGS["c2"], n)
    cfg = gta.synth.Config(**{**cfg.__dict__, "d": d})
    return gta.generate(cfg, seed=seed)


def _p(t):
    return None if t is None else t.data_ptr()


def _st():
    return torch.cuda.current_stream().cuda_stream


def test_row_range_stages_match_whole_graph():
    X = torch.from_numpy(_data(20000)).cuda()
    ids, _ = gta.build_bucket(X, 16, 32, 3)
    N, M, K = ids.shape[0], 32, 16
    san = gta.sanitize(ids)
    pruned = gta.prune(san, K)
    final = gta.reverse_merge(pruned)
    lib = L.lib()
    for row0, n_rows in [(0, N), (0, 7000), (7000, 9000), (16000, 4000), (19999, 1)]:
        s = torch.empty((n_rows, M), dtype=torch.int32, device="cuda")
        L.check(lib.gta_sanitize_rows(_p(ids[row0:row0 + n_rows]), n_rows, row0, N, M, _p(s), _st()))
        assert torch.equal(s, san[row0:row0 + n_rows])
        top2 = torch.randint(0, 16, (n_rows, 2), dtype=torch.int32, device="cuda")
        top2[:, 1] = (top2[:, 0] + 1) % 16
        for t2 in (None, top2):
            pr = torch.empty((n_rows, K), dtype=torch.int32, device="cuda")
            L.check(lib.gta_prune_rows(_p(san), N, M, K, row0, n_rows, _p(t2), 16, _p(pr), _st()))
            assert torch.equal(pr, pruned[row0:row0 + n_rows])
        rv = torch.empty((n_rows, K), dtype=torch.int32, device="cuda")
        L.check(lib.gta_reverse_merge_rows(_p(pruned), N, K, row0, n_rows, _p(rv), _st()))
        assert torch.equal(rv, final[row0:row0 + n_rows])
    bad = torch.empty((10, K), dtype=torch.int32, device="cuda")
    assert lib.gta_prune_rows(_p(san), N, M, K, N - 5, 10, None, 16, _p(bad), _st()) == L.GTA_EINVAL


def test_centroid_partials_and_grouping():
    rng = np.random.default_rng(0)
    Xs = torch.from_numpy(rng.integers(0, 256, (5000, 40)).astype(np.float32)).cuda()
    a = torch.from_numpy(rng.integers(0, 12, 5000).astype(np.int32)).cuda()
    a[a == 7] = 3  # one empty centroid keeps its value
    C = torch.from_numpy(rng.normal(size=(12, 40)).astype(np.float32)).cuda()
    st = gd.CudaStages()
    sums, cts = st.centroid_sums(Xs, a, 12)
    ref = torch.zeros((12, 40), dtype=torch.float64, device="cuda").index_add_(0, a.long(), Xs.double())
    assert torch.equal(sums, ref)
    assert torch.equal(cts, torch.bincount(a.long(), minlength=12))
    newC = st.centroid_means(sums, cts, C)
    exp = (ref / cts.clamp(min=1)[:, None].double()).float()
    exp[7] = C[7]
    assert torch.equal(newC, exp)
    # grouping: stable by (bucket, other)
    b = torch.from_numpy(rng.integers(0, 9, 3000).astype(np.int32)).cuda()
    o = torch.from_numpy(rng.integers(0, 9, 3000).astype(np.int32)).cuda()
    order, offs = st.group_memberships(b, o, 9)
    key = (b.long() * 9 + o.long()).cpu().numpy()
    assert np.array_equal(order.cpu().numpy(), np.argsort(key, kind="stable"))
    assert np.array_equal(offs.cpu().numpy()[1:], np.cumsum(np.bincount(b.cpu().numpy(), minlength=9)))
    # rows gathered from a shard, zero outside it
    Xu = torch.from_numpy(rng.integers(0, 256, (100, 8)).astype(np.uint8)).cuda()
    ids = torch.tensor([1000, 1050, 999, 1099, 1100], dtype=torch.int32, device="cuda")
    g = st.gather_rows(Xu, 1000, ids)
    assert torch.equal(g[0], Xu[0].float()) and torch.equal(g[1], Xu[50].float()) and torch.equal(g[3], Xu[99].float())
    assert not g[2].any() and not g[4].any()


def _memberships(X, top2, B):
    """Every membership (point p, slot s) as received row 2p+s: rows, global ids, grouping."""
    st = gd.CudaStages()
    bucket = top2.reshape(-1).contiguous()
    other = top2.flip(1).reshape(-1).contiguous()
    p_of = torch.arange(bucket.numel(), device="cuda") // 2
    R = X[p_of].contiguous()
    gid = p_of.to(torch.int32)
    order, offsets = st.group_memberships(bucket, other, B)
    ol = order.long()
    return st, R, gid, order, offsets, bucket[ol], other[ol].contiguous()


def _two_phases(st, R, gid, order, offsets, bucket_s, partner_s, M, rng=None, seed2=None):
    """Both passes; phase 2's seeds from phase 1's lists, or seed2 (a whole run's seeds: the
    all-reduce of the sharded build)."""
    n, N = R.shape[0], R.shape[0] // 2
    lid = torch.full((n, M), -1, dtype=torch.int32, device="cuda")
    ldist = torch.full((n, M), float("inf"), dtype=torch.float32, device="cuda")
    run = (lambda ph, sd: st.bucket_knn_rows_phased(R, order, gid, offsets, partner_s, M, ph, sd, lid, ldist)) \
        if rng is None else \
        (lambda ph, sd: st.bucket_knn_rows_ranged(R, order, gid, offsets, partner_s, M, ph, sd, rng[0], rng[1], lid,
                                                  ldist))
    run(1, None)
    seed = torch.full((N,), float("inf"), dtype=torch.float32, device="cuda")
    lower = partner_s > bucket_s
    seed[gid[order.long()][lower].long()] = ldist[lower, M - 1]
    run(2, seed if seed2 is None else seed2)
    return lid, ldist, seed


@pytest.mark.parametrize("kind", ["u8", "f32", "f32_long"])
def test_ranged_rows_match_whole_buckets(kind):
    """gta_bucket_knn_rows_ranged fills exactly the rows of each bucket's range, with the lists of
    the whole-bucket call (a split bucket's pieces on several ranks put together); rows outside
    the ranges keep their contents.  f32_long: buckets of 70000 rows (column chunks)."""
    rng = np.random.default_rng(4)
    if kind == "u8":
        X = torch.from_numpy(_data(30000, d=128, seed=5)).cuda()
        B, M = 6, 32
    elif kind == "f32":
        X = torch.from_numpy(_data(30000, d=96, seed=5).astype(np.float32) * 0.37).cuda()
        B, M = 6, 32
    else:
        X = torch.from_numpy(rng.normal(size=(70000, 32)).astype(np.float32)).cuda()
        B, M = 2, 32
    _, _, _, top2 = gta.build_bucket(X, B, M, 2, 0, 42, with_extras=True)
    st, R, gid, order, offsets, bucket_s, partner_s = _memberships(X, top2, B)
    full_i, full_d, seed = _two_phases(st, R, gid, order, offsets, bucket_s, partner_s, M)
    off = offsets.cpu().numpy()
    sizes = np.diff(off)
    # three pieces per bucket, cut at a multiple of 128 and at an arbitrary row
    cuts = [np.array([0, (n // 3) // 128 * 128, max((n // 3) // 128 * 128, 2 * n // 3 + 5), n]) for n in sizes]
    got_i = torch.full_like(full_i, -1)
    got_d = torch.full_like(full_d, float("inf"))
    for k in range(3):
        lo = torch.tensor([min(c[k], c[3]) for c in cuts], dtype=torch.int64)
        hi = torch.tensor([min(c[k + 1], c[3]) for c in cuts], dtype=torch.int64)
        pi, pd, _ = _two_phases(st, R, gid, order, offsets, bucket_s, partner_s, M, (lo, hi), seed)
        inside = np.zeros(R.shape[0], bool)
        for b in range(B):
            inside[off[b] + lo[b]: off[b] + hi[b]] = True
        ins = torch.from_numpy(inside).cuda()
        assert (pi[~ins] == -1).all() and torch.isinf(pd[~ins]).all()  # untouched outside the range
        got_i[ins] = pi[ins]
        got_d[ins] = pd[ins]
    assert torch.equal(got_i, full_i)
    assert torch.equal(got_d, full_d)
    # a range outside its bucket is refused before device work
    bad = torch.tensor([0] * B, dtype=torch.int64)
    badh = torch.tensor([int(n) + 1 for n in sizes], dtype=torch.int64)
    with pytest.raises(L.GtaError):
        st.bucket_knn_rows_ranged(R, order, gid, offsets, partner_s, M, 1, None, bad, badh, got_i, got_d)


@pytest.mark.parametrize("dtype", ["u8", "f32"])
def test_shard_packing_matches_host_restatement(dtype):
    """gta_shard_pack_memberships / _pack_lists / _member_rows / _lower_seeds against the host
    restatement the gloo tests use (dist_helpers.OracleStages), on random placements with split
    buckets (several holders), uneven rank row ranges and rows outside every range."""
    rng = np.random.default_rng(9)
    n_local, d, B, world, row0, M = 5000, 24, 40, 5, 12345, 16
    X = rng.integers(0, 256, (n_local, d)).astype(np.uint8)
    if dtype == "f32":
        X = rng.normal(size=(n_local, d)).astype(np.float32)
    c1 = rng.integers(0, B, n_local)
    top2 = np.stack([c1, (c1 + rng.integers(1, B, n_local)) % B], 1).astype(np.int32)
    holders = np.zeros(B, np.int64)
    for b in range(B):
        for r in rng.choice(world, int(rng.integers(1, 4)), replace=False):
            holders[b] |= 1 << int(r)
    cs, hs = gd.CudaStages(), dist_helpers.OracleStages()
    Xd, t2d = torch.from_numpy(X).cuda(), torch.from_numpy(top2).cuda()
    got = cs.pack_memberships(Xd, row0, t2d, torch.from_numpy(holders), world)
    want = hs.pack_memberships(torch.from_numpy(X), row0, torch.from_numpy(top2), torch.from_numpy(holders), world)
    assert got[2] == want[2]
    assert torch.equal(got[0].cpu(), want[0]) and torch.equal(got[1].cpu(), want[1])
    # lists: received rows grouped by (bucket, other), ranges inside each bucket, owners by row ranges
    n_r = 7000
    bucket = rng.integers(0, B, n_r).astype(np.int32)
    other = rng.integers(0, B, n_r).astype(np.int32)
    gid = rng.permutation(100000)[:n_r].astype(np.int32)  # one received row per point
    order, offsets = cs.group_memberships(torch.from_numpy(bucket).cuda(), torch.from_numpy(other).cuda(), B)
    sizes = np.diff(offsets.cpu().numpy())
    lo = np.array([int(rng.integers(0, s + 1)) for s in sizes], np.int64)
    hi = np.array([int(rng.integers(l, s + 1)) for l, s in zip(lo, sizes)], np.int64)
    starts = [0, 20000, 20001, 55000, 90000, 100000]
    lid = torch.from_numpy(rng.integers(0, 100000, (n_r, M)).astype(np.int32)).cuda()
    ldist = torch.from_numpy(rng.random((n_r, M)).astype(np.float32)).cuda()
    gid_t = torch.from_numpy(gid).cuda()
    lo_t, hi_t = torch.from_numpy(lo), torch.from_numpy(hi)
    got = cs.pack_lists(lid, ldist, order, gid_t, offsets, lo_t, hi_t, starts, world)
    want = hs.pack_lists(lid.cpu(), ldist.cpu(), order.cpu(), gid_t.cpu(), offsets.cpu(), lo_t, hi_t, starts, world)
    assert got[3] == want[3]
    for a, b in zip(got[:3], want[:3]):
        assert torch.equal(a.cpu(), b)
    partner = torch.from_numpy(other).cuda()[order.long()].contiguous()
    sd = cs.lower_seeds(ldist, order, gid_t, offsets, partner, lo_t, hi_t, 100000)
    hsd = hs.lower_seeds(ldist.cpu(), order.cpu(), gid_t.cpu(), offsets.cpu(), partner.cpu(), lo_t, hi_t, 100000)
    assert torch.equal(sd.cpu(), hsd)
    # member rows: each local point receives its two lists in a shuffled order
    meta = np.stack([np.repeat(np.arange(n_local) + row0, 2), top2.reshape(-1)], 1).astype(np.int32)
    meta = meta[rng.permutation(meta.shape[0])]
    mr = cs.member_rows(torch.from_numpy(meta).cuda(), row0, n_local, t2d)
    assert torch.equal(mr.cpu(), hs.member_rows(torch.from_numpy(meta), row0, n_local, torch.from_numpy(top2)))
    # a bucket with no holder, a list of a point outside the rows: data errors
    bad_h = holders.copy()
    bad_h[int(top2[0, 0])] = 0
    with pytest.raises(L.GtaError) as e:
        cs.pack_memberships(Xd, row0, t2d, torch.from_numpy(bad_h), world)
    assert e.value.code == L.GTA_EDATA
    meta[0, 0] = row0 + n_local
    with pytest.raises(L.GtaError) as e:
        cs.member_rows(torch.from_numpy(meta).cuda(), row0, n_local, t2d)
    assert e.value.code == L.GTA_EDATA


def _run_ranks(world, X, prm):
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(dist_helpers.nccl_worker, args=(world, _free_port(), X, prm, out), nprocs=world,
                           join=True, start_method="spawn")
        return [dict(np.load(f"{out}/rank{r}.npz")) for r in range(world)]


def _check_against_single(world, split_share=1.0):
    N, B, M, K = 60000, 16, 32, 16
    X = _data(N, d=128, seed=11)
    prm = dict(n_buckets=B, knn_degree=M, graph_degree=K, kmeans_iters=4, kmeans_sample=0, seed=42,
               split_share=split_share)
    parts = _run_ranks(world, X, prm)
    Xd = torch.from_numpy(X).cuda()
    ids, dists, C, top2 = gta.build_bucket(Xd, B, M, 4, 0, 42, with_extras=True)
    graph = gta.build_cagra(Xd, B, M, K, 4, 0, 42)
    for p in parts:
        assert np.array_equal(p["C"], C.cpu().numpy())
    assert np.array_equal(np.concatenate([p["top2"] for p in parts]), top2.cpu().numpy())
    assert np.array_equal(np.concatenate([p["ids"] for p in parts]), ids.cpu().numpy())
    assert np.array_equal(np.concatenate([p["dists"] for p in parts]), dists.cpu().numpy())
    assert np.array_equal(np.concatenate([p["graph"] for p in parts]), graph.cpu().numpy())


def test_sharded_one_rank_matches_single_gpu_build():
    _check_against_single(1)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("split_share", [1.0, 0.05])
def test_sharded_two_ranks_match_single_gpu_build(split_share):
    """split_share 0.05: most buckets cut into row ranges on both ranks."""
    _check_against_single(2, split_share)
