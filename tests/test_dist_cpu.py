"""The sharded (multi-GPU) build's host logic on CPU ranks (gloo, worlds 2 to 8).

Every per-rank computation is done by the CPU oracle (tests/dist_helpers.py), so
these tests check what the driver in gta/dist.py adds: row ranges, bucket
placement, the all-to-all exchanges of points and lists, the grouping of the
received memberships, the per-point merge rows and the gathers of the id
tables.  The concatenated per-rank results must equal the single-process oracle
pipeline bit for bit (u8 data, so the fp64 centroid sums are exact)."""
import socket
import tempfile
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402

from oracle import oracle as orc  # noqa: E402
import gta.dist as gd  # noqa: E402
import dist_helpers  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data(n, d, n_centres, seed):
    rng = np.random.default_rng(seed)
    centres = rng.uniform(0, 255, (n_centres, d))
    lab = rng.integers(0, n_centres, n)
    return np.clip(np.rint(centres[lab] + rng.normal(0, 20, (n, d))), 0, 255).astype(np.uint8)


def test_place_buckets_is_deterministic_and_balanced():
    rng = np.random.default_rng(5)
    sizes = rng.integers(10, 500, 64).tolist()
    own = gd.place_buckets(sizes, 4)
    assert own == gd.place_buckets(sizes, 4)
    load = np.zeros(4)
    for b, r in enumerate(own):
        load[r] += sizes[b] ** 2
    # LPT: within the largest single item of the ideal share
    assert load.max() - load.mean() <= max(s * s for s in sizes)
    assert set(own) == {0, 1, 2, 3}
    assert gd.place_buckets([5, 5], 1) == [0, 0]


def test_place_pieces_splits_a_dominant_bucket_over_distinct_ranks():
    sizes = [5000, 300, 280, 260, 250, 240, 230, 220]
    for world in (2, 4, 8):
        pcs = gd.place_pieces(sizes, world)
        assert pcs == gd.place_pieces(sizes, world)
        big = [p for p in pcs if p[0] == 0]
        assert len(big) == world  # 5000^2 is almost the whole job
        assert len({p[1] for p in big}) == world  # distinct ranks
        assert big[0][2] == 0 and big[-1][3] == 5000
        assert all(a[3] == b[2] for a, b in zip(big, big[1:]))  # contiguous row ranges
        assert all(p[2] % 128 == 0 for p in big)
        for b in range(1, len(sizes)):  # the others stay whole
            assert [(p[2], p[3]) for p in pcs if p[0] == b] == [(0, sizes[b])]
        load = np.zeros(world)
        for b, r, lo, hi in pcs:
            load[r] += (hi - lo) * sizes[b]
        assert load.max() <= 1.15 * load.mean()
    # whole buckets only: one piece each, the placement of place_buckets
    pcs = gd.place_pieces(sizes, 4, float("inf"))
    assert [(p[2], p[3]) for p in pcs] == [(0, n) for n in sizes]
    assert [p[1] for p in pcs] == gd.place_buckets(sizes, 4)
    # a bucket is never cut below the alignment
    assert [(p[2], p[3]) for p in gd.place_pieces([200, 10], 4) if p[0] == 0] == [(0, 200)]


def test_place_pieces_properties():
    """For any sizes, ranks and split share: every bucket's pieces tile [0, n) in order, sit on
    distinct ranks, are cut at multiples of 128 and are non-empty (a bucket of n > 0 rows); the
    placement is the same on every call."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies

    @hyp.settings(max_examples=300, deadline=None)
    @hyp.given(sizes=st.lists(st.integers(0, 3000), min_size=1, max_size=40), world=st.integers(1, 8),
               share=st.sampled_from([0.01, 0.1, 0.5, 1.0, float("inf")]))
    def check(sizes, world, share):
        pcs = gd.place_pieces(sizes, world, share)
        assert pcs == gd.place_pieces(sizes, world, share)
        assert pcs == sorted(pcs, key=lambda p: (p[0], p[2]))
        for b, n in enumerate(sizes):
            mine = [p for p in pcs if p[0] == b]
            assert mine and mine[0][2] == 0 and mine[-1][3] == n
            assert all(a[3] == c[2] for a, c in zip(mine, mine[1:]))
            assert len({p[1] for p in mine}) == len(mine) <= world
            assert all(0 <= p[1] < world for p in mine)
            assert all(p[2] % 128 == 0 for p in mine)
            if n > 0:
                assert all(p[3] > p[2] for p in mine)
            if world == 1 or share == float("inf") or n < 256:
                assert len(mine) == 1

    check()


@pytest.mark.parametrize("world,counts,split", [(2, [1300, 1700], 1.0), (3, [1000, 1000, 1000], 1.0),
                                                (2, [1300, 1700], 0.05), (3, [1000, 1000, 1000], 0.05),
                                                (4, [700, 800, 750, 750], 0.05),
                                                (8, [375] * 8, 0.05)])
def test_sharded_build_matches_single_pipeline(world, counts, split):
    N, d, B, M, K, iters = sum(counts), 16, 8, 16, 8, 3
    X = _data(N, d, 20, seed=7)
    rng = np.random.default_rng(1)
    C0 = X[rng.choice(N, B, replace=False)].astype(np.float32)
    prm = dict(n_buckets=B, knn_degree=M, graph_degree=K, kmeans_iters=iters, kmeans_sample=0, seed=42,
               split_share=split)

    # the single-process oracle pipeline on the same sample
    n_s = max(orc.default_sample_size(N), B)
    sid = orc.kmeans_sample_ids(N, n_s, 42)
    ref = orc.build_knn_graph(X, C0, B, M, iters, sample_ids=sid)
    g_ref = orc.optimize(orc.sanitize(ref["knn_ids"])[0], K)

    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(dist_helpers.gloo_worker, args=(world, _free_port(), X, counts, C0, prm, out),
                           nprocs=world, join=True, start_method="spawn")
        parts = [np.load(f"{out}/rank{r}.npz") for r in range(world)]
    ids = np.concatenate([p["ids"] for p in parts])
    dists = np.concatenate([p["dists"] for p in parts])
    graph = np.concatenate([p["graph"] for p in parts]).view(np.uint32)
    top2 = np.concatenate([p["top2"] for p in parts])
    for p in parts:
        np.testing.assert_array_equal(p["C"], ref["centroids"])
        np.testing.assert_array_equal(p["owner"], parts[0]["owner"])
    pcs = parts[0]["pieces"]
    assert set(pcs[:, 1].tolist()) == set(range(world))  # every rank holds a piece of some bucket
    if split < 1.0:  # buckets cut into row ranges on several ranks
        assert len(pcs) > B
    np.testing.assert_array_equal(top2, ref["top2"])
    np.testing.assert_array_equal(ids, ref["knn_ids"])
    np.testing.assert_array_equal(dists, ref["knn_dists"])
    np.testing.assert_array_equal(graph, g_ref)


def test_bad_bucket_on_one_rank_raises_on_every_rank():
    """A row without a valid bucket on one rank (a fault made on the host) ends the build with
    status 5 (data check failed) on every rank, promptly: the flag rides on the bucket sizes'
    all-reduce, so no rank is left waiting in a later collective for the process-group timeout."""
    world, counts, B = 3, [400, 500, 600], 6
    X = _data(sum(counts), 16, 12, seed=9)
    C0 = X[np.random.default_rng(2).choice(sum(counts), B, replace=False)].astype(np.float32)
    prm = dict(n_buckets=B, knn_degree=8, graph_degree=0, kmeans_iters=1, kmeans_sample=0, seed=42)
    t0 = time.monotonic()
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(dist_helpers.gloo_fault_worker, args=(world, _free_port(), X, counts, C0, prm, 1, out),
                           nprocs=world, join=True, start_method="spawn")
        status = [int(np.load(f"{out}/rank{r}.npy")[0]) for r in range(world)]
    assert status == [5] * world
    assert time.monotonic() - t0 < 90  # well under the 120 s process-group timeout
