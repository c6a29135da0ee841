"""The oracle's restatement of the reference bucketing's balanced choice and pool tables, pinned
to the reference's own loops: the committed fixture (tests/golden/bucket2_assign.npz, made by
tests/golden/make_golden.py from bucket.cu:2277-2302 and :5317-5347 compiled into oracle/_ref)
and, when oracle/_ref/libgta_ref_assign.so was built here, the loops themselves on more inputs."""
import os

import numpy as np
import pytest

from oracle import oracle as orc

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "bucket2_assign.npz"))


@pytest.mark.parametrize("name", ["mix", "few"])
@pytest.mark.parametrize("rule", [0, 1])
def test_balanced_choice_matches_reference_fixture(name, rule):
    t2, t2d, cid = GOLD[f"top2_{name}"], GOLD[f"top2d_{name}"], GOLD[f"cid_{name}"]
    got = orc.balanced_assign(t2, cid.size, cid, t2d, rule)
    np.testing.assert_array_equal(got, GOLD[f"assign_{name}_rule{rule}"])


def test_balanced_rules_differ_and_centroids_stay():
    t2, t2d, cid = GOLD["top2_few"], GOLD["top2d_few"], GOLD["cid_few"]
    a0, a1 = GOLD["assign_few_rule0"], GOLD["assign_few_rule1"]
    assert (a0 != a1).any()  # the fixture tells the two rules apart
    assert (a0[cid] == np.arange(cid.size)).all() and (a1[cid] == np.arange(cid.size)).all()
    # the second centroid is taken for some points, the first for most
    nc = np.setdiff1d(np.arange(t2.shape[0]), cid)
    took2 = (a0[nc] == t2[nc, 1]) & (t2[nc, 0] != t2[nc, 1])
    assert 0 < took2.sum() < nc.size


def test_pool_tables_match_reference_fixture():
    assign, adj = GOLD["pool_assign"], GOLD["pool_adj"]
    B = adj.shape[0]
    off, mem, sb, so, ps = orc.pool_tables(assign, B, adj.astype(np.int64).clip(max=2**31 - 1).astype(np.int32))
    np.testing.assert_array_equal(off, GOLD["pool_off"])
    np.testing.assert_array_equal(mem, GOLD["pool_members"])
    np.testing.assert_array_equal(sb, GOLD["pool_seg_bucket"])
    np.testing.assert_array_equal(so, GOLD["pool_seg_ofs"].astype(np.int64))
    np.testing.assert_array_equal(ps, GOLD["pool_size"])
    assert (sb == -1).any()  # neighbours past the last bucket dropped


R = orc.ref_assign_lib()
needs_ref = pytest.mark.skipif(R is None, reason="oracle/_ref/libgta_ref_assign.so not built (reference tree absent)")


def _ref_assign(t2, t2d, cid, rule, batch):
    a = np.full(t2.shape[0], -1, np.int32)
    R.ref_balanced_assign(orc._p(t2), orc._p(t2d), t2.shape[0], cid.size, orc._p(cid), rule, batch, orc._p(a))
    return a


@needs_ref
@pytest.mark.parametrize("seed", range(6))
def test_balanced_choice_matches_reference_loop(seed):
    rng = np.random.default_rng(100 + seed)
    N = int(rng.integers(50, 5000))
    B = int(rng.integers(2, 40))
    cid = rng.choice(N, B, replace=False).astype(np.int32)
    c1 = rng.integers(0, B, N)
    c2 = np.where(rng.random(N) < 0.05, c1, (c1 + rng.integers(1, B, N)) % B)  # a few equal pairs
    t2 = np.ascontiguousarray(np.stack([c1, c2], 1).astype(np.int32))
    d1 = rng.uniform(0.0, 3.0, N).astype(np.float32)
    t2d = np.ascontiguousarray(np.stack([d1, (d1 * rng.uniform(1.0, 1.5, N)).astype(np.float32)], 1))
    for rule in (0, 1):
        want = _ref_assign(t2, t2d, cid, rule, int(rng.integers(1, 2000)))
        np.testing.assert_array_equal(orc.balanced_assign(t2, B, cid, t2d, rule), want)


@needs_ref
@pytest.mark.parametrize("seed", range(4))
def test_pool_tables_match_reference_loop(seed):
    rng = np.random.default_rng(200 + seed)
    N, B, P = int(rng.integers(10, 3000)), int(rng.integers(2, 60)), int(rng.integers(0, 9))
    assign = rng.integers(0, B, N).astype(np.int32)
    adj = rng.integers(0, B + 3, (B, P)).astype(np.uint32)  # ids >= B dropped by both
    off = np.empty(B + 1, np.int64)
    mem = np.empty(N, np.int32)
    sb = np.empty((B, P + 1), np.int32)
    so = np.empty((B, P + 1), np.int32)
    ps = np.empty(B, np.int64)
    R.ref_pool_tables(orc._p(assign), N, B, orc._p(adj), P, orc._p(off), orc._p(mem), orc._p(sb), orc._p(so),
                      orc._p(ps))
    o2, m2, sb2, so2, ps2 = orc.pool_tables(assign, B, adj.astype(np.int32))
    np.testing.assert_array_equal(o2, off)
    np.testing.assert_array_equal(m2, mem)
    np.testing.assert_array_equal(sb2, sb)
    np.testing.assert_array_equal(so2, so.astype(np.int64))
    np.testing.assert_array_equal(ps2, ps)
