"""The seeded higher-bucket rows leave every merged list unchanged (CPU, oracle only).

The GPU build computes each point's lower-bucket list in full, then its higher-bucket list
only over the columns at or below the lower list's M-th distance that are not also members of
the lower bucket.  The merge (bucketDemo/buildBucket/src/bucket.cu:5025-5059: running side
first on equal distance, ids of the running list dropped from the new one) must then give the
same lists as the merge of two full lists.  Tie-heavy integer data exercises the equal-distance
cases of that argument.
"""
import numpy as np
import pytest

from oracle import oracle as orc


def _seeded_lists(X, top2, offsets, members, mem_row, li, ld, M):
    """Replace every higher-bucket row of (li, ld) by its seeded restriction."""
    li2, ld2 = li.copy(), ld.copy()
    Xf = X.astype(np.float64)
    N = X.shape[0]
    bucket_of_row = np.repeat(np.arange(len(offsets) - 1), np.diff(offsets))
    for p in range(N):
        r_lo, r_hi = mem_row[p]
        b_lo = bucket_of_row[r_lo]
        b_hi = bucket_of_row[r_hi]
        seed = ld[r_lo, M - 1]
        cols = members[offsets[b_hi]:offsets[b_hi + 1]].astype(np.int64)
        keep = (cols != p) & ~np.any(top2[cols] == b_lo, axis=1)
        cols = cols[keep]
        d = ((Xf[cols] - Xf[p]) ** 2).sum(1)
        ok = d <= seed
        cols, d = cols[ok], d[ok]
        o = np.lexsort((cols, d))[:M]
        li2[r_hi] = -1
        ld2[r_hi] = np.inf
        li2[r_hi, :len(o)] = cols[o]
        ld2[r_hi, :len(o)] = d[o]
    return li2, ld2


@pytest.mark.parametrize("seed,levels,B,M", [(0, 3, 6, 16), (1, 2, 5, 8), (2, 6, 9, 32)])
def test_seeded_higher_rows_give_the_same_merged_lists(seed, levels, B, M):
    rng = np.random.default_rng(seed)
    N, d = 500, 6
    X = rng.integers(0, levels, size=(N, d)).astype(np.uint8)   # many equal distances
    t0 = rng.integers(0, B, size=N)
    t1 = (t0 + rng.integers(1, B, size=N)) % B                  # two distinct buckets per point
    top2 = np.stack([t0, t1], 1).astype(np.int32)
    offsets, members, mem_row = orc.build_csr(top2, B)
    li, ld = orc.bucket_knn(X.astype(np.float32), offsets, members, M)
    full_n, full_d = orc.merge_memberships(li, ld, mem_row)
    li2, ld2 = _seeded_lists(X, top2, offsets, members, mem_row, li, ld, M)
    assert (li2 != li).any()                                    # the restriction did drop entries
    got_n, got_d = orc.merge_memberships(li2, ld2, mem_row)
    np.testing.assert_array_equal(got_n, full_n)
    np.testing.assert_array_equal(got_d, full_d)
