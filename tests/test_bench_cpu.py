"""bench.py's host-side helpers on CPU tensors: the exact ground truth the recall and the
parity block are measured against."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import bench  # noqa: E402


def _brute(X, Q, k, exclude=None):
    d = ((Q[:, None, :].astype(np.float64) - X[None, :, :].astype(np.float64)) ** 2).sum(-1)
    if exclude is not None:
        d[np.arange(len(Q)), exclude] = np.inf
    return np.argsort(d, axis=1, kind="stable")[:, :k]


@pytest.mark.parametrize("n,col_chunk,q_chunk", [(1000, 1 << 18, 2048), (1000, 300, 7), (1030, 256, 64)])
def test_exact_knn_matches_brute_force(n, col_chunk, q_chunk):
    """Blocked over queries and columns (a last column block smaller than k included), with and
    without the query's own row excluded; distinct distances, so the ids are unique."""
    rng = np.random.default_rng(3)
    X = rng.normal(size=(n, 24)).astype(np.float32)
    q = rng.choice(n, 150, replace=False)
    ex = torch.from_numpy(q)
    got = bench.exact_knn(torch.from_numpy(X), torch.from_numpy(X[q]), 32, exclude=ex, q_chunk=q_chunk,
                          col_chunk=col_chunk)
    np.testing.assert_array_equal(got, _brute(X, X[q], 32, exclude=q))
    Q = rng.normal(size=(40, 24)).astype(np.float32)
    got = bench.exact_knn(torch.from_numpy(X), torch.from_numpy(Q), 10, q_chunk=q_chunk, col_chunk=col_chunk)
    np.testing.assert_array_equal(got, _brute(X, Q, 10))
    assert bench.exact_knn(torch.from_numpy(X), torch.from_numpy(Q[:0]), 10).shape == (0, 10)
