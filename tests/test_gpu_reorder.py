"""Bucket-contiguous renumbering on the GPU, through the C ABI: the bucket reorder, row
permutation and graph renumbering kernels against the oracle and the reference's own
translate_ids / bucket_order output (committed fixture); bad ids and non-permutations are
refused with status 5."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import gta  # noqa: E402
from gta import _lib as L  # noqa: E402
from oracle import oracle as orc  # noqa: E402

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("n,B,ordered", [(1, 1, False), (1000, 7, True), (200_003, 256, True), (50_000, 300, False)])
def test_bucket_reorder(n, B, ordered):
    rng = np.random.default_rng(n)
    top2 = rng.integers(0, B, (n, 2)).astype(np.int32)
    order = rng.permutation(B).astype(np.int32) if ordered else None
    want_inv, want_off = orc.bucket_reorder(top2.reshape(-1), B, order=order, stride=2)
    inv, off = gta.bucket_reorder(dev(top2), B, order=dev(order) if ordered else None)
    np.testing.assert_array_equal(inv.cpu().numpy().view(np.uint32), want_inv)
    np.testing.assert_array_equal(off.cpu().numpy(), want_off)
    inv_h, off_h = gta.bucket_reorder(top2[:, 0].copy(), B, order=order)  # host arrays, 1-D assignment
    np.testing.assert_array_equal(inv_h, want_inv)
    np.testing.assert_array_equal(off_h, want_off)


def test_bucket_reorder_refuses_bad_input():
    with pytest.raises(gta.GtaError) as e:
        gta.bucket_reorder(np.array([0, 3, 1], np.int32), 3)  # bucket 3 of 3
    assert e.value.code == L.GTA_EDATA
    with pytest.raises(gta.GtaError) as e:
        gta.bucket_reorder(np.array([0, 1, 1], np.int32), 2, order=np.array([1, 1], np.int32))
    assert e.value.code == L.GTA_EDATA


@pytest.mark.parametrize("n,d,dtype", [(1, 3, np.uint8), (4097, 128, np.uint8), (3001, 100, np.float32),
                                       (777, 13, np.int8)])
def test_permute_rows(n, d, dtype):
    rng = np.random.default_rng(d)
    X = (rng.integers(-128, 128, (n, d)) if dtype == np.int8 else rng.integers(0, 255, (n, d))).astype(dtype)
    inv = rng.permutation(n).astype(np.uint32)
    np.testing.assert_array_equal(gta.permute_rows(dev(X), dev(inv.view(np.int32))).cpu().numpy(), X[inv])
    np.testing.assert_array_equal(gta.permute_rows(X, inv), X[inv])


def test_permute_graph_matches_reference_translate(golden):
    f = golden("reorder.npz")
    inv = f["translate_inv"]
    out = gta.permute_graph(dev(f["translate_g"].view(np.int32)), dev(inv.view(np.int32)), True, False)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), f["translate_bin"])
    out = gta.permute_graph(f["translate_g_pad"].astype(np.int32), inv, True, True)
    np.testing.assert_array_equal(out.astype(np.int64), f["translate_npy"])
    fwd = gta.permute_graph(f["translate_g"], inv, False, False)
    want, bad = orc.permute_graph(f["translate_g"], inv, False, False)
    assert bad == 0
    np.testing.assert_array_equal(fwd, want)
    np.testing.assert_array_equal(gta.permute_graph(fwd, inv, True, False).view(np.uint32), f["translate_g"])


def test_permute_graph_refuses_bad_input():
    g = np.array([[1, 2], [0, 2], [0, 1]], np.int32)
    for bad_g, inv, pad in ((np.array([[1, 5], [0, 2], [0, 1]], np.int32), [0, 1, 2], True),  # id >= n
                            (np.array([[1, -1], [0, 2], [0, 1]], np.int32), [0, 1, 2], False),  # padding not allowed
                            (g, [0, 0, 2], True),  # not a permutation
                            (g, [0, 1, 3], True)):  # out of range
        with pytest.raises(gta.GtaError) as e:
            gta.permute_graph(dev(bad_g), dev(np.array(inv, np.int32)), True, pad)
        assert e.value.code == L.GTA_EDATA


@pytest.mark.parametrize("B,k,window", [(16, 4, 0), (256, 32, 0), (300, 16, 5)])
def test_bucket_order(B, k, window):
    rng = np.random.default_rng(B)
    C = rng.integers(0, 256, (B, 24)).astype(np.float32)  # integer centroids: exact distances, ties by id
    C[5] = C[3]  # a duplicate centroid
    order, knn = gta.bucket_order(dev(C), k, window)
    ids, _ = orc.topk_assign(C, C, k + 1)
    want_knn = np.empty((B, k), np.int32)
    for b in range(B):
        row = list(ids[b])
        row.remove(b) if b in row else row.pop()
        want_knn[b] = row[:k]
    np.testing.assert_array_equal(knn.cpu().numpy(), want_knn)
    w = window if window > 0 else max(4 * k, 16)
    np.testing.assert_array_equal(order.cpu().numpy(), orc.bucket_order(want_knn, w))
    order_h, knn_h = gta.bucket_order(C, k, window)
    np.testing.assert_array_equal(order_h, order.cpu().numpy())
