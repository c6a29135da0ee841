"""The reverse-edge merge that allocates nothing (gta_reverse_merge_noalloc).

Some callers cannot allocate device memory at the moment they call in: a
serving process whose allocator reserved all of device memory up front, or a
latency-critical loop where cudaMalloc / cudaFree would synchronize the device
and stall its other streams.  gta_reverse_merge_noalloc serves them with scratch
that lives in a fixed array inside the library.  These tests call it through the
C ABI and check it gives exactly what gta_reverse_merge gives, on two calls in a
row (the shared scratch keeps the previous call's contents, so the second call
checks that the counters are cleared), and that oversized graphs are refused.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from gta import _lib as L  # noqa: E402

pytestmark = pytest.mark.gpu


def _graph(rng, n, k, big_hub=False):
    """A pruned-graph-shaped input: k distinct non-self ids per row, a few hubs; with
    ``big_hub``, node 0 is in most rows, an in-degree far above 512."""
    g = np.empty((n, k), np.uint32)
    hubs = rng.choice(n, 8, replace=False)
    for i in range(n):
        pool = rng.choice(n, k + 12, replace=False)
        pool = pool[pool != i][:k]
        if i % 3 == 0:
            pool[-1] = hubs[i % 8] if hubs[i % 8] != i and hubs[i % 8] not in pool[:-1] else pool[-1]
        if big_hub and i != 0 and i % 5 != 0 and 0 not in pool:
            pool[int(rng.integers(0, k))] = 0
        g[i] = pool
    return g


def _pool_used():
    """(default memory pool, bytes of it in use): the stream-ordered allocator the library
    falls back to for any scratch it takes outside its arena."""
    from cuda.bindings import runtime as rt

    err, pool = rt.cudaDeviceGetDefaultMemPool(torch.cuda.current_device())
    assert err == rt.cudaError_t.cudaSuccess
    err, used = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent)
    assert err == rt.cudaError_t.cudaSuccess
    return pool, int(used)


def _pool_high(pool, reset=False):
    from cuda.bindings import driver as drv
    from cuda.bindings import runtime as rt

    attr = rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh
    if reset:
        (err,) = rt.cudaMemPoolSetAttribute(pool, attr, drv.cuuint64_t(0))
        assert err == rt.cudaError_t.cudaSuccess
        return 0
    err, high = rt.cudaMemPoolGetAttribute(pool, attr)
    assert err == rt.cudaError_t.cudaSuccess
    return int(high)


def _noalloc(dev_graph, k, out=None):
    n = dev_graph.shape[0]
    if out is None:
        out = torch.empty((n, k), dtype=torch.int32, device="cuda")
    rc = L.lib().gta_reverse_merge_noalloc(ctypes.c_void_p(dev_graph.data_ptr()), n, k,
                                           ctypes.c_void_p(out.data_ptr()),
                                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


def _existing(dev_graph, k):
    n = dev_graph.shape[0]
    out = torch.empty((n, k), dtype=torch.int32, device="cuda")
    L.check(L.lib().gta_reverse_merge(ctypes.c_void_p(dev_graph.data_ptr()), n, k, ctypes.c_void_p(out.data_ptr()),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return out


def test_noalloc_matches_existing_entry_point_twice():
    rng = np.random.default_rng(2024)
    # two calls in a row, different sizes; the second graph has a hub of in-degree ~2300
    shapes = [(5000, 32), (3000, 16)]
    graphs = [torch.from_numpy(_graph(rng, n, k, big_hub=(i == 1)).view(np.int32)).cuda()
              for i, (n, k) in enumerate(shapes)]
    assert int((graphs[1] == 0).sum()) > 2000
    expected = [_existing(g, k) for g, (_, k) in zip(graphs, shapes)]
    outs = [torch.full((n, k), -7, dtype=torch.int32, device="cuda") for n, k in shapes]
    again = torch.full(shapes[0], -7, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    # every buffer is allocated before the measurement: the calls themselves must take nothing
    # from the stream-ordered pool (its high watermark stays at the usage before the calls)
    pool, used_before = _pool_used()
    _pool_high(pool, reset=True)
    for g, (_, k), ref, out in zip(graphs, shapes, expected, outs):
        rc, got = _noalloc(g, k, out)
        assert rc == L.GTA_OK, L.lib().gta_last_error()
        torch.cuda.synchronize()
        assert torch.equal(got, ref)  # integer graph: exact
    # the same graph again after a different one: still exact
    rc, again = _noalloc(graphs[0], shapes[0][1], again)
    assert rc == L.GTA_OK
    torch.cuda.synchronize()
    assert torch.equal(again, expected[0])
    assert _pool_high(pool) <= used_before, "a no-allocation call took memory from the stream-ordered pool"


def test_noalloc_reports_out_of_range_ids():
    """An id outside [0, n) is a data error (GTA_EDATA), as in gta_reverse_merge; the error word
    lives in the fixed scratch, and the next call starts with it cleared."""
    rng = np.random.default_rng(7)
    g = _graph(rng, 400, 8)
    bad = g.copy()
    bad[17, 3] = 400
    rc, _ = _noalloc(torch.from_numpy(bad.view(np.int32)).cuda(), 8)
    assert rc == L.GTA_EDATA
    assert b"outside" in L.lib().gta_last_error()
    gd = torch.from_numpy(g.view(np.int32)).cuda()
    rc, got = _noalloc(gd, 8)
    assert rc == L.GTA_OK
    torch.cuda.synchronize()
    assert torch.equal(got, _existing(gd, 8))


def test_noalloc_rejects_graphs_beyond_its_scratch():
    max_rows = L.lib().gta_reverse_merge_noalloc_max_rows()
    max_edges = L.lib().gta_reverse_merge_noalloc_max_edges()
    assert max_rows == 131072 and max_edges == 2097152
    g = torch.zeros((max_rows + 1, 1), dtype=torch.int32, device="cuda")
    rc, _ = _noalloc(g, 1)
    assert rc == L.GTA_EINVAL
    assert b"too large" in L.lib().gta_last_error()
    g2 = torch.zeros((70000, 32), dtype=torch.int32, device="cuda")  # 2.24M edges
    rc, _ = _noalloc(g2, 32)
    assert rc == L.GTA_EINVAL
