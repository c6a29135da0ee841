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


def _graph(rng, n, k):
    """A pruned-graph-shaped input: k distinct non-self ids per row, a few hubs."""
    g = np.empty((n, k), np.uint32)
    hubs = rng.choice(n, 8, replace=False)
    for i in range(n):
        pool = rng.choice(n, k + 12, replace=False)
        pool = pool[pool != i][:k]
        if i % 3 == 0:
            pool[-1] = hubs[i % 8] if hubs[i % 8] != i and hubs[i % 8] not in pool[:-1] else pool[-1]
        g[i] = pool
    return g


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
    shapes = [(5000, 32), (3000, 16)]  # two calls in a row, different sizes
    graphs = [torch.from_numpy(_graph(rng, n, k).view(np.int32)).cuda() for n, k in shapes]
    expected = [_existing(g, k) for g, (_, k) in zip(graphs, shapes)]
    outs = [torch.full((n, k), -7, dtype=torch.int32, device="cuda") for n, k in shapes]
    again = torch.full(shapes[0], -7, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
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
    # every buffer was allocated before the measurement; the calls themselves took no device memory
    assert torch.cuda.mem_get_info()[0] == free_before


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
