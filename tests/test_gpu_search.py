"""Device graph search (gta_search) against the reference's search.py rule:
the golden fixture made by the reference's own graph_search_single, and the
oracle's restatement on a graph built by this library.  8-bit data, so every
distance is an exact float32 integer and the results must match bit for bit."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import gta  # noqa: E402
from gta import _lib as L  # noqa: E402
from oracle import oracle as orc  # noqa: E402

pytestmark = pytest.mark.gpu


def test_search_matches_reference_fixture(golden):
    f = golden("search.npz")
    topk, ef = int(f["topk"]), int(f["ef"])
    # device arrays
    ids, dists = gta.search(torch.from_numpy(f["base"]).cuda(), torch.from_numpy(f["graph"].view(np.int32)).cuda(),
                            torch.from_numpy(f["queries"]).cuda(), topk, ef, entries=f["entries"])
    np.testing.assert_array_equal(dists.cpu().numpy(), f["dists"])
    np.testing.assert_array_equal(ids.cpu().numpy(), f["ids"])
    # host arrays, entries drawn like the reference
    ids_h, dists_h = gta.search(f["base"], f["graph"], f["queries"], topk, ef, num_entry=4, seed=42)
    np.testing.assert_array_equal(ids_h, f["ids"])
    np.testing.assert_array_equal(dists_h, f["dists"])


@pytest.mark.parametrize("ef,topk,ne", [(64, 10, 4), (200, 10, 4), (16, 16, 1)])
def test_search_matches_oracle_on_built_graph(ef, topk, ne):
    cfg = gta.scaled(gta.CONFIGS["c2"], 40000)
    X = gta.generate(cfg, seed=5)
    base, Q = X[:38000], X[38000:38400]
    g = gta.build_cagra(torch.from_numpy(base).cuda(), 10, 32, 16, 4)
    entries = gta.search_entries(base.shape[0], Q.shape[0], ne, 42)
    ids, dists = gta.search(torch.from_numpy(base).cuda(), g, torch.from_numpy(Q).cuda(), topk, ef, entries=entries)
    ri, rd = orc.graph_search(base, g.cpu().numpy().view(np.uint32), Q, entries, topk, ef)
    np.testing.assert_array_equal(dists.cpu().numpy(), rd)
    np.testing.assert_array_equal(ids.cpu().numpy(), ri)


def test_search_rejects_bad_arguments():
    b = torch.zeros((100, 16), dtype=torch.uint8, device="cuda")
    g = torch.zeros((100, 8), dtype=torch.int32, device="cuda")
    with pytest.raises(gta.GtaError) as e:
        gta.search(b, g, b[:4], topk=10, ef=300)
    assert e.value.code == L.GTA_EINVAL
