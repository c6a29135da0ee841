"""The reference-bucketing build (gta_build_bucket2: KMeans|| data-point centroids, balanced
1-way buckets, own + nprobe pools) on the GPU against the oracle's restatement of the same
steps.  Every distance on both sides is the exact fp32 chain, so centroids, buckets and lists
must agree bit for bit (8-bit and float data)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import gta  # noqa: E402
from gta import _lib as L  # noqa: E402
from oracle import oracle as orc  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg_name,n,M,nprobe,ratio,rounds,rule", [
    ("c2", 20000, 32, 8, 0.01, 1, "default"),    # ~200 buckets: the FP32-pipe assignment path
    ("c2", 60000, 64, 16, 0.01, 1, "default"),   # ~600 buckets: the tensor-core assignment path
    ("c2", 12000, 16, 4, 0.02, 2, "default"),    # two rounds merged
    ("c1", 10000, 32, 6, 0.01, 1, "default"),    # float data
    ("c2", 20000, 32, 8, 0.01, 1, "diskjoin"),   # BUCKET2_ASSIGN_RULE=diskjoin
    ("c1", 10000, 32, 6, 0.01, 1, "diskjoin"),
])
def test_build_bucket2_vs_oracle(cfg_name, n, M, nprobe, ratio, rounds, rule):
    cfg = gta.scaled(gta.CONFIGS[cfg_name], n)
    X = gta.generate(cfg, seed=3)
    ids, dists, assign, cid = gta.build_bucket2(torch.from_numpy(X).cuda(), M, nprobe, ratio, 7, rounds,
                                                with_extras=True, assign_rule=rule)
    ri, rd, ra, rc = orc.build_bucket2(X, M, nprobe, ratio, 7, rounds, assign_rule={"default": 0, "diskjoin": 1}[rule])
    np.testing.assert_array_equal(cid.cpu().numpy(), rc)
    np.testing.assert_array_equal(assign.cpu().numpy(), ra)
    np.testing.assert_array_equal(dists.cpu().numpy(), rd)
    np.testing.assert_array_equal(ids.cpu().numpy(), ri)


def test_build_bucket2_host_arrays_and_graph():
    cfg = gta.scaled(gta.CONFIGS["c2"], 15000)
    X = gta.generate(cfg, seed=4)
    ids, dists = gta.build_bucket2(X, 32, 8, 0.01, 11)
    ri, rd, _, _ = orc.build_bucket2(X, 32, 8, 0.01, 11)
    np.testing.assert_array_equal(ids, ri)
    np.testing.assert_array_equal(dists, rd)
    # the lists feed the CAGRA optimize like the 2-way build's
    g = gta.optimize_knn(ids, 16)
    np.testing.assert_array_equal(g, orc.optimize(orc.sanitize(ri)[0], 16))


def test_build_bucket2_rejects_bad_parameters():
    X = torch.zeros((100, 8), dtype=torch.uint8, device="cuda")
    for kw in ({"knn_degree": 0}, {"knn_degree": 8, "nprobe": 200}, {"knn_degree": 8, "centroid_ratio": 2.0},
               {"knn_degree": 8, "assign_rule": "other"}):
        with pytest.raises(gta.GtaError) as e:
            gta.build_bucket2(X, **kw)
        assert e.value.code == L.GTA_EINVAL
