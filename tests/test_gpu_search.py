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


def test_eval_command_line(golden, tmp_path):
    """python -m gta.eval search over files: the recall lines of the reference's search.py
    for the fixture's queries (their results are the reference's own)."""
    import os
    import subprocess
    import sys

    from gta import eval as ev

    f = golden("search.npz")
    gta.write_dataset(str(tmp_path / "base.u8bin"), f["base"])
    gta.write_dataset(str(tmp_path / "query.u8bin"), f["queries"])
    np.save(tmp_path / "index.npy", f["graph"].astype(np.int64))
    dd = ((f["queries"][:, None, :].astype(np.int64) - f["base"][None].astype(np.int64)) ** 2).sum(-1)
    gt = np.argsort(dd, axis=1, kind="stable")[:, :10]  # exact integers: ties by id
    with open(tmp_path / "gt.ibin", "wb") as fh:
        np.array(gt.shape, np.int32).tofile(fh)
        gt.astype(np.int32).tofile(fh)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PYTHONPATH=os.path.join(root, "gpu-talored-ann_b200"))
    r = subprocess.run([sys.executable, "-m", "gta.eval", "search", "--base", str(tmp_path / "base.u8bin"),
                        "--query", str(tmp_path / "query.u8bin"), "--index", str(tmp_path / "index.npy"),
                        "--gt", str(tmp_path / "gt.ibin"), "--topk", "10", "--ef", str(int(f["ef"])),
                        "--num-entry", "4"], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr
    want = ev.recall_vs_gt(f["ids"].astype(np.int64), gt, 10)
    assert f"Recall@10 (recall mean overlap): {want[2]:.6f}" in r.stdout, r.stdout
    assert f"Recall@10 (hit GT[:,0])         : {want[0]:.6f}" in r.stdout, r.stdout
