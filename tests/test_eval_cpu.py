"""The evaluation front end (gta.eval, the reference's search.py command line) on the host:
recall figures against the reference's own recall_vs_gt (committed fixture), the set-wise
index comparison, and the index / ground-truth readers."""
import numpy as np
import pytest

import gta
from gta import eval as ev


def test_recall_vs_gt_matches_reference(golden):
    f = golden("eval_recall.npz")
    np.testing.assert_array_equal(np.array(ev.recall_vs_gt(f["pred"], f["gt"], int(f["topk"]))), f["recall"])
    np.testing.assert_array_equal(np.array(ev.recall_vs_gt(f["pred"], f["gt"], 5)), f["recall_k5"])


def test_compare_setwise(tmp_path, capsys):
    a = np.array([[1, 2, 3, -1], [4, 5, 6, 7], [0, 1, 2, 3]], np.int64)
    b = np.array([[3, 2, 1, 9], [8, 9, 10, 11], [3, 2, 1, 0]], np.int64)
    np.save(tmp_path / "a.npy", a)
    np.save(tmp_path / "b.npy", b)
    csv = tmp_path / "o" / "c.csv"
    m = ev.compare_indices_setwise(str(tmp_path / "a.npy"), str(tmp_path / "b.npy"), 3, str(csv))
    # k = 3: row 0 {1,2,3} vs {3,2,1} -> 1; row 1 -> 0; row 2 {0,1,2} vs {3,2,1} -> 2/3
    assert m == pytest.approx((1.0 + 0.0 + 2.0 / 3.0) / 3.0, abs=1e-6)
    out = capsys.readouterr().out
    assert "HitsAny@3               : 0.666667" in out and "SetEqual@3              : 0.333333" in out
    assert csv.read_text().splitlines()[1] == "0,3,3,3,1.000000"


def test_readers(tmp_path):
    gt = np.arange(12, dtype=np.int32).reshape(3, 4)
    with open(tmp_path / "gt.ibin", "wb") as f:
        np.array([3, 4], np.int32).tofile(f)
        gt.tofile(f)
    np.testing.assert_array_equal(ev.load_ibin(str(tmp_path / "gt.ibin")), gt)
    g = np.arange(10, dtype=np.uint32).reshape(5, 2)
    gta.write_graph(str(tmp_path / "g.bin"), g)
    np.testing.assert_array_equal(ev.load_index(str(tmp_path / "g.bin")), g.astype(np.int64))
    np.save(tmp_path / "bad.npy", np.zeros(4))
    with pytest.raises(ValueError):
        ev.load_index(str(tmp_path / "bad.npy"))
