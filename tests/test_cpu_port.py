"""The CPU port that bench.py times as the reference's CPU path (oracle/cpu_port.py), pinned
to outputs of the reference's own Python code (fixtures made by tests/golden/make_golden.py):

  * kmeans_pp_centers  -- bucketDemo/build_bucket.py:189-229, the same torch RNG calls, so the
                          same centres as the reference's own run (kmeans_top2.npz, B = 12, seed 42);
  * one Lloyd step     -- bucketDemo/build_bucket.py:232-262 (kmeans_top2.npz, 5 iterations);
  * prune_graph        -- bucketDemo/prune.py:8-83, the occlusion rule (occlusion.npz).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import cpu_port  # noqa: E402


def test_kmeans_pp_centers_equal_the_reference(golden):
    f = golden("kmeans_top2.npz")
    X = torch.from_numpy(f["X"])
    _, C0 = cpu_port.kmeans_pp_centers(X, f["C0"].shape[0], seed=42)
    np.testing.assert_array_equal(C0.numpy(), f["C0"])


def test_lloyd_steps_equal_the_reference(golden):
    f = golden("kmeans_top2.npz")
    X = torch.from_numpy(f["X"])
    C = torch.from_numpy(f["C0"].copy())
    for _ in range(int(f["iters"])):
        C = cpu_port.lloyd_step(X, C)
    np.testing.assert_allclose(C.numpy(), f["C"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("cap,key", [(None, "pruned"), (8, "pruned_k8")])
def test_occlusion_prune_equals_the_reference(golden, cap, key):
    f = golden("occlusion.npz")
    np.testing.assert_array_equal(cpu_port.prune_graph(f["X"], f["neighbors"], cap), f[key])


def test_occlusion_prune_row_sample(golden):
    """``rows`` limits the work to a sample (the timed CPU leg); the sampled rows equal the full run."""
    f = golden("occlusion.npz")
    rows = np.arange(3, 600, 37)
    part = cpu_port.prune_graph(f["X"], f["neighbors"], 8, rows=rows)
    np.testing.assert_array_equal(part[rows], f["pruned_k8"][rows])
    assert (np.delete(part, rows, axis=0) == -1).all()
