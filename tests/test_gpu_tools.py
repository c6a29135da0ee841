"""The command-line tools on the GPU, end to end through files: bucket2's outputs equal the
library's build and the oracle's optimize of it; optimize (with and without the L2 sort)
equals the oracle's sanitize -> sort -> prune -> reverse edges; bucket2 -t merges rounds
exactly as the merge rule says."""
import os
import subprocess

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import gta  # noqa: E402
from oracle import oracle as orc  # noqa: E402

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "gpu-talored-ann_b200", "bin")


def run(*args):
    r = subprocess.run([str(a) for a in args], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    return r


@pytest.fixture(scope="module")
def data(tmp_path_factory):
    d = tmp_path_factory.mktemp("tools")
    cfg = gta.scaled(gta.CONFIGS["c2"], 6000, n_buckets=6)
    X = gta.generate(cfg, seed=3)
    path = d / "base.u8bin"
    gta.write_dataset(str(path), X)
    return d, path, X


@pytest.mark.parametrize("rounds", [1, 2])
def test_bucket2_outputs(data, rounds):
    d, path, X = data
    out = d / f"out{rounds}"
    run(os.path.join(BIN, "bucket2"), "-i", path, "-o", out, "--neighbors-m", 32, "--fused-optimize-degree", 16,
        "--bucketing", "top2", "--n-buckets", 6, "--kmeans-iters", 5, "--seed", 7, "-t", rounds, "--knn-k", 16)
    sub = out / f"k16p16m32t{rounds}"
    ids = gta.read_knn(str(sub / "vector_knn.bin"))
    dists = np.fromfile(sub / "vector_dists.bin", dtype=np.float32, offset=12).reshape(ids.shape)
    graph = gta.read_graph(str(sub / "final_graph.bin"))
    npy = np.load(sub / "neighbors.npy")
    inv = gta.read_u32(str(sub / "inverse_perm.bin"))
    # the library's build with the same parameters (rounds merged by the reference's merge rule)
    ri, rd = gta.build_bucket(X, 6, 32, 5, 0, 7)
    for r in range(1, rounds):
        ni, nd = gta.build_bucket(X, 6, 32, 5, 0, 7 + r)
        ri, rd = orc.merge_lists(ri, rd, ni, nd)
    li, ld, cent, top2 = gta.build_bucket(X, 6, 32, 5, 0, 7, rounds=rounds, with_extras=True)
    np.testing.assert_array_equal(li, ri)
    # renumbering: centroid kNN (k = min(knn-k, B-1)) -> bucket order -> nearest-bucket ranges
    ck = 5
    cid, _ = orc.topk_assign(cent, cent, ck + 1)
    adj = np.array([[v for v in row if v != b][:ck] for b, row in enumerate(cid)], np.int32)
    order = orc.bucket_order(adj, max(4 * ck, 16))
    want_inv, want_off = orc.bucket_reorder(top2[:, 0].copy(), 6, order=order)
    np.testing.assert_array_equal(inv, want_inv)
    np.testing.assert_array_equal(np.fromfile(sub / "bucket_offsets.bin", dtype=np.uint32, offset=4), want_off)
    np.testing.assert_array_equal(np.fromfile(sub / "bucket_process_order.bin", dtype=np.int32, offset=4), order)
    np.testing.assert_array_equal(gta.read_graph(str(sub / "centroid_knn.bin")).view(np.int32), adj)
    np.testing.assert_array_equal(gta.read_dataset(str(sub / "data_reordered.u8bin")), X[inv])
    ids_new, bad = orc.permute_graph(ri, inv, False, True)
    assert bad == 0
    np.testing.assert_array_equal(ids, ids_new)
    np.testing.assert_array_equal(dists, rd[inv])
    np.testing.assert_array_equal(npy, ids_new.astype(np.int64))
    # final graph: optimize in the reordered space, translated back to the input order
    g_new = orc.optimize(orc.sanitize(ids_new)[0], 16)
    want_graph, _ = orc.permute_graph(g_new, inv, True, False)
    np.testing.assert_array_equal(graph, want_graph.view(np.uint32))
    # translate_ids on the reordered-space graph, as .bin and as .npy
    gta.write_graph(str(sub / "graph_new_ids.bin"), g_new)
    run(os.path.join(BIN, "translate_ids"), "-g", sub / "graph_new_ids.bin", "-p", sub / "inverse_perm.bin",
        "-o", sub / "translated.bin")
    np.testing.assert_array_equal(gta.read_graph(str(sub / "translated.bin")), graph)
    run(os.path.join(BIN, "translate_ids"), "-g", sub / "neighbors.npy", "-p", sub / "inverse_perm.bin",
        "-o", sub / "neighbors_orig.npy")
    np.testing.assert_array_equal(np.load(sub / "neighbors_orig.npy"), ri.astype(np.int64))


def test_bucket2_reference_bucketing(data):
    """The default bucketing: the reference tool's (KMeans||, balanced 1-way, own + nprobe pools)."""
    d, path, X = data
    out = d / "outref"
    run(os.path.join(BIN, "bucket2"), "-i", path, "-o", out, "--neighbors-m", 32, "--fused-optimize-degree", 16,
        "--centroid-ratio", 0.005, "--nprobe", 6, "--knn-k", 8, "--seed", 9)
    sub = out / "k8p6m32t1"
    ri, rd, ra, rc = orc.build_bucket2(X, 32, 6, 0.005, 9)
    B = rc.size
    cent = X[rc].astype(np.float32)
    cid, _ = orc.topk_assign(cent, cent, 9)
    adj = np.array([[v for v in row if v != b][:8] for b, row in enumerate(cid)], np.int32)
    order = orc.bucket_order(adj, max(4 * 8, 16))
    inv, _ = orc.bucket_reorder(ra, B, order=order)
    np.testing.assert_array_equal(gta.read_u32(str(sub / "inverse_perm.bin")), inv)
    ids_new, _ = orc.permute_graph(ri, inv, False, True)
    np.testing.assert_array_equal(gta.read_knn(str(sub / "vector_knn.bin")), ids_new)
    g_new = orc.optimize(orc.sanitize(ids_new)[0], 16)
    want, _ = orc.permute_graph(g_new, inv, True, False)
    np.testing.assert_array_equal(gta.read_graph(str(sub / "final_graph.bin")), want.view(np.uint32))


def test_optimize_tool_sorts_and_prunes(data):
    d, path, X = data
    ids, _ = gta.build_bucket(X, 6, 32, 5, 0, 7)
    rng = np.random.default_rng(0)
    shuffled = np.take_along_axis(ids, np.argsort(rng.random(ids.shape), axis=1), axis=1)
    shuffled[::7, -3:] = -1  # padding the sanitize step must replace
    knn = d / "shuffled_knn.bin"
    gta.write_knn(str(knn), shuffled)
    out = d / "cagra_graph.bin"
    run(os.path.join(BIN, "optimize"), "-i", path, "-g", knn, "-o", out, "--output-degree", 16, "--save-npy")
    san, _ = orc.sanitize(shuffled)
    want = orc.optimize(orc.sort_rows_l2(X, san.view(np.int32)).view(np.uint32), 16)
    got = gta.read_graph(str(out))
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(np.load(d / "cagra_graph.npy"), want.astype(np.int64))
    # the library entry the tool calls, on device arrays
    gd = gta.optimize_knn(torch.from_numpy(shuffled).cuda(), 16, X=torch.from_numpy(X).cuda())
    np.testing.assert_array_equal(gd.cpu().numpy().view(np.uint32), want)
    # --skip-sort on already ascending lists
    knn2 = d / "vector_knn.bin"
    gta.write_knn(str(knn2), ids)
    out2 = d / "cagra_graph2.bin"
    run(os.path.join(BIN, "optimize"), "-i", path, "-g", knn2, "-o", out2, "--output-degree", 16, "--skip-sort")
    np.testing.assert_array_equal(gta.read_graph(str(out2)), orc.optimize(orc.sanitize(ids)[0], 16))


def test_optimize_tool_refuses_with_exit_2(data):
    d, path, X = data
    ids, _ = gta.build_bucket(X, 6, 32, 5, 0, 7)
    knn = d / "vk.bin"
    gta.write_knn(str(knn), ids)
    for extra in (["--force-chunked"], ["--gpu-fit-margin", "1e9"]):
        r = subprocess.run([os.path.join(BIN, "optimize"), "-i", str(path), "-g", str(knn), "-o", str(d / "x.bin")]
                           + extra, capture_output=True, text=True, timeout=120)
        assert r.returncode == 2, r.stderr
