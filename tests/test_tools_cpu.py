"""The command-line tools (bucket2, optimize) without a GPU: they are built next to
libgta.so, print their option list, and fail with the reference tools' exit codes on
bad arguments (1 = error) before touching the device."""
import os
import subprocess

import numpy as np
import pytest

import gta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "gpu-talored-ann_b200", "bin")


def tool(name):
    p = os.path.join(BIN, name)
    if not os.path.exists(p):
        pytest.skip(f"{name} is not built (make -C gpu-talored-ann_b200/csrc)")
    return p


def run(*args):
    return subprocess.run(list(args), capture_output=True, text=True, timeout=60)


@pytest.mark.parametrize("name,opts", [
    ("bucket2", ["--input", "--output", "--neighbors-m", "--fused-optimize-degree", "--seed", "--iterations",
                 "--knn-k", "--nprobe", "--skip-dists", "--skip-npy", "--out-of-core", "--centroid-ratio",
                 "--bucketing"]),
    ("optimize", ["--input", "--knn-graph", "--output", "--output-degree", "--skip-sort", "--save-npy",
                  "--force-chunked", "--gpu-fit-margin"]),
    ("translate_ids", ["--graph", "--inverse-perm", "--output", "--out-buffer-mb"]),
])
def test_help_lists_reference_options(name, opts):
    r = run(tool(name), "--help")
    assert r.returncode == 0
    for o in opts:
        assert o in r.stdout, f"{name} --help does not list {o}"


def test_bucket2_argument_errors(tmp_path):
    b2 = tool("bucket2")
    r = run(b2, "-o", str(tmp_path))
    assert r.returncode == 1 and "FATAL" in r.stderr and "--input" in r.stderr
    data = str(tmp_path / "x.u8bin")
    gta.write_dataset(data, np.zeros((10, 8), np.uint8))
    r = run(b2, "-i", data, "-o", str(tmp_path), "--neighbors-m", "0")
    assert r.returncode == 1 and "neighbors-m" in r.stderr
    r = run(b2, "-i", data, "-o", str(tmp_path), "--neighbors-m", "8", "--fused-optimize-degree", "9")
    assert r.returncode == 1 and "fused-optimize-degree" in r.stderr
    r = run(b2, "-i", data, "-o", str(tmp_path), "--neighbors-m", "8", "-t", "0")
    assert r.returncode == 1 and "iterations" in r.stderr
    r = run(b2, "-i", data, "-o", str(tmp_path), "--neighbors-m", "8", "--bucketing", "random")
    assert r.returncode == 1 and "--bucketing" in r.stderr
    r = run(b2, "-i", data, "-o", str(tmp_path), "--neighbors-m", "8", "--nprobe", "200")
    assert r.returncode == 1 and "nprobe" in r.stderr
    r = run(b2, "-i", data, "-o", str(tmp_path), "--bogus", "1")
    assert r.returncode == 1 and "unknown option" in r.stderr


def test_optimize_argument_errors(tmp_path):
    op = tool("optimize")
    data = str(tmp_path / "x.u8bin")
    knn = str(tmp_path / "vector_knn.bin")
    gta.write_dataset(data, np.zeros((10, 8), np.uint8))
    gta.write_knn(knn, np.zeros((12, 4), np.int32))
    r = run(op, "-i", data, "-g", knn, "-o", str(tmp_path / "g.bin"))
    assert r.returncode == 1 and "!= dataset N" in r.stderr
    gta.write_knn(knn, np.zeros((10, 4), np.int32))
    r = run(op, "-i", data, "-g", knn, "-o", str(tmp_path / "g.bin"), "--output-degree", "5")
    assert r.returncode == 1 and "> input degree" in r.stderr
    r = run(op, "-i", data, "-g", knn, "-o", str(tmp_path / "g.bin"), "--output-degree", "0")
    assert r.returncode == 1 and "must be > 0" in r.stderr


def test_translate_ids_argument_errors(tmp_path):
    tr = tool("translate_ids")
    g = str(tmp_path / "g.bin")
    gta.write_graph(g, np.zeros((5, 2), np.uint32))
    gta.write_u32(str(tmp_path / "inv.bin"), np.arange(4, dtype=np.uint32))
    r = run(tr, "-g", g, "-p", str(tmp_path / "inv.bin"), "-o", str(tmp_path / "o.bin"))
    assert r.returncode == 1 and "graph N=5" in r.stderr
    r = run(tr, "-g", g, "-o", str(tmp_path / "o.bin"))
    assert r.returncode == 1 and "--inverse-perm" in r.stderr
