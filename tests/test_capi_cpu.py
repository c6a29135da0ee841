"""CPU checks of libgta: the shared library loads, exports every entry point
declared in include/gta.h, and its host-only file I/O keeps the reference's
byte layouts.  Compute entry points are called here only with arguments they reject before
any device work (no GPU)."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import gta
from gta import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gta.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(gta_\w+)\s*\(", src, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    names = _declared()
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/gta.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (gta_\w+)", out))
    assert set(names) <= exported
    assert L.lib().gta_version().startswith(b"gta-b200")


def test_dataset_roundtrip_f32_u8_i8(tmp_path):
    rng = np.random.default_rng(0)
    for ext, X in ((".fbin", rng.normal(size=(37, 13)).astype(np.float32)),
                   (".u8bin", rng.integers(0, 256, (41, 16)).astype(np.uint8)),
                   (".i8bin", rng.integers(-128, 128, (9, 7)).astype(np.int8))):
        p = str(tmp_path / f"x{ext}")
        gta.write_dataset(p, X)
        raw = open(p, "rb").read()
        assert np.frombuffer(raw[:8], np.int32).tolist() == [X.shape[0], X.shape[1]]  # BIGANN header
        np.testing.assert_array_equal(gta.read_dataset(p), X)
        np.testing.assert_array_equal(gta.read_dataset(p, 3, 5), X[3:8])


def test_knn_and_graph_layouts(tmp_path):
    rng = np.random.default_rng(1)
    ids = rng.integers(-1, 1000, (50, 8)).astype(np.int32)
    p = str(tmp_path / "vector_knn.bin")
    gta.write_knn(p, ids)
    raw = open(p, "rb").read()
    assert np.frombuffer(raw[:8], np.int64)[0] == 50 and np.frombuffer(raw[8:12], np.int32)[0] == 8
    np.testing.assert_array_equal(np.frombuffer(raw[12:], np.int32).reshape(50, 8), ids)
    np.testing.assert_array_equal(gta.read_knn(p), ids)
    g = rng.integers(0, 1000, (50, 4)).astype(np.uint32)
    pg = str(tmp_path / "final_graph.bin")
    gta.write_graph(pg, g)
    np.testing.assert_array_equal(gta.read_graph(pg), g)
    pd = str(tmp_path / "vector_dists.bin")
    dd = rng.random((50, 8)).astype(np.float32)
    gta.write_knn_dists(pd, dd)
    np.testing.assert_array_equal(np.frombuffer(open(pd, "rb").read()[12:], np.float32).reshape(50, 8), dd)


def test_npy_writer(tmp_path):
    ids = np.arange(24, dtype=np.int32).reshape(6, 4) - 3
    p = str(tmp_path / "neighbors.npy")
    gta.write_npy(p, ids)
    got = np.load(p)
    assert got.dtype == np.int64 and got.shape == (6, 4)
    np.testing.assert_array_equal(got, ids.astype(np.int64))


def test_file_errors(tmp_path):
    p = str(tmp_path / "bad.fbin")
    with open(p, "wb") as f:
        np.array([100, 8], np.int32).tofile(f)
        np.zeros(10, np.float32).tofile(f)  # truncated payload
    with pytest.raises(gta.GtaError) as e:
        gta.read_dataset(p)
    assert e.value.code == L.GTA_EDATA
    with pytest.raises(gta.GtaError) as e:
        gta.read_dataset(str(tmp_path / "x.txt"))
    assert e.value.code == L.GTA_EINVAL
    with pytest.raises(gta.GtaError) as e:
        gta.read_knn(str(tmp_path / "missing.bin"))
    assert e.value.code == L.GTA_EINVAL


def test_phased_bucket_knn_rejects_bad_arguments_before_device_work():
    """gta_bucket_knn_rows_phased takes phase 1 or 2, and phase 2 needs the seeds."""
    f = L.lib().gta_bucket_knn_rows_phased
    dummy = ctypes.c_void_p(16)  # never dereferenced: the checks come first
    args = lambda phase, seed: (dummy, L.GTA_U8, 100, 16, dummy, dummy, dummy, dummy, 4, 8, phase, seed, dummy,
                                dummy, ctypes.c_void_p(0))
    assert f(*args(3, dummy)) == L.GTA_EINVAL
    assert b"bad argument" in L.lib().gta_last_error()
    assert f(*args(2, ctypes.c_void_p(0))) == L.GTA_EINVAL
    assert f(*args(0, dummy)) == L.GTA_EINVAL


def test_ranged_bucket_knn_and_shard_entry_points_reject_bad_arguments():
    """The sharded build's entry points check their arguments before any device work."""
    lib = L.lib()
    d = ctypes.c_void_p(16)  # never dereferenced: the checks come first
    z = ctypes.c_void_p(0)
    # ranged kNN: both row-range arrays or neither (the ranged entry needs both)
    assert lib.gta_bucket_knn_rows_ranged(d, L.GTA_F32, 100, 16, d, d, d, d, 4, 8, 1, z, z, z, d, d, z) == L.GTA_EINVAL
    assert lib.gta_bucket_knn_rows_ranged(d, L.GTA_F32, 100, 16, d, d, d, d, 4, 8, 1, z, d, z, d, d, z) == L.GTA_EINVAL
    cnt = (ctypes.c_int64 * 65)()
    # membership packing: 1 to 64 ranks, a known dtype, both send buffers or neither
    pm = lib.gta_shard_pack_memberships
    assert pm(d, L.GTA_U8, 10, 8, 0, d, 4, d, 65, cnt, z, z, 0, z) == L.GTA_EINVAL
    assert pm(d, 7, 10, 8, 0, d, 4, d, 2, cnt, z, z, 0, z) == L.GTA_EINVAL
    assert pm(d, L.GTA_U8, 10, 8, 0, d, 4, d, 2, cnt, d, z, 0, z) == L.GTA_EINVAL
    assert pm(d, L.GTA_U8, 10, 8, 0, d, 4, z, 2, cnt, z, z, 0, z) == L.GTA_EINVAL
    # list packing: owner ranges in order, buffers all or none
    pl = lib.gta_shard_pack_lists
    lo = (ctypes.c_int64 * 4)()
    hi = (ctypes.c_int64 * 4)()
    bad_starts = (ctypes.c_int64 * 3)(0, 50, 40)
    good_starts = (ctypes.c_int64 * 3)(0, 40, 50)
    assert pl(d, d, 10, 8, d, d, d, 4, lo, hi, bad_starts, 2, cnt, z, z, z, 0, z) == L.GTA_EINVAL
    assert pl(d, d, 10, 8, d, d, d, 4, lo, hi, good_starts, 2, cnt, d, z, z, 0, z) == L.GTA_EINVAL
    assert lib.gta_shard_member_rows(z, 5, 0, 10, d, d, z) == L.GTA_EINVAL
    assert lib.gta_shard_lower_seeds(d, 8, 10, d, d, d, d, 4, lo, hi, 100, z, z) == L.GTA_EINVAL


def test_synthetic_generators_are_seeded():
    cfg = gta.scaled(gta.CONFIGS["c2"], 2000)
    a, b = gta.generate(cfg, seed=5), gta.generate(cfg, seed=5)
    assert a.dtype == np.uint8 and a.shape == (2000, 128)
    np.testing.assert_array_equal(a, b)
    c4 = gta.generate(gta.scaled(gta.CONFIGS["c4"], 500), seed=1)
    np.testing.assert_allclose(np.linalg.norm(c4, axis=1), 1.0, rtol=1e-5)
    c3 = gta.generate(gta.scaled(gta.CONFIGS["c3"], 300), seed=1)
    assert (c3 >= 0).all() and c3.shape[1] == 960


def test_shard_generator_is_seeded_per_shard():
    cfg = gta.scaled(gta.CONFIGS["c2"], 3000)
    np.testing.assert_array_equal(gta.generate_shard(cfg, 0, seed=9), gta.generate(cfg, seed=9))
    s1 = gta.generate_shard(cfg, 1, seed=9)
    assert s1.shape == (3000, 128) and not np.array_equal(s1, gta.generate(cfg, seed=9))
    np.testing.assert_array_equal(s1, gta.generate_shard(cfg, 1, seed=9))
    assert not np.array_equal(s1, gta.generate_shard(cfg, 2, seed=9))


@pytest.mark.parametrize("n,b,req,n_s,pool", [(1_000_000, 256, 0, 100_000, 5120), (100_000_000, 8192, 0, 10_000_000,
                                                                                      16384),
                                              (8_000_000, 2048, 0, 800_000, 20480), (10_000, 16, 10_000, 10_000, 320),
                                              (5_000, 600, 0, 600, 600)])
def test_kmeans_sizes(n, b, req, n_s, pool):
    """Host-only sizing rule shared by the single- and multi-GPU builds."""
    import ctypes

    bp = L.gta_bucket_params(n_buckets=b, kmeans_sample=req, seed=7)
    a, c, s = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_uint64()
    L.check(L.lib().gta_kmeans_sizes(n, ctypes.byref(bp), ctypes.byref(a), ctypes.byref(c), ctypes.byref(s)))
    assert (a.value, c.value) == (n_s, pool)
    assert s.value != 7


def test_npy_reader_and_u32_files(tmp_path):
    ids = np.array([[0, 5, -1], [7, 2147483647, 3]], np.int32)
    p = str(tmp_path / "n.npy")
    gta.write_npy(p, ids)
    np.testing.assert_array_equal(gta.read_npy_i64(p), ids)
    np.save(tmp_path / "np.npy", ids.astype(np.int64))  # numpy's own writer
    np.testing.assert_array_equal(gta.read_npy_i64(str(tmp_path / "np.npy")), ids)
    np.save(tmp_path / "big.npy", np.array([[1 << 31]], np.int64))
    with pytest.raises(gta.GtaError):
        gta.read_npy_i64(str(tmp_path / "big.npy"))
    np.save(tmp_path / "f.npy", np.zeros((2, 2), np.float32))
    with pytest.raises(gta.GtaError):
        gta.read_npy_i64(str(tmp_path / "f.npy"))
    v = np.arange(10, dtype=np.uint32) * 7
    gta.write_u32(str(tmp_path / "inv.bin"), v)
    np.testing.assert_array_equal(gta.read_u32(str(tmp_path / "inv.bin")), v)
    assert (tmp_path / "inv.bin").stat().st_size == 40  # raw, no header


def test_host_resident_needs_a_contiguous_host_array():
    """host_resident datasets are read in place: a strided view is refused before any device work."""
    X = np.zeros((100, 16), np.uint8)
    with pytest.raises(gta.GtaError) as e:
        gta.build_bucket(X[:, ::2], 4, 8, host_resident=True)
    assert e.value.code == L.GTA_EINVAL


def test_strided_host_arrays_are_refused_with_a_status():
    """Every entry point takes C-contiguous buffers: a strided host view raises GtaError (status 1),
    not an assertion that optimised Python would skip."""
    X = np.zeros((64, 16), np.float32)
    with pytest.raises(gta.GtaError) as e:
        gta.build_bucket(X[:, ::2], 4, 8)
    assert e.value.code == L.GTA_EINVAL


def test_stage_wrappers_refuse_host_arrays_before_device_work():
    """The stage entry points read device memory: numpy arguments are refused (status 1) before
    anything is allocated or launched, and mixed host / device arguments likewise."""
    X = np.zeros((64, 16), np.float32)
    mem = np.arange(64, dtype=np.int32)
    off = np.array([0, 64], np.int64)
    g = np.zeros((64, 8), np.int32)
    for call in (lambda: gta.bucket_knn(X, mem, off, 8), lambda: gta.prune(g, 4), lambda: gta.reverse_merge(g),
                 lambda: gta.sanitize(g), lambda: gta.assign_topk(X, X[:4], 2), lambda: gta.kmeans_fit(X, X[:4], 1)):
        with pytest.raises(gta.GtaError) as e:
            call()
        assert e.value.code == L.GTA_EINVAL
    fake_dev = type("FakeCudaTensor", (), {"is_cuda": True})()  # a device-side argument beside host X
    with pytest.raises(gta.GtaError) as e:
        gta.permute_rows(X, fake_dev)
    assert e.value.code == L.GTA_EINVAL
