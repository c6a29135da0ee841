"""ctypes binding of libgta.so (the C ABI declared in include/gta.h).

The library is built in-tree (gpu-talored-ann_b200/lib/libgta.so) by
``gpu-talored-ann_b200/csrc/Makefile``.  Loading fails loudly when it is
missing: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libgta.so")
CSRC = os.path.join(PKG_DIR, "csrc")

GTA_OK, GTA_EINVAL, GTA_ENOMEM, GTA_ECUDA, GTA_ENCCL, GTA_EDATA = range(6)
GTA_ROWS_INTEGER = 1
GTA_F32, GTA_U8, GTA_I8 = 0, 1, 2
GTA_L2, GTA_IP = 0, 1

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_U64 = ctypes.c_uint64


class GtaError(RuntimeError):
    """Raised for a non-zero status of a libgta entry point."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[gta status {code}] {msg}")
        self.code = code


class gta_dataset(ctypes.Structure):
    _fields_ = [("data", _P), ("n", _I64), ("d", _I32), ("dtype", _I32), ("metric", _I32), ("on_device", _I32)]


class gta_bucket_params(ctypes.Structure):
    _fields_ = [
        ("n_buckets", _I32), ("kmeans_iters", _I32), ("knn_degree", _I32), ("rounds", _I32),
        ("kmeans_sample", _I64), ("seed", _U64),
        ("init_centroids", _P), ("init_on_device", _I32), ("out_on_device", _I32),
        ("centroids_out", _P), ("top2_out", _P), ("device_budget", _I64),
    ]


class gta_bucket2_params(ctypes.Structure):
    _fields_ = [
        ("knn_degree", _I32), ("nprobe", _I32), ("knn_k", _I32), ("rounds", _I32),
        ("centroid_ratio", ctypes.c_float), ("assign_rule", _I32), ("seed", _U64),
        ("out_on_device", _I32), ("reserved1", _I32),
        ("assign_out", _P), ("centroid_ids_out", _P), ("n_buckets_out", ctypes.POINTER(_I32)),
    ]


class gta_cagra_params(ctypes.Structure):
    _fields_ = [("bucket", gta_bucket_params), ("graph_degree", _I32), ("reserved0", _I32)]


_SIGS = {
    "gta_build_bucket": [ctypes.POINTER(gta_dataset), ctypes.POINTER(gta_bucket_params), _P, _P, _P],
    "gta_optimize": [_P, _I64, _I32, _I32, _P, _I32, _P],
    "gta_build_cagra": [ctypes.POINTER(gta_dataset), ctypes.POINTER(gta_cagra_params), _P, _P],
    "gta_build_bucket2": [ctypes.POINTER(gta_dataset), ctypes.POINTER(gta_bucket2_params), _P, _P, _P],
    "gta_optimize_knn": [ctypes.POINTER(gta_dataset), _P, _I64, _I32, _I32, _P, _I32, _P],
    "gta_kmeans_fit": [_P, _I64, _I32, _P, _I32, _I32, _P, _P],
    "gta_kmeans_init": [_P, _I64, _I32, _I32, _U64, _P, _P],
    "gta_assign_topk": [_P, _I64, _I32, _P, _I32, _I32, _P, _P, _P],
    "gta_assign_topk_ex": [_P, _I64, _I32, _P, _I32, _I32, _P, _P, _I32, _P],
    "gta_build_memberships": [_P, _I64, _I32, _P, _P, _P, _P],
    "gta_bucket_knn": [_P, _I32, _I64, _I32, _P, _P, _I32, _I32, _P, _P, _P],
    "gta_merge_memberships": [_P, _P, _P, _I64, _I32, _P, _P, _P],
    "gta_merge_lists": [_P, _P, _P, _P, _I64, _I32, _P, _P, _P],
    "gta_sanitize": [_P, _I64, _I32, _P, _P],
    "gta_sort_rows": [_P, _I64, _I32, _P, _I32, _P, _P],
    "gta_prune": [_P, _I64, _I32, _I32, _P, _P],
    "gta_reverse_merge": [_P, _I64, _I32, _P, _P],
    "gta_reverse_merge_noalloc": [_P, _I64, _I32, _P, _P],
    "gta_search": [ctypes.POINTER(gta_dataset), _P, _I64, _P, _I32, _P, _I32, _I32, _I32, _P, _P, _P],
    "gta_bucket_order": [_P, _I32, _I32, _I32, _I32, _P, _P, _I32, _P],
    "gta_bucket_reorder": [_P, _I64, _I32, _I32, _P, _P, _P, _I32, _P],
    "gta_permute_rows": [_P, _I64, _I64, _P, _P, _I32, _P],
    "gta_permute_graph": [_P, _I64, _I32, _P, _I32, _I32, _P, _I32, _P],
    "gta_kmeans_sizes": [_I64, ctypes.POINTER(gta_bucket_params), ctypes.POINTER(_I64), ctypes.POINTER(_I64),
                         ctypes.POINTER(_U64)],
    "gta_sample_ids": [_I64, _I64, _U64, _P, _P],
    "gta_gather_rows": [_P, _I32, _I64, _I32, _I64, _P, _I64, _P, _P],
    "gta_centroid_sums": [_P, _I64, _I32, _P, _I32, _P, _P, _P],
    "gta_centroid_means": [_P, _P, _I32, _I32, _P, _P],
    "gta_group_memberships": [_P, _P, _I64, _I32, _P, _P, _P],
    "gta_bucket_knn_rows": [_P, _I32, _I64, _I32, _P, _P, _P, _I32, _I32, _P, _P, _P],
    "gta_bucket_knn_rows_phased": [_P, _I32, _I64, _I32, _P, _P, _P, _P, _I32, _I32, _I32, _P, _P, _P, _P],
    "gta_bucket_knn_rows_ranged": [_P, _I32, _I64, _I32, _P, _P, _P, _P, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P],
    "gta_shard_pack_memberships": [_P, _I32, _I64, _I32, _I64, _P, _I32, _P, _I32, _P, _P, _P, _I64, _P],
    "gta_shard_pack_lists": [_P, _P, _I64, _I32, _P, _P, _P, _I32, _P, _P, _P, _I32, _P, _P, _P, _P, _I64, _P],
    "gta_shard_member_rows": [_P, _I64, _I64, _I64, _P, _P, _P],
    "gta_shard_lower_seeds": [_P, _I32, _I64, _P, _P, _P, _P, _I32, _P, _P, _I64, _P, _P],
    "gta_sanitize_rows": [_P, _I64, _I64, _I64, _I32, _P, _P],
    "gta_prune_rows": [_P, _I64, _I32, _I32, _I64, _I64, _P, _I32, _P, _P],
    "gta_reverse_merge_rows": [_P, _I64, _I32, _I64, _I64, _P, _P],
    "gta_read_dataset_header": [ctypes.c_char_p, ctypes.POINTER(_I64), ctypes.POINTER(_I32), ctypes.POINTER(_I32)],
    "gta_read_dataset": [ctypes.c_char_p, _I64, _I64, _P],
    "gta_write_dataset": [ctypes.c_char_p, _P, _I64, _I32, _I32],
    "gta_write_knn": [ctypes.c_char_p, _P, _I64, _I32],
    "gta_read_knn_header": [ctypes.c_char_p, ctypes.POINTER(_I64), ctypes.POINTER(_I32)],
    "gta_read_knn": [ctypes.c_char_p, _P],
    "gta_write_knn_dists": [ctypes.c_char_p, _P, _I64, _I32],
    "gta_write_graph": [ctypes.c_char_p, _P, _I64, _I32],
    "gta_read_graph_header": [ctypes.c_char_p, ctypes.POINTER(_I64), ctypes.POINTER(_I32)],
    "gta_read_graph": [ctypes.c_char_p, _P],
    "gta_write_npy_i64": [ctypes.c_char_p, _P, _I64, _I32],
    "gta_read_npy_i64_header": [ctypes.c_char_p, ctypes.POINTER(_I64), ctypes.POINTER(_I32)],
    "gta_read_npy_i64": [ctypes.c_char_p, _P],
    "gta_write_u32": [ctypes.c_char_p, _P, _I64],
    "gta_read_u32_count": [ctypes.c_char_p, ctypes.POINTER(_I64)],
    "gta_read_u32": [ctypes.c_char_p, _P],
    "gta_profile_enable": [_I32],
    "gta_release_workspace": [],
    "gta_device_memory": [ctypes.POINTER(_I64), ctypes.POINTER(_I64)],
    "gta_profile_get": [_I32, ctypes.c_char_p, _I32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_double)],
    "gta_profile_counters": [_I32, ctypes.POINTER(ctypes.c_double), _I32],
}

_lib = None


def build(jobs: int = 3) -> str:
    """Compile libgta.so for sm_100a (nvcc cross-compiles without a GPU)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", CSRC, f"-j{jobs}"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libgta.so is not built ({LIB_PATH}); run `make -C {CSRC}`")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        L.gta_last_error.restype = ctypes.c_char_p
        L.gta_last_error.argtypes = []
        L.gta_version.restype = ctypes.c_char_p
        L.gta_version.argtypes = []
        L.gta_profile_count.restype = ctypes.c_int
        L.gta_profile_count.argtypes = []
        L.gta_launch_count.restype = ctypes.c_longlong
        L.gta_launch_count.argtypes = []
        for fn in ("gta_reverse_merge_noalloc_max_rows", "gta_reverse_merge_noalloc_max_edges"):
            getattr(L, fn).restype = ctypes.c_int64
            getattr(L, fn).argtypes = []
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != GTA_OK:
        raise GtaError(rc, lib().gta_last_error().decode(errors="replace"))


def profile_enable(on: bool) -> None:
    """Start (clearing old records) or stop per-stage CUDA-event timing inside libgta."""
    check(lib().gta_profile_enable(1 if on else 0))


def profile_records():
    """[(stage name, elapsed ms, algorithmic units, counters)] recorded since profile_enable(True)."""
    out = []
    name = ctypes.create_string_buffer(64)
    ms, units = ctypes.c_float(), ctypes.c_double()
    cnt = (ctypes.c_double * 8)()
    for i in range(lib().gta_profile_count()):
        check(lib().gta_profile_get(i, name, 64, ctypes.byref(ms), ctypes.byref(units)))
        check(lib().gta_profile_counters(i, cnt, 8))
        out.append((name.value.decode(), ms.value, units.value, tuple(cnt)))
    return out


def launch_count() -> int:
    """This library's own kernel launches since it was loaded."""
    return int(lib().gta_launch_count())
