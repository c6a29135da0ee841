"""gta: B200-native bucketed kNN-graph and CAGRA-style graph build (host layer over libgta.so)."""
from ._lib import GtaError, LIB_PATH, build, lib  # noqa: F401
from .api import (  # noqa: F401
    assign_topk,
    bucket_knn,
    build_bucket,
    build_cagra,
    build_memberships,
    kmeans_fit,
    kmeans_init,
    merge_lists,
    merge_memberships,
    optimize,
    prune,
    read_dataset,
    read_graph,
    read_knn,
    reverse_merge,
    sanitize,
    search,
    search_entries,
    sort_rows,
    write_dataset,
    write_graph,
    write_knn,
    write_knn_dists,
    write_npy,
)
from .synth import CONFIGS, generate, generate_queries, generate_shard, scaled  # noqa: F401
