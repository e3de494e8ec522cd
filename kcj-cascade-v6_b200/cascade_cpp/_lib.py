"""ctypes binding of the C ABI in include/cascade_b200.h.

The library is the product: there is no CPU fallback. Importing this module
without the built ``libcascade_b200.so`` raises ImportError with the build
command.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcascade_b200.so")

CB_OK = 0
CB_ERR_ARG = 1
CB_ERR_CUDA = 2
CB_ERR_NOSPACE = 3
CB_ERR_BUFSIZE = 4
CB_ERR_TIMEOUT = 5
CB_ERR_NCCL = 6
CB_ERR_STATE = 7
CB_ERR_DEVICE = 8
CB_PROMOTE_EVERY_HIT = 0
CB_PROMOTE_LOCALITY = 1
CB_SELFTEST_HASH_WAIT = 1
CB_SELFTEST_FAIL_MOVES = 2
CB_SELFTEST_GET_ERROR = 3

CB_MEM_DEVICE = 0
CB_MEM_HOST = 1

CB_PUT_STORED = 0
CB_PUT_DEDUP = 1
CB_PUT_FAILED = 2

CB_FOUND_MISS = 0
CB_FOUND_LOCAL_HBM = 1
CB_FOUND_LOCAL_DRAM = 2
CB_FOUND_REMOTE_HBM = 3
CB_FOUND_REMOTE_DRAM = 4
CB_FOUND_NOT_COPIED = 0x80

CB_UID_BYTES = 128


class cb_config(C.Structure):
    _fields_ = [
        ("gpu_capacity_bytes", C.c_uint64),
        ("dram_capacity_bytes", C.c_uint64),
        ("device", C.c_int32),
        ("dedup_enabled", C.c_int32),
        ("semantic_eviction", C.c_int32),
        ("promote_on_hit", C.c_int32),
        ("index_log2", C.c_int32),
        ("copy_engine", C.c_int32),
        ("staging_bytes", C.c_uint64),
        ("profile", C.c_int32),
        ("hash_lanes", C.c_int32),
        ("replica_bytes", C.c_uint64),
        ("locality_aware", C.c_int32),
        ("promotion_threshold", C.c_uint32),
        ("kv_compression", C.c_int32),
        ("prefix_replication", C.c_int32),
        ("collective_timeout_ms", C.c_uint64),
        ("promotion_rule", C.c_int32),
        ("reserved32", C.c_int32),
        ("pipeline_blocks", C.c_uint64),
        ("hash_sms", C.c_int32),
        ("reserved32b", C.c_int32),
    ]


STATS_FIELDS = [
    "local_gpu_used", "local_dram_used", "cluster_gpu_used", "cluster_dram_used",
    "local_gpu_hits", "local_dram_hits", "remote_gpu_hits", "remote_dram_hits",
    "lustre_hits", "misses", "dedup_hits", "dedup_bytes_saved",
    "gpu_evictions", "dram_evictions", "prefix_blocks_protected", "promotions_to_local",
    "compression_savings", "total_blocks", "prefix_blocks",
    "evicted_bytes", "promoted_bytes", "dropped_blocks", "kernel_launches",
    "sha_ns", "sha_bytes", "sha_launches", "scatter_ns", "scatter_bytes", "scatter_launches",
    "gather_ns", "gather_bytes", "gather_launches", "tier_ns", "tier_bytes", "tier_launches",
    "peer_bytes_read", "peer_bytes_written", "prefix_replicated_blocks",
    "coll_ns", "coll_bytes", "coll_calls",
]


class cb_stats(C.Structure):
    _fields_ = [(f, C.c_uint64) for f in STATS_FIELDS]


class cb_location(C.Structure):
    _fields_ = [
        ("node_id", C.c_int32),
        ("gpu_id", C.c_int32),
        ("offset", C.c_uint64),
        ("size", C.c_uint64),
        ("is_gpu", C.c_int32),
        ("is_prefix", C.c_int32),
    ]


# (name, restype, argtypes) — exactly the entry points of cascade_b200.h.
_P = C.c_void_p
_U8P = C.POINTER(C.c_uint8)
_U64P = C.POINTER(C.c_uint64)
SIGNATURES = [
    ("cb_config_init", None, [C.POINTER(cb_config)]),
    ("cb_create", C.c_int, [C.POINTER(cb_config), C.POINTER(_P)]),
    ("cb_destroy", C.c_int, [_P]),
    ("cb_last_error", C.c_char_p, [_P]),
    ("cb_selftest", C.c_int, [_P, C.c_int32]),
    ("cb_get_views", C.c_int, [_P, _P, C.c_int32, _P, _P, _P, _P]),
    ("cb_release_views", C.c_int, [_P, _P, C.c_int32]),
    ("cb_kv_compress_batch", C.c_int, [_P, _P, _P, _P, C.c_int32, _P]),
    ("cb_kv_decompress_batch", C.c_int, [_P, _P, _P, _P, _P, C.c_int32, _P, _P]),
    ("cb_hash_batch", C.c_int, [_P, _P, _P, C.c_int32, C.c_int32, _P, _P]),
    ("cb_put_batch", C.c_int, [_P, _P, _P, _P, _P, C.c_int32, C.c_int32, _P, _P, _P]),
    ("cb_get_batch", C.c_int, [_P, _P, C.c_int32, _P, _P, C.c_int32, _P, _P, _P]),
    ("cb_contains_batch", C.c_int, [_P, _P, C.c_int32, _P]),
    ("cb_locate", C.c_int, [_P, _P, C.POINTER(cb_location), C.POINTER(C.c_int32)]),
    ("cb_evict", C.c_int, [_P, C.c_uint64, _U64P]),
    ("cb_get_stats", C.c_int, [_P, C.POINTER(cb_stats)]),
    ("cb_clear", C.c_int, [_P]),
    ("cb_sync", C.c_int, [_P]),
    ("cb_dht_unique_id", C.c_int, [_P]),
    ("cb_dht_attach", C.c_int, [_P, C.c_int32, C.c_int32, _P]),
    ("cb_dht_barrier", C.c_int, [_P]),
    ("cb_sync_metadata", C.c_int, [_P]),
    ("cb_rank", C.c_int, [_P, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    ("cb_put_batch_async", C.c_int, [_P, _P, _P, _P, _P, C.c_int32, C.c_int32, _P, _P, _P, _P]),
    ("cb_put_wait", C.c_int, [_P, C.c_uint64, _P]),
    ("cb_put_placed", C.c_int, [_P, _P]),
    ("cb_get_batch_async", C.c_int, [_P, _P, C.c_int32, _P, _P, _P, _P, _P]),
    ("cb_hash_batch_noalloc", C.c_int, [C.c_int32, _P, _P, C.c_int32, _P, _P]),
    ("cb_owner_rank", C.c_int32, [_P, C.c_int32]),
    ("cb_dht_route", C.c_int, [_P, C.c_int32, C.c_int32, _P, _P, _P]),
    ("cb_planner_create", C.c_int, [C.c_uint64, C.c_uint64, C.c_int32, C.c_int32, C.POINTER(_P)]),
    ("cb_planner_destroy", C.c_int, [_P]),
    ("cb_dht_plan_put", C.c_int, [_P, _P, _P, _P, C.c_int32, _P, _P]),
]

CB_NOALLOC_MAX_BLOCKS = 4096


def load(path: str = LIB_PATH) -> C.CDLL:
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build the CUDA library with "
            "`python kcj-cascade-v6_b200/build.py` (or __graft_entry__.build())")
    lib = C.CDLL(path)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


class CascadeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[cb {code}] {msg}")
        self.code = code
