"""B200-native ``cascade_cpp``: drop-in for the reference's pybind module.

Mirrors the Python surface of cascade_Code/cpp/python/bindings.cpp —
``DistributedStore`` / ``DistributedConfig`` / ``DistributedStats`` /
``BlockLocation`` (bindings.cpp:91-171), ``CascadeStore`` / ``CascadeConfig``
/ ``CascadeStats`` (bindings.cpp:15-85) and ``compute_block_id``
(bindings.cpp:176-179) — over the C ABI of ``include/cascade_b200.h``.
Adds ``batch_put`` / ``batch_get`` (the reference's C++-only
``put_batch``/``get_batch``, include/cascade_distributed.hpp:359-365) and
accepts CUDA tensors (any dtype, reinterpreted as bytes) besides numpy
arrays. Every byte moved and every SHA-256 runs in the sm_100a kernels of
``libcascade_b200.so``; nothing here computes on the CPU.

Block IDs: ``compute_block_id`` returns the first 16 SHA-256 bytes as 32
lowercase hex chars, exactly like cascade_core.cpp:47-58. The store keys a
block by those 16 bytes; a caller ID that is not 32 lowercase hex chars (the
reference allows any string, e.g. ``"synth_b12"``) is keyed by a 16-byte
BLAKE2b of the string, with a per-store check that no two strings share one.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import os
import re
import threading
import warnings
from typing import Iterable, Sequence

import numpy as np

from . import _lib as L
from ._lib import CascadeError

try:  # torch is plumbing (device buffers, streams, process groups)
    import torch
except Exception:  # pragma: no cover - torch is present in this image
    torch = None

__all__ = [
    "DistributedConfig", "DistributedStore", "DistributedStats", "BlockLocation",
    "CascadeConfig", "CascadeStore", "CascadeStats", "compute_block_id",
    "compute_block_ids", "block_id_to_key", "key_to_block_id", "CascadeError", "KVCompressor",
    "PutFuture", "DhtPlanner", "dht_route",
]

_lib_handle = None
_lib_lock = threading.Lock()
_cache_lock = threading.Lock()  # the per-device helper stores (hashing, KVCompressor)


def _native_lib():
    global _lib_handle
    if _lib_handle is None:
        with _lib_lock:
            if _lib_handle is None:
                _lib_handle = L.load()
    return _lib_handle


# --------------------------------------------------------------------- ids

_HEX32 = re.compile(r"[0-9a-f]{32}\Z")


def block_id_to_key(block_id: str) -> bytes:
    """16-byte store key of a BlockId string."""
    if _HEX32.match(block_id):
        return bytes.fromhex(block_id)
    return hashlib.blake2b(block_id.encode("utf-8", "surrogatepass"), digest_size=16,
                           person=b"cascade-b200-id").digest()


def key_to_block_id(key: bytes) -> str:
    return bytes(key).hex()


def owner_rank(block_id: str, world: int) -> int:
    """Rank that owns ``block_id`` in a ``world``-rank DHT (cb_owner_rank)."""
    k = np.frombuffer(block_id_to_key(block_id), np.uint8).copy()
    return int(_native_lib().cb_owner_rank(C.c_void_p(k.ctypes.data), int(world)))


def dht_route(keys: np.ndarray, world: int):
    """Writer-side DHT routing of a batch of 16-byte keys (cb_dht_route):
    (owner per key, send order grouped by owner in batch order, keys per
    owner). Host-only."""
    keys = np.ascontiguousarray(keys, np.uint8).reshape(-1, 16)
    n = len(keys)
    owner = np.zeros(n, np.int32)
    order = np.zeros(n, np.int32)
    counts = np.zeros(int(world), np.uint32)
    rc = _native_lib().cb_dht_route(_ptr(keys), n, int(world), _ptr(owner), _ptr(order), _ptr(counts))
    if rc:
        raise CascadeError(rc, "cb_dht_route: bad arguments")
    return owner, order, counts


class DhtPlanner:
    """A DHT owner's host policy without a GPU (cb_planner_create /
    cb_dht_plan_put): the function an owner runs on the requests of one put
    step, in (source rank, batch index) order."""

    def __init__(self, gpu_capacity: int, dram_capacity: int = 0, semantic_eviction: bool = True,
                 dedup_enabled: bool = True):
        self._lib = _native_lib()
        self._p = C.c_void_p()
        rc = self._lib.cb_planner_create(int(gpu_capacity), int(dram_capacity), int(bool(semantic_eviction)),
                                         int(bool(dedup_enabled)), C.byref(self._p))
        if rc:
            raise CascadeError(rc, "cb_planner_create failed")

    def plan_put(self, keys: np.ndarray, sizes: np.ndarray, prefix: np.ndarray | None = None):
        """-> (status per request: CB_PUT_*, location word per request)."""
        keys = np.ascontiguousarray(keys, np.uint8).reshape(-1, 16)
        n = len(keys)
        sizes = np.ascontiguousarray(sizes, np.uint64)
        pf = None if prefix is None else np.ascontiguousarray(prefix, np.uint8)
        status = np.zeros(n, np.uint8)
        loc = np.zeros(n, np.uint64)
        rc = self._lib.cb_dht_plan_put(self._p, _ptr(keys), _ptr(sizes), _ptr(pf), n, _ptr(status), _ptr(loc))
        if rc:
            raise CascadeError(rc, "cb_dht_plan_put failed")
        return status, loc

    def close(self):
        if self._p:
            self._lib.cb_planner_destroy(self._p)
            self._p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ buffers

def _block_view(data, writable: bool = False):
    """(address, nbytes, mem_kind, device_index, keepalive) of a block buffer."""
    if torch is not None and isinstance(data, torch.Tensor):
        t = data
        if not t.is_contiguous():
            if writable:
                raise ValueError("output tensor must be contiguous")
            t = t.contiguous()
        kind = L.CB_MEM_DEVICE if t.is_cuda else L.CB_MEM_HOST
        dev = t.device.index if t.is_cuda else -1
        return t.data_ptr(), t.numel() * t.element_size(), kind, dev, t
    if isinstance(data, (bytes, bytearray, memoryview)) and not writable:
        a = np.frombuffer(data, dtype=np.uint8)
    else:
        a = np.asarray(data)
        if a.dtype != np.uint8:
            if writable:
                a = a.view(np.uint8) if a.flags.c_contiguous else a
            else:
                # pybind11 array_t<uint8_t> force-casts by value (bindings.cpp:152-155)
                a = a.astype(np.uint8)
        if not a.flags.c_contiguous:
            if writable:
                raise ValueError("output array must be C-contiguous")
            a = np.ascontiguousarray(a)
        if writable and not a.flags.writeable:
            raise ValueError("output array is read-only")
    return a.ctypes.data, a.nbytes, L.CB_MEM_HOST, -1, a


def _ptr(a: np.ndarray | None):
    return None if a is None else C.c_void_p(a.ctypes.data)


# ------------------------------------------------------------------- native

class _Native:
    """Owns one cb_store (one GPU of this process)."""

    def __init__(self, cfg: L.cb_config):
        lib = _native_lib()
        h = C.c_void_p()
        rc = lib.cb_create(C.byref(cfg), C.byref(h))
        if rc:
            raise CascadeError(rc, lib.cb_last_error(None).decode(errors="replace"))
        self.lib = lib
        self.h = h
        self.device = cfg.device  # calls on one store are serialised by the library's own mutex

    def _check(self, rc: int):
        if rc:
            raise CascadeError(rc, self.lib.cb_last_error(self.h).decode(errors="replace"))

    def stream_ptr(self, kind: int):
        if kind == L.CB_MEM_DEVICE and torch is not None and torch.cuda.is_available():
            return C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        return None

    def hash(self, ptrs: np.ndarray, sizes: np.ndarray, kind: int) -> np.ndarray:
        n = len(ptrs)
        dig = np.empty((n, 32), np.uint8)
        if n:
            self._check(self.lib.cb_hash_batch(self.h, _ptr(ptrs), _ptr(sizes), n, kind, _ptr(dig),
                                               self.stream_ptr(kind)))
        return dig

    def put(self, ptrs, sizes, kind, keys_in=None, prefix=None):
        n = len(ptrs)
        keys = np.empty((n, 16), np.uint8)
        status = np.empty(n, np.uint8)
        # called even for n == 0: in a DHT every rank takes part in each batch
        self._check(self.lib.cb_put_batch(self.h, _ptr(ptrs), _ptr(sizes), _ptr(prefix), _ptr(keys_in), n,
                                          kind, _ptr(keys), _ptr(status), self.stream_ptr(kind)))
        return keys, status

    def get(self, keys, outs, caps, kind):
        n = len(keys)
        sizes = np.zeros(n, np.uint64)
        found = np.zeros(n, np.uint8)
        self._check(self.lib.cb_get_batch(self.h, _ptr(keys), n, _ptr(outs), _ptr(caps), kind,
                                          _ptr(sizes), _ptr(found), self.stream_ptr(kind)))
        return sizes, found

    def put_async(self, ptrs, sizes, kind, keys_out, status_out, keys_in=None, prefix=None) -> int:
        t = C.c_uint64(0)
        self._check(self.lib.cb_put_batch_async(self.h, _ptr(ptrs), _ptr(sizes), _ptr(prefix), _ptr(keys_in),
                                                len(ptrs), kind, _ptr(keys_out), _ptr(status_out), C.byref(t),
                                                self.stream_ptr(kind)))
        return t.value

    def put_wait(self, ticket: int = 0) -> int:
        placed = C.c_uint64(0)
        self._check(self.lib.cb_put_wait(self.h, int(ticket), C.byref(placed)))
        return placed.value

    def put_placed(self) -> int:
        placed = C.c_uint64(0)
        self._check(self.lib.cb_put_placed(self.h, C.byref(placed)))
        return placed.value

    def get_async(self, keys, outs, caps):
        n = len(keys)
        sizes = np.zeros(n, np.uint64)
        found = np.zeros(n, np.uint8)
        self._check(self.lib.cb_get_batch_async(self.h, _ptr(keys), n, _ptr(outs), _ptr(caps), _ptr(sizes),
                                                _ptr(found), self.stream_ptr(L.CB_MEM_DEVICE)))
        return sizes, found

    def kv_compress(self, srcs, sizes, dsts):
        self._check(self.lib.cb_kv_compress_batch(self.h, _ptr(srcs), _ptr(sizes), _ptr(dsts), len(srcs),
                                                  self.stream_ptr(L.CB_MEM_DEVICE)))

    def kv_decompress(self, srcs, comp_sizes, orig_sizes, dsts) -> np.ndarray:
        ok = np.zeros(len(srcs), np.uint8)
        self._check(self.lib.cb_kv_decompress_batch(self.h, _ptr(srcs), _ptr(comp_sizes), _ptr(orig_sizes),
                                                    _ptr(dsts), len(srcs), _ptr(ok),
                                                    self.stream_ptr(L.CB_MEM_DEVICE)))
        return ok

    def contains(self, keys) -> np.ndarray:
        n = len(keys)
        found = np.zeros(n, np.uint8)
        self._check(self.lib.cb_contains_batch(self.h, _ptr(keys), n, _ptr(found)))
        return found

    def locate(self, key: bytes):
        loc = L.cb_location()
        found = C.c_int32(0)
        k = np.frombuffer(key, np.uint8).copy()
        self._check(self.lib.cb_locate(self.h, _ptr(k), C.byref(loc), C.byref(found)))
        return loc if found.value else None

    def stats(self) -> L.cb_stats:
        st = L.cb_stats()
        self._check(self.lib.cb_get_stats(self.h, C.byref(st)))
        return st

    def evict(self, nbytes: int) -> int:
        out = C.c_uint64(0)
        self._check(self.lib.cb_evict(self.h, nbytes, C.byref(out)))
        return out.value

    def clear(self):
        self._check(self.lib.cb_clear(self.h))

    def sync(self):
        self._check(self.lib.cb_sync(self.h))

    def close(self):
        if self.h:
            self.lib.cb_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------ block ID hash

_hashers: dict[int, _Native] = {}


def _hasher(device: int) -> _Native:
    with _cache_lock:  # one helper store per device, also when threads race here
        h = _hashers.get(device)
        if h is None:
            cfg = L.cb_config()
            _native_lib().cb_config_init(C.byref(cfg))
            cfg.gpu_capacity_bytes = 0
            cfg.dram_capacity_bytes = 0
            cfg.index_log2 = 8
            cfg.device = device
            h = _hashers[device] = _Native(cfg)
        return h


def _default_device() -> int:
    if torch is not None and torch.cuda.is_available():
        return torch.cuda.current_device()
    return int(os.environ.get("LOCAL_RANK", "0"))


def compute_block_id(data) -> str:
    """SHA-256 of the block on the GPU -> first 16 bytes as 32 hex chars.

    Same result as cascade_core.cpp:47-58 / bindings.cpp:176-179. One block
    is one serial SHA-256 chain, so a single call is latency bound; hash many
    blocks at once with :func:`compute_block_ids`.
    """
    return compute_block_ids([data])[0]


def compute_block_ids(blocks: Sequence) -> list[str]:
    """Block IDs of many blocks in one GPU launch (one chain per block)."""
    views = [_block_view(b) for b in blocks]
    if not views:
        return []
    kinds = {v[2] for v in views}
    if len(kinds) != 1:
        raise ValueError("blocks must be all host or all device buffers")
    kind = kinds.pop()
    dev = views[0][3] if kind == L.CB_MEM_DEVICE else _default_device()
    h = _hasher(dev)
    ptrs = np.array([v[0] for v in views], np.uint64)
    sizes = np.array([v[1] for v in views], np.uint64)
    dig = h.hash(ptrs, sizes, kind)
    return [row[:16].tobytes().hex() for row in dig]


# ----------------------------------------------------------- KV compressor

class KVCompressor:
    """KVCompressor (include/cascade.hpp:397-418, src/cascade_core.cpp:
    908-967) on the GPU: INT8 compression of fp16 KV blocks into
    [f32 scale][i8 zero_point][3 zero bytes][size/2 x i8], the format of
    DRAM-tier blocks under ``kv_compression``. Blocks are contiguous CUDA
    uint8 tensors of one device; the batched forms take one launch pair per
    batch."""

    _stores: dict = {}

    @staticmethod
    def compressed_size(original_size: int) -> int:
        return 8 + int(original_size) // 2

    @staticmethod
    def original_size(compressed_size: int) -> int:
        return (int(compressed_size) - 8) * 2

    @classmethod
    def _native(cls, device: int) -> "_Native":
        with _cache_lock:
            n = cls._stores.get(device)
            if n is None:
                c = L.cb_config()
                _native_lib().cb_config_init(C.byref(c))
                c.gpu_capacity_bytes = 0  # no pool: the store only lends its scratch buffers and stream
                c.dram_capacity_bytes = 0
                c.index_log2 = 4
                c.device = device
                n = cls._stores[device] = _Native(c)
            return n

    @staticmethod
    def _check_blocks(blocks) -> int:
        dev = None
        for b in blocks:
            if not (torch is not None and isinstance(b, torch.Tensor) and b.is_cuda and b.dtype == torch.uint8
                    and b.is_contiguous()):
                raise TypeError("KVCompressor works on contiguous CUDA uint8 tensors")
            if dev is not None and b.device.index != dev:
                raise ValueError("all blocks of a batch must be on one device")
            dev = b.device.index
        return 0 if dev is None else dev

    @classmethod
    def compress_batch(cls, blocks):
        dev = cls._check_blocks(blocks)
        for b in blocks:
            if b.numel() < 2:
                raise ValueError("compression needs at least one 16-bit value")
        outs = [torch.empty(cls.compressed_size(b.numel()), dtype=torch.uint8, device=b.device) for b in blocks]
        if blocks:
            cls._native(dev).kv_compress(np.array([b.data_ptr() for b in blocks], np.uint64),
                                         np.array([b.numel() for b in blocks], np.uint64),
                                         np.array([o.data_ptr() for o in outs], np.uint64))
        return outs

    @classmethod
    def compress(cls, block):
        return cls.compress_batch([block])[0]

    @classmethod
    def decompress_batch(cls, packed, original_sizes):
        """Returns one tensor of (original_size/2)*2 bytes per block, or None
        where the packed block is too short (the reference's false)."""
        dev = cls._check_blocks(packed)
        outs = [torch.empty(int(s) // 2 * 2, dtype=torch.uint8, device=p.device)
                for p, s in zip(packed, original_sizes)]
        if not packed:
            return []
        ok = cls._native(dev).kv_decompress(np.array([p.data_ptr() for p in packed], np.uint64),
                                            np.array([p.numel() for p in packed], np.uint64),
                                            np.array([int(s) for s in original_sizes], np.uint64),
                                            np.array([o.data_ptr() for o in outs], np.uint64))
        return [o if k else None for o, k in zip(outs, ok)]

    @classmethod
    def decompress(cls, packed, original_size: int):
        return cls.decompress_batch([packed], [original_size])[0]


# ------------------------------------------------------------------- config

class DistributedConfig:
    """Fields of DistributedConfig (include/cascade_distributed.hpp:186-213),
    plus B200 fields (device, promote_on_hit, copy_engine, index_log2,
    staging_bytes)."""

    def __init__(self):
        self.gpu_capacity_per_device = 32 * 1024 ** 3
        self.dram_capacity = 64 * 1024 ** 3
        self.num_gpus_per_node = 4
        self.staging_buffer_size = 16 * 1024 * 1024
        self.num_staging_buffers = 32
        self.semantic_eviction = True
        self.prefix_replication = True
        self.dedup_enabled = True
        self.locality_aware = True
        self.promotion_threshold = 3
        self.kv_compression = False
        self.sync_metadata = False
        self.lustre_path = ""
        self.aggregated_lustre = True
        self.agg_file_size = 256 * 1024 * 1024
        # B200 additions
        self.device = None            # default: LOCAL_RANK / current CUDA device
        # DRAM-tier get hits back to HBM: None = DistributedStore::get's rule
        # (locality-gated, distributed_backend.cpp:721-724: a store's own DRAM
        # hits are local accesses and are never promoted), True = every hit
        # (CascadeStore::get's rule, cascade_core.cpp:1303-1307), False = never
        self.promote_on_hit = None
        self.copy_engine = 0          # 0 auto (TMA bulk), 1 TMA bulk, 2 LSU vectors
        self.index_log2 = 16
        self.staging_bytes = 1 << 30  # device staging for host-memory callers
        self.dht = None               # None: shard over all ranks when WORLD_SIZE > 1
        self.replica_bytes = 0        # DHT: HBM for replicas of hot remote blocks (0 = auto)
        self.profile = False          # time every kernel with CUDA events (stats *_ns)
        self.hash_lanes = 32          # reserved (the SHA-256 kernel runs 32 chains per warp)
        self.collective_timeout_ms = 0  # DHT: abort a collective after this long (0 = 600 s)
        self.pipeline_blocks = 0      # pipelined puts: blocks hashing at once (0 = 65536)
        self.hash_sms = 0             # pipelined puts: SMs their SHA-256 may use (0 = all; DHT: all but 8)


class CascadeConfig:
    """Fields of CascadeConfig (include/cascade.hpp:47-82). The SHM tier maps
    to the pinned DRAM arena; Lustre and prefetch are out of scope."""

    def __init__(self):
        self.gpu_capacity_bytes = 32 * 1024 ** 3
        self.gpu_device_id = 0
        self.use_gpu = True
        self.shm_capacity_bytes = 64 * 1024 ** 3
        self.shm_path = "/dev/shm/cascade"
        self.lustre_path = "/pscratch/sd/s/sgkim/cascade_store"
        self.lustre_stripe_size = 1024 * 1024
        self.lustre_stripe_count = 16
        self.dedup_enabled = True
        self.compression_enabled = True
        self.num_io_threads = 8
        self.semantic_eviction = True
        self.promotion_enabled = True
        self.prefetch_enabled = True
        self.prefetch_threads = 2
        self.prefetch_queue_size = 64
        self.kv_compression = False
        self.aggregated_lustre = False
        self.agg_file_size = 256 * 1024 * 1024
        self.copy_engine = 0
        self.index_log2 = 16
        self.staging_bytes = 1 << 30
        self.pipeline_blocks = 0      # pipelined puts: blocks hashing at once (0 = 65536)
        self.hash_sms = 0             # pipelined puts: SMs their SHA-256 may use (0 = all; DHT: all but 8)


class _Record:
    _fields: Sequence[str] = ()

    def __init__(self, **kw):
        for f in self._fields:
            setattr(self, f, kw.get(f, 0))


class DistributedStats(_Record):
    """DistributedStore::Stats (include/cascade_distributed.hpp:386-409)."""
    _fields = L.STATS_FIELDS

    def __repr__(self):  # same shape as bindings.cpp:137-146
        hits = (self.local_gpu_hits + self.local_dram_hits + self.remote_gpu_hits
                + self.remote_dram_hits + self.lustre_hits)
        return (f"DistributedStats(gpu={self.local_gpu_used // (1024 * 1024)}MB"
                f", dram={self.local_dram_used // (1024 * 1024)}MB, hits={hits}"
                f", dedup={self.dedup_hits}, promotions={self.promotions_to_local}"
                f", prefix={self.prefix_blocks})")


class CascadeStats(_Record):
    """CascadeStore::Stats (include/cascade.hpp:501-519)."""
    _fields = ["gpu_used", "shm_used", "gpu_hits", "shm_hits", "lustre_hits", "misses",
               "dedup_hits", "gpu_evictions", "shm_evictions", "promotions_to_gpu",
               "promotions_to_shm", "prefetch_completed", "compression_savings_bytes",
               "shm_puts", "lustre_puts"]

    def __repr__(self):  # same shape as bindings.cpp:56-65
        return (f"CascadeStats(gpu={self.gpu_used // (1024 * 1024)}MB"
                f", shm={self.shm_used // (1024 * 1024)}MB"
                f", hits={self.gpu_hits + self.shm_hits + self.lustre_hits}"
                f", dedup={self.dedup_hits}"
                f", evictions={self.gpu_evictions + self.shm_evictions}"
                f", promotions={self.promotions_to_gpu + self.promotions_to_shm}"
                f", prefetch={self.prefetch_completed}"
                f", compression_saved={self.compression_savings_bytes // (1024 * 1024)}MB)")


class BlockLocation(_Record):
    """BlockLocation (include/cascade_distributed.hpp:62-80)."""
    _fields = ["node_id", "gpu_id", "offset", "size", "is_gpu", "is_prefix"]

    def __repr__(self):
        return (f"BlockLocation(node_id={self.node_id}, gpu_id={self.gpu_id}, offset={self.offset}, "
                f"size={self.size}, is_gpu={self.is_gpu}, is_prefix={self.is_prefix})")


# -------------------------------------------------------------------- store

class _PoolSpan:
    """A span of the HBM pool exposed through __cuda_array_interface__ so
    that torch can alias it without a copy."""

    def __init__(self, addr: int, size: int):
        self.__cuda_array_interface__ = {"shape": (int(size),), "typestr": "|u1", "data": (int(addr), False),
                                         "version": 3, "strides": None}


class _StoreBase:
    _miss_size_is_buffer_len = True

    def _init_native(self, cfg: L.cb_config):
        self._n = _Native(cfg)
        self._device = cfg.device
        self._strkeys: dict[bytes, str] = {}
        # pipelined puts: ticket -> what the library reads or writes when the
        # batch is placed (inputs, output arrays), kept alive until then
        self._inflight: dict[int, tuple] = {}

    def _release_placed(self, placed: int | None = None):
        if not self._inflight:
            return
        if placed is None:
            placed = self._n.put_placed()
        for t in [t for t in self._inflight if t <= placed]:
            del self._inflight[t]

    # -- ids
    def _key(self, block_id: str) -> bytes:
        k = block_id_to_key(block_id)
        if not _HEX32.match(block_id):
            prev = self._strkeys.setdefault(k, block_id)
            if prev != block_id:
                raise CascadeError(L.CB_ERR_STATE, f"block id key collision: {prev!r} vs {block_id!r}")
        return k

    def _keys(self, ids: Iterable[str]) -> np.ndarray:
        ks = [self._key(i) for i in ids]
        return np.frombuffer(b"".join(ks), np.uint8).reshape(len(ks), 16).copy()

    def _check_device(self, views):
        kinds = {v[2] for v in views}
        if len(kinds) > 1:
            raise ValueError("a batch must be all host or all device buffers")
        kind = kinds.pop() if kinds else L.CB_MEM_HOST
        if kind == L.CB_MEM_DEVICE:
            for v in views:
                if v[3] != self._device:
                    raise ValueError(f"tensor on cuda:{v[3]} but store on cuda:{self._device}")
        return kind

    # -- single block API (bindings.cpp:152-161)
    def put(self, block_id: str, data, is_prefix: bool = False) -> bool:
        v = _block_view(data)
        kind = self._check_device([v])
        keys = self._keys([block_id])
        _, status = self._n.put(np.array([v[0]], np.uint64), np.array([v[1]], np.uint64), kind,
                                keys_in=keys, prefix=np.array([1 if is_prefix else 0], np.uint8))
        return int(status[0]) != L.CB_PUT_FAILED

    def get(self, block_id: str, out):
        v = _block_view(out, writable=True)
        kind = self._check_device([v])
        sizes, found = self._n.get(self._keys([block_id]), np.array([v[0]], np.uint64),
                                   np.array([v[1]], np.uint64), kind)
        if int(found[0]) & 0x0F == L.CB_FOUND_MISS:
            # DistributedStore binding reports len(out) on a miss
            # (bindings.cpp:158-160); CascadeStore's reports 0 (:77-80).
            return (False, v[1] if self._miss_size_is_buffer_len else 0)
        return (True, int(sizes[0]))

    def contains(self, block_id: str) -> bool:
        return bool(self._n.contains(self._keys([block_id]))[0])

    # -- batch API
    def batch_put(self, blocks: Sequence, is_prefix: Sequence[bool] | None = None,
                  ids: Sequence[str] | None = None, return_status: bool = False):
        """Store many blocks with one GPU pass.

        ``ids=None``: every block is hashed on the GPU and stored under its
        content ID (the IDs ``compute_block_id`` returns). With ``ids``: the
        caller's IDs, exactly DistributedStore::put_batch semantics
        (distributed_backend.cpp:813-841). Dedup is sequential in batch
        order. Returns the IDs (and, with ``return_status``, per-block
        CB_PUT_* codes: 0 stored, 1 dedup hit, 2 failed).
        """
        views = [_block_view(b) for b in blocks]
        kind = self._check_device(views)
        ptrs = np.array([v[0] for v in views], np.uint64)
        sizes = np.array([v[1] for v in views], np.uint64)
        keys_in = self._keys(ids) if ids is not None else None
        prefix = None if is_prefix is None else np.array([1 if p else 0 for p in is_prefix], np.uint8)
        keys, status = self._n.put(ptrs, sizes, kind, keys_in=keys_in, prefix=prefix)
        out_ids = list(ids) if ids is not None else [k.tobytes().hex() for k in keys]
        return (out_ids, status.tolist()) if return_status else out_ids

    def batch_get(self, ids: Sequence[str], outs: Sequence):
        """Fetch many blocks into ``outs`` (one buffer per ID) with one GPU
        pass. Returns ``(found: list[bool], sizes: list[int])``; a found block
        whose buffer is too small reports its size and is not written."""
        views = [_block_view(o, writable=True) for o in outs]
        if len(views) != len(ids):
            raise ValueError("ids and outs differ in length")
        kind = self._check_device(views)
        sizes, found = self._n.get(self._keys(ids), np.array([v[0] for v in views], np.uint64),
                                   np.array([v[1] for v in views], np.uint64), kind)
        return [(int(f) & 0x0F) != L.CB_FOUND_MISS for f in found], [int(s) for s in sizes]

    # -- raw pointer API (no per-block Python objects; used by bench.py)
    def put_ptrs(self, ptrs: np.ndarray, sizes: np.ndarray, device_memory: bool,
                 keys: np.ndarray | None = None, prefix: np.ndarray | None = None):
        kind = L.CB_MEM_DEVICE if device_memory else L.CB_MEM_HOST
        return self._n.put(np.ascontiguousarray(ptrs, np.uint64), np.ascontiguousarray(sizes, np.uint64),
                           kind, keys_in=keys, prefix=prefix)

    def put_ptrs_async(self, ptrs: np.ndarray, sizes: np.ndarray, keys_out: np.ndarray | None = None,
                       status_out: np.ndarray | None = None, prefix: np.ndarray | None = None,
                       keys: np.ndarray | None = None, device_memory: bool = True) -> int:
        """Pipelined put of one batch of device blocks (cb_put_batch_async):
        launches the batch's SHA-256 and returns a ticket at once; batches
        are placed in ticket order (same IDs, statuses and dedup counts as
        put_ptrs one batch after the other). ``keys_out`` ((n, 16) uint8) and
        ``status_out`` ((n,) uint8), when given, are filled when the batch
        is placed: after ``wait_puts`` covering the ticket, or any other
        call of the store. The blocks must stay unchanged until then."""
        ptrs = np.ascontiguousarray(ptrs, np.uint64)
        sizes = np.ascontiguousarray(sizes, np.uint64)
        for a, shape in ((keys_out, (len(ptrs), 16)), (status_out, (len(ptrs),))):
            if a is not None and (a.dtype != np.uint8 or a.shape != shape or not a.flags.c_contiguous
                                  or not a.flags.writeable):
                raise ValueError(f"output must be a writable C-contiguous uint8 array of shape {shape}")
        prefix = None if prefix is None else np.ascontiguousarray(prefix, np.uint8)
        keys = None if keys is None else np.ascontiguousarray(keys, np.uint8)
        kind = L.CB_MEM_DEVICE if device_memory else L.CB_MEM_HOST
        t = self._n.put_async(ptrs, sizes, kind, keys_out, status_out, keys_in=keys, prefix=prefix)
        self._inflight[t] = (keys_out, status_out)
        self._release_placed()
        return t

    def wait_puts(self, ticket: int = 0) -> int:
        """Places every pipelined batch up to ``ticket`` (0: all) and waits
        for their device work. Returns the highest ticket placed."""
        placed = self._n.put_wait(ticket)
        self._release_placed(placed)
        return placed

    def batch_put_async(self, blocks: Sequence, is_prefix: Sequence[bool] | None = None,
                        ids: Sequence[str] | None = None) -> "PutFuture":
        """Pipelined ``batch_put`` of CUDA tensors: returns a future at once;
        ``future.result()`` gives the IDs (and statuses) once the batch is
        placed. Batches are placed in submission order, so IDs, statuses and
        dedup counts are those of ``batch_put`` called batch after batch."""
        views = [_block_view(b) for b in blocks]
        kind = self._check_device(views)
        n = len(views)
        ptrs = np.array([v[0] for v in views], np.uint64)
        sizes = np.array([v[1] for v in views], np.uint64)
        keys_in = self._keys(ids) if ids is not None else None
        prefix = None if is_prefix is None else np.array([1 if p else 0 for p in is_prefix], np.uint8)
        keys = np.empty((n, 16), np.uint8)
        status = np.empty(n, np.uint8)
        t = self._n.put_async(ptrs, sizes, kind, keys, status, keys_in=keys_in, prefix=prefix)
        self._inflight[t] = (keys, status, views)
        self._release_placed()
        return PutFuture(self, t, keys, status, None if ids is None else list(ids))

    def get_ptrs_async(self, keys: np.ndarray, outs: np.ndarray, caps: np.ndarray):
        """Stream-ordered get into device buffers (cb_get_batch_async):
        returns (sizes, found) final at once; the bytes land in order on the
        current CUDA stream."""
        return self._n.get_async(np.ascontiguousarray(keys, np.uint8), np.ascontiguousarray(outs, np.uint64),
                                 np.ascontiguousarray(caps, np.uint64))

    def batch_get_async(self, ids: Sequence[str], outs: Sequence):
        """``batch_get`` into CUDA tensors, stream-ordered: (found, sizes)
        are final when it returns, the bytes land in order on the current
        CUDA stream (read them on that stream)."""
        views = [_block_view(o, writable=True) for o in outs]
        if len(views) != len(ids):
            raise ValueError("ids and outs differ in length")
        if self._check_device(views) != L.CB_MEM_DEVICE:
            raise ValueError("batch_get_async writes CUDA tensors; use batch_get for host buffers")
        sizes, found = self._n.get_async(self._keys(ids), np.array([v[0] for v in views], np.uint64),
                                         np.array([v[1] for v in views], np.uint64))
        return [(int(f) & 0x0F) != L.CB_FOUND_MISS for f in found], [int(s) for s in sizes]

    def get_views(self, ids: Sequence[str]):
        """Zero-copy batch_get: one CUDA uint8 tensor per ID that aliases the
        block where it sits in this store's HBM pool (no copy; for HBM hits no
        kernel either), or None for a miss (and for a DRAM-tier block that
        could not be promoted). Each view pins its block (never evicted or
        moved) until ``release_views`` is called for that ID. Views are
        read-only by contract: a block is its content hash, and they alias
        memory the store owns: drop them before ``close()``."""
        keys = self._keys(ids)
        n = len(keys)
        addrs = np.zeros(n, np.uint64)
        sizes = np.zeros(n, np.uint64)
        found = np.zeros(n, np.uint8)
        if n:
            self._n._check(self._n.lib.cb_get_views(self._n.h, _ptr(keys), n, _ptr(addrs), _ptr(sizes), _ptr(found),
                                                    self._n.stream_ptr(L.CB_MEM_DEVICE)))
        out = []
        for a, s, f in zip(addrs.tolist(), sizes.tolist(), found.tolist()):
            if (f & 0x0F) != L.CB_FOUND_LOCAL_HBM:
                out.append(None)
            elif s == 0:
                out.append(torch.empty(0, dtype=torch.uint8, device=f"cuda:{self._device}"))
            else:
                out.append(torch.as_tensor(_PoolSpan(a, s), device=f"cuda:{self._device}"))
        return out

    def release_views(self, ids: Sequence[str]):
        """Drops one view pin of each ID (views obtained by ``get_views``)."""
        keys = self._keys(ids)
        if len(keys):
            self._n._check(self._n.lib.cb_release_views(self._n.h, _ptr(keys), len(keys)))

    def get_ptrs(self, keys: np.ndarray, outs: np.ndarray, caps: np.ndarray, device_memory: bool):
        kind = L.CB_MEM_DEVICE if device_memory else L.CB_MEM_HOST
        return self._n.get(np.ascontiguousarray(keys, np.uint8), np.ascontiguousarray(outs, np.uint64),
                           np.ascontiguousarray(caps, np.uint64), kind)

    def evict(self, nbytes: int) -> int:
        """Demote LRU HBM blocks (prefix blocks last) to the DRAM tier."""
        return self._n.evict(int(nbytes))

    def clear(self):
        self._n.clear()
        self._strkeys.clear()
        self._inflight.clear()  # placed or dropped by the clear

    def flush(self):
        self._n.sync()

    def close(self):
        self._n.close()


class PutFuture:
    """Result of ``batch_put_async``: ``result()`` waits until the batch is
    placed and returns its IDs (with ``return_status``, also the per-block
    CB_PUT_* codes)."""

    def __init__(self, store: "_StoreBase", ticket: int, keys: np.ndarray, status: np.ndarray, ids):
        self._store, self.ticket, self._keys, self._status, self._ids = store, ticket, keys, status, ids

    def done(self) -> bool:
        return self._store._n.put_placed() >= self.ticket

    def result(self, return_status: bool = False):
        if not self.done():
            self._store.wait_puts(self.ticket)
        out = self._ids if self._ids is not None else [k.tobytes().hex() for k in self._keys]
        return (out, self._status.tolist()) if return_status else out


def _resolve_device(dev) -> int:
    if dev is not None:
        return int(dev)
    if "LOCAL_RANK" in os.environ:
        return int(os.environ["LOCAL_RANK"])
    return _default_device()


_warned: set[str] = set()


def _warn_once(msg: str):
    if msg not in _warned:
        _warned.add(msg)
        warnings.warn(msg, stacklevel=3)


class DistributedStore(_StoreBase):
    """Drop-in for cascade_cpp.DistributedStore (bindings.cpp:150-170).

    One process per GPU. With WORLD_SIZE > 1 (torch.distributed initialised,
    or RANK/WORLD_SIZE in the environment) the stores of all ranks form one
    hash-sharded DHT over NVLink: owner = first 8 ID bytes (big-endian) mod
    world; lookups travel by NCCL all-to-all and payloads by peer loads.
    """

    _miss_size_is_buffer_len = True

    def __init__(self, cfg: DistributedConfig | None = None):
        cfg = cfg or DistributedConfig()
        if cfg.lustre_path:
            _warn_once("the Lustre tier is out of scope; lustre_path ignored")
        c = L.cb_config()
        _native_lib().cb_config_init(C.byref(c))
        c.gpu_capacity_bytes = int(cfg.gpu_capacity_per_device)
        c.dram_capacity_bytes = int(cfg.dram_capacity)
        c.device = _resolve_device(cfg.device)
        c.dedup_enabled = 1 if cfg.dedup_enabled else 0
        c.semantic_eviction = 1 if cfg.semantic_eviction else 0
        c.promote_on_hit = 0 if cfg.promote_on_hit is False else 1
        c.promotion_rule = L.CB_PROMOTE_EVERY_HIT if cfg.promote_on_hit is True else L.CB_PROMOTE_LOCALITY
        c.index_log2 = int(cfg.index_log2)
        c.copy_engine = int(cfg.copy_engine)
        c.staging_bytes = int(cfg.staging_bytes)
        c.profile = 1 if cfg.profile else 0
        c.hash_lanes = int(cfg.hash_lanes)
        c.locality_aware = 1 if cfg.locality_aware else 0
        c.promotion_threshold = int(cfg.promotion_threshold)
        c.replica_bytes = int(cfg.replica_bytes)
        c.kv_compression = 1 if cfg.kv_compression else 0
        c.prefix_replication = 1 if cfg.prefix_replication else 0
        c.collective_timeout_ms = int(cfg.collective_timeout_ms)
        c.pipeline_blocks = int(cfg.pipeline_blocks)
        c.hash_sms = int(getattr(cfg, "hash_sms", 0))
        self._init_native(c)
        self._rank, self._world = 0, 1
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if torch is not None and torch.distributed.is_available() and torch.distributed.is_initialized():
            world = torch.distributed.get_world_size()
        if world > 1 and cfg.dht is not False:
            self._attach_dht()

    def _attach_dht(self):
        import torch.distributed as dist
        # The DHT's own collectives are a few bytes; keep NCCL off NVLink
        # multicast (NVLS) so a rank that dies cannot leave a bound multicast
        # object behind on the other GPUs.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        if not dist.is_initialized():
            dist.init_process_group(backend="gloo", init_method="env://")
        rank, world = dist.get_rank(), dist.get_world_size()
        uid = np.zeros(L.CB_UID_BYTES, np.uint8)
        if rank == 0:
            self._n._check(self._n.lib.cb_dht_unique_id(_ptr(uid)))
        obj = [uid.tobytes()]
        dist.broadcast_object_list(obj, src=0)
        uid = np.frombuffer(obj[0], np.uint8).copy()
        self._n._check(self._n.lib.cb_dht_attach(self._n.h, rank, world, _ptr(uid)))
        self._rank, self._world = rank, world

    @property
    def rank(self) -> int:
        return self._rank

    @property
    def world_size(self) -> int:
        return self._world

    def locate(self, block_id: str):
        loc = self._n.locate(self._key(block_id))
        if loc is None:
            return None
        return BlockLocation(node_id=loc.node_id, gpu_id=loc.gpu_id, offset=loc.offset, size=loc.size,
                             is_gpu=bool(loc.is_gpu), is_prefix=bool(loc.is_prefix))

    def get_stats(self) -> DistributedStats:
        st = self._n.stats()
        return DistributedStats(**{f: getattr(st, f) for f in L.STATS_FIELDS})

    def sync_metadata(self):
        """DistributedStore::sync_metadata (distributed_backend.cpp:1323-1382).
        Block locations need no replication (every block has one owner rank
        that answers lookups); the prefix registry is merged cluster-wide and,
        with ``prefix_replication``, every rank copies the other ranks' prefix
        blocks into its local HBM (sync_prefix_registry /
        broadcast_prefix_data, :958-1217). Collective; ends with a barrier."""
        self._n.sync()
        self._n._check(self._n.lib.cb_sync_metadata(self._n.h))
        if self._world > 1:
            self._n._check(self._n.lib.cb_dht_barrier(self._n.h))

    def barrier(self):
        self._n.sync()
        if self._world > 1:
            self._n._check(self._n.lib.cb_dht_barrier(self._n.h))


class CascadeStore(_StoreBase):
    """Drop-in for cascade_cpp.CascadeStore (bindings.cpp:71-85): HBM tier
    plus the pinned DRAM arena standing in for the SHM tier."""

    _miss_size_is_buffer_len = False

    def __init__(self, cfg: CascadeConfig | None = None):
        cfg = cfg or CascadeConfig()
        c = L.cb_config()
        _native_lib().cb_config_init(C.byref(c))
        c.gpu_capacity_bytes = int(cfg.gpu_capacity_bytes) if cfg.use_gpu else 0
        c.dram_capacity_bytes = int(cfg.shm_capacity_bytes)
        c.device = int(cfg.gpu_device_id)
        c.dedup_enabled = 1 if cfg.dedup_enabled else 0
        c.semantic_eviction = 1 if cfg.semantic_eviction else 0
        c.promote_on_hit = 1 if cfg.promotion_enabled else 0
        c.promotion_rule = L.CB_PROMOTE_EVERY_HIT  # CascadeStore::get promotes every SHM hit
        c.index_log2 = int(cfg.index_log2)
        c.copy_engine = int(cfg.copy_engine)
        c.staging_bytes = int(cfg.staging_bytes)
        c.kv_compression = 1 if cfg.kv_compression else 0
        c.pipeline_blocks = int(cfg.pipeline_blocks)
        c.hash_sms = int(getattr(cfg, "hash_sms", 0))
        self._init_native(c)

    def get_stats(self) -> CascadeStats:
        st = self._n.stats()
        return CascadeStats(gpu_used=st.local_gpu_used, shm_used=st.local_dram_used,
                            gpu_hits=st.local_gpu_hits, shm_hits=st.local_dram_hits,
                            lustre_hits=0, misses=st.misses, dedup_hits=st.dedup_hits,
                            gpu_evictions=st.gpu_evictions, shm_evictions=st.dram_evictions,
                            promotions_to_gpu=st.promotions_to_local, promotions_to_shm=0,
                            prefetch_completed=0, compression_savings_bytes=st.compression_savings, shm_puts=0,
                            lustre_puts=0)
