"""ORACLE — test infrastructure only (see oracle/__init__.py).

Sequential CPU restatement of the store semantics on the Cascade hot path:

* ``block_id`` / ``block_ids``: compute_block_id
  (cascade_Code/cpp/src/cascade_core.cpp:47-58) through the plain-C FIPS
  180-4 restatement in ``sha256_oracle.c`` (ctypes).
* ``SequentialStore``: DistributedStore::put (src/distributed_backend.cpp:
  601-692; dedup check :604-608), put_batch (:813-841, sequential), get
  (:698-795, bytes only), contains (:797-802), with the pybind return
  conventions of python/bindings.cpp:152-161.
* ``TierModel``: the prefix-protected demotion rule of
  GPUBackend::evict_lru_semantic / evict_for_space (src/gpu_backend.cu:
  482-537) and DistributedDRAMBackend::evict_for_space
  (src/distributed_backend.cpp:240-284), with exact LRU order.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from collections import OrderedDict

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            subprocess.run(["make", "-C", _HERE, "all"], check=True, capture_output=True)
        lib = C.CDLL(_LIB_PATH)
        lib.oracle_sha256.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p]
        lib.oracle_sha256.restype = None
        lib.oracle_sha256_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]
        lib.oracle_sha256_batch.restype = None
        lib.oracle_sha256_constants.argtypes = [C.c_void_p, C.c_void_p]
        lib.oracle_sha256_constants.restype = None
        _lib = lib
    return _lib


def sha256(data) -> bytes:
    a = np.ascontiguousarray(np.frombuffer(bytes(data), np.uint8) if isinstance(data, (bytes, bytearray))
                             else np.asarray(data, np.uint8))
    out = np.empty(32, np.uint8)
    _load().oracle_sha256(C.c_void_p(a.ctypes.data if a.size else 0), a.size, C.c_void_p(out.ctypes.data))
    return out.tobytes()


def sha256_batch(packed: np.ndarray, offsets, sizes) -> np.ndarray:
    packed = np.ascontiguousarray(packed, np.uint8)
    off = np.ascontiguousarray(offsets, np.uint64)
    sz = np.ascontiguousarray(sizes, np.uint64)
    out = np.empty((len(off), 32), np.uint8)
    if len(off):
        _load().oracle_sha256_batch(C.c_void_p(packed.ctypes.data), C.c_void_p(off.ctypes.data),
                                    C.c_void_p(sz.ctypes.data), len(off), C.c_void_p(out.ctypes.data))
    return out


def block_id(data) -> str:
    return sha256(data)[:16].hex()


def constants() -> tuple[list[int], list[int]]:
    k = np.empty(64, np.uint32)
    h = np.empty(8, np.uint32)
    _load().oracle_sha256_constants(C.c_void_p(k.ctypes.data), C.c_void_p(h.ctypes.data))
    return [int(x) for x in k], [int(x) for x in h]


class SequentialStore:
    """Bytes-level model of one rank's DistributedStore."""

    def __init__(self, dedup_enabled: bool = True):
        self.dedup_enabled = dedup_enabled
        self.blocks: dict[str, bytes] = {}
        self.prefix: set[str] = set()
        self.dedup_hits = 0
        self.dedup_bytes_saved = 0
        self.misses = 0

    def put(self, block_id: str, data: bytes, is_prefix: bool = False) -> tuple[bool, int]:
        """Returns (stored_ok, status) with status 0 new, 1 dedup hit."""
        if block_id in self.blocks:
            if self.dedup_enabled:
                self.dedup_hits += 1
                self.dedup_bytes_saved += len(data)
            return True, 1
        self.blocks[block_id] = bytes(data)
        if is_prefix:
            self.prefix.add(block_id)
        return True, 0

    def put_batch(self, ids, datas, is_prefix=None) -> list[int]:
        flags = is_prefix or [False] * len(ids)
        return [self.put(i, d, p)[1] for i, d, p in zip(ids, datas, flags)]

    def get(self, block_id: str):
        d = self.blocks.get(block_id)
        if d is None:
            self.misses += 1
            return False, None
        return True, d

    def contains(self, block_id: str) -> bool:
        return block_id in self.blocks


class TierModel:
    """HBM/DRAM placement under the prefix-protected LRU demotion rule.

    Logical-capacity model (the reference checks ``used + size > capacity``,
    src/gpu_backend.cu:307); allocation fragmentation is not modelled, so use
    equal block sizes when comparing placements exactly.

    With ``compress`` (kv_compression) a block >= 64 B that enters DRAM is
    held as KVCompressor output, 8 + size/2 bytes
    (src/distributed_backend.cpp:611-620, :898-903), and its size becomes
    (size/2)*2, what a read returns (:712-719).
    """

    def __init__(self, hbm_cap: int, dram_cap: int, semantic: bool = True, compress: bool = False):
        self.hbm_cap, self.dram_cap, self.semantic = hbm_cap, dram_cap, semantic
        self.compress = compress
        self.hbm: OrderedDict[str, int] = OrderedDict()   # id -> size, last = MRU
        self.dram: OrderedDict[str, int] = OrderedDict()  # id -> bytes held in DRAM
        self.size: dict[str, int] = {}                    # id -> size a read returns
        self.prefix: set[str] = set()
        self.dropped: list[str] = []
        self.evictions = 0
        self.compression_savings = 0

    def _to_dram(self, k: str, size: int) -> int:
        """Bytes block k of `size` bytes occupies in DRAM (and its new size)."""
        if self.compress and size >= 64:
            self.size[k] = size // 2 * 2
            return 8 + size // 2
        self.size[k] = size
        return size

    def _victim_hbm(self):
        order = list(self.hbm.keys())
        if self.semantic:
            for k in order:
                if k not in self.prefix:
                    return k
        return order[0] if order else None

    def _room_dram(self, size: int) -> bool:
        if self.dram_cap == 0 or size > self.dram_cap:
            return False
        while sum(self.dram.values()) + size > self.dram_cap:
            cands = [k for k in self.dram if not (self.semantic and k in self.prefix)]
            if not cands:
                return False
            v = cands[0]
            del self.dram[v]
            self.dropped.append(v)
        return True

    def _demote_one(self) -> bool:
        v = self._victim_hbm()
        if v is None:
            return False
        size = self.hbm.pop(v)
        self.evictions += 1
        dsize = 8 + size // 2 if self.compress and size >= 64 else size
        if self._room_dram(dsize):
            self.dram[v] = self._to_dram(v, size)
            self.compression_savings += size - dsize
        else:
            self.dropped.append(v)
        return True

    def put(self, k: str, size: int, is_prefix: bool = False) -> str:
        if k in self.hbm or k in self.dram:
            return "dedup"
        if is_prefix:
            self.prefix.add(k)
        while sum(self.hbm.values()) + size > self.hbm_cap:
            if not self._demote_one():
                break
        if sum(self.hbm.values()) + size <= self.hbm_cap:
            self.hbm[k] = size
            self.size[k] = size
            return "hbm"
        dsize = 8 + size // 2 if self.compress and size >= 64 else size
        if self._room_dram(dsize):
            self.dram[k] = self._to_dram(k, size)
            self.compression_savings += size - dsize
            return "dram"
        return "failed"

    def touch(self, k: str):
        if k in self.hbm:
            self.hbm.move_to_end(k)
        elif k in self.dram:
            self.dram.move_to_end(k)

    def promote(self, k: str) -> bool:
        if k not in self.dram:
            return False
        size = self.size[k]
        # the promoted block itself is never a DRAM victim while room is made
        while sum(self.hbm.values()) + size > self.hbm_cap:
            v = self._victim_hbm()
            if v is None:
                return False
            vs = self.hbm.pop(v)
            self.evictions += 1
            vd = 8 + vs // 2 if self.compress and vs >= 64 else vs
            cands_ok = self.dram_cap > 0 and vd <= self.dram_cap
            while cands_ok and sum(self.dram.values()) + vd > self.dram_cap:
                cands = [x for x in self.dram if x != k and not (self.semantic and x in self.prefix)]
                if not cands:
                    cands_ok = False
                    break
                del self.dram[cands[0]]
                self.dropped.append(cands[0])
            if cands_ok:
                self.dram[v] = self._to_dram(v, vs)
                self.compression_savings += vs - vd
            else:
                self.dropped.append(v)
        del self.dram[k]
        self.hbm[k] = size
        return True

    def tier(self, k: str) -> str | None:
        if k in self.hbm:
            return "hbm"
        if k in self.dram:
            return "dram"
        return None


class LocalityTracker:
    """DistributedStore::record_access / should_promote_local
    (src/distributed_backend.cpp:1224-1265; AccessRecord,
    include/cascade_distributed.hpp:162-180): per block, total and windowed
    access counts; when a window of 8 accesses is full, the remote fraction
    of the window enters an EMA with alpha 0.3 (float32 arithmetic, like the
    reference). A block may be promoted after >= threshold accesses with an
    EMA above 0.5."""

    WINDOW = 8
    ALPHA = np.float32(0.3)

    def __init__(self, threshold: int = 3):
        self.threshold = threshold
        self.rec: dict[str, list] = {}  # id -> [total, window_total, window_remote, ema(float32)]

    def record(self, k: str, remote: bool):
        r = self.rec.setdefault(k, [0, 0, 0, np.float32(0.0)])
        r[0] += 1
        r[1] += 1
        if remote:
            r[2] += 1
        if r[1] >= self.WINDOW:
            cur = np.float32(r[2]) / np.float32(r[1])
            r[3] = np.float32(self.ALPHA * cur + (np.float32(1.0) - self.ALPHA) * r[3])
            r[1] = r[2] = 0

    def should_promote(self, k: str) -> bool:
        r = self.rec.get(k)
        return r is not None and r[0] >= self.threshold and float(r[3]) > 0.5


def distributed_gets(model: TierModel, tracker: LocalityTracker, batches, locality_aware: bool = True):
    """Tier of every get of a 1-rank DistributedStore (DistributedStore::get,
    src/distributed_backend.cpp:698-795) over ``batches`` of IDs: an HBM hit
    or a DRAM hit (recorded as a local access), promoted only when
    ``locality_aware and should_promote_local`` (:721-724). Returns
    (codes per batch: 1 HBM / 2 DRAM / 0 miss, counters)."""
    ctr = {"local_gpu_hits": 0, "local_dram_hits": 0, "misses": 0, "promotions_to_local": 0}
    out = []
    for batch in batches:
        codes = []
        for k in batch:
            t = model.tier(k)
            if t is None:
                ctr["misses"] += 1
                codes.append(0)
                continue
            model.touch(k)
            tracker.record(k, remote=False)
            if t == "hbm":
                ctr["local_gpu_hits"] += 1
                codes.append(1)
            else:
                ctr["local_dram_hits"] += 1
                codes.append(2)
                if locality_aware and tracker.should_promote(k) and model.promote(k):
                    ctr["promotions_to_local"] += 1
        out.append(codes)
    return out, ctr
