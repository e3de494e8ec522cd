"""Python mirror checks that need no GPU: the KVCompressor size helpers
(include/cascade.hpp:409-417), argument checks that reject non-CUDA input
before any native call, the zero-copy view span, and the config fields the
C ABI reads."""
import ctypes as C

import numpy as np
import pytest

import cascade_cpp
from cascade_cpp import _lib as L

torch = pytest.importorskip("torch")


def test_kv_compressor_sizes():
    K = cascade_cpp.KVCompressor
    assert K.compressed_size(917_504) == 8 + 458_752
    assert K.compressed_size(65) == 8 + 32
    assert K.original_size(K.compressed_size(4096)) == 4096
    assert K.original_size(8 + 32) == 64


def test_kv_compressor_rejects_host_tensors():
    with pytest.raises(TypeError):
        cascade_cpp.KVCompressor.compress(torch.zeros(64, dtype=torch.uint8))
    with pytest.raises(TypeError):
        cascade_cpp.KVCompressor.compress_batch([np.zeros(64, np.uint8)])
    assert cascade_cpp.KVCompressor.compress_batch([]) == []


def test_pool_span_interface():
    span = cascade_cpp._PoolSpan(0x7f0000001000, 4096)
    ai = span.__cuda_array_interface__
    assert ai["shape"] == (4096,) and ai["typestr"] == "|u1" and ai["data"] == (0x7f0000001000, False)
    assert ai["version"] == 3 and ai["strides"] is None


def test_new_config_fields_reach_the_c_struct():
    c = L.cb_config()
    lib = cascade_cpp._native_lib()
    lib.cb_config_init(C.byref(c))
    assert c.kv_compression == 0 and c.prefix_replication == 0 and c.collective_timeout_ms == 0
    cfg = cascade_cpp.DistributedConfig()
    assert cfg.kv_compression is False and cfg.prefix_replication is True
    assert cfg.collective_timeout_ms == 0


def test_connector_rejects_non_cuda_caches():
    from cascade_cpp.connector import KVPageConnector
    with pytest.raises(TypeError):
        KVPageConnector(None, torch.zeros(4, 16))
    with pytest.raises(TypeError):
        KVPageConnector(None, np.zeros((4, 16)))


def test_hex_ids_parse_to_their_bytes():
    rng = np.random.default_rng(21)
    for _ in range(64):
        k = rng.integers(0, 256, 16, dtype=np.uint8).tobytes()
        bid = k.hex()
        assert cascade_cpp.block_id_to_key(bid) == k
        assert cascade_cpp.key_to_block_id(cascade_cpp.block_id_to_key(bid)) == bid


def test_other_ids_are_hashed_deterministically_and_distinctly():
    lower = "0123456789abcdef0123456789abcdef"
    others = [lower.upper(), lower[:-1], lower + "0", "", "block-7", "blöck-7", "block-8"]
    keys = [cascade_cpp.block_id_to_key(s) for s in others]
    assert all(len(k) == 16 for k in keys)
    assert keys == [cascade_cpp.block_id_to_key(s) for s in others]  # deterministic
    assert len(set(keys)) == len(keys)
    assert cascade_cpp.block_id_to_key(lower) not in keys  # hex parse and string hash stay apart


def test_owner_rank_matches_oracle_rule():
    from oracle.dht_oracle import owner
    rng = np.random.default_rng(22)
    ids = [rng.integers(0, 256, 16, dtype=np.uint8).tobytes().hex() for _ in range(256)]
    ids += ["ff" * 16, "00" * 16, "80" + "00" * 15]
    for world in (1, 2, 3, 4, 7, 8):
        assert [cascade_cpp.owner_rank(b, world) for b in ids] == [owner(b, world) for b in ids]


def test_helper_store_caches_create_one_store_per_device(monkeypatch):
    # threads that hash (or compress) at once on a device share one helper store
    import threading
    import time
    made = []

    class FakeNative:
        def __init__(self, cfg):
            time.sleep(0.02)  # widen the window a racing thread would use
            made.append(cfg.device)

    monkeypatch.setattr(cascade_cpp, "_Native", FakeNative)
    monkeypatch.setattr(cascade_cpp, "_hashers", {})
    monkeypatch.setattr(cascade_cpp.KVCompressor, "_stores", {})
    for get in (cascade_cpp._hasher, cascade_cpp.KVCompressor._native):
        made.clear()
        got = []
        ts = [threading.Thread(target=lambda: got.append(get(3))) for _ in range(8)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        assert made == [3] and len({id(g) for g in got}) == 1
