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
