"""Paged-KV connector (cascade_cpp.connector): pages of a paged KV cache
saved from and loaded into the cache in place. IDs must equal
compute_block_id of each page, a duplicated page is a dedup hit, and a load
into other page slots must reproduce the saved bytes."""
import numpy as np
import pytest

import cascade_cpp
from cascade_cpp.connector import KVPageConnector

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def test_pages_round_trip_in_place():
    g = torch.Generator(device=DEV).manual_seed(11)
    # 32 pages shaped like Qwen2.5-7B KV blocks: 28 layers x (K,V) x 4 heads x 16 tokens x 128, fp16
    kv = torch.randn(32, 28, 2, 4, 16, 128, generator=g, dtype=torch.float16, device=DEV)
    kv[5].copy_(kv[3])
    cfg = cascade_cpp.DistributedConfig()
    cfg.gpu_capacity_per_device = 64 << 20
    cfg.dram_capacity = 0
    cfg.device = 0
    store = cascade_cpp.DistributedStore(cfg)
    conn = KVPageConnector(store, kv)
    assert conn.page_bytes == 917_504
    ids, status = conn.save(range(32), return_status=True)
    assert ids == cascade_cpp.compute_block_ids([kv[p] for p in range(32)])
    assert status[5] == 1 and status.count(1) == 1 and status.count(0) == 31
    saved = kv.clone()
    kv.zero_()
    src = np.random.default_rng(3).permutation(32)
    dst = np.arange(32)
    assert conn.load([ids[s] for s in src], dst) == [True] * 32
    for s, d in zip(src, dst):
        assert torch.equal(kv[d], saved[s])
    assert conn.load(["0" * 32], [0]) == [False]
    with pytest.raises(IndexError):
        conn.save([32])
