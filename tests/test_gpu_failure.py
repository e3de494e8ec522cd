"""Failure detection on the GPU without a GPU fault: a bounded device wait is
made to run out on purpose (cb_selftest: a hash whose input is announced but
never published). The kernel gives up after its short poll budget, raises its
error word, both of its warps leave, and the call returns CB_ERR_TIMEOUT; the
store and the CUDA context stay usable."""
import time

import numpy as np
import pytest

import cascade_cpp
from cascade_cpp import _lib as L

from helpers import gen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_store_stays_usable():
    cfg = cascade_cpp.DistributedConfig()
    cfg.gpu_capacity_per_device = 64 << 20
    cfg.dram_capacity = 0
    cfg.device = 0
    store = cascade_cpp.DistributedStore(cfg)
    n = store._n
    for _ in range(2):
        t0 = time.perf_counter()
        rc = n.lib.cb_selftest(n.h, L.CB_SELFTEST_HASH_WAIT)
        dt = time.perf_counter() - t0
        assert rc == L.CB_ERR_TIMEOUT
        assert b"timed out" in n.lib.cb_last_error(n.h)
        assert dt < 5.0, dt
    # the store (and the context) still work
    blocks = [gen("kv_fp16", 900 + i, 4096) for i in range(8)]
    ids = store.batch_put([torch.from_numpy(b).to("cuda:0") for b in blocks])
    outs = [torch.empty(4096, dtype=torch.uint8, device="cuda:0") for _ in ids]
    found, sizes = store.batch_get(ids, outs)
    assert all(found)
    assert all(np.array_equal(o.cpu().numpy(), b) for o, b in zip(outs, blocks))
    assert n.lib.cb_selftest(n.h, 99) == L.CB_ERR_ARG


def test_failure_after_planning_refuses_data_calls_until_clear():
    # A put whose room-making demotion fails (injected on the host before any
    # copy is issued) leaves placements the memory does not back: the store
    # must refuse reads instead of returning those bytes, until clear().
    cfg = cascade_cpp.DistributedConfig()
    cfg.gpu_capacity_per_device = 4 * 65536 + 1024  # room for four 64 KiB blocks
    cfg.dram_capacity = 16 << 20
    cfg.device = 0
    store = cascade_cpp.DistributedStore(cfg)
    n = store._n
    blocks = [torch.from_numpy(gen("kv_fp16", 950 + i, 65536)).to("cuda:0") for i in range(5)]
    ids = store.batch_put(blocks[:4])
    assert n.lib.cb_selftest(n.h, L.CB_SELFTEST_FAIL_MOVES) == L.CB_OK
    with pytest.raises(cascade_cpp.CascadeError) as e:
        store.batch_put(blocks[4:])  # needs a demotion: the injected failure
    assert e.value.code == L.CB_ERR_NOSPACE
    outs = [torch.empty(65536, dtype=torch.uint8, device="cuda:0") for _ in ids]
    with pytest.raises(cascade_cpp.CascadeError) as e:
        store.batch_get(ids, outs)
    assert e.value.code == L.CB_ERR_STATE and "injected" in str(e.value)
    with pytest.raises(cascade_cpp.CascadeError) as e:
        store.contains(ids[0])
    assert e.value.code == L.CB_ERR_STATE
    store.get_stats()  # statistics still answer
    store.clear()
    ids = store.batch_put(blocks[:4]) + store.batch_put(blocks[4:])  # the demotion now runs
    assert store.get_stats().local_dram_used > 0
    outs = [torch.empty(65536, dtype=torch.uint8, device="cuda:0") for _ in ids]
    found, sizes = store.batch_get(ids, outs)
    assert all(found) and sizes == [65536] * 5
    assert all(torch.equal(o, b) for o, b in zip(outs, blocks))
