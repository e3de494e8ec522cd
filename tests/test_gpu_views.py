"""Zero-copy gets (cb_get_views / cb_release_views): torch tensors aliasing
blocks in the HBM pool. Bytes must equal what a copying get returns (the
oracle's bytes, or the INT8 round trip for a block that went through the
compressed DRAM tier); viewed blocks must stay in place while pinned."""
import numpy as np
import pytest

import cascade_cpp
from oracle import kvquant as KQ

from helpers import gen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def make_store(hbm, dram=1 << 28, **kw):
    cfg = cascade_cpp.DistributedConfig()
    cfg.gpu_capacity_per_device = hbm
    cfg.dram_capacity = dram
    cfg.device = 0
    for k, v in kw.items():
        setattr(cfg, k, v)
    return cascade_cpp.DistributedStore(cfg)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def test_views_alias_the_pool_without_kernels():
    sizes = [917_504, 4096, 65, 1, 300_003]
    blocks = [gen("kv_fp16", 500 + i, s) for i, s in enumerate(sizes)]
    store = make_store(64 << 20)
    ids = store.batch_put([dev(b) for b in blocks])
    k0 = store.get_stats().kernel_launches
    views = store.get_views(ids + ["0" * 32])
    assert store.get_stats().kernel_launches == k0  # host metadata only
    assert views[-1] is None
    for b, v in zip(blocks, views):
        assert v.dtype == torch.uint8 and v.is_cuda and v.numel() == b.size
        assert np.array_equal(v.cpu().numpy(), b)
    # two views of one block alias the same memory
    again = store.get_views(ids[:1])
    assert again[0].data_ptr() == views[0].data_ptr()
    store.release_views(ids[:1])
    store.release_views(ids)
    with pytest.raises(cascade_cpp.CascadeError):
        store.release_views(ids[:1])  # no view left


def test_pinned_blocks_stay_in_hbm():
    S = 1 << 20
    blocks = [gen("kv_fp16", 600 + i, S) for i in range(12)]
    store = make_store(4 * S)
    ids = [store.batch_put([dev(b)])[0] for b in blocks[:4]]
    views = store.get_views(ids[:2])
    for b in blocks[4:10]:
        ids.append(store.batch_put([dev(b)])[0])  # each put demotes an unpinned LRU block
    assert store.locate(ids[0]).is_gpu and store.locate(ids[1]).is_gpu
    assert not store.locate(ids[2]).is_gpu and not store.locate(ids[3]).is_gpu
    for b, v in zip(blocks[:2], views):  # still the same bytes at the same place
        assert np.array_equal(v.cpu().numpy(), b)
    with pytest.raises(cascade_cpp.CascadeError):
        store.clear()  # would hand the viewed memory out again
    store.release_views(ids[:2])
    for b in blocks[10:12]:
        ids.append(store.batch_put([dev(b)])[0])
    assert not store.locate(ids[0]).is_gpu  # demoted once released
    store.clear()


@pytest.mark.parametrize("compress", [False, True])
def test_view_of_a_dram_block_promotes_it(compress):
    S = 65_536 * 3 + 6
    blocks = [gen("kv_fp16", 700 + i, S) for i in range(3)]
    store = make_store(8 * S, kv_compression=compress)
    ids = store.batch_put([dev(b) for b in blocks])
    store.evict(8 * S)
    assert not any(store.locate(i).is_gpu for i in ids)
    views = store.get_views(ids)
    assert all(store.locate(i).is_gpu for i in ids)
    for b, v in zip(blocks, views):
        want = KQ.roundtrip(b) if compress else b.tobytes()
        assert v.cpu().numpy().tobytes() == want
    store.release_views(ids)


def test_view_without_promotion_reports_dram():
    S = 4096
    store = make_store(8 * S, promote_on_hit=False)
    ids = store.batch_put([dev(gen("uniform_u8", 800, S))])
    store.evict(8 * S)
    assert store.get_views(ids) == [None]
    with pytest.raises(cascade_cpp.CascadeError):
        store.release_views(ids)  # nothing was pinned
