"""GPU store parity through the C ABI: IDs, dedup decisions and bytes against
the reference-generated fixtures and the oracle."""
import hashlib

import numpy as np
import pytest

import cascade_cpp
from cascade_cpp import workloads as W
from oracle import store_oracle as O

from helpers import load

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def make_store(hbm=1 << 30, dram=0, engine=0, cls="dist", **kw):
    if cls == "dist":
        cfg = cascade_cpp.DistributedConfig()
        cfg.gpu_capacity_per_device = hbm
        cfg.dram_capacity = dram
        cfg.device = 0
        cfg.copy_engine = engine
        for k, v in kw.items():
            setattr(cfg, k, v)
        return cascade_cpp.DistributedStore(cfg)
    cfg = cascade_cpp.CascadeConfig()
    cfg.gpu_capacity_bytes = hbm
    cfg.shm_capacity_bytes = dram
    cfg.gpu_device_id = 0
    cfg.copy_engine = engine
    for k, v in kw.items():
        setattr(cfg, k, v)
    return cascade_cpp.CascadeStore(cfg)


def scenario_blocks(sc):
    src, is_prefix = W.dedup_mix(sc["n_blocks"], sc["n_prefix"], sc["dup_frac"], sc["mix_seed"])
    uniq = {int(s): W.kv_block_fp16(sc["block_seed_base"] + int(s), sc["size"]) for s in np.unique(src)}
    return src, is_prefix, uniq


@pytest.mark.parametrize("name", ["mix_small_4k", "mix_qwen7b_128"])
@pytest.mark.parametrize("batch", [1, 32, 256])
@pytest.mark.parametrize("memory", ["device", "host"])
def test_scenario_parity(name, batch, memory):
    sc = next(s for s in load("store_scenarios.json")["scenarios"] if s["name"] == name)
    src, is_prefix, uniq = scenario_blocks(sc)
    blocks = [uniq[int(s)] for s in src]
    if memory == "device":
        blocks = [torch.from_numpy(b).to(DEV) for b in blocks]
    store = make_store()
    ids, status = [], []
    for i in range(0, len(blocks), batch):
        r_ids, r_st = store.batch_put(blocks[i:i + batch], is_prefix=list(is_prefix[i:i + batch]),
                                      return_status=True)
        ids += r_ids
        status += r_st
    assert ids == sc["ids"]
    assert status == sc["status"]
    st = store.get_stats()
    assert st.dedup_hits == sc["ref_dedup_hits"]
    assert st.dedup_bytes_saved == sc["ref_dedup_hits"] * sc["size"]
    assert st.total_blocks == sc["unique"]
    assert st.prefix_blocks == sc["n_prefix"]
    uids = list(dict.fromkeys(ids))
    order = np.random.default_rng(sc["get_order_seed"]).permutation(len(uids))
    req = [uids[j] for j in order]
    if memory == "device":
        outs = [torch.empty(sc["size"], dtype=torch.uint8, device=DEV) for _ in req]
    else:
        outs = [np.empty(sc["size"], np.uint8) for _ in req]
    for i in range(0, len(req), batch):
        found, sizes = store.batch_get(req[i:i + batch], outs[i:i + batch])
        assert all(found) and sizes == [sc["size"]] * len(found)
    got = [hashlib.sha256((o.cpu().numpy() if memory == "device" else o).tobytes()).hexdigest()[:16]
           for o in outs]
    assert got == sc["get_digest16"]
    out = np.empty(sc["size"], np.uint8) if memory == "host" else torch.empty(sc["size"], dtype=torch.uint8,
                                                                                 device=DEV)
    # DistributedStore binding reports len(out) on a miss (bindings.cpp:156-161)
    assert store.get("0" * 32, out) == (False, sc["size"])
    assert store.get_stats().misses == 1
    store.close()


def test_cascade_store_miss_reports_zero():
    store = make_store(cls="cascade")
    out = np.empty(64, np.uint8)
    assert store.get("f" * 32, out) == (False, 0)
    b = np.arange(64, dtype=np.uint8)
    bid = cascade_cpp.compute_block_id(b)
    assert store.put(bid, b)
    assert store.get(bid, out) == (True, 64) and np.array_equal(out, b)
    assert store.get_stats().gpu_hits == 1


def test_caller_ids_any_string():
    store = make_store()
    rng = np.random.default_rng(0)
    blocks = [rng.integers(0, 256, 5000, dtype=np.uint8) for _ in range(5)]
    ids = ["synth_b12", "rank0_block_7", "E3B0C44298FC1C149AFBF4C8996FB924", "x", "synth_b12"]
    _, status = store.batch_put(blocks, ids=ids, return_status=True)
    assert status == [0, 0, 0, 0, 1]
    assert store.contains("synth_b12") and not store.contains("synth_b13")
    out = np.empty(5000, np.uint8)
    assert store.get("E3B0C44298FC1C149AFBF4C8996FB924", out) == (True, 5000)
    assert np.array_equal(out, blocks[2])
    assert store.get("synth_b12", out) == (True, 5000) and np.array_equal(out, blocks[0])
    # the lower-case hex string is a different ID
    assert not store.contains("e3b0c44298fc1c149afbf4c8996fb924")


def test_single_put_get_contains_locate():
    store = make_store()
    b = torch.randint(0, 256, (917504,), dtype=torch.uint8, device=DEV)
    bid = cascade_cpp.compute_block_id(b)
    assert bid == O.block_id(b.cpu().numpy())
    assert store.put(bid, b, is_prefix=True)
    assert store.put(bid, b)  # dedup hit still returns True
    assert store.contains(bid)
    loc = store.locate(bid)
    assert loc.is_gpu and loc.is_prefix and loc.size == 917504 and loc.node_id == 0 and loc.gpu_id == 0
    out = torch.empty_like(b)
    assert store.get(bid, out) == (True, 917504)
    assert torch.equal(out, b)
    assert store.locate("0" * 32) is None
    assert store.rank == 0 and store.world_size == 1


def test_output_too_small_reports_size_and_writes_nothing():
    store = make_store()
    b = torch.randint(0, 256, (10000,), dtype=torch.uint8, device=DEV)
    bid = store.batch_put([b])[0]
    small = torch.full((9999,), 7, dtype=torch.uint8, device=DEV)
    assert store.get(bid, small) == (True, 10000)
    assert int((small != 7).sum()) == 0
    host_small = np.full(100, 7, np.uint8)
    found, sizes = store.batch_get([bid], [host_small])
    assert found == [True] and sizes == [10000] and (host_small == 7).all()


SIZES = [0, 1, 15, 16, 17, 4095, 65535, 65536, 65537, 131072 + 5, 917504, 1 << 20, 3 * 65536 + 48]


@pytest.mark.parametrize("engine", [1, 2])
@pytest.mark.parametrize("out_shift", [0, 16, 3])
def test_copy_engines_sizes_and_alignment(engine, out_shift):
    store = make_store(engine=engine)
    rng = np.random.default_rng(engine * 10 + out_shift)
    host = [rng.integers(0, 256, s, dtype=np.uint8) for s in SIZES]
    src = [torch.from_numpy(h).to(DEV) for h in host]
    ids = store.batch_put(src)
    arena = torch.zeros(sum(SIZES) + 64 * len(SIZES) + out_shift, dtype=torch.uint8, device=DEV)
    outs, off = [], out_shift
    for s in SIZES:
        outs.append(arena[off:off + s])
        off += s + 64
    found, sizes = store.batch_get(ids, outs)
    assert all(found) and sizes == SIZES
    for o, h in zip(outs, host):
        assert np.array_equal(o.cpu().numpy(), h)


def test_unaligned_sources():
    store = make_store(engine=1)
    base = torch.randint(0, 256, (1 << 21,), dtype=torch.uint8, device=DEV)
    views = [base[3 + 70001 * i: 3 + 70001 * i + 70000] for i in range(10)]
    ids = store.batch_put(views)
    host = base.cpu().numpy()
    assert ids == [O.block_id(host[3 + 70001 * i: 3 + 70001 * i + 70000]) for i in range(10)]
    outs = [torch.empty(70000, dtype=torch.uint8, device=DEV) for _ in ids]
    store.batch_get(ids, outs)
    for i, o in enumerate(outs):
        assert torch.equal(o, views[i])


@pytest.mark.parametrize("semantic", [True, False])
def test_tiering_matches_model_and_bytes_survive(semantic):
    S = 256 * 1024
    store = make_store(hbm=8 * S, dram=20 * S, semantic_eviction=semantic, promote_on_hit=False)
    model = O.TierModel(8 * S, 20 * S, semantic=semantic)
    rng = np.random.default_rng(77)
    blocks, ids = {}, []
    for i in range(26):
        b = rng.integers(0, 256, S, dtype=np.uint8)
        pf = i % 7 == 0
        bid = store.batch_put([torch.from_numpy(b).to(DEV)], is_prefix=[pf])[0]
        model.put(bid, S, pf)
        blocks[bid] = b
        ids.append(bid)
    for bid in ids:
        loc = store.locate(bid)
        want = model.tier(bid)
        assert (loc is None) == (want is None)
        if loc is not None:
            assert loc.is_gpu == (want == "hbm"), bid
    st = store.get_stats()
    assert st.gpu_evictions == model.evictions
    assert st.local_gpu_used == sum(model.hbm.values()) and st.local_dram_used == sum(model.dram.values())
    live = [b for b in ids if model.tier(b)]
    outs = [torch.empty(S, dtype=torch.uint8, device=DEV) for _ in live]
    found, sizes = store.batch_get(live, outs)
    assert all(found)
    for bid, o in zip(live, outs):
        assert np.array_equal(o.cpu().numpy(), blocks[bid])
    st = store.get_stats()
    assert st.local_dram_hits == sum(1 for b in live if model.tier(b) == "dram")


def test_promotion_on_dram_hit():
    S = 128 * 1024
    store = make_store(hbm=4 * S, dram=16 * S, promote_on_hit=True)
    rng = np.random.default_rng(5)
    blocks = [rng.integers(0, 256, S, dtype=np.uint8) for _ in range(8)]
    ids = store.batch_put([torch.from_numpy(b).to(DEV) for b in blocks[:4]])
    ids += store.batch_put([torch.from_numpy(b).to(DEV) for b in blocks[4:]])
    assert not store.locate(ids[0]).is_gpu
    out = torch.empty(S, dtype=torch.uint8, device=DEV)
    assert store.get(ids[0], out) == (True, S)
    assert np.array_equal(out.cpu().numpy(), blocks[0])
    assert store.locate(ids[0]).is_gpu  # promoted back to HBM
    st = store.get_stats()
    assert st.promotions_to_local == 1 and st.local_dram_hits == 1
    for i, bid in enumerate(ids):  # everything still intact after the moves
        assert store.get(bid, out) == (True, S)
        assert np.array_equal(out.cpu().numpy(), blocks[i])


@pytest.mark.parametrize("cls", ["dist", "cascade"])
def test_dram_hit_promotion_rule_matches_oracle(cls):
    """DistributedStore promotes a DRAM hit only under its locality rule
    (distributed_backend.cpp:721-724: locality_aware, >= 3 accesses, EMA of
    the remote-access rate > 0.5), which a store's own accesses never meet;
    CascadeStore promotes every DRAM hit (cascade_core.cpp:1303-1307). Tier
    codes of every get, hit counters and promotions equal the oracle's."""
    S = 128 * 1024
    rng = np.random.default_rng(21)
    blocks = [rng.integers(0, 256, S, dtype=np.uint8) for _ in range(16)]
    store = make_store(hbm=8 * S, dram=32 * S, cls=cls)
    ids = [store.batch_put([torch.from_numpy(b).to(DEV)])[0] for b in blocks]
    model = O.TierModel(8 * S, 32 * S)
    for i in ids:
        assert model.put(i, S) in ("hbm", "dram")
    if cls == "dist":  # placement after the puts (only DistributedStore has locate)
        assert [store.locate(i).is_gpu for i in ids] == [model.tier(i) == "hbm" for i in ids]
    batches = [[ids[j] for j in rng.integers(0, 16, 8)] for _ in range(12)]
    if cls == "dist":
        want, ctr = O.distributed_gets(model, O.LocalityTracker(3), batches)
    else:
        want, ctr = [], {"local_gpu_hits": 0, "local_dram_hits": 0, "promotions_to_local": 0}
        for b in batches:  # CascadeStore: touch the batch, then promote its DRAM hits in order
            codes = [1 if model.tier(k) == "hbm" else 2 for k in b]
            for k in b:
                model.touch(k)
            for k, c in zip(b, codes):
                if c == 2 and model.tier(k) == "dram" and model.promote(k):
                    ctr["promotions_to_local"] += 1
            ctr["local_gpu_hits"] += codes.count(1)
            ctr["local_dram_hits"] += codes.count(2)
            want.append(codes)
    outs = [torch.empty(S, dtype=torch.uint8, device=DEV) for _ in range(8)]
    for b, w in zip(batches, want):
        keys = np.frombuffer(b"".join(bytes.fromhex(k) for k in b), np.uint8).reshape(-1, 16)
        sizes, found = store.get_ptrs(keys, np.array([o.data_ptr() for o in outs], np.uint64),
                                      np.full(8, S, np.uint64), True)
        assert list(found) == w
        for k, o in zip(b, outs):
            assert np.array_equal(o.cpu().numpy(), blocks[ids.index(k)])
    st = store.get_stats()
    gpu_hits = st.gpu_hits if cls == "cascade" else st.local_gpu_hits
    dram_hits = st.shm_hits if cls == "cascade" else st.local_dram_hits
    promos = st.promotions_to_gpu if cls == "cascade" else st.promotions_to_local
    assert (gpu_hits, dram_hits, promos) == (ctr["local_gpu_hits"], ctr["local_dram_hits"],
                                             ctr["promotions_to_local"])
    if cls == "dist":
        assert promos == 0 and dram_hits > 0
        assert [store.locate(i).is_gpu for i in ids] == [model.tier(i) == "hbm" for i in ids]
    else:
        assert promos > 0


def test_explicit_evict_then_get():
    S = 1 << 20
    store = make_store(hbm=16 * S, dram=16 * S)
    rng = np.random.default_rng(8)
    blocks = [rng.integers(0, 256, S, dtype=np.uint8) for _ in range(6)]
    ids = store.batch_put(blocks)
    assert store.evict(3 * S) == 3 * S
    assert [store.locate(b).is_gpu for b in ids] == [False] * 3 + [True] * 3
    outs = [np.empty(S, np.uint8) for _ in ids]
    found, _ = store.batch_get(ids, outs)
    assert all(found) and all(np.array_equal(o, b) for o, b in zip(outs, blocks))


def test_block_larger_than_hbm_pool_goes_to_dram():
    store = make_store(hbm=1 << 20, dram=8 << 20)
    b = np.random.default_rng(1).integers(0, 256, 3 << 20, dtype=np.uint8)
    bid = store.batch_put([b])[0]
    assert not store.locate(bid).is_gpu
    out = np.empty(3 << 20, np.uint8)
    assert store.get(bid, out) == (True, 3 << 20) and np.array_equal(out, b)


def test_no_space_anywhere_fails():
    store = make_store(hbm=1 << 20, dram=0)
    b = np.zeros(2 << 20, np.uint8)
    ids, status = store.batch_put([b], return_status=True)
    assert status == [2]
    assert not store.contains(ids[0])


def test_clear_resets():
    store = make_store()
    ids = store.batch_put([np.arange(100, dtype=np.uint8)])
    store.clear()
    assert not store.contains(ids[0])
    st = store.get_stats()
    assert st.total_blocks == 0 and st.dedup_hits == 0 and st.local_gpu_used == 0
    assert store.batch_put([np.arange(100, dtype=np.uint8)], return_status=True)[1] == [0]


def test_index_growth_keeps_everything():
    store = make_store(index_log2=6)  # 64 slots: forces several rebuilds
    rng = np.random.default_rng(11)
    blocks = [rng.integers(0, 256, 300, dtype=np.uint8) for _ in range(700)]
    ids = []
    for i in range(0, 700, 100):
        ids += store.batch_put(blocks[i:i + 100])
    outs = [np.empty(300, np.uint8) for _ in ids]
    found, _ = store.batch_get(ids, outs)
    assert all(found) and all(np.array_equal(o, b) for o, b in zip(outs, blocks))


@pytest.mark.parametrize("use_side_stream", [False, True])
def test_put_is_ordered_after_pending_torch_writes(use_side_stream):
    """Blocks written by torch kernels still in flight on the caller's current
    stream (the default stream, or a side stream) must be hashed and stored
    after those writes land."""
    store = make_store(hbm=4 << 30)
    size, n = 5 << 20, 64
    buf = torch.empty(n * size, dtype=torch.uint8, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(9)
    s = torch.cuda.Stream() if use_side_stream else torch.cuda.current_stream()
    with torch.cuda.stream(s):
        for rnd in range(3):
            buf.view(torch.bfloat16).copy_(torch.randn(n * size // 2, generator=g, device=DEV, dtype=torch.bfloat16))
            views = [buf[i * size:(i + 1) * size] for i in range(n)]
            ids = store.batch_put(views)  # no synchronize between the writes and the put
            host = buf.cpu().numpy()
            for i in (0, n // 2, n - 1):
                assert ids[i] == O.block_id(host[i * size:(i + 1) * size]), (rnd, i)
            out = torch.empty(size, dtype=torch.uint8, device=DEV)
            assert store.get(ids[0], out)[0] and torch.equal(out, views[0])


@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("size,stride_pad", [(917504, 0), (300_000, 0), (262_144 + 17, 4096 + 3)])
def test_host_put_overlapped_copy_and_hash(pinned, size, stride_pad):
    """Equal-size host blocks at a constant stride take the overlapped path
    (segment-major copies on a second stream, hash gated per segment)."""
    n = 96
    stride = size + stride_pad
    rng = np.random.default_rng(size)
    packed = torch.empty(n * stride, dtype=torch.uint8, pin_memory=pinned)
    packed.copy_(torch.from_numpy(rng.integers(0, 256, n * stride, dtype=np.uint8)))
    host = packed.numpy()
    store = make_store(hbm=2 << 30)
    ptrs = (np.uint64(host.ctypes.data) + np.arange(n, dtype=np.uint64) * np.uint64(stride)).astype(np.uint64)
    sizes = np.full(n, size, np.uint64)
    for rnd in range(2):
        keys, status = store.put_ptrs(ptrs, sizes, device_memory=False)
        want = [O.block_id(host[i * stride:i * stride + size]) for i in range(n)]
        assert [k.tobytes().hex() for k in keys] == want
        assert (status == rnd).all()  # second round: all dedup hits
    outs = torch.empty(n * size, dtype=torch.uint8, device=DEV)
    optrs = (np.uint64(outs.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(size)).astype(np.uint64)
    s, f = store.get_ptrs(keys, optrs, sizes, device_memory=True)
    assert (f == 1).all()
    got = outs.cpu().numpy()
    for i in range(n):
        assert np.array_equal(got[i * size:(i + 1) * size], host[i * stride:i * stride + size])


def test_config2_slice_device_roundtrip():
    """2048 Qwen2.5-7B blocks (config-2 shape, 25 % copies) in batches of
    1024: IDs equal the oracle's on a sample, every get is byte-exact."""
    n, size = 2048, W.QWEN7B_BLOCK
    src, is_prefix = W.dedup_mix(n, 64, 0.25, 3)
    uniq = np.unique(src)
    g = torch.Generator(device=DEV).manual_seed(3)
    pool = torch.randn(len(uniq) * size // 2, generator=g, device=DEV, dtype=torch.float16).view(torch.uint8)
    pos = {int(s): i for i, s in enumerate(uniq)}
    blocks = [pool[pos[int(s)] * size:(pos[int(s)] + 1) * size] for s in src]
    store = make_store(hbm=4 << 30)
    ids = []
    for i in range(0, n, 1024):
        ids += store.batch_put(blocks[i:i + 1024], is_prefix=list(is_prefix[i:i + 1024]))
    assert store.get_stats().dedup_hits == n - len(uniq)
    for j in [0, 1, 500, 2047]:
        assert ids[j] == O.block_id(blocks[j].cpu().numpy())
    order = np.random.default_rng(4).permutation(n)
    outs = torch.empty(1024 * size, dtype=torch.uint8, device=DEV)
    for i in range(0, n, 1024):
        sel = order[i:i + 1024]
        views = [outs[k * size:(k + 1) * size] for k in range(len(sel))]
        found, sizes = store.batch_get([ids[j] for j in sel], views)
        assert all(found)
        want = torch.stack([blocks[j] for j in sel])
        assert torch.equal(outs.view(len(sel), size), want)


@pytest.mark.parametrize("buffers", ["numpy", "pinned_views", "pinned_separate"])
def test_dram_hits_into_host_buffers(buffers):
    """Large plain DRAM-tier blocks (copied by the copy engines) read into
    host memory: pageable numpy arrays, views of one pinned buffer (runs
    merged into one copy), and separate pinned tensors (never merged across
    allocations). Bytes must equal what was put."""
    S = 1 << 20
    blocks = [W.kv_block_fp16(4000 + i, S) for i in range(12)]
    store = make_store(hbm=16 * S, dram=64 * S)
    ids = store.batch_put([torch.from_numpy(b).to(DEV) for b in blocks])
    store.evict(16 * S)
    assert not any(store.locate(i).is_gpu for i in ids)
    if buffers == "numpy":
        outs = [np.empty(S, np.uint8) for _ in ids]
    elif buffers == "pinned_views":
        big = torch.empty(len(ids) * S, dtype=torch.uint8, pin_memory=True)
        outs = [big[k * S:(k + 1) * S] for k in range(len(ids))]
    else:
        outs = [torch.empty(S, dtype=torch.uint8, pin_memory=True) for _ in ids]
    found, sizes = store.batch_get(ids, outs)
    assert all(found) and sizes == [S] * len(ids)
    for o, b in zip(outs, blocks):
        got = o if isinstance(o, np.ndarray) else o.numpy()
        assert np.array_equal(got, b)
