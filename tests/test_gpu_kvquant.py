"""INT8 KV compression on the GPU (kv_compression) against the reference's own
compressor: the golden vectors of tests/golden/kvquant_vectors.json were
produced by KVCompressor::compress/decompress (cascade_Code/cpp/src/
cascade_core.cpp:908-967) compiled from the reference sources; the oracle
(oracle/kvquant_oracle.c) is pinned to them on the CPU.

Covers the standalone compressor (cb_kv_compress_batch /
cb_kv_decompress_batch, every packed byte), and the store paths that use it:
demotion (evict), direct DRAM placement, gets from the DRAM tier into device
and host buffers, promotion on hit, blocks below 64 B and odd sizes."""
import hashlib

import numpy as np
import pytest

import cascade_cpp
from cascade_cpp import KVCompressor
from oracle import kvquant as KQ

from helpers import gen, load

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda:0"
VEC = load("kvquant_vectors.json")["vectors"]
LOCAL_HBM, LOCAL_DRAM = 1, 2


def sha(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


def dev(a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def test_compress_matches_reference_vectors():
    blocks = [dev(gen(v["kind"], v["seed"], v["size"])) for v in VEC]
    packed = KVCompressor.compress_batch(blocks)
    for v, p in zip(VEC, packed):
        b = p.cpu().numpy().tobytes()
        assert len(b) == v["compressed_size"]
        assert b[:64].hex() == v["compressed_head"], (v["kind"], v["size"])
        assert sha(b) == v["compressed_sha256"], (v["kind"], v["size"])
    outs = KVCompressor.decompress_batch(packed, [v["size"] for v in VEC])
    for v, o in zip(VEC, outs):
        b = o.cpu().numpy().tobytes()
        assert len(b) == v["decompressed_size"] and sha(b) == v["decompressed_sha256"], (v["kind"], v["size"])


@pytest.mark.parametrize("shift", [1, 2, 8, 24])
def test_unaligned_buffers_take_the_scalar_path(shift):
    # blocks at odd offsets (sub-tensor views of one allocation): same bytes
    rng = np.random.default_rng(shift)
    sizes = [64, 65, 1000, 70_001]
    raw = [rng.standard_normal(s // 2 + 1).astype(np.float16).view(np.uint8)[:s] for s in sizes]
    big = torch.zeros(sum(s + 64 for s in sizes) + 64, dtype=torch.uint8, device=DEV)
    views, off = [], shift
    for r in raw:
        v = big[off:off + r.size]
        v.copy_(dev(r))
        views.append(v)
        off += r.size + 37
    packed = KVCompressor.compress_batch(views)
    for r, p in zip(raw, packed):
        assert p.cpu().numpy().tobytes() == KQ.compress(r)
    # packed output at unaligned addresses as well
    n = cascade_cpp.KVCompressor._native(0)
    pd = torch.zeros(sum(8 + s // 2 + 16 for s in sizes) + 64, dtype=torch.uint8, device=DEV)
    dviews, off = [], shift
    for s in sizes:
        dviews.append(pd[off:off + 8 + s // 2])
        off += 8 + s // 2 + 11
    n.kv_compress(np.array([v.data_ptr() for v in views], np.uint64), np.array(sizes, np.uint64),
                  np.array([d.data_ptr() for d in dviews], np.uint64))
    torch.cuda.synchronize()
    for r, d in zip(raw, dviews):
        assert d.cpu().numpy().tobytes() == KQ.compress(r)
    # unpack into unaligned outputs too
    ob = torch.zeros(sum(sizes) + 256, dtype=torch.uint8, device=DEV)
    outs, off = [], shift
    for s in sizes:
        outs.append(ob[off:off + s // 2 * 2])
        off += s + 3
    pk = torch.zeros(sum(p.numel() for p in packed) + 64, dtype=torch.uint8, device=DEV)
    pviews, off = [], shift
    for p in packed:
        pv = pk[off:off + p.numel()]
        pv.copy_(p)
        pviews.append(pv)
        off += p.numel() + 5
    ok = n.kv_decompress(np.array([p.data_ptr() for p in pviews], np.uint64),
                         np.array([p.numel() for p in pviews], np.uint64),
                         np.array(sizes, np.uint64), np.array([o.data_ptr() for o in outs], np.uint64))
    torch.cuda.synchronize()
    assert ok.tolist() == [1] * len(sizes)
    for r, o in zip(raw, outs):
        assert o.cpu().numpy().tobytes() == KQ.roundtrip(r)


def test_decompress_short_buffer_is_refused():
    p = KVCompressor.compress(dev(gen("kv_fp16", 1, 256)))
    assert KVCompressor.decompress(p[:-1].contiguous(), 256) is None
    assert KVCompressor.decompress(p, 256) is not None
    with pytest.raises(ValueError):
        KVCompressor.compress(torch.zeros(1, dtype=torch.uint8, device=DEV))


def make_store(hbm, dram, cls="dist", **kw):
    if cls == "dist":
        cfg = cascade_cpp.DistributedConfig()
        cfg.gpu_capacity_per_device = hbm
        cfg.dram_capacity = dram
        cfg.device = 0
        cfg.kv_compression = True
        for k, v in kw.items():
            setattr(cfg, k, v)
        return cascade_cpp.DistributedStore(cfg)
    cfg = cascade_cpp.CascadeConfig()
    cfg.gpu_capacity_bytes = hbm
    cfg.shm_capacity_bytes = dram
    cfg.gpu_device_id = 0
    cfg.kv_compression = True
    for k, v in kw.items():
        setattr(cfg, k, v)
    return cascade_cpp.CascadeStore(cfg)


def codes_and_bytes(store, ids, sizes, device_memory=True):
    keys = np.frombuffer(b"".join(bytes.fromhex(i) for i in ids), np.uint8).reshape(-1, 16)
    if device_memory:
        outs = [torch.zeros(max(s, 1), dtype=torch.uint8, device=DEV) for s in sizes]
        ptrs = [o.data_ptr() for o in outs]
    else:
        outs = [np.zeros(max(s, 1), np.uint8) for s in sizes]
        ptrs = [o.ctypes.data for o in outs]
    got_sizes, found = store.get_ptrs(keys, np.array(ptrs, np.uint64), np.array(sizes, np.uint64), device_memory)
    torch.cuda.synchronize()
    data = [(o.cpu().numpy() if device_memory else o)[:int(s)].tobytes() for o, s in zip(outs, got_sizes)]
    return [int(f) for f in found], [int(s) for s in got_sizes], data


@pytest.mark.parametrize("cls", ["dist", "cascade"])
@pytest.mark.parametrize("memory", ["device", "host"])
def test_demoted_blocks_read_back_through_the_int8_tier(cls, memory):
    S = 917_504  # one Qwen2.5-7B KV page (fp16)
    sizes = [S] * 6 + [40, 4097, 63, 64]
    blocks = [gen("kv_fp16", 100 + i, s) for i, s in enumerate(sizes)]
    store = make_store(hbm=3 * S, dram=1 << 30, cls=cls, promote_on_hit=False) if cls == "dist" else \
        make_store(hbm=3 * S, dram=1 << 30, cls=cls, promotion_enabled=False)
    # one put per block: each put demotes the oldest pages (packed) to DRAM
    ids = [store.batch_put([dev(b)])[0] for b in blocks]
    st = store.get_stats()
    assert st.gpu_evictions == 4
    found, got, data = codes_and_bytes(store, ids, [s + 1 for s in sizes], memory == "device")
    in_dram = [i for i, f in enumerate(found) if f == LOCAL_DRAM]
    assert in_dram and all(f in (LOCAL_HBM, LOCAL_DRAM) for f in found)
    packed_bytes, saved = 0, 0
    for i, (b, f, g, d) in enumerate(zip(blocks, found, got, data)):
        if f == LOCAL_DRAM and b.size >= 64:
            want = KQ.roundtrip(b)
            packed_bytes += 8 + b.size // 2
            saved += b.size - (8 + b.size // 2)
        else:
            want = b.tobytes()
            packed_bytes += b.size if f == LOCAL_DRAM else 0
        assert g == len(want) and d == want, (i, f, g)
    used = st.shm_used if cls == "cascade" else st.local_dram_used
    assert used == packed_bytes
    savings = st.compression_savings_bytes if cls == "cascade" else st.compression_savings
    assert savings == saved


def test_evict_then_promote_on_hit():
    S = 65_536 + 2
    blocks = [gen("kv_fp16", 200 + i, S) for i in range(4)]
    store = make_store(hbm=8 * S, dram=1 << 28, promote_on_hit=True)  # CascadeStore's every-hit rule
    ids = store.batch_put([dev(b) for b in blocks])
    store.evict(4 * S)
    st = store.get_stats()
    assert st.gpu_evictions == 4 and st.local_dram_used == 4 * (8 + S // 2)
    want = [KQ.roundtrip(b) for b in blocks]
    found, got, data = codes_and_bytes(store, ids, [S] * 4)
    assert found == [LOCAL_DRAM] * 4 and data == want
    # promoted by that get (unpacked into HBM): the same bytes, now from HBM
    found, got, data = codes_and_bytes(store, ids, [S] * 4)
    assert found == [LOCAL_HBM] * 4 and data == want and got == [S] * 4
    st = store.get_stats()
    assert st.local_dram_used == 0 and st.local_gpu_used == 4 * S and st.promotions_to_local == 4
    # a second demotion packs the already-unpacked blocks: same bytes again
    # (compress(decompress(compress(x))) == compress(x) is not required; the
    # read must equal the oracle's round trip of what HBM held)
    store.evict(4 * S)
    found, _, data2 = codes_and_bytes(store, ids, [S] * 4)
    assert found == [LOCAL_DRAM] * 4
    assert data2 == [KQ.roundtrip(np.frombuffer(w, np.uint8)) for w in want]


def test_block_larger_than_hbm_is_packed_into_dram():
    S = 3 * 1024 * 1024 + 5
    b = gen("int16_full", 7, S)
    store = make_store(hbm=1 << 20, dram=1 << 28)
    ids, status = store.batch_put([dev(b)], return_status=True)
    assert status == [0]
    found, got, data = codes_and_bytes(store, ids, [S])
    assert found == [LOCAL_DRAM] and got == [S - 1] and data == [KQ.roundtrip(b)]
    assert store.get_stats().local_dram_used == 8 + S // 2


def test_golden_vectors_through_the_store():
    # every golden block is put, demoted (packed on the GPU), and read back:
    # the bytes equal the reference's decompress(compress(block))
    vec = [v for v in VEC if v["size"] <= 2 * 1024 * 1024]
    blocks = [gen(v["kind"], v["seed"], v["size"]) for v in vec]
    store = make_store(hbm=64 << 20, dram=256 << 20)
    ids = store.batch_put([dev(b) for b in blocks])
    store.evict(64 << 20)
    found, got, data = codes_and_bytes(store, ids, [v["size"] for v in vec])
    assert found == [LOCAL_DRAM] * len(vec)
    for v, g, d in zip(vec, got, data):
        assert g == v["decompressed_size"] and sha(d) == v["decompressed_sha256"], (v["kind"], v["size"])


@pytest.mark.parametrize("compress", [False, True])
def test_get_promotions_overlapped_with_demotions(compress):
    """Gets whose DRAM hits are promoted while the demotions that make room
    run beside the gather: many DRAM hits per batch, repeated keys, outputs
    too small to copy, and requested HBM blocks chosen as victims. Every
    copied block must read back as expected: the bytes it was put with,
    or, each time it comes back from the (INT8) DRAM tier, the oracle's
    round trip of what it held before."""
    S = 1 << 20
    rng = np.random.default_rng(7 if compress else 8)
    blocks = [gen("kv_fp16", 300 + i, S) for i in range(40)]
    cfg = cascade_cpp.DistributedConfig()
    cfg.gpu_capacity_per_device = 8 * S
    cfg.dram_capacity = 1 << 30
    cfg.device = 0
    cfg.kv_compression = compress
    cfg.promote_on_hit = True  # every DRAM hit is promoted (CascadeStore's rule)
    store = cascade_cpp.DistributedStore(cfg)
    ids = [store.batch_put([dev(b)])[0] for b in blocks]
    exp = [b.tobytes() for b in blocks]
    promoted = 0
    for it in range(25):
        pick = [int(x) for x in rng.integers(0, 40, 16)]
        pick += pick[:3]  # repeats
        caps = [S if rng.random() > 0.15 else S // 2 for _ in pick]
        found, got, data = codes_and_bytes(store, [ids[j] for j in pick], caps)
        read_from_dram = set()
        for j, f, g, d, c in zip(pick, found, got, data, caps):
            tier = f & 0x0F
            assert tier in (LOCAL_HBM, LOCAL_DRAM), (it, j, f)
            if c < S:
                assert f & 0x80, (it, j, f)  # found, not copied
                continue
            # a DRAM hit reads back the round trip of what the block held;
            # repeats in one batch read the same DRAM copy
            want = KQ.roundtrip(exp[j]) if tier == LOCAL_DRAM and compress else exp[j]
            assert d == want, (it, j, f)
            if tier == LOCAL_DRAM:
                read_from_dram.add(j)
        # a promoted block now holds in HBM what the get returned; one that
        # could not be promoted (HBM full of this batch's promotions) still
        # holds its packed copy in DRAM
        for j in read_from_dram:
            if store.locate(ids[j]).is_gpu:
                if compress:
                    exp[j] = KQ.roundtrip(exp[j])
                promoted += 1
    assert promoted > 20
    st = store.get_stats()
    assert st.local_gpu_used <= 8 * S and st.total_blocks == 40
    # everything still reads back as tracked
    found, got, data = codes_and_bytes(store, ids, [S] * 40)
    for j, (f, d) in enumerate(zip(found, data)):
        want = KQ.roundtrip(exp[j]) if (f & 0x0F) == LOCAL_DRAM and compress else exp[j]
        assert d == want, j
