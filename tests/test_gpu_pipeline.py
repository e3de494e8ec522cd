"""Stream-ordered puts and gets (cb_put_batch_async / cb_put_wait /
cb_get_batch_async) through the C ABI, against the fixtures the reference
generated and the oracle.

Pipelined puts are placed in ticket order, so every result must equal the
synchronous put of the same batches one after the other
(DistributedStore::put_batch, distributed_backend.cpp:813-841): IDs,
per-block statuses, dedup counts, tier placement; stream-ordered gets must
return what synchronous gets return (DistributedStore::get_batch, :844-870).
"""
import ctypes as C
import hashlib

import numpy as np
import pytest

import cascade_cpp
from cascade_cpp import _lib as L
from cascade_cpp import workloads as W
from oracle import store_oracle as O

from helpers import load

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def make_store(hbm=1 << 30, dram=0, **kw):
    cfg = cascade_cpp.DistributedConfig()
    cfg.gpu_capacity_per_device = hbm
    cfg.dram_capacity = dram
    cfg.device = 0
    for k, v in kw.items():
        setattr(cfg, k, v)
    return cascade_cpp.DistributedStore(cfg)


def dev_blocks(arrays):
    """One device buffer holding the blocks back to back; (buffer, ptrs, sizes)."""
    sizes = np.array([a.size for a in arrays], np.uint64)
    offs = np.concatenate([[0], np.cumsum([((int(s) + 255) // 256) * 256 for s in sizes])]).astype(np.uint64)
    host = np.zeros(int(offs[-1]) + 256, np.uint8)
    for a, o in zip(arrays, offs[:-1]):
        host[int(o):int(o) + a.size] = a
    buf = torch.from_numpy(host).to(DEV)
    ptrs = (np.uint64(buf.data_ptr()) + offs[:-1]).astype(np.uint64)
    return buf, ptrs, sizes


@pytest.mark.parametrize("name", ["mix_small_4k", "mix_qwen7b_128"])
@pytest.mark.parametrize("batch", [1, 32, 64])
@pytest.mark.parametrize("pipeline_blocks", [0, 40])
def test_pipelined_put_matches_reference_scenarios(name, batch, pipeline_blocks):
    sc = next(s for s in load("store_scenarios.json")["scenarios"] if s["name"] == name)
    src, is_prefix = W.dedup_mix(sc["n_blocks"], sc["n_prefix"], sc["dup_frac"], sc["mix_seed"])
    uniq = {int(s): W.kv_block_fp16(sc["block_seed_base"] + int(s), sc["size"]) for s in np.unique(src)}
    buf, ptrs, sizes = dev_blocks([uniq[int(s)] for s in src])
    store = make_store(pipeline_blocks=pipeline_blocks)
    n = len(src)
    keys = np.zeros((n, 16), np.uint8)
    status = np.full(n, 9, np.uint8)
    prefix = is_prefix.astype(np.uint8)
    tickets = [store.put_ptrs_async(ptrs[i:i + batch], sizes[i:i + batch], keys_out=keys[i:i + batch],
                                    status_out=status[i:i + batch], prefix=prefix[i:i + batch])
               for i in range(0, n, batch)]
    assert tickets == list(range(tickets[0], tickets[0] + len(tickets)))
    assert store.wait_puts() == tickets[-1]
    assert [k.tobytes().hex() for k in keys] == sc["ids"]
    assert status.tolist() == sc["status"]
    st = store.get_stats()
    assert st.dedup_hits == sc["ref_dedup_hits"]
    assert st.dedup_bytes_saved == sc["ref_dedup_hits"] * sc["size"]
    assert st.total_blocks == sc["unique"]
    assert st.prefix_blocks == sc["n_prefix"]
    # stream-ordered gets in the reference's shuffled order, bytes checked
    uids = list(dict.fromkeys(sc["ids"]))
    order = np.random.default_rng(sc["get_order_seed"]).permutation(len(uids))
    req = [uids[j] for j in order]
    outs = [torch.empty(sc["size"], dtype=torch.uint8, device=DEV) for _ in req]
    for i in range(0, len(req), batch):
        found, got = store.batch_get_async(req[i:i + batch], outs[i:i + batch])
        assert all(found) and got == [sc["size"]] * len(found)
    digests = [hashlib.sha256(o.cpu().numpy().tobytes()).hexdigest()[:16] for o in outs]
    assert digests == sc["get_digest16"]
    store.close()


def test_many_small_batches_in_flight_sequential_dedup():
    """Batches of 16 blocks, hundreds submitted before any wait: duplicates
    inside a batch, across adjacent batches and across far-apart batches are
    decided exactly like a sequential put of the whole stream; IDs equal the
    oracle's SHA-256."""
    rng = np.random.default_rng(3)
    n_uniq, n = 700, 3200
    uniq = [rng.integers(0, 256, int(s), dtype=np.uint8) for s in rng.integers(1, 9000, n_uniq)]
    src = rng.integers(0, n_uniq, n)
    src[100:140] = src[60:100]  # a run of repeats one batch later
    buf, ptrs, sizes = dev_blocks([uniq[s] for s in src])
    store = make_store()
    keys = np.zeros((n, 16), np.uint8)
    status = np.full(n, 9, np.uint8)
    for i in range(0, n, 16):
        store.put_ptrs_async(ptrs[i:i + 16], sizes[i:i + 16], keys_out=keys[i:i + 16], status_out=status[i:i + 16])
    store.wait_puts()
    seen, want = set(), []
    for s in src:
        want.append(1 if s in seen else 0)
        seen.add(s)
    assert status.tolist() == want
    for j in range(0, n, 97):
        assert keys[j].tobytes() == O.sha256(uniq[src[j]])[:16]
    st = store.get_stats()
    assert st.dedup_hits == n - len(seen) and st.total_blocks == len(seen)


def test_future_api_and_interleaved_sync_calls():
    """batch_put_async futures, a synchronous put between pipelined ones
    (it settles the pipeline first, so dedup order is submission order),
    and a get that sees every put submitted before it."""
    rng = np.random.default_rng(4)
    blocks = [torch.from_numpy(rng.integers(0, 256, 5000, dtype=np.uint8)).to(DEV) for _ in range(6)]
    store = make_store()
    f1 = store.batch_put_async(blocks[0:3])
    ids2, st2 = store.batch_put(blocks[2:4], return_status=True)  # block 2 was submitted before: a hit
    f3 = store.batch_put_async(blocks[3:6])
    ids1, st1 = f1.result(return_status=True)
    assert st1 == [0, 0, 0] and st2 == [1, 0]
    outs = [torch.empty(5000, dtype=torch.uint8, device=DEV) for _ in range(6)]
    ids3 = [cascade_cpp.compute_block_id(b) for b in blocks[3:6]]
    found, sizes = store.batch_get_async(ids1 + ids3, outs)  # f3 not waited for: still visible
    assert all(found) and sizes == [5000] * 6
    for o, b in zip(outs, blocks):
        assert torch.equal(o, b)
    assert f3.result(return_status=True) == (ids3, [1, 0, 0])
    assert store.get_stats().dedup_hits == 2


def test_async_get_codes_sizes_and_too_small_outputs():
    rng = np.random.default_rng(5)
    sizes = [0, 1, 17, 4096, 65536 + 3, 300000]
    blocks = [torch.from_numpy(rng.integers(0, 256, s, dtype=np.uint8)).to(DEV) for s in sizes]
    store = make_store()
    ids = store.batch_put(blocks)
    req = ids + ["0" * 32]
    caps = sizes + [64]
    caps[4] = 100  # too small: found, size reported, nothing written
    outs = [torch.full((max(c, 1),), 7, dtype=torch.uint8, device=DEV)[:c] for c in caps]
    keys = np.frombuffer(b"".join(bytes.fromhex(i) for i in req), np.uint8).reshape(-1, 16)
    got_sizes, found = store.get_ptrs_async(keys, np.array([o.data_ptr() for o in outs], np.uint64),
                                            np.array(caps, np.uint64))
    want_sizes, want_found = store.get_ptrs(keys, np.array([o.data_ptr() for o in outs], np.uint64),
                                            np.array(caps, np.uint64), True)
    assert got_sizes.tolist() == want_sizes.tolist() == sizes + [0]
    assert found.tolist() == want_found.tolist()
    assert found[4] == L.CB_FOUND_LOCAL_HBM | L.CB_FOUND_NOT_COPIED and found[6] == L.CB_FOUND_MISS
    for k, (o, b) in enumerate(zip(outs, blocks)):
        if k != 4:
            assert torch.equal(o, b)
    assert bool((outs[4] == 7).all())


def test_async_get_of_dram_blocks_takes_the_synchronous_path():
    S = 256 * 1024
    rng = np.random.default_rng(6)
    blocks = [torch.from_numpy(rng.integers(0, 256, S, dtype=np.uint8)).to(DEV) for _ in range(8)]
    store = make_store(hbm=16 * S, dram=64 * S)
    ids = store.batch_put(blocks)
    store.evict(5 * S)
    tiers = [store.locate(i).is_gpu for i in ids]
    assert tiers.count(False) == 5
    outs = [torch.empty(S, dtype=torch.uint8, device=DEV) for _ in ids]
    found, sizes = store.batch_get_async(ids, outs)
    assert all(found) and sizes == [S] * 8
    for o, b in zip(outs, blocks):
        assert torch.equal(o, b)
    st = store.get_stats()
    assert st.local_dram_hits == 5 and st.local_gpu_hits == 3 and st.promotions_to_local == 0


def test_pipelined_puts_with_demotions_match_the_tier_model():
    """A small HBM pool under pipelined puts: LRU demotions run inside the
    placements; tiers equal the oracle's model and every byte survives."""
    S = 128 * 1024
    rng = np.random.default_rng(7)
    arrays = [rng.integers(0, 256, S, dtype=np.uint8) for _ in range(40)]
    buf, ptrs, sizes = dev_blocks(arrays)
    store = make_store(hbm=10 * S, dram=64 * S)
    keys = np.zeros((40, 16), np.uint8)
    for i in range(0, 40, 4):
        store.put_ptrs_async(ptrs[i:i + 4], sizes[i:i + 4], keys_out=keys[i:i + 4])
    store.wait_puts()
    model = O.TierModel(10 * S, 64 * S)
    ids = [k.tobytes().hex() for k in keys]
    for i in ids:
        model.put(i, S)
    assert [store.locate(i).is_gpu for i in ids] == [model.tier(i) == "hbm" for i in ids]
    outs = [np.empty(S, np.uint8) for _ in ids]
    found, _ = store.batch_get(ids, outs)
    assert all(found) and all(np.array_equal(o, a) for o, a in zip(outs, arrays))


def test_pool_extents_are_not_reused_under_a_pending_gather():
    """A stream-ordered gather of a block, then pipelined puts that demote
    that block and write new blocks into the pool: the gather still returns
    the old block's bytes (the placements wait for it on the device)."""
    S = 1 << 20
    rng = np.random.default_rng(8)
    old = [torch.from_numpy(rng.integers(0, 256, S, dtype=np.uint8)).to(DEV) for _ in range(4)]
    store = make_store(hbm=4 * S, dram=64 * S)
    ids = store.batch_put(old)
    outs = [torch.empty(S, dtype=torch.uint8, device=DEV) for _ in range(4)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # the gathers run on a stream of their own
        torch.cuda._sleep(20_000_000)  # keep that stream busy, so the gathers are still queued
        found, _ = store.batch_get_async(ids, outs)
    assert all(found)
    new = [torch.from_numpy(rng.integers(0, 256, S, dtype=np.uint8)).to(DEV) for _ in range(4)]
    f = store.batch_put_async(new)  # demotes all four old blocks and reuses their extents
    f.result()
    side.synchronize()
    for o, b in zip(outs, old):
        assert torch.equal(o, b)
    assert not any(store.locate(i).is_gpu for i in ids)


def test_async_put_is_ordered_after_the_callers_stream():
    store = make_store()
    s = torch.cuda.Stream()
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device=DEV)
    with torch.cuda.stream(s):
        torch.cuda._sleep(20_000_000)
        buf.fill_(42)
        f = store.batch_put_async([buf])  # hashed after the fill on s
    assert f.result() == [hashlib.sha256(bytes([42]) * (1 << 20)).hexdigest()[:32]]


def test_get_error_surfaces_at_the_next_settling_call():
    lib = cascade_cpp._native_lib()
    store = make_store()
    b = torch.arange(256, dtype=torch.uint8, device=DEV)
    ids = store.batch_put([b])
    assert lib.cb_selftest(store._n.h, L.CB_SELFTEST_GET_ERROR) == L.CB_OK
    out = torch.empty(256, dtype=torch.uint8, device=DEV)
    found, _ = store.batch_get_async(ids, [out])  # the error is raised on the device, later
    assert found == [True]
    assert lib.cb_sync(store._n.h) == L.CB_ERR_DEVICE
    assert b"device-side check failed" in lib.cb_last_error(store._n.h)
    # nothing was lost: the store goes on serving
    assert lib.cb_sync(store._n.h) == L.CB_OK
    out2 = torch.empty(256, dtype=torch.uint8, device=DEV)
    assert store.batch_get(ids, [out2])[0] == [True] and torch.equal(out2, b)
    assert torch.equal(out, b)


def test_clear_places_then_drops_pipelined_batches():
    rng = np.random.default_rng(9)
    blocks = [torch.from_numpy(rng.integers(0, 256, 4096, dtype=np.uint8)).to(DEV) for _ in range(8)]
    store = make_store()
    fs = [store.batch_put_async(blocks[i:i + 2]) for i in range(0, 8, 2)]
    store.clear()
    assert store.get_stats().total_blocks == 0
    assert all(f.done() for f in fs)
    assert store.batch_put(blocks[:1], return_status=True)[1] == [0]


def test_pipelined_ids_match_the_golden_vectors():
    """The pipelined put hashes with the many-chain kernel: its IDs of every
    golden vector (FIPS examples, every padding edge 0..129 B, KV pages,
    1 MB of 'a') equal the reference's, in one launch and spread over
    launches of different sizes; unaligned sources too."""
    from helpers import gen
    vec = load("sha256_vectors.json")["vectors"]
    blocks = [np.ascontiguousarray(gen(v["gen"], v["seed"], v["size"])) for v in vec]
    for shift in (0, 3):
        arrays = [np.concatenate([np.zeros(shift, np.uint8), b]) for b in blocks]
        buf, ptrs, sizes = dev_blocks(arrays)
        ptrs = (ptrs + np.uint64(shift)).astype(np.uint64)
        sizes = (sizes - np.uint64(shift)).astype(np.uint64)
        for batch in (len(vec), 5):
            store = make_store(dedup_enabled=False)
            keys = np.zeros((len(vec), 16), np.uint8)
            for i in range(0, len(vec), batch):
                store.put_ptrs_async(ptrs[i:i + batch], sizes[i:i + batch], keys_out=keys[i:i + batch])
            store.wait_puts()
            assert [k.tobytes().hex() for k in keys] == [v["block_id"] for v in vec], (shift, batch)
            store.close()


def test_pipelined_ids_of_ragged_warps():
    """The many-chain kernel copies two 64-byte chunks of each of a warp's 32
    blocks at a time through shared memory, up to the shortest block of the
    warp, and each lane then reads the rest of its own block; a warp with an
    unaligned block reads all of it lane by lane. IDs of 1024 blocks of
    2-12 KB (sizes not multiples of 64; about 1 in 40 at an address that is
    not a multiple of 16) equal the oracle's, in one launch and over batches
    of 96."""
    rng = np.random.default_rng(4242)
    n = 1024
    sizes = rng.integers(2048, 12289, n)
    shifts = np.where(rng.integers(0, 40, n) == 0, rng.integers(1, 16, n), 0)
    blocks = [rng.integers(0, 256, int(s), dtype=np.uint8) for s in sizes]
    arrays = [np.concatenate([np.zeros(int(sh), np.uint8), b]) for sh, b in zip(shifts, blocks)]
    buf, ptrs, _ = dev_blocks(arrays)
    ptrs = (ptrs + shifts.astype(np.uint64)).astype(np.uint64)
    sz = sizes.astype(np.uint64)
    want = [O.block_id(b) for b in blocks]
    for batch in (n, 96):
        store = make_store(dedup_enabled=False)
        keys = np.zeros((n, 16), np.uint8)
        for i in range(0, n, batch):
            store.put_ptrs_async(ptrs[i:i + batch], sz[i:i + batch], keys_out=keys[i:i + batch])
        store.wait_puts()
        assert [k.tobytes().hex() for k in keys] == want, batch
        store.close()


def test_hash_launches_confined_to_part_of_the_sms():
    """cb_config.hash_sms: the pipelined puts' SHA-256 launches run on hash
    streams of a green context holding part of the SMs (the rest stay free
    for collectives and copies). IDs, statuses, dedup counts and every byte
    read back equal the reference scenario's."""
    sc = next(s for s in load("store_scenarios.json")["scenarios"] if s["name"] == "mix_qwen7b_128")
    src, is_prefix = W.dedup_mix(sc["n_blocks"], sc["n_prefix"], sc["dup_frac"], sc["mix_seed"])
    uniq = {int(s): W.kv_block_fp16(sc["block_seed_base"] + int(s), sc["size"]) for s in np.unique(src)}
    buf, ptrs, sizes = dev_blocks([uniq[int(s)] for s in src])
    store = make_store(hash_sms=64)
    n = len(src)
    keys = np.zeros((n, 16), np.uint8)
    status = np.full(n, 9, np.uint8)
    prefix = is_prefix.astype(np.uint8)
    for i in range(0, n, 16):
        store.put_ptrs_async(ptrs[i:i + 16], sizes[i:i + 16], keys_out=keys[i:i + 16], status_out=status[i:i + 16],
                             prefix=prefix[i:i + 16])
    store.wait_puts()
    assert [k.tobytes().hex() for k in keys] == sc["ids"]
    assert status.tolist() == sc["status"]
    assert store.get_stats().dedup_hits == sc["ref_dedup_hits"]
    uids = list(dict.fromkeys(sc["ids"]))
    outs = [torch.empty(sc["size"], dtype=torch.uint8, device=DEV) for _ in uids]
    found, _ = store.batch_get(uids, outs)
    assert all(found)
    by_id = {sc["ids"][j]: uniq[int(src[j])] for j in range(n)}
    for u, o in zip(uids, outs):
        assert np.array_equal(o.cpu().numpy(), by_id[u])
    store.close()
