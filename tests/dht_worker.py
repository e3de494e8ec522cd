"""One rank of the multi-GPU DHT parity check (run by tests/test_gpu_dht.py
through torch.distributed.run, one process per GPU). Exits non-zero on any
mismatch with the DhtOracle."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "kcj-cascade-v6_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import cascade_cpp  # noqa: E402
from oracle import store_oracle as O  # noqa: E402
from oracle.dht_oracle import DhtOracle, owner  # noqa: E402


def batches(world, seed):
    rng = np.random.default_rng(seed)
    sizes = [0, 1, 63, 64, 65, 4096, 65537, 917504, 300_003, 5000]
    pool = [rng.integers(0, 256, int(sizes[i % len(sizes)]), dtype=np.uint8) for i in range(48)]
    items = []
    for r in range(world):
        sel = rng.integers(0, 48, 64)
        items.append([(int(s), bool(s % 7 == 0)) for s in sel])
    return pool, items


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    cfg = cascade_cpp.DistributedConfig()
    cfg.gpu_capacity_per_device = 1 << 30
    cfg.dram_capacity = 0
    cfg.device = local
    store = cascade_cpp.DistributedStore(cfg)
    assert store.rank == rank and store.world_size == world

    pool, items = batches(world, 11)
    ids_all = [[O.block_id(pool[s]) for s, _ in items[r]] for r in range(world)]
    ora = DhtOracle(world)
    want_status = ora.put_step([[(ids_all[r][i], pool[s].tobytes(), pf) for i, (s, pf) in enumerate(items[r])]
                                 for r in range(world)])

    # phase 1: device tensors, GPU hashing
    blocks = [torch.from_numpy(pool[s].copy()).to(dev) for s, _ in items[rank]]
    ids, status = store.batch_put(blocks, is_prefix=[pf for _, pf in items[rank]], return_status=True)
    assert ids == ids_all[rank], "ids"
    assert status == want_status[rank], ("status", status, want_status[rank])
    st = store.get_stats()
    assert st.dedup_hits == ora.dedup_hits[rank], ("dedup", st.dedup_hits, ora.dedup_hits[rank])

    # every rank reads every stored block, shuffled, into device buffers
    uniq = sorted({b for r in range(world) for b in ids_all[r]})
    order = np.random.default_rng(rank).permutation(len(uniq))
    req = [uniq[j] for j in order]
    by_id = {O.block_id(p): p for p in pool}
    outs = [torch.empty(len(by_id[b]), dtype=torch.uint8, device=dev) for b in req]
    found, sizes = store.batch_get(req, outs)
    assert all(found), "found"
    for b, o, s in zip(req, outs, sizes):
        assert s == len(by_id[b]) and np.array_equal(o.cpu().numpy(), by_id[b]), ("bytes", b)
    # repeated keys in one batch (fetched once, fanned out locally)
    rep = req[:7] * 3 + [req[0]]
    routs = [torch.empty(len(by_id[b]), dtype=torch.uint8, device=dev) for b in rep]
    found, sizes = store.batch_get(rep, routs)
    assert all(found) and all(np.array_equal(o.cpu().numpy(), by_id[b]) for o, b in zip(routs, rep)), "repeats"
    # locality promotion: a remote block fetched 16 times (EMA of the remote
    # rate passes 0.5 after two windows of 8) is replicated into local HBM
    # and served locally from then on
    hot = next(b for b in uniq if owner(b, world) != rank and len(by_id[b]) > 0)
    p0 = store.get_stats().promotions_to_local
    hk = np.frombuffer(bytes.fromhex(hot), np.uint8).reshape(1, 16)
    hout = torch.empty(len(by_id[hot]), dtype=torch.uint8, device=dev)
    optr = np.array([hout.data_ptr()], np.uint64)
    cap = np.array([hout.numel()], np.uint64)
    codes = []
    for _ in range(20):  # same number of collective calls on every rank
        s, f = store.get_ptrs(hk, optr, cap, True)
        codes.append(int(f[0]))
    # CB_FOUND_REMOTE_HBM (3) until promoted, CB_FOUND_LOCAL_HBM (1) after
    assert codes[0] == 3 and codes[-1] == 1, codes
    first_local = codes.index(1)
    assert all(c == 3 for c in codes[:first_local]) and all(c == 1 for c in codes[first_local:]), codes
    assert first_local >= 8, codes  # the EMA needs two full windows of remote accesses
    assert np.array_equal(hout.cpu().numpy(), by_id[hot]), "replica bytes"
    assert store.get_stats().promotions_to_local == p0 + 1

    # prefix registry + replication (sync_metadata): a rank's registry holds
    # the prefix blocks it stored; after the sync it holds the cluster's, and
    # every prefix block owned by another rank has a local copy, so gets of
    # it are served from local HBM without NVLink traffic
    # (a prefix-flagged copy that is a dedup hit registers nothing: the empty
    # block is stored first from a non-prefix copy here)
    assert store.get_stats().prefix_blocks == len(ora.registry[rank])
    union = ora.sync_prefixes()
    store.sync_metadata()
    st = store.get_stats()
    assert st.prefix_blocks == len(union), (st.prefix_blocks, len(union))
    remote_pref = sorted(b for b in union if owner(b, world) != rank and len(by_id[b]) > 0)
    assert st.prefix_replicated_blocks == len(remote_pref), (st.prefix_replicated_blocks, len(remote_pref))
    pk = np.frombuffer(b"".join(bytes.fromhex(b) for b in remote_pref), np.uint8).reshape(-1, 16)
    pouts = [torch.empty(len(by_id[b]), dtype=torch.uint8, device=dev) for b in remote_pref]
    pr0 = store.get_stats().peer_bytes_read
    s_, codes = store.get_ptrs(pk, np.array([o.data_ptr() for o in pouts], np.uint64),
                               np.array([o.numel() for o in pouts], np.uint64), True)
    assert all(int(c) == 1 for c in codes), codes  # CB_FOUND_LOCAL_HBM: the replica
    assert store.get_stats().peer_bytes_read == pr0
    for b, o in zip(remote_pref, pouts):
        assert np.array_equal(o.cpu().numpy(), by_id[b]), ("prefix replica bytes", b)
    # host-memory outputs too
    houts = [np.empty(len(by_id[b]), np.uint8) for b in req[:20]]
    found, sizes = store.batch_get(req[:20], houts)
    assert all(found) and all(np.array_equal(h, by_id[b]) for h, b in zip(houts, req[:20])), "host get"

    # contains / locate / miss
    missing = "f" * 32
    got = store.batch_get([missing], [torch.empty(16, dtype=torch.uint8, device=dev)])
    assert got[0] == [False], "miss"
    assert store.contains(uniq[0]) and not store.contains(missing)
    loc = store.locate(uniq[0])
    assert loc is not None and loc.node_id == owner(uniq[0], world) and loc.is_gpu
    assert store.locate(missing) is None

    # phase 2: host numpy blocks, everything is already stored
    ids2, status2 = store.batch_put([pool[s] for s, _ in items[rank]], return_status=True)
    assert ids2 == ids_all[rank] and status2 == [1] * len(ids2), "phase 2"

    # cluster usage sums the shards; total blocks per owner add up
    st = store.get_stats()
    t = torch.tensor([st.total_blocks, st.local_gpu_used], dtype=torch.int64)
    dist.all_reduce(t)
    assert int(t[0]) == len(uniq), ("total_blocks", int(t[0]), len(uniq))
    assert st.cluster_gpu_used == int(t[1])

    store.clear()
    assert not store.contains(uniq[0])

    # pipelined puts: four steps of 16 blocks per rank submitted before any
    # wait, each placed in submission order by the collective DHT put; the
    # statuses equal the oracle's four sequential steps
    ora2 = DhtOracle(world)
    futs = []
    for j in range(4):
        part = items[rank][16 * j:16 * (j + 1)]
        futs.append(store.batch_put_async([torch.from_numpy(pool[s].copy()).to(dev) for s, _ in part],
                                          is_prefix=[pf for _, pf in part]))
    want2 = [ora2.put_step([[(ids_all[r][16 * j + i], pool[s].tobytes(), pf)
                             for i, (s, pf) in enumerate(items[r][16 * j:16 * (j + 1)])] for r in range(world)])
             for j in range(4)]
    store.wait_puts()  # all four placed in one grouped collective step
    for j, f in enumerate(futs):
        got_ids, got_st = f.result(return_status=True)
        assert got_ids == ids_all[rank][16 * j:16 * (j + 1)], ("pipelined ids", j)
        assert got_st == want2[j][rank], ("pipelined status", j, got_st, want2[j][rank])
    assert store.get_stats().dedup_hits == ora2.dedup_hits[rank], "pipelined dedup"
    outs = [torch.empty(len(by_id[b]), dtype=torch.uint8, device=dev) for b in req]
    found, sizes = store.batch_get(req, outs)
    assert all(found) and all(np.array_equal(o.cpu().numpy(), by_id[b]) for o, b in zip(outs, req)), "pipelined bytes"
    store.clear()
    store.barrier()
    store.close()
    dist.destroy_process_group()
    print(f"rank {rank}: DHT parity ok ({len(uniq)} unique blocks)", flush=True)


if __name__ == "__main__":
    main()
