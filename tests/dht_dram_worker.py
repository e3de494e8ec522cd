"""One rank of the DHT DRAM-tier check (run by tests/test_gpu_dht.py through
torch.distributed.run, one process per GPU). Exits non-zero on a mismatch.

Every owner has a small HBM pool (8 blocks) and a pinned DRAM tier. Each
rank puts 24 blocks per step in three pipelined steps, with duplicates
inside and across ranks; owners hold far more than their HBM, so they demote
to DRAM, and blocks that find no HBM room inside their own step go straight
to the owner's DRAM tier through its outbox. Statuses and dedup counts must
equal the DhtOracle's; then every rank reads every block back - blocks in a
peer's DRAM tier come through that peer's outbox - and the bytes must equal
what was put (with kv_compression: the INT8 round trip for blocks that went
through a DRAM tier)."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "kcj-cascade-v6_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import cascade_cpp  # noqa: E402
from cascade_cpp import _lib as L  # noqa: E402
from oracle import kvquant as KQ  # noqa: E402
from oracle import store_oracle as O  # noqa: E402
from oracle.dht_oracle import DhtOracle, owner  # noqa: E402

S = 256 * 1024


def main():
    compress = len(sys.argv) > 1 and sys.argv[1] == "compress"
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    cfg = cascade_cpp.DistributedConfig()
    cfg.gpu_capacity_per_device = 8 * S
    cfg.dram_capacity = 256 * S
    cfg.device = local
    cfg.kv_compression = compress
    cfg.locality_aware = False
    cfg.prefix_replication = False
    store = cascade_cpp.DistributedStore(cfg)

    rng = np.random.default_rng(21)
    pool = [W_kv(1000 + i) for i in range(60)]
    steps = []
    for _ in range(3):
        steps.append([[int(s) for s in rng.integers(0, 60, 24)] for _ in range(world)])
    ids = [O.block_id(p) for p in pool]
    ora = DhtOracle(world)
    tickets = []
    results = []
    for st in steps:
        blocks = [torch.from_numpy(pool[s].copy()).to(dev) for s in st[rank]]
        results.append((store.batch_put_async(blocks), blocks))
        tickets.append(ora.put_step([[(ids[s], pool[s].tobytes(), False) for s in st[r]] for r in range(world)]))
    store.wait_puts()  # the three steps placed as one group (batch order kept by the owners)
    for (fut, _), want in zip(results, tickets):
        got_ids, got_status = fut.result(return_status=True)
        assert got_status == want[rank], ("status", got_status, want[rank])
    assert store.get_stats().dedup_hits == ora.dedup_hits[rank], "dedup"

    stored = sorted({ids[s] for st in steps for r in range(world) for s in st[r]})
    by_id = {ids[i]: pool[i] for i in range(60)}
    in_dram = {b: not store.locate(b).is_gpu for b in stored}
    assert sum(in_dram.values()) > len(stored) // 2, "most blocks live in the owners' DRAM tiers"
    order = np.random.default_rng(rank).permutation(len(stored))
    req = [stored[j] for j in order]
    outs = [torch.empty(S, dtype=torch.uint8, device=dev) for _ in req]
    st0 = store.get_stats()
    for i in range(0, len(req), 16):  # same number of collective calls on every rank
        found, sizes = store.batch_get(req[i:i + 16], outs[i:i + 16])
        assert all(found), "found"
    codes = []
    keys = np.frombuffer(b"".join(bytes.fromhex(b) for b in req), np.uint8).reshape(-1, 16)
    for i in range(0, len(req), 16):
        _, f = store.get_ptrs(keys[i:i + 16], np.array([o.data_ptr() for o in outs[i:i + 16]], np.uint64),
                              np.full(len(keys[i:i + 16]), S, np.uint64), True)
        codes += [int(c) for c in f]
    for b, o, c in zip(req, outs, codes):
        want = by_id[b].tobytes()
        if compress and in_dram[b]:
            want = KQ.roundtrip(by_id[b])
        assert o.cpu().numpy().tobytes() == want, ("bytes", b, in_dram[b])
        remote = owner(b, world) != rank
        if in_dram[b]:
            assert c == (L.CB_FOUND_REMOTE_DRAM if remote else L.CB_FOUND_LOCAL_DRAM), (b, c)
        else:
            assert c == (L.CB_FOUND_REMOTE_HBM if remote else L.CB_FOUND_LOCAL_HBM), (b, c)
    st1 = store.get_stats()
    assert st1.remote_dram_hits > st0.remote_dram_hits, "remote DRAM hits"
    # the owners' tiers are unchanged by the reads
    assert all(in_dram[b] == (not store.locate(b).is_gpu) for b in stored), "tiers"
    store.clear()
    store.barrier()
    store.close()
    dist.destroy_process_group()
    print(f"rank {rank}: DHT DRAM parity ok ({len(stored)} blocks, "
          f"{sum(in_dram.values())} in DRAM tiers, compress={compress})", flush=True)


def W_kv(seed):
    from cascade_cpp import workloads as W
    return W.kv_block_fp16(seed, S)


if __name__ == "__main__":
    main()
