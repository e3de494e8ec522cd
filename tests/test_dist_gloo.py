"""N>1 host-side logic on CPU: 2 and 4 gloo ranks run the DHT put protocol
with the library's own host functions - writer-side routing
(cb_dht_route: owner per key, per-owner buckets in batch order, counts) and
owner-side planning (cb_dht_plan_put: sequential dedup in (source rank,
index) order), the functions cb_put_batch runs on a DHT member - with gloo
collectives in place of NCCL, and must reach exactly the sequential
DhtOracle's decisions."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _batches(world):
    """Per-rank batches with cross-rank and intra-rank duplicates."""
    rng = np.random.default_rng(7)
    pool = [rng.integers(0, 256, 512, dtype=np.uint8).tobytes() for _ in range(24)]
    items = []
    for r in range(world):
        sel = rng.integers(0, 24, 40)
        items.append([(int(s), bool(s % 5 == 0)) for s in sel])
    return pool, items


def _alltoallv(recv, send, rank, world):
    """Grouped point-to-point exchange (what the library does with
    ncclGroupStart / ncclSend / ncclRecv / ncclGroupEnd)."""
    reqs = []
    for r in range(world):
        if r == rank:
            recv[r].copy_(send[r])
            continue
        if send[r].numel():
            reqs.append(dist.isend(send[r].contiguous(), r))
        if recv[r].numel():
            reqs.append(dist.irecv(recv[r], r))
    for q in reqs:
        q.wait()


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import cascade_cpp
    from oracle import store_oracle as O
    from oracle.dht_oracle import owner as oracle_owner

    pool, items = _batches(world)
    mine = [(O.block_id(pool[s]), pool[s], pf) for s, pf in items[rank]]
    keys = np.frombuffer(b"".join(bytes.fromhex(b) for b, _, _ in mine), np.uint8).reshape(-1, 16)
    # writer side: the library's routing
    owners, order, counts = cascade_cpp.dht_route(keys, world)
    assert owners.tolist() == [oracle_owner(b, world) for b, _, _ in mine]
    allc = [torch.zeros(world, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(allc, torch.from_numpy(counts.astype(np.int64)))
    rcount = [int(allc[r][rank]) for r in range(world)]
    # requests (key bytes, size, prefix) in send order, all-to-all
    rows = [list(keys[i]) + [len(mine[i][1]), int(mine[i][2])] for i in order.tolist()]
    send, o = [], 0
    for r in range(world):
        send.append(torch.tensor(rows[o:o + int(counts[r])], dtype=torch.int64).reshape(-1, 18))
        o += int(counts[r])
    recv = [torch.zeros((rcount[r], 18), dtype=torch.int64) for r in range(world)]
    _alltoallv(recv, send, rank, world)
    # owner side: the library's planning over (source rank, index) order
    req = torch.cat(recv).numpy()
    planner = cascade_cpp.DhtPlanner(1 << 30)
    status, loc = planner.plan_put(req[:, :16].astype(np.uint8), req[:, 16].astype(np.uint64),
                                   req[:, 17].astype(np.uint8))
    # every stored block got a distinct pool extent
    stored = [int(x) for x, st in zip(loc, status) if st == 0]
    assert len(set(stored)) == len(stored)
    replies, o = [], 0
    for r in range(world):
        replies.append(torch.from_numpy(status[o:o + rcount[r]].astype(np.int64)).reshape(-1, 1))
        o += rcount[r]
    back = [torch.zeros((int(counts[r]), 1), dtype=torch.int64) for r in range(world)]
    _alltoallv(back, replies, rank, world)
    flat = torch.cat(back).reshape(-1).tolist()
    status_mine = [None] * len(mine)
    for j, i in enumerate(order.tolist()):
        status_mine[i] = flat[j]
    out[rank] = status_mine
    planner.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_dht_protocol_gloo_ranks(world):
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, port, out), nprocs=world, start_method="spawn", join=True)
    from oracle import store_oracle as O
    from oracle.dht_oracle import DhtOracle
    pool, items = _batches(world)
    ora = DhtOracle(world)
    want = ora.put_step([[(O.block_id(pool[s]), pool[s], pf) for s, pf in items[r]] for r in range(world)])
    for r in range(world):
        assert out[r] == want[r], r
    # cross-rank duplicates exist and the lowest (rank, index) copy is stored
    assert sum(map(sum, want)) > 0


def _prefix_worker(rank, world, port, out):
    """sync_metadata's prefix exchange (csrc/dht.cu dht_sync_prefixes): each
    owner all-gathers one record per prefix block it holds, padded to the
    largest count; every rank merges the keys into its registry and plans a
    local copy of each prefix block another rank owns (non-empty)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import store_oracle as O
    from oracle.dht_oracle import DhtOracle, owner

    pool, items = _batches(world)
    ora = DhtOracle(world)
    ora.put_step([[(O.block_id(pool[s]), pool[s], pf) for s, pf in items[r]] for r in range(world)])
    # what this rank's policy holds: the prefix blocks it owns
    held = sorted({b for r in range(world) for b in ora.registry[r] if owner(b, world) == rank})
    count = torch.tensor([len(held)], dtype=torch.int64)
    counts = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(counts, count)
    max_n = max(int(c) for c in counts)
    rec = torch.zeros((max_n, 17), dtype=torch.int64)  # 16 key bytes + size
    for j, b in enumerate(held):
        rec[j, :16] = torch.tensor(list(bytes.fromhex(b)))
        rec[j, 16] = len(next(pool[s] for s, _ in sum(items, []) if O.block_id(pool[s]) == b))
    recs = [torch.zeros_like(rec) for _ in range(world)]
    dist.all_gather(recs, rec)
    registry = set(ora.registry[rank])
    plan = []
    for r in range(world):
        for j in range(int(counts[r])):
            row = recs[r][j].tolist()
            b = bytes(row[:16]).hex()
            registry.add(b)
            if r != rank and row[16] > 0:
                plan.append(b)
    out[rank] = (sorted(registry), sorted(plan))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_prefix_registry_sync_gloo_ranks(world):
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_prefix_worker, args=(world, port, out), nprocs=world, start_method="spawn", join=True)
    from oracle import store_oracle as O
    from oracle.dht_oracle import DhtOracle, owner
    pool, items = _batches(world)
    ora = DhtOracle(world)
    ora.put_step([[(O.block_id(pool[s]), pool[s], pf) for s, pf in items[r]] for r in range(world)])
    union = ora.sync_prefixes()
    assert union and all(ora.registry[r] == union for r in range(world))
    for r in range(world):
        reg, plan = out[r]
        assert set(reg) == union
        assert set(plan) == {b for b in union if owner(b, world) != r}
