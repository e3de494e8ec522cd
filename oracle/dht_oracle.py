"""ORACLE — test infrastructure only (see oracle/__init__.py).

Sequential restatement of the multi-rank store semantics of the B200 DHT:
every block has one owner rank, owner = first 8 ID bytes (big-endian) mod
world; within one collective put step an owner applies the requests it
receives in (source rank, batch index) order with the sequential dedup rule
of DistributedStore::put (cascade_Code/cpp/src/distributed_backend.cpp:
604-608), so among byte-identical blocks put in the same step the lowest
(rank, index) is stored and every other copy is a dedup hit; a get returns
the bytes stored by the owner.

Prefix registry (DistributedStore::prefix_registry_, distributed_backend.cpp:
680-683, 958-1024): a rank registers each prefix block it stores (not a dedup
hit); sync_metadata makes every rank's registry the union.
"""
from __future__ import annotations

from .store_oracle import SequentialStore


def owner(block_id: str, world: int) -> int:
    return int.from_bytes(bytes.fromhex(block_id)[:8], "big") % world


class DhtOracle:
    def __init__(self, world: int):
        self.world = world
        self.shards = [SequentialStore() for _ in range(world)]
        self.dedup_hits = [0] * world  # counted on the putting rank
        self.registry = [set() for _ in range(world)]

    def put_step(self, items: list[list[tuple[str, bytes, bool]]]) -> list[list[int]]:
        """items[r] = rank r's batch [(id, bytes, is_prefix)]; returns per-rank
        status lists (0 stored, 1 dedup hit)."""
        status = [[None] * len(b) for b in items]
        # owners process requests grouped by owner, then (rank, index) order
        for o in range(self.world):
            for r, batch in enumerate(items):
                for i, (bid, data, pf) in enumerate(batch):
                    if owner(bid, self.world) != o:
                        continue
                    _, st = self.shards[o].put(bid, data, pf)
                    status[r][i] = st
                    self.dedup_hits[r] += st
                    if st == 0 and pf:
                        self.registry[r].add(bid)
        return status

    def sync_prefixes(self) -> set:
        """sync_prefix_registry: every rank's registry becomes the union."""
        u = set().union(*self.registry)
        self.registry = [set(u) for _ in range(self.world)]
        return u

    def get(self, block_id: str):
        return self.shards[owner(block_id, self.world)].get(block_id)

    def contains(self, block_id: str) -> bool:
        return self.shards[owner(block_id, self.world)].contains(block_id)
