"""Generates the golden fixtures of tests/golden/ from the REFERENCE itself.

Run in a container that has the reference sources (it builds oracle/_ref with
`make -C oracle ref` first):

    python tests/golden/make_golden.py

Every expected value comes from the reference's compiled CPU path
(compute_block_id, cascade_core.cpp:47-58; CascadeStore put/get/contains,
cascade_core.cpp:1211-1352) through oracle/_ref/cascade_ref, cross-checked
with Python hashlib (the reference drivers' convention,
benchmark/run_benchmark.py:119). Blocks are not stored: each fixture entry
names the seeded generator (cascade_cpp.workloads) that rebuilds its bytes.
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "kcj-cascade-v6_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle", "_ref"))

from cascade_cpp import workloads as W  # noqa: E402

SIZES = [0, 1, 3, 55, 56, 57, 63, 64, 65, 100, 119, 120, 121, 127, 128, 129, 191, 192, 1000,
         4095, 4096, 4097, 65536, 65537, W.QWEN7B_BLOCK, W.QWEN7B_BLOCK + 13, 1048573]


def gen(kind: str, seed: int, size: int) -> np.ndarray:
    if kind == "uniform_u8":
        return W.uniform_block(seed, size)
    if kind == "kv_fp16":
        return W.kv_block_fp16(seed, size)
    if kind == "kv_bf16":
        return W.kv_block_bf16(seed, size)
    if kind == "fips_abc":
        return np.frombuffer(b"abc", np.uint8)
    if kind == "fips_448":
        return np.frombuffer(b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq", np.uint8)
    if kind == "fips_million_a":
        return np.full(1_000_000, ord("a"), np.uint8)
    raise ValueError(kind)


def main():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref"], check=True)
    import cascade_ref  # noqa: E402  (the reference, compiled from its sources)

    vectors = []
    cases = [("fips_abc", 0, 3), ("fips_448", 0, 56), ("fips_million_a", 0, 1_000_000)]
    cases += [("uniform_u8", 1000 + i, s) for i, s in enumerate(SIZES)]
    cases += [("kv_fp16", 7, W.QWEN7B_BLOCK), ("kv_fp16", 8, 4096), ("kv_bf16", 9, W.QWEN72B_BLOCK)]
    for kind, seed, size in cases:
        b = gen(kind, seed, size)
        assert b.size == size
        full = hashlib.sha256(b.tobytes()).hexdigest()
        rid = cascade_ref.compute_block_id(np.ascontiguousarray(b))
        assert rid == full[:32], (kind, seed, size)
        vectors.append({"gen": kind, "seed": seed, "size": size, "sha256": full, "block_id": rid})
    with open(os.path.join(HERE, "sha256_vectors.json"), "w") as f:
        json.dump({"source": "reference compute_block_id + hashlib", "vectors": vectors}, f, indent=1)

    # Config-1-shaped dedup stream through the reference CascadeStore (SHM
    # tier), sequential put then shuffled get.
    scenarios = []
    for name, n_blocks, n_prefix, size, seed in [("mix_small_4k", 160, 8, 4096, 11),
                                                 ("mix_qwen7b_128", 128, 8, W.QWEN7B_BLOCK, 12)]:
        src, is_prefix = W.dedup_mix(n_blocks, n_prefix, 0.25, seed)
        uniq = {int(s): W.kv_block_fp16(100_000 * seed + int(s), size) for s in np.unique(src)}
        shm = f"/dev/shm/cascade_golden_{os.getpid()}"
        store = cascade_ref.CascadeStore(shm_capacity=2 * len(uniq) * size + (1 << 20), shm_path=shm)
        ids, status = [], []
        for i, s in enumerate(src):
            b = uniq[int(s)]
            bid = cascade_ref.compute_block_id(b)
            known = store.contains(bid)
            assert store.put(bid, b, bool(is_prefix[i]))
            ids.append(bid)
            status.append(1 if known else 0)
        st = store.stats()
        order = np.random.default_rng(seed + 1).permutation(len(uniq))
        uids = list(dict.fromkeys(ids))
        got = []
        out = np.empty(size, np.uint8)
        for j in order:
            found, sz = store.get(uids[j], out)
            assert found and sz == size
            got.append(hashlib.sha256(out.tobytes()).hexdigest()[:16])
        missing = "0" * 32
        miss = store.get(missing, out)
        scenarios.append({
            "name": name, "n_blocks": n_blocks, "n_prefix": n_prefix, "dup_frac": 0.25, "size": size,
            "mix_seed": seed, "block_seed_base": 100_000 * seed, "gen": "kv_fp16",
            "ids": ids, "status": status, "ref_dedup_hits": st["dedup_hits"],
            "unique": len(uids), "get_order_seed": seed + 1,
            "get_digest16": got, "ref_miss_result": [bool(miss[0]), int(miss[1])],
        })
        del store
        shutil.rmtree(shm, ignore_errors=True)

    # Full config 1: 4096 Qwen2.5-7B blocks, 64 prefix, 25 % copies. Only a
    # checksum of the ID stream is stored (sha256 over the newline-joined IDs).
    src, is_prefix = W.dedup_mix(4096, 64, 0.25, 2024)
    uniq_ids = {}
    for s in np.unique(src):
        uniq_ids[int(s)] = cascade_ref.compute_block_id(W.kv_block_fp16(int(s), W.QWEN7B_BLOCK))
    ids = [uniq_ids[int(s)] for s in src]
    seen, hits = set(), 0
    for bid in ids:
        hits += bid in seen
        seen.add(bid)
    cfg1 = {"n_blocks": 4096, "n_prefix": 64, "dup_frac": 0.25, "mix_seed": 2024, "size": W.QWEN7B_BLOCK,
            "gen": "kv_fp16 seed = unique index", "unique": len(seen), "dedup_hits": hits,
            "ids_sha256": hashlib.sha256("\n".join(ids).encode()).hexdigest(),
            "first_ids": ids[:4], "last_ids": ids[-4:]}
    with open(os.path.join(HERE, "store_scenarios.json"), "w") as f:
        json.dump({"source": "reference CascadeStore (cascade_core.cpp) via oracle/_ref",
                   "scenarios": scenarios, "config1": cfg1}, f, indent=1)
    print("wrote", len(vectors), "vectors,", len(scenarios), "scenarios, config1 unique", len(seen))


if __name__ == "__main__":
    main()
