"""The oracle is pinned against the reference before it is trusted.

Golden fixtures (tests/golden/*.json) were produced by the reference's own
compiled CPU path (oracle/_ref, tests/golden/make_golden.py) and hashlib.
"""
import hashlib
import os
import re

import numpy as np
import pytest

from cascade_cpp import workloads as W
from oracle import store_oracle as O

from helpers import gen, load

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def test_constants_derived_match_cuda_table():
    k, h0 = O.constants()
    src = open(os.path.join(ROOT, "kcj-cascade-v6_b200", "csrc", "sha256_core.cuh")).read()
    table = src[src.index("kSha256K[64]"):src.index("};", src.index("kSha256K[64]"))]
    cuda_k = [int(x, 16) for x in re.findall(r"0x([0-9a-f]{8})u", table)]
    assert cuda_k == k
    h0_src = src[src.index("#define CB_SHA256_H0"):]
    h0_src = h0_src[:h0_src.index("}")]
    assert [int(x, 16) for x in re.findall(r"0x([0-9a-f]{8})u", h0_src)] == h0


def test_oracle_matches_reference_vectors():
    vec = load("sha256_vectors.json")["vectors"]
    assert len(vec) >= 30
    for v in vec:
        b = gen(v["gen"], v["seed"], v["size"])
        d = O.sha256(b)
        assert d.hex() == v["sha256"], v
        assert O.block_id(b) == v["block_id"], v


@pytest.mark.parametrize("size", [0, 1, 55, 56, 63, 64, 65, 119, 120, 128, 1000, 70001])
def test_oracle_vs_hashlib_random(size):
    rng = np.random.default_rng(size)
    b = rng.integers(0, 256, size, dtype=np.uint8)
    assert O.sha256(b) == hashlib.sha256(b.tobytes()).digest()


def test_oracle_batch_form():
    rng = np.random.default_rng(5)
    sizes = rng.integers(0, 3000, 40)
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]])
    packed = rng.integers(0, 256, int(sizes.sum()), dtype=np.uint8)
    d = O.sha256_batch(packed, offs, sizes)
    for i in range(40):
        assert d[i].tobytes() == hashlib.sha256(packed[offs[i]:offs[i] + sizes[i]].tobytes()).digest()


@pytest.mark.parametrize("name", ["mix_small_4k", "mix_qwen7b_128"])
def test_sequential_store_matches_reference_scenario(name):
    sc = next(s for s in load("store_scenarios.json")["scenarios"] if s["name"] == name)
    src, is_prefix = W.dedup_mix(sc["n_blocks"], sc["n_prefix"], sc["dup_frac"], sc["mix_seed"])
    uniq = {int(s): W.kv_block_fp16(sc["block_seed_base"] + int(s), sc["size"]) for s in np.unique(src)}
    store = O.SequentialStore()
    ids = [O.block_id(uniq[int(s)]) for s in src]
    assert ids == sc["ids"]
    status = store.put_batch(ids, [uniq[int(s)].tobytes() for s in src], list(map(bool, is_prefix)))
    assert status == sc["status"]
    assert store.dedup_hits == sc["ref_dedup_hits"] == sc["n_blocks"] - sc["unique"]
    uids = list(dict.fromkeys(ids))
    order = np.random.default_rng(sc["get_order_seed"]).permutation(len(uids))
    got = [hashlib.sha256(store.get(uids[j])[1]).hexdigest()[:16] for j in order]
    assert got == sc["get_digest16"]
    assert store.get("0" * 32) == (False, None)
    assert sc["ref_miss_result"][0] is False


def test_config1_id_stream_checksum():
    """Full config 1: 4096 Qwen2.5-7B blocks, 25 % copies of 64 prefix blocks."""
    c = load("store_scenarios.json")["config1"]
    src, _ = W.dedup_mix(c["n_blocks"], c["n_prefix"], c["dup_frac"], c["mix_seed"])
    uniq = np.unique(src)
    packed = np.concatenate([W.kv_block_fp16(int(s), c["size"]) for s in uniq])
    offs = np.arange(len(uniq), dtype=np.uint64) * c["size"]
    dig = O.sha256_batch(packed, offs, np.full(len(uniq), c["size"], np.uint64))
    idmap = {int(s): dig[i, :16].tobytes().hex() for i, s in enumerate(uniq)}
    ids = [idmap[int(s)] for s in src]
    assert hashlib.sha256("\n".join(ids).encode()).hexdigest() == c["ids_sha256"]
    assert len(set(ids)) == c["unique"] == 3072
    assert len(ids) - len(set(ids)) == c["dedup_hits"] == 1024
    assert ids[:4] == c["first_ids"]


def test_tier_model_protection_rule():
    m = O.TierModel(hbm_cap=4 * 100, dram_cap=100 * 100)
    for i in range(4):
        m.put(f"p{i}", 100, is_prefix=True)
    for i in range(6):
        m.put(f"n{i}", 100)
    # n0 found HBM full of prefix blocks only: the LRU prefix block (p0) went.
    # From then on every victim is the non-prefix block in HBM.
    assert m.tier("p0") == "dram"
    assert [k for k in m.hbm] == ["p1", "p2", "p3", "n5"]
    assert [k for k in m.dram] == ["p0", "n0", "n1", "n2", "n3", "n4"]
    assert m.evictions == 6


def test_locality_tracker_follows_the_reference_rule():
    # EMA updates once per window of 8 accesses: after one all-remote window
    # the EMA is 0.3 (no promotion), after two it is 0.3 + 0.7 * 0.3 = 0.51
    t = O.LocalityTracker(threshold=3)
    for i in range(15):
        t.record("a", remote=True)
        assert not t.should_promote("a"), i
    t.record("a", remote=True)
    assert t.should_promote("a")
    # local accesses only: the EMA stays 0, never promoted
    for _ in range(100):
        t.record("b", remote=False)
    assert not t.should_promote("b")
    # half remote windows: EMA converges to 0.5 from below, never > 0.5
    for i in range(400):
        t.record("c", remote=i % 2 == 0)
    assert not t.should_promote("c")
