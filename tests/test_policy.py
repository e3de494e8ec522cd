"""Host policy of the store (csrc/policy.cpp) on the CPU: extent allocator,
sequential dedup, and prefix-protected demotion checked against the
oracle's TierModel (restating src/gpu_backend.cu:482-537 and
src/distributed_backend.cpp:240-284)."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

from oracle.store_oracle import SequentialStore, TierModel

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(ROOT, "kcj-cascade-v6_b200", "csrc")


@pytest.fixture(scope="module")
def ph(tmp_path_factory):
    out = tmp_path_factory.mktemp("policy") / "libpolicy_harness.so"
    # CB_SANITIZE=1 builds the harness with ASan + UBSan; run pytest with
    # LD_PRELOAD="$(gcc -print-file-name=libasan.so) $(gcc -print-file-name=libubsan.so)"
    # and ASAN_OPTIONS=detect_leaks=0 so the runtimes load first.
    opt = (["-O1", "-g", "-fno-omit-frame-pointer", "-fsanitize=address,undefined",
            "-fno-sanitize-recover=undefined"] if os.environ.get("CB_SANITIZE") == "1" else ["-O2"])
    subprocess.run(["g++", *opt, "-std=c++17", "-shared", "-fPIC", f"-I{CSRC}",
                    os.path.join(HERE, "native", "policy_harness.cpp"), os.path.join(CSRC, "policy.cpp"),
                    "-o", str(out)], check=True)
    lib = C.CDLL(str(out))
    V, U64, I = C.c_void_p, C.c_uint64, C.c_int
    lib.ph_create.restype = V
    lib.ph_create.argtypes = [U64, U64, I]
    lib.ph_destroy.argtypes = [V]
    lib.ph_set_compression.argtypes = [V, I]
    for f in ("ph_pin", "ph_unpin"):
        getattr(lib, f).restype = I
        getattr(lib, f).argtypes = [V, U64, U64]
    lib.ph_size.restype = I
    lib.ph_size.argtypes = [V, U64, U64, C.POINTER(U64)]
    lib.ph_put.restype = I
    lib.ph_put.argtypes = [V, V, V, V, I, I, V, V, I, V, C.POINTER(I), V, C.POINTER(I)]
    lib.ph_find.restype = I
    lib.ph_find.argtypes = [V, U64, U64, C.POINTER(U64)]
    lib.ph_touch.argtypes = [V, U64, U64]
    lib.ph_promote.restype = I
    lib.ph_promote.argtypes = [V, U64, U64]
    lib.ph_evict.restype = U64
    lib.ph_evict.argtypes = [V, U64]
    lib.ph_counters.argtypes = [V, V]
    lib.ph_alloc_create.restype = V
    lib.ph_alloc_create.argtypes = [U64]
    lib.ph_alloc_destroy.argtypes = [V]
    lib.ph_alloc.restype = U64
    lib.ph_alloc.argtypes = [V, U64]
    lib.ph_free.argtypes = [V, U64, U64]
    for f in ("ph_alloc_free_bytes", "ph_alloc_extents", "ph_alloc_largest"):
        getattr(lib, f).restype = U64
        getattr(lib, f).argtypes = [V]
    return lib


class Pol:
    def __init__(self, lib, hbm, dram, semantic=True, compress=False):
        self.lib, self.p = lib, lib.ph_create(hbm, dram, 1 if semantic else 0)
        self.names = {}
        if compress:
            lib.ph_set_compression(self.p, 1)

    def key(self, name):
        k = self.names.setdefault(name, (len(self.names) + 1, 0xABC))
        return k

    def put(self, names, sizes, prefix=None, dedup=True):
        n = len(names)
        keys = np.array([self.key(x) for x in names], np.uint64).reshape(-1)
        sz = np.array(sizes, np.uint64)
        pf = np.array(prefix if prefix is not None else [0] * n, np.uint8)
        st = np.zeros(n, np.uint8)
        moves = np.zeros((4096, 7), np.uint64)
        dropped = np.zeros((4096, 2), np.uint64)
        places = np.zeros((max(n, 1), 4), np.uint64)
        nd, npl = C.c_int(0), C.c_int(0)
        nm = self.lib.ph_put(self.p, keys.ctypes.data, sz.ctypes.data, pf.ctypes.data, n, 1 if dedup else 0,
                             st.ctypes.data, moves.ctypes.data, 4096, dropped.ctypes.data, C.byref(nd),
                             places.ctypes.data, C.byref(npl))
        return st.tolist(), moves[:nm], dropped[:nd.value], places[:npl.value]

    def tier(self, name):
        off = C.c_uint64(0)
        lo, hi = self.key(name)
        t = self.lib.ph_find(self.p, lo, hi, C.byref(off))
        return {-1: None, 0: "hbm", 1: "dram"}[t]

    def touch(self, name):
        self.lib.ph_touch(self.p, *self.key(name))

    def promote(self, name):
        return self.lib.ph_promote(self.p, *self.key(name))

    def size(self, name):
        sz = C.c_uint64(0)
        packed = self.lib.ph_size(self.p, *self.key(name), C.byref(sz))
        return int(sz.value), packed

    def counters(self):
        out = np.zeros(11, np.uint64)
        self.lib.ph_counters(self.p, out.ctypes.data)
        return dict(zip(["hbm_used", "dram_used", "size", "dedup_hits", "dedup_bytes", "gpu_evictions",
                         "dram_evictions", "dropped", "prefix_blocks", "promotions", "compression_savings"],
                        map(int, out)))


def test_allocator_best_fit_and_coalesce(ph):
    a = ph.ph_alloc_create(1 << 20)
    offs = [ph.ph_alloc(a, 1000) for _ in range(10)]  # rounded to 1024
    assert offs == [i * 1024 for i in range(10)]
    for o in offs[2:5]:
        ph.ph_free(a, o, 1000)
    assert ph.ph_alloc_extents(a) == 2  # [2048, 5120) coalesced + tail
    assert ph.ph_alloc(a, 3000) == 2048  # best fit into the 3 KiB hole
    ph.ph_free(a, 2048, 3000)
    for o in offs[:2] + offs[5:]:
        ph.ph_free(a, o, 1000)
    assert ph.ph_alloc_extents(a) == 1 and ph.ph_alloc_free_bytes(a) == 1 << 20
    assert ph.ph_alloc(a, (1 << 20) + 1) == 2 ** 64 - 1
    ph.ph_alloc_destroy(a)


def test_allocator_random_never_overlaps(ph):
    rng = np.random.default_rng(3)
    cap = 1 << 24
    a = ph.ph_alloc_create(cap)
    live = {}
    for step in range(3000):
        if live and rng.random() < 0.45:
            o = rng.choice(list(live))
            ph.ph_free(a, int(o), int(live.pop(o)))
        else:
            s = int(rng.integers(1, 200_000))
            o = ph.ph_alloc(a, s)
            if o != 2 ** 64 - 1:
                r = (s + 255) // 256 * 256
                for lo, ls in live.items():
                    lr = (ls + 255) // 256 * 256
                    assert o + r <= lo or lo + lr <= o
                assert o % 256 == 0 and o + r <= cap
                live[o] = s
    used = sum((s + 255) // 256 * 256 for s in live.values())
    assert ph.ph_alloc_free_bytes(a) == cap - used
    ph.ph_alloc_destroy(a)


def test_sequential_dedup_matches_oracle(ph):
    rng = np.random.default_rng(9)
    names = [f"b{int(x)}" for x in rng.integers(0, 40, 300)]
    pol = Pol(ph, 1 << 30, 0)
    ora = SequentialStore()
    got = []
    for i in range(0, 300, 37):  # uneven batches
        st, _, _, _ = pol.put(names[i:i + 37], [1000] * len(names[i:i + 37]))
        got += st
    want = [ora.put(n, b"x" * 1000)[1] for n in names]
    assert got == want
    c = pol.counters()
    assert c["dedup_hits"] == ora.dedup_hits and c["dedup_bytes"] == ora.dedup_bytes_saved
    assert c["size"] == len(set(names))


def test_dedup_disabled_counts_nothing(ph):
    pol = Pol(ph, 1 << 30, 0)
    st, _, _, _ = pol.put(["a", "a", "b"], [10, 10, 10], dedup=False)
    assert st == [0, 1, 0] and pol.counters()["dedup_hits"] == 0


@pytest.mark.parametrize("semantic,compress", [(True, False), (False, False), (True, True), (False, True)])
def test_demotion_matches_tier_model(ph, semantic, compress):
    S = 64 * 1024
    rng = np.random.default_rng((4 if semantic else 5) + (10 if compress else 0))
    pol = Pol(ph, 10 * S, 25 * S, semantic=semantic, compress=compress)
    model = TierModel(10 * S, 25 * S, semantic=semantic, compress=compress)
    for step in range(200):
        op = rng.random()
        name = f"k{int(rng.integers(0, 60))}"
        if op < 0.6:
            pf = bool(rng.random() < 0.15)
            st, moves, dropped, _ = pol.put([name], [S], [1 if pf else 0])
            r = model.put(name, S, pf)
            assert (st[0] == 1) == (r == "dedup")
        elif op < 0.85:
            pol.touch(name)
            model.touch(name)
        else:
            if model.tier(name) == "dram":
                assert pol.promote(name) >= 1
                assert model.promote(name)
        for k in list(pol.names):
            assert pol.tier(k) == model.tier(k), (step, k)
    c = pol.counters()
    assert c["gpu_evictions"] == model.evictions
    assert c["hbm_used"] == sum(model.hbm.values()) and c["dram_used"] == sum(model.dram.values())
    assert c["compression_savings"] == model.compression_savings


def test_prefix_never_evicted_while_nonprefix_evictable(ph):
    S = 1 << 20
    pol = Pol(ph, 4 * S, 100 * S)
    pol.put(["p0", "p1"], [S, S], [1, 1])
    for i in range(20):
        _, moves, _, _ = pol.put([f"n{i}"], [S])
        for mv in moves:
            name = next(k for k, v in pol.names.items() if v == (int(mv[0]), int(mv[1])))
            assert not name.startswith("p"), name
    assert pol.tier("p0") == "hbm" and pol.tier("p1") == "hbm"


def test_batch_never_evicts_its_own_placements(ph):
    S = 1 << 20
    pol = Pol(ph, 4 * S, 100 * S)
    st, moves, _, places = pol.put([f"x{i}" for i in range(6)], [S] * 6)
    # 4 fit in HBM; the other 2 cannot displace same-batch blocks -> DRAM tier
    assert st == [0] * 6 and len(moves) == 0
    assert [int(p[2]) for p in places] == [0, 0, 0, 0, 1, 1]


def test_dram_full_drops_lru_nonprefix(ph):
    S = 1 << 20
    pol = Pol(ph, 2 * S, 2 * S)
    for i in range(6):
        pol.put([f"b{i}"], [S])
    assert [pol.tier(f"b{i}") for i in range(6)] == [None, None, "dram", "dram", "hbm", "hbm"]
    c = pol.counters()
    assert c["dropped"] == 2 and c["dram_evictions"] == 2 and c["size"] == 4


def test_explicit_evict(ph):
    S = 1 << 20
    pol = Pol(ph, 8 * S, 8 * S)
    pol.put([f"b{i}" for i in range(8)], [S] * 8)
    assert ph.ph_evict(pol.p, 3 * S) == 3 * S
    assert [pol.tier(f"b{i}") for i in range(3)] == ["dram"] * 3


def test_compression_packs_demotions_and_unpacks_promotions(ph):
    # kv_compression: DRAM copies of blocks >= 64 B hold 8 + size/2 bytes
    # (src/distributed_backend.cpp:898-903); a packed block reads back as
    # (size/2)*2 bytes; smaller blocks move as they are.
    S = 4097  # odd: the last byte is not kept once packed
    pol = Pol(ph, 3 * 4352, 1 << 20, compress=True)
    pol.put(["a", "b", "c"], [S, S, 40])
    _, moves, _, _ = pol.put(["d", "e"], [S, S])
    ops = {next(k for k, v in pol.names.items() if v == (int(m[0]), int(m[1]))): int(m[6]) for m in moves}
    assert ops == {"a": 1, "b": 1}  # kMovePack, oldest first
    assert pol.tier("a") == "dram" and pol.size("a") == (4096, 1)
    assert pol.tier("c") == "hbm" and pol.size("c") == (40, 0)
    c = pol.counters()
    assert c["dram_used"] == 2 * (8 + S // 2)
    assert c["compression_savings"] == 2 * (S - (8 + S // 2))
    nm = pol.promote("a")
    assert nm >= 1
    assert pol.tier("a") == "hbm" and pol.size("a") == (4096, 0)
    # the promotion move unpacks; "a" is now an even 4096-byte HBM block
    assert pol.counters()["hbm_used"] == sum(
        sz for n, sz in [("a", 4096), ("c", 40), ("d", S), ("e", S)] if pol.tier(n) == "hbm")


def test_compression_small_blocks_stay_raw(ph):
    pol = Pol(ph, 256, 1 << 20, compress=True)
    pol.put(["s0"], [63])
    _, moves, _, _ = pol.put(["s1"], [63])
    assert len(moves) == 1 and int(moves[0][6]) == 0  # kMoveCopy
    assert pol.size("s0") == (63, 0) and pol.counters()["compression_savings"] == 0


def test_compression_direct_dram_placement_is_packed(ph):
    # a block larger than the whole HBM pool goes to DRAM at put time,
    # compressed (distributed_backend.cpp:615-620, :643-652)
    pol = Pol(ph, 1024, 1 << 20, compress=True)
    st, _, _, places = pol.put(["big"], [100_001])
    assert st == [0] and int(places[0][2]) == 1  # DRAM tier
    assert pol.size("big") == (100_000, 1)
    assert pol.counters()["dram_used"] == 8 + 50_000


def test_pinned_blocks_are_never_victims(ph):
    # zero-copy views pin blocks: a pinned block is neither demoted nor
    # dropped, whatever the LRU order, until its last pin is released
    S = 1 << 20
    pol = Pol(ph, 4 * S, 100 * S)
    pol.put(["v0", "v1", "a", "b"], [S] * 4)
    assert ph.ph_pin(pol.p, *pol.key("v0")) == 1 and ph.ph_pin(pol.p, *pol.key("v1")) == 1
    assert ph.ph_pin(pol.p, *pol.key("v0")) == 1  # two views of v0
    for i in range(6):
        pol.put([f"n{i}"], [S])
    assert pol.tier("v0") == "hbm" and pol.tier("v1") == "hbm"
    assert pol.tier("a") == "dram" and pol.tier("b") == "dram"
    # with every HBM block pinned but two, a put still finds room
    st, _, _, _ = pol.put(["x"], [S])
    assert st == [0] and pol.tier("x") == "hbm"
    assert ph.ph_unpin(pol.p, *pol.key("v1")) == 1
    assert ph.ph_unpin(pol.p, *pol.key("v1")) == 0  # no view left
    pol.put(["y"], [S])
    pol.put(["z"], [S])
    assert pol.tier("v1") == "dram" and pol.tier("v0") == "hbm"
    ph.ph_unpin(pol.p, *pol.key("v0"))
    pol.put(["w"], [S])
    assert pol.tier("v0") == "hbm"  # one pin left


@pytest.mark.parametrize("semantic", [True, False])
def test_reference_semantic_eviction_scenario(ph, semantic):
    # The reference's own check (benchmark/scripts/v6_distributed_bench.py:
    # 151-207): 5 MB GPU, 20 MB DRAM, dedup off, 10 prefix then 40 regular
    # 2 MB blocks put one by one; with semantic eviction every prefix block
    # must still be readable afterwards. Placement equals the oracle model's.
    S, MB = 2 << 20, 1 << 20
    pol = Pol(ph, 5 * MB, 20 * MB, semantic=semantic)
    model = TierModel(5 * MB, 20 * MB, semantic=semantic)
    names = [f"prefix_{i:04d}" for i in range(10)] + [f"regular_{i:04d}" for i in range(40)]
    for nm in names:
        pf = nm.startswith("prefix")
        st, _, _, _ = pol.put([nm], [S], [1 if pf else 0], dedup=False)
        assert st == [0]
        model.put(nm, S, pf)
    assert [pol.tier(n) for n in names] == [model.tier(n) for n in names]
    kept = sum(pol.tier(f"prefix_{i:04d}") is not None for i in range(10))
    if semantic:
        assert kept == 10  # the reference's "10/10 prefix readback"
    else:
        assert kept < 10   # plain LRU drops old prefix blocks like any other
    c = pol.counters()
    # prefix_blocks counts prefix blocks the store holds: a dropped block is
    # gone here (the reference would still hold it on its Lustre tier)
    assert c["size"] == 12 and c["prefix_blocks"] == kept
