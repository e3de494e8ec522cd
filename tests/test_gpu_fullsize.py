"""Config 2 at its full size, checked through properties that do not need
the oracle to process 60 GB: 65,536 Qwen2.5-7B blocks (917,504 B fp16
N(0,1), 25 % byte-identical copies of 64 prefix blocks) put in batches of
1024 from HBM, then every unique block read back in shuffled order.

* dedup decisions equal sequential dedup of the put stream (a position is a
  hit iff its block occurred earlier), counts and saved bytes included;
* one ID per distinct block: equal blocks share an ID, distinct ones differ;
* IDs of a seeded sample of 256 blocks equal the CPU oracle's SHA-256;
* every block read back equals its source bytes and re-hashes on the GPU to
  the ID it was requested by.

It holds ~91 GB of HBM and runs in well under a minute; it runs whenever
the GPU has at least 100 GB free."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

N_BLOCKS, BLOCK, BATCH = 65536, 917504, 1024
NEED_FREE = 100 * 10**9  # inputs 45 GB + pool 45 GB + read-back buffers


def _free_hbm() -> int:
    if not torch.cuda.is_available():
        return 0
    torch.cuda.empty_cache()  # blocks cached by earlier tests in this process
    return torch.cuda.mem_get_info(0)[0]


def test_config2_full_size_properties():
    if _free_hbm() < NEED_FREE:
        pytest.skip(f"needs {NEED_FREE / 1e9:.0f} GB of free HBM, {_free_hbm() / 1e9:.0f} GB free")
    import cascade_cpp
    from cascade_cpp import workloads as W
    from oracle.store_oracle import sha256

    dev = torch.device("cuda", 0)
    src, is_prefix = W.dedup_mix(N_BLOCKS, 64, 0.25, 2024)
    uniq = np.unique(src)
    assert len(uniq) == 49152
    g = torch.Generator(device=dev).manual_seed(1000)
    pool = torch.empty(len(uniq) * BLOCK, dtype=torch.uint8, device=dev)
    flat = pool.view(torch.float16)
    chunk = 4096 * BLOCK // 2
    for o in range(0, flat.numel(), chunk):
        m = min(chunk, flat.numel() - o)
        flat[o:o + m] = torch.randn(m, generator=g, device=dev, dtype=torch.float16)
    pos = np.searchsorted(uniq, src)  # unique-block index of every put position
    ptrs = (np.uint64(pool.data_ptr()) + pos.astype(np.uint64) * np.uint64(BLOCK)).astype(np.uint64)
    sizes = np.full(N_BLOCKS, BLOCK, np.uint64)

    cfg = cascade_cpp.DistributedConfig()
    cfg.gpu_capacity_per_device = len(uniq) * BLOCK + (256 << 20)
    cfg.dram_capacity = 0
    cfg.device = 0
    cfg.index_log2 = 18
    store = cascade_cpp.DistributedStore(cfg)

    keys = np.empty((N_BLOCKS, 16), np.uint8)
    status = np.empty(N_BLOCKS, np.uint8)
    for i in range(0, N_BLOCKS, BATCH):
        k, st = store.put_ptrs(ptrs[i:i + BATCH], sizes[i:i + BATCH], True,
                               prefix=is_prefix[i:i + BATCH].astype(np.uint8))
        keys[i:i + BATCH] = k
        status[i:i + BATCH] = st

    # sequential dedup of the stream: hit iff the block occurred earlier
    seen = np.zeros(len(uniq), bool)
    want = np.empty(N_BLOCKS, np.uint8)
    for j, p in enumerate(pos):
        want[j] = 1 if seen[p] else 0
        seen[p] = True
    assert np.array_equal(status, want)
    st = store.get_stats()
    assert st.dedup_hits == N_BLOCKS - len(uniq) == 16384
    assert st.dedup_bytes_saved == 16384 * BLOCK
    assert st.total_blocks == len(uniq)

    # one ID per distinct block
    first = np.full(len(uniq), -1, np.int64)
    for j, p in enumerate(pos):
        if first[p] < 0:
            first[p] = j
    ukeys = keys[first]
    assert len({k.tobytes() for k in ukeys}) == len(uniq)
    assert all(np.array_equal(keys[j], ukeys[p]) for j, p in enumerate(pos))

    # seeded sample against the CPU oracle
    rng = np.random.default_rng(7)
    for u in rng.choice(len(uniq), 256, replace=False):
        host = pool[u * BLOCK:(u + 1) * BLOCK].cpu().numpy()
        assert sha256(host)[:16] == ukeys[u].tobytes(), int(u)

    # read every unique block back in shuffled order; bytes and re-hash
    out = torch.empty(BATCH * BLOCK, dtype=torch.uint8, device=dev)
    outs = (np.uint64(out.data_ptr()) + np.arange(BATCH, dtype=np.uint64) * np.uint64(BLOCK)).astype(np.uint64)
    caps = np.full(BATCH, BLOCK, np.uint64)
    order = rng.permutation(len(uniq))
    for i in range(0, len(order), BATCH):
        sel = order[i:i + BATCH]
        m = len(sel)
        got_sizes, found = store.get_ptrs(ukeys[sel], outs[:m], caps[:m], True)
        assert (found == 1).all() and (got_sizes == BLOCK).all()
        ids = cascade_cpp.compute_block_ids([out[k * BLOCK:(k + 1) * BLOCK] for k in range(m)])
        assert ids == [ukeys[u].tobytes().hex() for u in sel]
        src_rows = pool.view(-1, BLOCK)[torch.from_numpy(sel).to(dev)]  # the requested blocks' source bytes
        assert torch.equal(out.view(BATCH, BLOCK)[:m], src_rows)
        del src_rows
    store.close()
