"""GPU SHA-256 / block-ID parity: the sm_100a kernel through the C ABI against
the golden vectors (from the reference) and the oracle."""
import hashlib
import numpy as np
import pytest

import cascade_cpp
from cascade_cpp import _lib as L
from cascade_cpp import workloads as W
from oracle import store_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from helpers import gen, load


def gpu_digests(blocks):
    """Full 32-byte digests via cb_hash_batch on device tensors."""
    h = cascade_cpp._hasher(0)
    ts = [torch.from_numpy(np.ascontiguousarray(b)).to("cuda:0") for b in blocks]
    ptrs = np.array([t.data_ptr() for t in ts], np.uint64)
    sizes = np.array([t.numel() for t in ts], np.uint64)
    return h.hash(ptrs, sizes, L.CB_MEM_DEVICE)


def test_golden_vectors_device():
    vec = load("sha256_vectors.json")["vectors"]
    blocks = [gen(v["gen"], v["seed"], v["size"]) for v in vec]
    dig = gpu_digests(blocks)
    for v, d in zip(vec, dig):
        assert d.tobytes().hex() == v["sha256"], v
    ids = cascade_cpp.compute_block_ids([torch.from_numpy(np.ascontiguousarray(b)).cuda() for b in blocks])
    assert ids == [v["block_id"] for v in vec]


def test_golden_vectors_host_memory():
    vec = load("sha256_vectors.json")["vectors"][:12]
    ids = cascade_cpp.compute_block_ids([gen(v["gen"], v["seed"], v["size"]) for v in vec])
    assert ids == [v["block_id"] for v in vec]


def test_single_compute_block_id_numpy_and_bytes():
    b = W.kv_block_fp16(7, W.QWEN7B_BLOCK)
    assert cascade_cpp.compute_block_id(b) == O.block_id(b)
    assert cascade_cpp.compute_block_id(b"abc") == hashlib.sha256(b"abc").hexdigest()[:32]


@pytest.mark.parametrize("shift", [1, 2, 3, 4, 5, 7, 8, 12, 13])
def test_unaligned_block_addresses(shift):
    base = torch.randint(0, 256, (1 << 20,), dtype=torch.uint8, device="cuda:0")
    sizes = [0, 1, 63, 64, 65, 1000, 65536 + 3, 300_001]
    views = [base[shift + 17 * i: shift + 17 * i + s] for i, s in enumerate(sizes)]
    ids = cascade_cpp.compute_block_ids(views)
    host = base.cpu().numpy()
    for i, s in enumerate(sizes):
        assert ids[i] == O.block_id(host[shift + 17 * i: shift + 17 * i + s])


@pytest.mark.parametrize("n", [1, 31, 32, 33, 97, 512, 1025])
def test_batch_sizes_random_lengths(n):
    rng = np.random.default_rng(n)
    sizes = rng.integers(0, 20_000, n)
    blocks = [rng.integers(0, 256, int(s), dtype=np.uint8) for s in sizes]
    dig = gpu_digests(blocks)
    for b, d in zip(blocks, dig):
        assert d.tobytes() == hashlib.sha256(b.tobytes()).digest()


def test_config1_full_scale_id_stream():
    """All 4096 config-1 IDs (3072 unique Qwen2.5-7B blocks) hashed on the
    GPU in one batch; checksum of the ID stream against the reference's."""
    c = load("store_scenarios.json")["config1"]
    src, _ = W.dedup_mix(c["n_blocks"], c["n_prefix"], c["dup_frac"], c["mix_seed"])
    uniq = np.unique(src)
    dev = torch.empty(len(uniq) * c["size"], dtype=torch.uint8, device="cuda:0")
    for i, s in enumerate(uniq):
        dev[i * c["size"]:(i + 1) * c["size"]].copy_(torch.from_numpy(W.kv_block_fp16(int(s), c["size"])))
    ids_u = cascade_cpp.compute_block_ids([dev[i * c["size"]:(i + 1) * c["size"]] for i in range(len(uniq))])
    idmap = dict(zip(map(int, uniq), ids_u))
    ids = [idmap[int(s)] for s in src]
    assert hashlib.sha256("\n".join(ids).encode()).hexdigest() == c["ids_sha256"]
