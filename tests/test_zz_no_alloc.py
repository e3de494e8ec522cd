"""cb_hash_batch_noalloc: the allocation-free hashing entry point.

It exists for callers that may not allocate GPU memory while they hash (an
engine holding nearly all HBM in its own pool, code inside an allocator
callback). The test calls it through the C ABI and checks its digests against
the regular store-based entry point (cb_hash_batch), bit for bit, on two calls
in a row with different inputs — the second call reuses the static scratch the
first one left behind. This file is collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest

import cascade_cpp
from cascade_cpp import _lib as L

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def noalloc_digests(lib, blocks):
    out = torch.empty((len(blocks), 32), dtype=torch.uint8, device="cuda:0")
    ptrs = np.array([b.data_ptr() for b in blocks], np.uint64)
    sizes = np.array([b.numel() for b in blocks], np.uint64)
    torch.cuda.synchronize()
    rc = lib.cb_hash_batch_noalloc(0, C.c_void_p(ptrs.ctypes.data), C.c_void_p(sizes.ctypes.data), len(blocks),
                                   C.c_void_p(out.data_ptr()), None)
    assert rc == L.CB_OK, lib.cb_last_error(None)
    return out.cpu().numpy()


def store_digests(blocks):
    h = cascade_cpp._hasher(0)
    ptrs = np.array([b.data_ptr() for b in blocks], np.uint64)
    sizes = np.array([b.numel() for b in blocks], np.uint64)
    return h.hash(ptrs, sizes, L.CB_MEM_DEVICE)


def test_noalloc_matches_store_path_twice():
    lib = cascade_cpp._native_lib()
    rng = np.random.default_rng(42)
    for call in range(2):
        sizes = rng.integers(0, 300_000, 97 + 31 * call)
        sizes[:3] = [0, 55, 917504]
        blocks = [torch.from_numpy(rng.integers(0, 256, int(s), dtype=np.uint8)).to("cuda:0") for s in sizes]
        got = noalloc_digests(lib, blocks)
        want = store_digests(blocks)
        assert np.array_equal(got, want), f"call {call}"


def test_noalloc_rejects_oversize_batch():
    lib = cascade_cpp._native_lib()
    n = L.CB_NOALLOC_MAX_BLOCKS + 1
    block = torch.zeros(64, dtype=torch.uint8, device="cuda:0")
    ptrs = np.full(n, block.data_ptr(), np.uint64)
    sizes = np.full(n, 64, np.uint64)
    out = torch.empty((n, 32), dtype=torch.uint8, device="cuda:0")
    rc = lib.cb_hash_batch_noalloc(0, C.c_void_p(ptrs.ctypes.data), C.c_void_p(sizes.ctypes.data), n,
                                   C.c_void_p(out.data_ptr()), None)
    assert rc == L.CB_ERR_ARG
    assert b"CB_NOALLOC_MAX_BLOCKS" in lib.cb_last_error(None)
