"""cb_hash_batch_noalloc: the allocation-free hashing entry point.

It exists for callers that may not allocate GPU memory while they hash: a
serving engine that reserved nearly all HBM for its own KV-cache pool and
forbids cudaMalloc while it serves, or code running inside an allocator
callback, which must not re-enter the allocator. The tests call it through
the C ABI and check:

* its digests against hashlib's SHA-256, bit for bit, on two calls in a row
  with different inputs (the second call reuses the static scratch the first
  one left behind);
* in a fresh process, that after the set-up call (n = 0) two hashing calls
  leave the device's free memory exactly where it was, i.e. nothing was
  allocated, and that the digests of that process are right too;
* that a call on a stream under capture is refused before it enqueues
  anything, and that oversize batches are refused.

This file is collected last on purpose.
"""
import ctypes as C
import hashlib
import json
import os
import subprocess
import sys

import numpy as np
import pytest

import cascade_cpp
from cascade_cpp import _lib as L

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def noalloc_digests(lib, blocks, stream=None):
    out = torch.empty((len(blocks), 32), dtype=torch.uint8, device="cuda:0")
    ptrs = np.array([b.data_ptr() for b in blocks], np.uint64)
    sizes = np.array([b.numel() for b in blocks], np.uint64)
    torch.cuda.synchronize()
    rc = lib.cb_hash_batch_noalloc(0, C.c_void_p(ptrs.ctypes.data), C.c_void_p(sizes.ctypes.data), len(blocks),
                                   C.c_void_p(out.data_ptr()), stream)
    assert rc == L.CB_OK, lib.cb_last_error(None)
    return out.cpu().numpy()


def test_noalloc_matches_sha256_twice():
    lib = cascade_cpp._native_lib()
    rng = np.random.default_rng(42)
    for call in range(2):
        sizes = rng.integers(0, 300_000, 97 + 31 * call)
        sizes[:4] = [0, 55, 64, 917504]
        host = [rng.integers(0, 256, int(s), dtype=np.uint8) for s in sizes]
        blocks = [torch.from_numpy(h).to("cuda:0") for h in host]
        got = noalloc_digests(lib, blocks)
        want = np.array([np.frombuffer(hashlib.sha256(h.tobytes()).digest(), np.uint8) for h in host])
        assert np.array_equal(got, want), f"call {call}"


def test_noalloc_allocates_nothing_in_a_fresh_process():
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([os.path.join(os.path.dirname(HERE), "kcj-cascade-v6_b200"),
                                         env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, os.path.join(HERE, "noalloc_child.py")], capture_output=True, text=True,
                       env=env, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["digests_ok"], res
    # after the set-up call, hashing calls change no free device memory
    assert res["free_after_setup"] == res["free_after_call1"] == res["free_after_call2"], res


def test_noalloc_refuses_a_capturing_stream():
    lib = cascade_cpp._native_lib()
    block = torch.zeros(64, dtype=torch.uint8, device="cuda:0")
    out = torch.empty((1, 32), dtype=torch.uint8, device="cuda:0")
    ptrs = np.array([block.data_ptr()], np.uint64)
    sizes = np.array([64], np.uint64)
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=s):
        rc = lib.cb_hash_batch_noalloc(0, C.c_void_p(ptrs.ctypes.data), C.c_void_p(sizes.ctypes.data), 1,
                                       C.c_void_p(out.data_ptr()), C.c_void_p(s.cuda_stream))
        out.add_(0)  # the capture itself is still valid after the refusal
    assert rc == L.CB_ERR_ARG
    assert b"captured" in lib.cb_last_error(None)
    del g
    # and the entry point still works afterwards
    assert np.array_equal(noalloc_digests(lib, [block])[0],
                          np.frombuffer(hashlib.sha256(bytes(64)).digest(), np.uint8))


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
