"""Child process of tests/test_zz_no_alloc.py: cb_hash_batch_noalloc in a
fresh process (nothing of the library has run on the GPU yet).

Inputs and outputs are allocated first; then the device's free memory is
read before the set-up call (n = 0), after it, and after each of two hashing
calls. Prints one JSON line."""
import ctypes as C
import hashlib
import json

import numpy as np
import torch

import cascade_cpp
from cascade_cpp import _lib as L


def main():
    lib = cascade_cpp._native_lib()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(9)
    calls = []
    for n in (64, 200):
        sizes = rng.integers(1, 200_000, n)
        host = [rng.integers(0, 256, int(s), dtype=np.uint8) for s in sizes]
        blocks = [torch.from_numpy(h).to(dev) for h in host]
        out = torch.zeros((n, 32), dtype=torch.uint8, device=dev)
        ptrs = np.array([b.data_ptr() for b in blocks], np.uint64)
        szs = np.array([b.numel() for b in blocks], np.uint64)
        calls.append((host, blocks, out, ptrs, szs))
    torch.cuda.synchronize()
    free = {"free_before_setup": torch.cuda.mem_get_info(0)[0]}
    rc = lib.cb_hash_batch_noalloc(0, None, None, 0, None, None)
    assert rc == L.CB_OK, lib.cb_last_error(None)
    free["free_after_setup"] = torch.cuda.mem_get_info(0)[0]
    ok = True
    for k, (host, blocks, out, ptrs, szs) in enumerate(calls):
        rc = lib.cb_hash_batch_noalloc(0, C.c_void_p(ptrs.ctypes.data), C.c_void_p(szs.ctypes.data), len(blocks),
                                       C.c_void_p(out.data_ptr()), None)
        assert rc == L.CB_OK, lib.cb_last_error(None)
        free[f"free_after_call{k + 1}"] = torch.cuda.mem_get_info(0)[0]
        got = out.cpu().numpy()
        want = np.array([np.frombuffer(hashlib.sha256(h.tobytes()).digest(), np.uint8) for h in host])
        ok = ok and bool(np.array_equal(got, want))
    print(json.dumps({**free, "digests_ok": ok}))


if __name__ == "__main__":
    main()
