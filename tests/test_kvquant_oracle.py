"""The INT8 KV compressor oracle (oracle/kvquant_oracle.c) pinned to the
reference's own outputs: tests/golden/kvquant_vectors.json was produced by
KVCompressor::compress/decompress (cascade_Code/cpp/src/cascade_core.cpp:
908-967) compiled from the reference sources (make_kvquant_golden.py)."""
import hashlib

import numpy as np
import pytest

from helpers import gen, load
from oracle import kvquant as KQ

VEC = load("kvquant_vectors.json")["vectors"]


@pytest.mark.parametrize("v", VEC, ids=lambda v: f"{v['kind']}-{v['size']}")
def test_oracle_matches_reference_vectors(v):
    a = gen(v["kind"], v["seed"], v["size"])
    assert hashlib.sha256(a.tobytes()).hexdigest() == v["input_sha256"]
    comp = KQ.compress(a)
    assert len(comp) == v["compressed_size"] == KQ.compressed_size(v["size"])
    assert comp[:64].hex() == v["compressed_head"]
    assert hashlib.sha256(comp).hexdigest() == v["compressed_sha256"]
    dec = KQ.decompress(comp, v["size"])
    assert len(dec) == v["decompressed_size"]
    assert hashlib.sha256(dec).hexdigest() == v["decompressed_sha256"]
    if "compressed" in v:
        assert comp.hex() == v["compressed"] and dec.hex() == v["decompressed"]


def test_header_fields():
    # max == min -> scale 1, zero point = low byte of min
    assert KQ.params(15360, 15360) == (1.0, 0)
    assert KQ.params(-32768, -32768) == (1.0, 0)
    assert KQ.params(-200, -200)[1] == 56  # -200 & 0xff as int8
    s, z = KQ.params(0, 255)
    assert s == 1.0 and z == 0
    # a mixed-sign fp16 block: min/scale leaves int8 and wraps
    s, z = KQ.params(-27000, 16000)
    assert s == np.float32(43000) / np.float32(255)
    assert z == np.int8(np.uint8(int(np.float32(-27000) / np.float32(s)) & 0xFF))


def test_decompress_short_buffer_fails():
    comp = KQ.compress(np.arange(64, dtype=np.uint8))
    assert KQ.decompress(comp[:-1], 64) is None
    assert KQ.decompress(comp, 64) is not None


def test_odd_size_drops_last_byte():
    a = gen("uniform_u8", 3, 101)
    comp = KQ.compress(a)
    assert len(comp) == 8 + 50
    assert len(KQ.decompress(comp, 101)) == 100


def _reference_module():
    import os
    import sys
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ref = os.path.join(here, "oracle", "_ref")
    if ref not in sys.path:
        sys.path.insert(0, ref)
    try:
        import cascade_ref  # the reference, compiled from its sources (oracle/Makefile)
    except ImportError:
        return None
    return cascade_ref if hasattr(cascade_ref, "kv_compress") else None


def test_oracle_matches_compiled_reference_on_random_blocks():
    ref = _reference_module()
    if ref is None:
        pytest.skip("oracle/_ref (the compiled reference) is not built here")
    rng = np.random.default_rng(2026)
    for t in range(300):
        kind = t % 5
        n = int(rng.integers(32, 3000))
        if kind == 0:
            a = rng.standard_normal(n).astype(np.float16).view(np.uint8)
        elif kind == 1:
            a = (rng.standard_normal(n) * 10 ** rng.uniform(-4, 4)).astype(np.float16).view(np.uint8)
        elif kind == 2:
            a = rng.integers(-32768, 32768, n, dtype=np.int64).astype(np.int16).view(np.uint8)
        elif kind == 3:
            a = rng.integers(0, 256, 2 * n + int(rng.integers(0, 2)), dtype=np.uint8)
        else:
            lo = int(rng.integers(-32768, 32767))
            a = rng.integers(lo, min(32768, lo + int(rng.integers(1, 600))), n).astype(np.int16).view(np.uint8)
        a = np.ascontiguousarray(a)
        comp = ref.kv_compress(a)
        assert KQ.compress(a) == comp, (t, kind, a.size)
        ok, dec = ref.kv_decompress(np.frombuffer(comp, np.uint8), a.size)
        assert ok and KQ.decompress(comp, a.size) == dec, (t, kind, a.size)
