"""Generates tests/golden/kvquant_vectors.json from the REFERENCE itself.

Run in a container that has the reference sources (it builds oracle/_ref with
`make -C oracle ref` first):

    python tests/golden/make_kvquant_golden.py

Every expected value is the output of the reference's own INT8 KV compressor,
KVCompressor::compress / decompress (cascade_Code/cpp/src/cascade_core.cpp:
908-967), compiled from its sources with the reference's Release arithmetic
(oracle/Makefile REF_CXXFLAGS) and called through oracle/_ref/cascade_ref.
Blocks are not stored: each entry names the seeded generator
(tests/helpers.gen) that rebuilds its bytes. Small cases keep the whole
compressed block; large ones its SHA-256, the first 64 bytes, and the SHA-256
of the decompressed block.
"""
from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "kcj-cascade-v6_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle", "_ref"))
sys.path.insert(0, os.path.dirname(HERE))

from helpers import gen  # noqa: E402

CASES = [
    ("uniform_u8", 1, 64), ("uniform_u8", 2, 65), ("uniform_u8", 3, 66), ("uniform_u8", 4, 127),
    ("uniform_u8", 5, 200), ("uniform_u8", 6, 4097), ("uniform_u8", 7, 65537),
    ("kv_fp16", 11, 64), ("kv_fp16", 12, 256), ("kv_fp16", 13, 4096), ("kv_fp16", 14, 917504),
    ("kv_fp16_pos", 21, 96), ("kv_fp16_pos", 22, 4096), ("kv_fp16_pos", 23, 917504),
    ("kv_fp16_small", 31, 128), ("kv_fp16_small", 32, 65536),
    ("int16_full", 41, 64), ("int16_full", 42, 8192), ("int16_full", 43, 1048576 + 6),
    ("const_i16", 32768 + 15360, 64), ("const_i16", 0, 1000), ("const_i16", 65535, 130),
    ("kv_bf16", 51, 4096), ("kv_bf16", 52, 5242880),
]
FULL_MAX = 512  # compressed blocks up to this size are stored whole


def main():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref"], check=True)
    import cascade_ref  # noqa: E402  (the reference, compiled from its sources)

    out = []
    for kind, seed, size in CASES:
        a = np.ascontiguousarray(gen(kind, seed, size))
        assert a.size == size, (kind, size, a.size)
        comp = cascade_ref.kv_compress(a)
        ok, dec = cascade_ref.kv_decompress(np.frombuffer(comp, np.uint8), size)
        assert ok and len(comp) == 8 + size // 2 and len(dec) == size // 2 * 2
        e = {"kind": kind, "seed": seed, "size": size,
             "input_sha256": hashlib.sha256(a.tobytes()).hexdigest(),
             "compressed_size": len(comp),
             "compressed_sha256": hashlib.sha256(comp).hexdigest(),
             "compressed_head": comp[:64].hex(),
             "decompressed_size": len(dec),
             "decompressed_sha256": hashlib.sha256(dec).hexdigest()}
        if len(comp) <= FULL_MAX:
            e["compressed"] = comp.hex()
            e["decompressed"] = dec.hex()
        out.append(e)
    doc = {"source": "KVCompressor::compress/decompress, cascade_Code/cpp/src/cascade_core.cpp:908-967, "
                     "compiled by oracle/Makefile (REF_CXXFLAGS) and called via oracle/ref_shim.cpp",
           "format": "[f32 scale][i8 zero_point][3 zero pad][size/2 x i8]",
           "vectors": out}
    with open(os.path.join(HERE, "kvquant_vectors.json"), "w") as f:
        json.dump(doc, f, indent=1)
    print(f"wrote {len(out)} vectors")


if __name__ == "__main__":
    main()
