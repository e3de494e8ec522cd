"""Shared test helpers: golden fixture loading and the seeded generators
the fixtures name."""
import json
import os

import numpy as np

from cascade_cpp import workloads as W

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    with open(os.path.join(GOLD, name)) as f:
        return json.load(f)


def gen(kind, seed, size):
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
