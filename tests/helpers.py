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
    if kind == "kv_fp16_pos":  # one sign only: the zero point stays inside int8
        return np.abs(W.kv_block_fp16(seed, size).view(np.float16)).view(np.uint8)
    if kind == "kv_fp16_small":
        rng = np.random.default_rng(seed)
        return (rng.standard_normal(size // 2) * 1e-3).astype(np.float16).view(np.uint8)
    if kind == "int16_full":  # both int16 extremes present
        rng = np.random.default_rng(seed)
        v = rng.integers(-32768, 32768, size // 2, dtype=np.int64).astype(np.int16)
        v[: min(2, v.size)] = [-32768, 32767][: min(2, v.size)]
        return v.view(np.uint8)
    if kind == "const_i16":  # max == min: scale 1
        return np.full(size // 2, seed - 32768, np.int16).view(np.uint8)
    if kind == "fips_abc":
        return np.frombuffer(b"abc", np.uint8)
    if kind == "fips_448":
        return np.frombuffer(b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq", np.uint8)
    if kind == "fips_million_a":
        return np.full(1_000_000, ord("a"), np.uint8)
    raise ValueError(kind)
