"""Seeded synthetic KV-block workloads with the shapes of the Cascade configs.

No dataset is involved: the reference's drivers generate blocks the same way
(seeded normal fp16 KV tensors, benchmark/scripts/v6_distributed_bench.py:42-54;
uniform bytes, script_example/01_throughput_scalability/throughput_driver.py:
71-83). Block sizes:

* Qwen2.5-7B : 28 layers x (K,V) x 4 KV heads x 128 x 16 tokens x 2 B = 917,504 B
* Qwen2.5-72B: 80 layers x (K,V) x 8 KV heads x 128 x 16 tokens x 2 B = 5,242,880 B
"""
from __future__ import annotations

import numpy as np

QWEN7B_BLOCK = 28 * 2 * 4 * 128 * 16 * 2
QWEN72B_BLOCK = 80 * 2 * 8 * 128 * 16 * 2


def kv_block_fp16(seed: int, nbytes: int = QWEN7B_BLOCK) -> np.ndarray:
    """N(0,1) fp16 values from default_rng(seed), as a uint8 byte view."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal(nbytes // 2).astype(np.float16).view(np.uint8)


def kv_block_bf16(seed: int, nbytes: int = QWEN72B_BLOCK) -> np.ndarray:
    """N(0,1) bf16 values (fp32 draws truncated to their upper 16 bits)."""
    rng = np.random.default_rng(seed)
    f = rng.standard_normal(nbytes // 2, dtype=np.float32)
    return (f.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)


def uniform_block(seed: int, nbytes: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, 256, nbytes, dtype=np.uint8)


def dedup_mix(n_blocks: int, n_prefix: int, dup_frac: float, seed: int):
    """Order of a put stream where ``dup_frac`` of the blocks are byte-identical
    copies of ``n_prefix`` prefix blocks (equal copies per prefix block).

    Returns ``(src, is_prefix)``: ``src[i]`` is the unique-block index put at
    position i (indices < n_prefix are prefix blocks), positions shuffled with
    default_rng(seed). Expected: n_blocks - n_dups unique IDs and n_dups dedup
    hits under sequential dedup.
    """
    n_dups = int(round(n_blocks * dup_frac))
    n_unique = n_blocks - n_dups
    assert n_prefix <= n_unique and n_dups % max(n_prefix, 1) == 0
    src = np.concatenate([np.arange(n_unique), np.repeat(np.arange(n_prefix), n_dups // max(n_prefix, 1))])
    src = np.random.default_rng(seed).permutation(src)
    return src, src < n_prefix


def zipf_keys(n_keys: int, n_draws: int, alpha: float, seed: int) -> np.ndarray:
    """Bounded Zipf draws: p(rank k) ~ k^-alpha over n_keys, seeded rank->key
    permutation."""
    rng = np.random.default_rng(seed)
    p = np.arange(1, n_keys + 1, dtype=np.float64) ** (-alpha)
    p /= p.sum()
    ranks = rng.choice(n_keys, size=n_draws, p=p)
    perm = rng.permutation(n_keys)
    return perm[ranks]
