"""Paged-KV connector: moves the pages of an inference engine's paged KV
cache to and from a store without per-page tensors or staging copies.

The cache is one CUDA tensor whose first dimension indexes pages
(``kv_cache[p]`` is one page, contiguous); a page is one store block, keyed by
the SHA-256 block ID of its bytes (``compute_block_id``). ``save`` hashes and
stores the selected pages straight from the cache (``batch_put`` on pointers
into it), ``load`` gathers stored blocks straight into the selected page
slots (``batch_get`` on pointers into it). This is the caller-side step the
reference's benchmark adapters perform with one host copy per block
(benchmark/adapters/cascade_adapter.py:141-199).
"""
from __future__ import annotations

from typing import Sequence

import numpy as np

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None

from . import block_id_to_key, key_to_block_id


class KVPageConnector:
    def __init__(self, store, kv_cache):
        if torch is None or not isinstance(kv_cache, torch.Tensor) or not kv_cache.is_cuda:
            raise TypeError("kv_cache must be a CUDA tensor")
        if kv_cache.dim() < 1 or kv_cache.shape[0] == 0:
            raise ValueError("kv_cache needs a leading page dimension")
        if not kv_cache[0].is_contiguous():
            raise ValueError("each page kv_cache[p] must be contiguous")
        self.store = store
        self.cache = kv_cache
        self.num_pages = int(kv_cache.shape[0])
        self.page_bytes = kv_cache[0].numel() * kv_cache.element_size()
        self.base = kv_cache.data_ptr()
        self.stride = kv_cache.stride(0) * kv_cache.element_size()

    def _ptrs(self, pages: Sequence[int]) -> np.ndarray:
        p = np.asarray(pages, dtype=np.int64).reshape(-1)
        if p.size and (p.min() < 0 or p.max() >= self.num_pages):
            raise IndexError("page index out of range")
        return (np.uint64(self.base) + p.astype(np.uint64) * np.uint64(self.stride)).astype(np.uint64)

    def save(self, pages: Sequence[int], is_prefix: Sequence[bool] | None = None,
             return_status: bool = False):
        """Store the given pages; returns their block IDs (and the per-page
        status: 0 stored, 1 already stored, 2 no space)."""
        ptrs = self._ptrs(pages)
        sizes = np.full(len(ptrs), self.page_bytes, np.uint64)
        prefix = None if is_prefix is None else np.asarray(is_prefix, np.uint8).reshape(-1)
        keys, status = self.store.put_ptrs(ptrs, sizes, True, prefix=prefix)
        ids = [key_to_block_id(bytes(k)) for k in keys]
        return (ids, [int(s) for s in status]) if return_status else ids

    def load(self, ids: Sequence[str], pages: Sequence[int]) -> list[bool]:
        """Fill the given page slots with the stored blocks of ``ids``;
        returns, per page, whether its block was found and copied."""
        if len(ids) != len(pages):
            raise ValueError("ids and pages differ in length")
        outs = self._ptrs(pages)
        keys = np.frombuffer(b"".join(block_id_to_key(i) for i in ids), np.uint8).reshape(-1, 16).copy()
        caps = np.full(len(outs), self.page_bytes, np.uint64)
        sizes, found = self.store.get_ptrs(keys, outs, caps, True)
        return [bool((int(f) & 0x0F) != 0 and not (int(f) & 0x80) and int(s) == self.page_bytes)
                for s, f in zip(sizes, found)]
