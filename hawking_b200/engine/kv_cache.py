"""Paged KV cache storage on the device.

One bf16 tensor per K and V: [layers, num_blocks, n_kv_heads, block_size, head_dim]. A block holds
``block_size`` consecutive tokens of one sequence; each head's tokens inside a block are contiguous
so the decode kernel reads whole rows. Block allocation, prefix sharing and copy-on-write live in
the C++ ``BlockManager``; this class owns the memory and the device-side block tables.
"""
from __future__ import annotations

from typing import Dict, Iterable, List, Optional, Tuple

import torch

from .._ext import native


class PagedKVCache:
    def __init__(self, layers: int, n_kv_heads: int, head_dim: int, num_blocks: int, block_size: int,
                 max_seqs: int, max_blocks_per_seq: int, device, prefix_cache: bool = True,
                 dtype=torch.bfloat16):
        if num_blocks * block_size >= 2 ** 31:
            raise ValueError("KV pool too large for int32 slot ids")
        self.layers, self.nkv, self.hd = layers, n_kv_heads, head_dim
        self.num_blocks, self.block_size = num_blocks, block_size
        self.k = torch.zeros(layers, num_blocks, n_kv_heads, block_size, head_dim, dtype=dtype, device=device)
        self.v = torch.zeros_like(self.k)
        self.max_seqs, self.max_blocks = max_seqs, max_blocks_per_seq
        self.block_tables = torch.zeros(max_seqs, max_blocks_per_seq, dtype=torch.int32, device=device)
        self._host_tables = torch.zeros(max_seqs, max_blocks_per_seq, dtype=torch.int32).pin_memory() \
            if torch.cuda.is_available() else torch.zeros(max_seqs, max_blocks_per_seq, dtype=torch.int32)
        self.bm = native().BlockManager(num_blocks, block_size, prefix_cache)
        self._row_of: Dict[int, int] = {}
        self._free_rows: List[int] = list(range(max_seqs - 1, -1, -1))
        self._synced_len: Dict[int, int] = {}

    @staticmethod
    def bytes_per_block(layers: int, n_kv_heads: int, head_dim: int, block_size: int, elem_bytes: int = 2) -> int:
        return 2 * layers * n_kv_heads * block_size * head_dim * elem_bytes

    # ---- table rows (one per live sequence) ----
    def row(self, seq_id: int) -> int:
        r = self._row_of.get(seq_id)
        if r is None:
            if not self._free_rows:
                raise RuntimeError("no free block-table rows")
            r = self._free_rows.pop()
            self._row_of[seq_id] = r
            self._synced_len[seq_id] = 0
        return r

    def drop(self, seq_id: int):
        r = self._row_of.pop(seq_id, None)
        if r is not None:
            self._free_rows.append(r)
        self._synced_len.pop(seq_id, None)
        if self.bm.has(seq_id):
            self.bm.release(seq_id)

    def sync_tables(self, seq_ids: Iterable[int]):
        """Copy changed block-table rows to the device."""
        for s in seq_ids:
            t = self.bm.table(s)
            if len(t) > self.max_blocks:
                raise RuntimeError("sequence exceeds max_blocks_per_seq")
            if self._synced_len.get(s, -1) == len(t):
                continue
            r = self.row(s)
            self._host_tables[r, : len(t)] = torch.tensor(t, dtype=torch.int32)
            self.block_tables[r].copy_(self._host_tables[r], non_blocking=True)
            self._synced_len[s] = len(t)

    def copy_blocks(self, pairs: List[Tuple[int, int]]):
        for src, dst in pairs:
            self.k[:, dst].copy_(self.k[:, src])
            self.v[:, dst].copy_(self.v[:, src])
