"""Paged fp16 KV cache (the reference has none: runners/engine.py:90-91 hold
one token's k/v and seq_len is fixed at 1, engine.py:64).

Layout in HBM: K and V are each one tensor fp16
[n_layers, n_pages, n_kv_heads, page_size, head_dim]; a page holds
``page_size`` consecutive positions of one KV head of one sequence, so the
attention kernel reads a (page, head) tile as one contiguous 16 KB block
(page_size 64 x 128 x 2 bytes).  ``block_table`` int32 [max_batch,
pages_per_seq] maps page j of sequence slot b to a pool page.  Row i of the
reference's implied [T, n_kv_heads*128] cache (kernels/attention.metal:33)
is position i here.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from .config import ModelConfig


class PagedKVCache:
    def __init__(self, cfg: ModelConfig, n_layers: int, max_batch: int, max_seq_len: int,
                 page_size: int = 64, device="cuda", n_pages: Optional[int] = None,
                 page_order: Optional[List[int]] = None):
        if max_seq_len <= 0 or page_size <= 0 or max_batch <= 0:
            raise ValueError("max_seq_len, page_size and max_batch must be positive")
        self.cfg = cfg
        self.n_layers = n_layers
        self.page_size = page_size
        self.max_batch = max_batch
        self.pages_per_seq = (max_seq_len + page_size - 1) // page_size
        self.max_seq_len = self.pages_per_seq * page_size
        self.n_pages = n_pages if n_pages is not None else max_batch * self.pages_per_seq
        if self.n_pages < self.pages_per_seq:
            raise ValueError("pool smaller than one sequence")
        self.device = torch.device(device)
        shape = (n_layers, self.n_pages, cfg.n_kv_heads, page_size, cfg.head_dim)
        self.k = torch.zeros(shape, dtype=torch.float16, device=self.device)
        self.v = torch.zeros(shape, dtype=torch.float16, device=self.device)
        self.block_table = torch.zeros(max_batch, self.pages_per_seq, dtype=torch.int32, device=self.device)
        order = list(page_order) if page_order is not None else list(range(self.n_pages))
        if sorted(order) != list(range(self.n_pages)):
            raise ValueError("page_order must be a permutation of the pool's pages")
        self._free: List[int] = order[::-1]
        self._owned: List[List[int]] = [[] for _ in range(max_batch)]

    # -- page allocation ----------------------------------------------------
    def reserve(self, slot: int, n_positions: int) -> None:
        """Make positions [0, n_positions) of ``slot`` addressable."""
        need = (n_positions + self.page_size - 1) // self.page_size
        if need > self.pages_per_seq:
            raise ValueError(f"{n_positions} positions exceed the cache capacity {self.max_seq_len}")
        owned = self._owned[slot]
        new = []
        while len(owned) < need:
            if not self._free:
                raise MemoryError("KV page pool exhausted")
            owned.append(self._free.pop())
            new.append(len(owned) - 1)
        if new:
            idx = torch.tensor(new, dtype=torch.long)
            vals = torch.tensor([owned[j] for j in new], dtype=torch.int32)
            self.block_table[slot, idx.to(self.device)] = vals.to(self.device)

    def release(self, slot: int) -> None:
        self._free.extend(reversed(self._owned[slot]))
        self._owned[slot] = []

    def release_all(self) -> None:
        for s in range(self.max_batch):
            self.release(s)

    def pages(self, slot: int) -> List[int]:
        return list(self._owned[slot])

    # -- views ---------------------------------------------------------------
    def layer(self, layer: int):
        return self.k[layer], self.v[layer]

    def write_positions(self, slot: int, layer: int, start: int, k_rows: torch.Tensor,
                        v_rows: torch.Tensor) -> None:
        """Scatter rows [T, n_kv_heads*head_dim] into positions start.. of ``slot``."""
        cfg = self.cfg
        T = k_rows.shape[0]
        self.reserve(slot, start + T)
        kr = k_rows.to(self.device, torch.float16).reshape(T, cfg.n_kv_heads, cfg.head_dim)
        vr = v_rows.to(self.device, torch.float16).reshape(T, cfg.n_kv_heads, cfg.head_dim)
        pos = torch.arange(start, start + T, device=self.device)
        pages = self.block_table[slot, (pos // self.page_size)].long()
        off = pos % self.page_size
        for h in range(cfg.n_kv_heads):
            self.k[layer, pages, h, off] = kr[:, h]
            self.v[layer, pages, h, off] = vr[:, h]

    def read_positions(self, slot: int, layer: int, n: int):
        """Rows [n, n_kv_heads*head_dim] of positions 0..n-1 (a copy)."""
        cfg = self.cfg
        pos = torch.arange(n, device=self.device)
        pages = self.block_table[slot, (pos // self.page_size)].long()
        off = pos % self.page_size
        k = torch.stack([self.k[layer, pages, h, off] for h in range(cfg.n_kv_heads)], dim=1)
        v = torch.stack([self.v[layer, pages, h, off] for h in range(cfg.n_kv_heads)], dim=1)
        return k.reshape(n, -1), v.reshape(n, -1)
