"""Paged KV cache: one pool per model, block tables per sequence row.

Replaces the reference's slot-contiguous cache
``K[num_slots][max_seq_len][Hkv][D]`` (model/model.py:324-336,
model/model_tp.py:410-426).  A "slot" of the reference API is a row of
``block_tables``; its tokens live in fixed-size blocks drawn from a shared
free list, so a sequence only holds the blocks its length needs.

Device layout (bf16), allocated once and zero-filled:
    k, v: [num_layers][num_blocks][num_kv_heads][block_size][128]
Every (block, kv head) is one contiguous ``block_size x 256``-byte panel, the
unit the attention kernels stream with TMA.

Host bookkeeping (block free list, per-row lengths) lives here; the device
copies (``block_tables`` int32 [rows][max_blocks], ``seqlens`` int32 [rows])
are what the kernels read.
"""
from __future__ import annotations

import numpy as np
import torch


class PagedKVCache:
    def __init__(self, num_layers: int, num_kv_heads: int, num_rows: int, max_seq_len: int, *,
                 block_size: int = 256, num_blocks: int | None = None, head_dim: int = 128,
                 device="cuda", dtype=torch.bfloat16):
        if head_dim != 128:
            raise ValueError("the B200 kernels are built for head_dim 128 (all Qwen3 models)")
        if block_size % 64:
            raise ValueError("block_size must be a multiple of 64")
        self.num_layers, self.num_kv_heads, self.block_size = num_layers, num_kv_heads, block_size
        self.num_rows = num_rows
        self.max_blocks = (max_seq_len + block_size - 1) // block_size + 1
        self.max_seq_len = max_seq_len
        if num_blocks is None:
            num_blocks = num_rows * self.max_blocks
        self.num_blocks = num_blocks
        shape = (num_layers, num_blocks, num_kv_heads, block_size, head_dim)
        # Zero-filled: masked tail tokens of a tile are multiplied by p = 0,
        # so the pool must never hold non-finite values.
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.block_tables = torch.full((num_rows, self.max_blocks), -1, dtype=torch.int32, device=device)
        self.seqlens = torch.zeros(num_rows, dtype=torch.int32, device=device)
        self._bt_host = np.full((num_rows, self.max_blocks), -1, dtype=np.int32)
        self._nblk = np.zeros(num_rows, dtype=np.int64)
        self.lengths = np.zeros(num_rows, dtype=np.int64)  # host mirror of seqlens
        self._free = list(range(num_blocks - 1, -1, -1))  # pop() yields the lowest id
        self._dirty = False

    # ------------------------------------------------------------ blocks
    @property
    def free_blocks(self) -> int:
        return len(self._free)

    def reserve(self, row: int, length: int) -> None:
        """Make row `row` able to hold `length` tokens (allocating blocks)."""
        need = (length + self.block_size - 1) // self.block_size
        if need > self.max_blocks:
            raise ValueError(f"sequence length {length} exceeds the cache limit {self.max_blocks * self.block_size}")
        have = int(self._nblk[row])
        if need <= have:
            return
        if need - have > len(self._free):
            raise RuntimeError(f"KV pool exhausted: need {need - have} blocks, {len(self._free)} free")
        for j in range(have, need):
            self._bt_host[row, j] = self._free.pop()
        self._nblk[row] = need
        self._dirty = True

    def release(self, row: int) -> None:
        """Return a row's blocks to the pool and reset its length (clear_slot)."""
        n = int(self._nblk[row])
        for j in range(n - 1, -1, -1):
            self._free.append(int(self._bt_host[row, j]))
        self._free.sort(reverse=True)
        self._bt_host[row, :] = -1
        self._nblk[row] = 0
        self.lengths[row] = 0
        self._dirty = True

    def sync(self) -> None:
        """Upload the block tables if any row changed (one small H2D copy)."""
        if self._dirty:
            self.block_tables.copy_(torch.from_numpy(self._bt_host), non_blocking=False)
            self._dirty = False

    def set_lengths(self, rows, lengths) -> None:
        """Host + device lengths for rows after a prefill."""
        rows = list(rows)
        for r, n in zip(rows, lengths):
            self.lengths[r] = int(n)
        idx = torch.tensor(rows, dtype=torch.int64)
        vals = torch.tensor([int(n) for n in lengths], dtype=torch.int32)
        self.seqlens.index_copy_(0, idx.to(self.seqlens.device), vals.to(self.seqlens.device))

    def clear_all(self) -> None:
        for r in range(self.num_rows):
            if self._nblk[r]:
                self.release(r)
        self.lengths[:] = 0
        self.seqlens.zero_()
        self.sync()

    # ------------------------------------------------------------ mapping
    def slot_of(self, row: int, pos: int) -> int:
        """Flat cache slot of token `pos` of `row` (host mirror)."""
        return int(self._bt_host[row, pos // self.block_size]) * self.block_size + pos % self.block_size

    def slot_mapping(self, row: int, start: int, end: int) -> np.ndarray:
        pos = np.arange(start, end)
        return self._bt_host[row, pos // self.block_size].astype(np.int64) * self.block_size + pos % self.block_size

    def gather(self, layer: int, row: int, length: int) -> tuple[torch.Tensor, torch.Tensor]:
        """K, V of the first `length` tokens of `row` as [length, Hkv, 128] (test/export helper)."""
        pos = torch.arange(length)
        blk = torch.from_numpy(self._bt_host[row]).long()[pos // self.block_size].to(self.k.device)
        off = (pos % self.block_size).to(self.k.device)
        k = self.k[layer][blk, :, off]
        v = self.v[layer][blk, :, off]
        return k, v
