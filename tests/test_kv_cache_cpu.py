"""Host bookkeeping of the paged KV cache on CPU tensors: block allocation
from the shared free list, release, slot mapping (the paged form of the
reference's flat index slot * max_seq_len + pos, llm.py:139-140) and gather."""
import numpy as np
import pytest
import torch

from awesome_acceleration_b200.kv_cache import PagedKVCache


def _cache(rows=4, max_seq_len=1000, bs=256, blocks=None):
    return PagedKVCache(2, 2, rows, max_seq_len, block_size=bs, num_blocks=blocks, device="cpu")


def test_reserve_allocates_lowest_free_blocks_and_release_returns_them():
    kv = _cache()
    kv.reserve(0, 300)          # 2 blocks
    kv.reserve(1, 1)            # 1 block
    kv.reserve(0, 512)          # still 2 blocks
    assert kv._bt_host[0, :2].tolist() == [0, 1] and kv._bt_host[1, 0] == 2
    kv.reserve(0, 513)          # a third block
    assert kv._bt_host[0, 2] == 3
    free0 = kv.free_blocks
    kv.release(0)
    assert kv.free_blocks == free0 + 3 and (kv._bt_host[0] == -1).all() and kv.lengths[0] == 0
    kv.reserve(2, 10)
    assert kv._bt_host[2, 0] == 0  # lowest id first again
    kv.sync()
    assert torch.equal(kv.block_tables, torch.from_numpy(kv._bt_host))


def test_limits_raise():
    kv = _cache(rows=2, max_seq_len=300, blocks=3)
    with pytest.raises(ValueError):
        kv.reserve(0, kv.max_blocks * 256 + 1)
    kv.reserve(0, 512)
    with pytest.raises(RuntimeError):
        kv.reserve(1, 512)  # 2 more blocks wanted, 1 free


def test_slot_mapping_and_gather_follow_the_block_table():
    kv = _cache(rows=3, max_seq_len=700, bs=64)
    rng = np.random.default_rng(0)
    kv.reserve(1, 10)
    kv.reserve(2, 200)          # interleaved allocation: row 2's blocks are not contiguous ids
    kv.reserve(1, 150)
    for row, n in ((1, 150), (2, 200)):
        sm = kv.slot_mapping(row, 0, n)
        assert sm.tolist() == [kv.slot_of(row, p) for p in range(n)]
        assert len(set(sm.tolist())) == n
        blk, off = sm // 64, sm % 64
        assert (off == np.arange(n) % 64).all() and (blk == kv._bt_host[row, np.arange(n) // 64]).all()
    assert not set(kv.slot_mapping(1, 0, 150)) & set(kv.slot_mapping(2, 0, 200))
    # write distinct values through the flat slots, read them back with gather
    flat_k = kv.k[1].view(kv.num_blocks, 2, 64, 128)
    vals = torch.from_numpy(rng.standard_normal((150, 2, 128)).astype(np.float32)).to(kv.k.dtype)
    for p, s in enumerate(kv.slot_mapping(1, 0, 150)):
        flat_k[s // 64, :, s % 64] = vals[p]
    k, _ = kv.gather(1, 1, 150)
    assert torch.equal(k, vals)


def test_set_lengths_and_clear_all():
    kv = _cache()
    kv.reserve(0, 5)
    kv.reserve(3, 700)
    kv.set_lengths([0, 3], [5, 700])
    assert kv.seqlens.tolist() == [5, 0, 0, 700] and kv.lengths.tolist() == [5, 0, 0, 700]
    kv.clear_all()
    assert kv.seqlens.tolist() == [0, 0, 0, 0] and (kv._bt_host == -1).all() and kv.free_blocks == kv.num_blocks
