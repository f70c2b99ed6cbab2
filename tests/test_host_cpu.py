"""Host-side policies of the B200 runtime that need no GPU: split-K choice,
decode-batch buckets, sampling seeds, the gate/up interleave."""
import torch

from awesome_acceleration_b200.kernels import pick_splits
from awesome_acceleration_b200.llm import sampling_seed
from awesome_acceleration_b200.runtime import Qwen3Runtime, interleave_gate_up


def test_pick_splits_invariants_and_cfg2_choices():
    for M in (1, 16, 128, 200, 256, 512):
        for N, K in ((4096, 1024), (6144, 1024), (1024, 2048), (1024, 3072), (1536, 4096), (4096, 1536)):
            d = pick_splits(M, N, K, max_elems=8 << 20)
            tiles = ((N + 127) // 128) * ((M + 127) // 128)
            assert (K // 64) % d == 0 and (d == 1 or tiles * d <= 148) and d * M * N <= 8 << 20
            assert d == 1 or 2 * d * M <= K  # fp32 partials no more bytes than the weights
    # the cfg2 decode step (M = 256): QKV 2, gate/up 1, o_proj 4, down_proj 6
    assert [pick_splits(256, n, k, max_elems=8 << 20) for n, k in ((4096, 1024), (6144, 1024), (1024, 2048),
                                                                    (1024, 3072))] == [2, 1, 4, 6]


def test_pick_skinny_splits_invariants():
    """Small-batch GEMM split counts: a divisor of K/64 (at most 64, which the
    tensor-parallel exchange takes), at most `target` CTAs unless the weight
    tiles alone exceed it, fp32 partials at most half the weight bytes."""
    from awesome_acceleration_b200.kernels import pick_skinny_splits
    shapes = ((4096, 1024), (6144, 1024), (1024, 2048), (1024, 3072), (6144, 4096), (24576, 4096), (4096, 12288),
              (512, 512), (1536, 4096))
    for M in (1, 8, 16, 32, 64):
        for N, K in shapes:
            for target in (148, 296, 444):
                d = pick_skinny_splits(M, N, K, target=target, max_elems=8 << 20)
                tiles = N // 128
                assert (K // 64) % d == 0 and 1 <= d <= 64
                assert d == 1 or (tiles * d <= target and 4 * d * M <= K and d * M * N <= 8 << 20)
                # the largest such divisor
                bigger = [e for e in range(d + 1, min(K // 64, 64) + 1) if (K // 64) % e == 0 and
                          tiles * e <= target and 4 * e * M <= K and e * M * N <= 8 << 20]
                assert not bigger, (M, N, K, target, d, bigger)
    # Qwen3-0.6B decode at one row, two CTAs per SM: QKV 8, gate/up 4, o 32, down 24
    assert [pick_skinny_splits(1, n, k) for n, k in ((4096, 1024), (6144, 1024), (1024, 2048), (1024, 3072))] == \
        [8, 4, 32, 24]


class _Rt:
    padded_batch = Qwen3Runtime.padded_batch

    def __init__(self, max_batch, graphs=True):
        self.max_batch, self.use_graphs = max_batch, graphs


def test_decode_batch_buckets():
    rt = _Rt(512)
    sizes = [rt.padded_batch(b) for b in range(1, 513)]
    assert all(b <= p <= 512 for b, p in zip(range(1, 513), sizes))
    assert sizes == sorted(sizes) and len(set(sizes)) <= 25  # 4 powers of two, 7 multiples of 8, 14 of 32
    assert [rt.padded_batch(b) for b in (1, 3, 5, 9, 63, 65, 256, 257)] == [1, 4, 8, 16, 64, 96, 256, 288]
    assert _Rt(434).padded_batch(430) == 434  # capped at max_batch
    assert _Rt(512, graphs=False).padded_batch(37) == 37  # eager runs the exact size


def test_sampling_seeds_are_distinct_int64():
    seeds = {sampling_seed(b, s, i) for b in (0, 1, 7) for s in range(1, 200) for i in range(8)}
    assert len(seeds) == 3 * 199 * 8
    assert all(0 <= x < 2 ** 63 for x in seeds)


def test_gate_up_interleave_groups_of_64():
    I, H = 256, 8
    gate = torch.arange(I).float().unsqueeze(1).expand(I, H)
    up = (1000 + torch.arange(I)).float().unsqueeze(1).expand(I, H)
    w = interleave_gate_up(gate, up)
    for j in range(I // 64):
        assert torch.equal(w[128 * j:128 * j + 64, 0], torch.arange(64 * j, 64 * j + 64).float())
        assert torch.equal(w[128 * j + 64:128 * j + 128, 0], 1000 + torch.arange(64 * j, 64 * j + 64).float())


def test_decode_batch_may_hold_every_kv_slot():
    """A decode step may hold every KV slot: with more than 256 slots (the
    Qwen3-32B model at TP4 holds ~450 sequences) the runtime's batch
    capacity is the slot count, so the scheduler can never build a decode
    batch larger than the buffers and graphs it stages into."""
    from awesome_acceleration_b200.model.model import Qwen3Config, Qwen3ForCausalLM
    from oracle.weights import TINY
    cfg = Qwen3Config(**{k: v for k, v in TINY.as_dict().items() if k in Qwen3Config.__annotations__})
    with torch.device("meta"):
        m = Qwen3ForCausalLM(cfg)
    m = m.to_empty(device="cpu").to(torch.bfloat16)
    for slots in (3, 256, 300, 450):
        m.init_kv_cache(slots, 16, torch.device("cpu"), torch.bfloat16, num_blocks=slots)
        assert m.max_batch == slots
    m.init_kv_cache(300, 16, torch.device("cpu"), torch.bfloat16, num_blocks=300, max_batch=64)
    assert m.max_batch == 64
