"""The bench's roofline arithmetic (no GPU): algorithmic bytes of one decode
attention launch and of the cfg2 decode phase."""
import types

import bench


def test_attention_bytes_per_launch():
    ctx = [1, 256, 257, 2048]
    hq, hkv, bs = 16, 8, 256
    kv = sum(ctx) * hkv * 128 * 2 * 2          # K and V, bf16
    qo = len(ctx) * hq * 128 * 2 * 2           # q in, o out
    bt = sum((c + bs - 1) // bs for c in ctx) * 4
    assert bench.attention_bytes(ctx, hq, hkv, bs) == kv + qo + bt
    # cfg3 at its mean context: about 2.42 GB per launch
    assert abs(bench.attention_bytes([2304] * 256, 16, 8, 256) / 1e9 - 2.42) < 0.01


def test_cfg2_decode_phase_bytes_and_fraction():
    cfg2 = types.SimpleNamespace(prompt=1024, out=1024, n_seqs=256)
    cfg = types.SimpleNamespace(num_hidden_layers=28, num_key_value_heads=8, head_dim=128)
    ph = bench.phase_summary(cfg2, steps=1, elapsed=10.0, prefill_s=1.0, cfg=cfg)
    n_dec = 1023
    kv_tok = 2 * 28 * 8 * 128 * 2            # 114,688 B per token, all layers
    ctx_sum = sum(1024 + 1 + t for t in range(n_dec))
    expect = n_dec * 1.192e9 + 256 * kv_tok * (ctx_sum + n_dec)
    assert abs(ph["decode_hbm_bytes"] - expect) / expect < 1e-9
    pk, _ = bench.peaks()
    assert abs(ph["decode_roofline_frac"] - expect / (pk["hbm_gbs"] * 1e9) / 9.0) < 1e-3
    assert ph["decode_ms_per_step"] == round(9.0 / n_dec * 1e3, 3)
