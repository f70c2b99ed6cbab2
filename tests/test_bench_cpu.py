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


def _streamed_param_bytes(cfg):
    """bf16 bytes of the projection weights plus the lm_head, counted from the
    model's own parameters (meta device): what one decode step streams."""
    import torch
    from awesome_acceleration_b200.model.model import Qwen3ForCausalLM
    with torch.device("meta"):
        m = Qwen3ForCausalLM(cfg)
    n = sum(p.numel() for name, p in m.named_parameters() if name.endswith("proj.weight"))
    head = m.model.embed_tokens.weight if m.lm_head is None else m.lm_head.weight
    return 2 * (n + head.numel())


def test_weight_bytes_match_the_model():
    from awesome_acceleration_b200.model.model import Qwen3Config
    c06 = Qwen3Config()
    assert bench.weight_bytes(c06) == _streamed_param_bytes(c06)
    assert abs(bench.weight_bytes(c06) / 1e9 - 1.19) < 0.01  # Qwen3-0.6B: ~1.19 GB per step
    c8 = Qwen3Config(**bench.QWEN3_8B_KW)
    assert bench.weight_bytes(c8) == _streamed_param_bytes(c8)
    assert bench.weight_bytes(c8, tp=4) == bench.weight_bytes(c8) / 4


def test_cfg2_decode_phase_bytes_and_fraction():
    from awesome_acceleration_b200.model.model import Qwen3Config
    cfg2 = types.SimpleNamespace(prompt=1024, out=1024, n_seqs=256)
    cfg = Qwen3Config()
    ph = bench.phase_summary(cfg2, steps=1, elapsed=10.0, prefill_s=1.0, cfg=cfg)
    n_dec = 1023
    kv_tok = 2 * 28 * 8 * 128 * 2            # 114,688 B per token, all layers
    ctx_sum = sum(1024 + 1 + t for t in range(n_dec))
    expect = n_dec * _streamed_param_bytes(cfg) + 256 * kv_tok * (ctx_sum + n_dec)
    assert abs(ph["decode_hbm_bytes"] - expect) / expect < 1e-9
    pk, _ = bench.peaks()
    assert abs(ph["decode_roofline_frac"] - expect / (pk["hbm_gbs"] * 1e9) / 9.0) < 1e-3
    assert ph["decode_ms_per_step"] == round(9.0 / n_dec * 1e3, 3)
