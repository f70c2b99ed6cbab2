"""Seeded random-init Qwen3 weights shared by the oracle, the golden-vector
generator and the GPU parity tests (test infrastructure).

Key names follow the reference checkpoint layout read by
``Qwen3ForCausalLM.from_pretrained`` (reference model/model.py:353-384) so the
same dict loads into the reference model, the oracle and the B200 model.

Every Linear / Embedding weight is N(0, std) drawn from one CPU
``torch.Generator`` in a fixed order; RMSNorm weights are ones (the
reference's own init, model/model.py:42) unless ``norm_jitter`` > 0, which
draws ``1 + norm_jitter * N(0,1)`` to exercise the weight multiply.
"""
from __future__ import annotations

from dataclasses import dataclass, asdict
import torch


@dataclass
class Qwen3Arch:
    """Architecture fields of the reference ``Qwen3Config`` (model/model.py:13-37)."""
    vocab_size: int = 151936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    max_position_embeddings: int = 40960
    rope_theta: float = 1000000.0
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = True
    bos_token_id: int = 151643
    eos_token_id: int = 151645

    def as_dict(self) -> dict:
        return asdict(self)


# Architectures named by the benchmark configs.
QWEN3_0_6B = Qwen3Arch()
QWEN3_8B = Qwen3Arch(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                     num_attention_heads=32, num_key_value_heads=8, tie_word_embeddings=False)
QWEN3_32B = Qwen3Arch(hidden_size=5120, intermediate_size=25600, num_hidden_layers=64,
                      num_attention_heads=64, num_key_value_heads=8, tie_word_embeddings=False)
# Small architectures for fast parity tests (same head_dim as every Qwen3).
TINY = Qwen3Arch(vocab_size=4096, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                 num_attention_heads=4, num_key_value_heads=2)
TINY_G4 = Qwen3Arch(vocab_size=3000, hidden_size=512, intermediate_size=768, num_hidden_layers=2,
                    num_attention_heads=8, num_key_value_heads=2)
# Qwen3-8B layer shapes and vocabulary with two layers (tensor-parallel parity case).
TP8B_2L = Qwen3Arch(hidden_size=4096, intermediate_size=12288, num_hidden_layers=2, num_attention_heads=32,
                    num_key_value_heads=8, tie_word_embeddings=False)


def init_weights(arch: Qwen3Arch, seed: int, std: float = 0.02, norm_jitter: float = 0.0,
                 dtype: torch.dtype = torch.float32) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    H, I, V = arch.hidden_size, arch.intermediate_size, arch.vocab_size
    D, Hq, Hkv = arch.head_dim, arch.num_attention_heads, arch.num_key_value_heads
    sd: dict[str, torch.Tensor] = {}

    def lin(name, shape):
        sd[name] = (torch.randn(shape, generator=g) * std).to(dtype)

    def norm(name, n):
        if norm_jitter > 0:
            sd[name] = (1.0 + norm_jitter * torch.randn(n, generator=g)).to(dtype)
        else:
            sd[name] = torch.ones(n, dtype=dtype)

    lin("model.embed_tokens.weight", (V, H))
    for i in range(arch.num_hidden_layers):
        p = f"model.layers.{i}."
        norm(p + "input_layernorm.weight", H)
        lin(p + "self_attn.q_proj.weight", (Hq * D, H))
        lin(p + "self_attn.k_proj.weight", (Hkv * D, H))
        lin(p + "self_attn.v_proj.weight", (Hkv * D, H))
        lin(p + "self_attn.o_proj.weight", (H, Hq * D))
        norm(p + "self_attn.q_norm.weight", D)
        norm(p + "self_attn.k_norm.weight", D)
        norm(p + "post_attention_layernorm.weight", H)
        lin(p + "mlp.gate_proj.weight", (I, H))
        lin(p + "mlp.up_proj.weight", (I, H))
        lin(p + "mlp.down_proj.weight", (H, I))
    norm("model.norm.weight", H)
    if not arch.tie_word_embeddings:
        lin("lm_head.weight", (V, H))
    return sd


def random_prompts(n: int, length: int, vocab: int, seed: int) -> list[list[int]]:
    """Uniform-random prompt token ids, as the benchmark configs specify."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n, length), generator=g).tolist()
