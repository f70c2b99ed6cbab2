"""Single-GPU Qwen3 with the reference's module interface on B200 kernels.

Mirrors yijichar/AWesome_ACceleration model/model.py: the same class names,
attribute names (``model.embed_tokens``, ``layers[i].self_attn._qkv_proj``,
``q_norm``, ``k_norm``, ``o_proj``, ``mlp.gate_proj`` ...), ``forward``
signature and KV-cache methods, so code written against the reference keeps
working.  The forward pass itself runs on the fused sm_100a kernels through
``awesome_acceleration_b200.runtime.Qwen3Runtime``; there is no eager-PyTorch
fallback.

Differences the caller can see:
  * the KV cache is paged (block tables, block_size 256) instead of
    slot-contiguous; ``_kv_cache`` / ``_v_cache`` are the layer's views of the
    paged pool ``[num_blocks][Hkv][block_size][128]`` and ``_cache_seqlens``
    is one tensor shared by all layers;
  * ``fuse_qkv()`` also builds the interleaved gate/up weight the fused
    SiLU-mul GEMM reads.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import torch
import torch.nn as nn

from .. import kernels as K
from ..kv_cache import PagedKVCache
from ..runtime import LayerWeights, Qwen3Runtime, interleave_gate_up, rope_table


@dataclass
class Qwen3Config:
    """Qwen 3 model configuration (model/model.py:13-37)."""
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
    hidden_act: str = "silu"
    tie_word_embeddings: bool = True
    bos_token_id: int = 151643
    eos_token_id: int = 151645

    @classmethod
    def from_json(cls, path: str):
        with open(path) as f:
            data = json.load(f)
        return cls(**{k: v for k, v in data.items() if k in cls.__annotations__})


class RMSNorm(nn.Module):
    """RMSNorm (model/model.py:40-52); forward runs aacc_rmsnorm."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, hidden_states):
        return K.rmsnorm(hidden_states.contiguous(), self.weight, self.eps)


class RotaryEmbedding(nn.Module):
    """Holds the reference's RoPE parameters (model/model.py:55-70).  The
    rotation itself is fused into the QKV GEMM epilogue; the table the
    kernels read is ``Qwen3ForCausalLM.rope`` ([max_pos][cos 64 | sin 64])."""

    def __init__(self, dim: int, max_position_embeddings: int = 2048, base: float = 10000.0):
        super().__init__()
        self.dim = dim
        self.max_position_embeddings = max_position_embeddings
        self.base = base
        inv_freq = 1.0 / (self.base ** (torch.arange(0, self.dim, 2).float() / self.dim))
        self.register_buffer("inv_freq", inv_freq, persistent=False)


class Attention(nn.Module):
    """GQA attention block parameters (model/model.py:102-154)."""

    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.head_dim = config.head_dim
        self.num_kv_groups = self.num_heads // self.num_kv_heads
        self._q_size = self.num_heads * self.head_dim
        self._kv_size = self.num_kv_heads * self.head_dim
        self.q_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.k_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self._qkv_proj = None
        self.q_proj = nn.Linear(self.hidden_size, self._q_size, bias=False)
        self.k_proj = nn.Linear(self.hidden_size, self._kv_size, bias=False)
        self.v_proj = nn.Linear(self.hidden_size, self._kv_size, bias=False)
        self.o_proj = nn.Linear(self._q_size, self.hidden_size, bias=False)
        self.rotary_emb = RotaryEmbedding(self.head_dim, config.max_position_embeddings, config.rope_theta)
        self.scaling = self.head_dim ** -0.5
        self._kv_cache = None
        self._v_cache = None
        self._cache_seqlens = None

    def fuse_qkv(self):
        """Concatenate [Q | K | V] rows into ``_qkv_proj`` (model/model.py:132-154)."""
        if self._qkv_proj is not None:
            return
        w = self.q_proj.weight
        self._qkv_proj = nn.Linear(self.hidden_size, self._q_size + 2 * self._kv_size, bias=False,
                                   device=w.device, dtype=w.dtype)
        with torch.no_grad():
            self._qkv_proj.weight.copy_(torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight], 0))
        del self.q_proj, self.k_proj, self.v_proj
        self.q_proj = self.k_proj = self.v_proj = None


class MLP(nn.Module):
    """SwiGLU MLP parameters (model/model.py:180-190)."""

    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.gate_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.down_proj = nn.Linear(config.intermediate_size, config.hidden_size, bias=False)
        self.act_fn = nn.SiLU()
        self._gate_up = None

    def fuse_gate_up(self):
        """Interleave gate/up rows into the layout the fused SiLU GEMM reads, then
        release the separate gate/up weights (their values live on in the fused
        copy), so the weights are held once."""
        if self._gate_up is not None:
            return
        with torch.no_grad():
            self._gate_up = interleave_gate_up(self.gate_proj.weight, self.up_proj.weight).contiguous()
            for lin in (self.gate_proj, self.up_proj):
                lin.weight.data = lin.weight.data.new_empty(0)


class TransformerBlock(nn.Module):
    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.self_attn = Attention(config)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.mlp = MLP(config)


class Qwen3Model(nn.Module):
    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([TransformerBlock(config) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)


class Qwen3ForCausalLM(nn.Module):
    """Qwen3 with LM head (model/model.py:289-401) on the B200 hot path."""

    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.config = config
        self.model = Qwen3Model(config)
        self.lm_head = None if config.tie_word_embeddings else nn.Linear(config.hidden_size, config.vocab_size,
                                                                        bias=False)
        self.kv: PagedKVCache | None = None
        self.runtime: Qwen3Runtime | None = None
        self.rope = None
        self.max_batch = 256
        self.use_cuda_graphs = True
        self.prefill_chunk_tokens = 32768

    # ------------------------------------------------------------------ setup
    def fuse_qkv(self):
        """Fuse QKV (and gate/up) projections of every layer."""
        for layer in self.model.layers:
            layer.self_attn.fuse_qkv()
            layer.mlp.fuse_gate_up()
        self.runtime = None

    def _lm_head_weight(self):
        return self.model.embed_tokens.weight if self.lm_head is None else self.lm_head.weight

    def init_kv_cache(self, num_slots: int, max_seq_len: int, device, dtype, *, block_size: int = 256,
                      num_blocks: int | None = None, max_batch: int | None = None):
        """Allocate the paged KV pool for `num_slots` sequences of up to
        `max_seq_len` tokens (model/model.py:324-336)."""
        if dtype != torch.bfloat16:
            raise ValueError("the B200 hot path computes in bf16")
        cfg = self.config
        self.kv = PagedKVCache(cfg.num_hidden_layers, cfg.num_key_value_heads, num_slots, max_seq_len,
                               block_size=block_size, num_blocks=num_blocks, device=device, dtype=dtype)
        self.max_batch = max_batch or num_slots or 1  # a decode step may hold every slot
        for i, layer in enumerate(self.model.layers):
            attn = layer.self_attn
            attn._kv_cache = self.kv.k[i]
            attn._v_cache = self.kv.v[i]
            attn._cache_seqlens = self.kv.seqlens
        self.runtime = None

    def _rt(self) -> Qwen3Runtime:
        if self.runtime is None:
            if self.kv is None:
                raise RuntimeError("KV cache is not initialized")
            cfg = self.config
            dev = self.model.embed_tokens.weight.device
            if self.rope is None or self.rope.device != dev:
                self.rope = rope_table(cfg.max_position_embeddings, cfg.head_dim, cfg.rope_theta, dev)
            layers = []
            for layer in self.model.layers:
                a, m = layer.self_attn, layer.mlp
                if a._qkv_proj is None or m._gate_up is None:
                    raise RuntimeError("call fuse_qkv() before running the model")
                layers.append(LayerWeights(layer.input_layernorm.weight.data, a._qkv_proj.weight.data,
                                           a.q_norm.weight.data, a.k_norm.weight.data, a.o_proj.weight.data,
                                           layer.post_attention_layernorm.weight.data, m._gate_up,
                                           m.down_proj.weight.data))
            self.runtime = Qwen3Runtime(
                hidden=cfg.hidden_size, intermediate=cfg.intermediate_size, num_q_heads=cfg.num_attention_heads,
                num_kv_heads=cfg.num_key_value_heads, vocab=cfg.vocab_size, eps=cfg.rms_norm_eps, layers=layers,
                embed=self.model.embed_tokens.weight.data, final_norm=self.model.norm.weight.data,
                lm_head=self._lm_head_weight().data, kv=self.kv, rope=self.rope, max_batch=self.max_batch,
                use_graphs=self.use_cuda_graphs, prefill_chunk_tokens=self.prefill_chunk_tokens)
        return self.runtime

    def clear_slot(self, idx: int):
        """Free a sequence's blocks and reset its length (model/model.py:338-341)."""
        self.kv.release(int(idx))
        self.kv.seqlens[int(idx)] = 0
        self.kv.sync()

    def clear_all_slots(self):
        """model/model.py:343-346."""
        self.kv.clear_all()

    # ------------------------------------------------------------------ forward
    @torch.inference_mode()
    def forward(self, input_ids, position_ids, slot_indices=None):
        """input_ids/position_ids [B, S] -> logits [B, S, V] (model/model.py:302-322).

        Decode (S == 1 with slots) appends one token per slot to the paged cache
        and attends over it; otherwise every row is a causal prefill whose K/V
        (first max(position)+1 tokens) is stored for its slot."""
        rt = self._rt()
        B, S = input_ids.shape
        if slot_indices is not None and S == 1:
            rows = [int(r) for r in slot_indices.tolist()]
            rt.load_decode_inputs(input_ids[:, 0].tolist(), position_ids[:, 0].tolist(), rows)
            logits = torch.empty((B, self.config.vocab_size), dtype=torch.bfloat16, device=input_ids.device)
            rt.decode_step(rows, logits=logits)
            return logits.unsqueeze(1)
        seqs = input_ids.tolist()
        pos = position_ids.tolist()
        temp = None
        if slot_indices is None:
            # The reference attends without storing K/V; attention here reads K/V
            # from a paged pool, so use a private scratch pool for the call.
            cfg = self.config
            temp = PagedKVCache(cfg.num_hidden_layers, cfg.num_key_value_heads, B, S,
                                block_size=self.kv.block_size, device=input_ids.device)
            rows = list(range(B))
            saved = (self.kv, self.runtime)
            self.kv, self.runtime = temp, None
            rt = self._rt()
        else:
            rows = [int(r) for r in slot_indices.tolist()]
        try:
            store = [max(p) + 1 for p in pos]
            _, logits = rt.prefill(seqs, rows, positions=pos, store_lengths=store, all_logits=True)
        finally:
            if temp is not None:
                self.kv, self.runtime = saved
        return logits.view(B, S, -1)

    # ------------------------------------------------------------------ loading
    @classmethod
    def from_pretrained(cls, model_path: str, config: Qwen3Config, device, dtype):
        """Load ``model.safetensors`` (model/model.py:353-384)."""
        from safetensors import safe_open
        f = Path(model_path) / "model.safetensors"
        if not f.exists():
            raise FileNotFoundError(f"No model.safetensors found in {model_path}")
        model = cls(config).to(dtype)
        sd = {}
        with safe_open(str(f), framework="pt", device=str(device)) as fh:
            for key in fh.keys():
                t = fh.get_tensor(key)
                sd[key] = t.to(dtype) if t.is_floating_point() else t
        model.load_state_dict(sd, strict=False)
        return model.to(device)

    @classmethod
    def random_init(cls, config: Qwen3Config, device, dtype=torch.bfloat16, seed: int = 0, std: float = 0.02):
        """Seeded N(0, std) weights generated on the device (norm weights = 1)."""
        with torch.device("meta"):
            model = cls(config)
        model = model.to_empty(device=device).to(dtype)
        g = torch.Generator(device=device).manual_seed(seed)
        with torch.no_grad():
            for name, p in model.named_parameters():
                if name.endswith("norm.weight") or "layernorm" in name:
                    p.fill_(1.0)
                else:
                    p.normal_(0.0, std, generator=g)
        return model

    # ------------------------------------------------------------------ PD export/import
    def export_request_kv(self, slot_idx: int, length: int, device="cpu") -> dict:
        """Per-layer K/V of the first `length` tokens as tensors [length, Hkv, 128]
        (model/model.py:156-166, :386-390).  On the CPU by default, as in the
        reference; `device` may name a GPU instead, so that a prefill engine
        hands a request to a decode engine in the same process with
        device-to-device copies of the gathered blocks (over NVLink when the
        target is another GPU) rather than through host memory.
        import_request_kv takes either."""
        out = []
        for i in range(self.config.num_hidden_layers):
            k, v = self.kv.gather(i, int(slot_idx), int(length))
            out.append({"k": k.to(device), "v": v.to(device), "seqlen": int(self.kv.lengths[int(slot_idx)])})
        return {"layers": out}

    def export_request_kv_ipc(self, slot_idx: int, length: int):
        """Hand a request's K/V to another process without host copies: returns
        (ticket, owner); send the picklable ticket, call owner.release() once
        the other side has imported it (awesome_acceleration_b200.kv_transfer)."""
        from ..kv_transfer import export_request_kv_ipc
        return export_request_kv_ipc(self, slot_idx, length)

    def import_request_kv_ipc(self, slot_idx: int, ticket) -> None:
        """Store a request exported by another process (export_request_kv_ipc)
        into slot_idx, reading its device buffer in place (same GPU or NVLink)."""
        from ..kv_transfer import import_request_kv_ipc
        import_request_kv_ipc(self, slot_idx, ticket)

    def import_request_kv(self, slot_idx: int, payload: dict, length: int):
        """Write exported K/V into `slot_idx` (model/model.py:168-177, :392-401)."""
        layers = payload["layers"]
        if len(layers) != self.config.num_hidden_layers:
            raise ValueError(f"Layer count mismatch: payload has {len(layers)}, "
                             f"model has {self.config.num_hidden_layers}")
        row = int(slot_idx)
        self.kv.reserve(row, int(length))
        self.kv.sync()
        dev = self.kv.k.device
        # The store kernel runs on the current device and stream: make that the
        # cache's device, whichever GPU the caller (or the payload) is on.
        with torch.cuda.device(dev):
            slots = torch.from_numpy(self.kv.slot_mapping(row, 0, int(length))).to(dev)
            for i, lp in enumerate(layers):
                k = lp["k"][:length].to(dev, torch.bfloat16).contiguous()
                v = lp["v"][:length].to(dev, torch.bfloat16).contiguous()
                K.kv_store(k.view(length, -1), v.view(length, -1), slots, self.kv.k[i], self.kv.v[i])
        seqlen = int(layers[0]["seqlen"])
        self.kv.set_lengths([row], [seqlen])
