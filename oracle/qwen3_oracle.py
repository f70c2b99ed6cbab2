"""CPU restatement of the reference Qwen3 hot path (test infrastructure).

Follows yijichar/AWesome_ACceleration:
  * RMSNorm              model/model.py:47-52
  * RotaryEmbedding      model/model.py:63-99
  * fused QKV            model/model.py:132-154 (rows [Q | K | V])
  * TransformerBlock     model/model.py:202-267 (decode branch :231-241)
  * Qwen3ForCausalLM     model/model.py:302-322 (tied lm_head :316-318)
  * LLM._prefill         llm.py:116-208 (packed varlen prefill, KV scatter at
                         ``slot*max_seq_len + pos`` :139-140, :171-175)
  * LLM._decode_step     llm.py:210-213; greedy sampling llm.py:215-219
with the flash-attn calls replaced by ``oracle.attention``.

Every op runs in the model dtype on CPU exactly as the reference's eager
PyTorch code does (each op rounds its output to the dtype), so a bf16 oracle
reproduces the reference's rounding points; fp32 runs are the parity pin
against the reference itself.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import attention as fa
from .weights import Qwen3Arch


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """model/model.py:47-52: fp32 variance, rsqrt, cast back, then weight multiply."""
    dt = x.dtype
    h = x.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(var + eps)
    return w * h.to(dt)


def rope_inv_freq(dim: int, theta: float) -> torch.Tensor:
    """model/model.py:63."""
    return 1.0 / (theta ** (torch.arange(0, dim, 2).float() / dim))


def rope_cos_sin(positions: torch.Tensor, dim: int, theta: float, dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin rows for ``positions`` exactly as the reference's cached table
    (model/model.py:72-78).

    The reference builds its model with ``cls(config).to(dtype)``
    (model/model.py:358), which also converts the non-persistent ``inv_freq``
    buffer (:64) to the model dtype; the table is then computed from
    ``arange(seq_len, dtype=inv_freq.dtype)`` (:75).  In a bf16 model both the
    positions and the frequencies are therefore bf16 (position 257 becomes
    256, ...), and ``t * inv_freq`` and cos/sin round to bf16.  In fp32 the
    same code is plain fp32."""
    inv = rope_inv_freq(dim, theta).to(dtype).to(positions.device)
    t = positions.to(dtype)
    freqs = t.unsqueeze(-1) * inv
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """model/model.py:94-99."""
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rope(q, k, cos, sin):
    """model/model.py:80-92 (cos/sin already gathered and broadcastable)."""
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


def paged_slot(block_table_row, pos: int, block_size: int) -> int:
    """Flat paged-cache slot of token ``pos`` of a sequence: the block-table
    restatement of the reference's ``slot*max_seq_len + pos`` (llm.py:139-140)."""
    return int(block_table_row[pos // block_size]) * block_size + pos % block_size


class Qwen3Oracle:
    """Single-GPU reference engine semantics on CPU (slot-contiguous KV cache,
    model/model.py:324-336)."""

    def __init__(self, arch: Qwen3Arch, state_dict: dict, dtype=torch.float32,
                 num_slots: int = 4, max_seq_len: int = 512, device="cpu"):
        self.arch = arch
        self.dtype = dtype
        self.max_seq_len = max_seq_len
        self.device = torch.device(device)
        self.w = {k: v.to(device=self.device, dtype=dtype) for k, v in state_dict.items()}
        a = arch
        self.q_size = a.num_attention_heads * a.head_dim
        self.kv_size = a.num_key_value_heads * a.head_dim
        self.scaling = a.head_dim ** -0.5
        self.wqkv = []
        for i in range(a.num_hidden_layers):
            p = f"model.layers.{i}.self_attn."
            self.wqkv.append(torch.cat([self.w[p + "q_proj.weight"], self.w[p + "k_proj.weight"],
                                        self.w[p + "v_proj.weight"]], 0))
        self.lm_head = self.w.get("lm_head.weight", self.w["model.embed_tokens.weight"])
        shape = (num_slots, max_seq_len, a.num_key_value_heads, a.head_dim)
        self.k_cache = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(a.num_hidden_layers)]
        self.v_cache = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(a.num_hidden_layers)]
        self.seqlens = torch.zeros(num_slots, dtype=torch.int32)

    def _lw(self, i, name):
        return self.w[f"model.layers.{i}.{name}"]

    def _mlp(self, i, x):
        """model/model.py:189-190."""
        g = F.linear(x, self._lw(i, "mlp.gate_proj.weight"))
        u = F.linear(x, self._lw(i, "mlp.up_proj.weight"))
        return F.linear(F.silu(g) * u, self._lw(i, "mlp.down_proj.weight"))

    def _qkv(self, i, x):
        a = self.arch
        qkv = F.linear(x, self.wqkv[i])
        q = qkv[..., :self.q_size].unflatten(-1, (a.num_attention_heads, a.head_dim))
        k = qkv[..., self.q_size:self.q_size + self.kv_size].unflatten(-1, (a.num_key_value_heads, a.head_dim))
        v = qkv[..., self.q_size + self.kv_size:].unflatten(-1, (a.num_key_value_heads, a.head_dim))
        eps = a.rms_norm_eps
        q = rms_norm(q, self._lw(i, "self_attn.q_norm.weight"), eps)
        k = rms_norm(k, self._lw(i, "self_attn.k_norm.weight"), eps)
        return q, k, v

    def final_hidden_prefill(self, sequences: list[list[int]], slots: list[int]) -> torch.Tensor:
        """llm.py:116-198; returns the final-normed hidden of the last token of each sequence."""
        a = self.arch
        eps = a.rms_norm_eps
        lens = [len(s) for s in sequences]
        T = sum(lens)
        dev = self.device
        flat = torch.tensor([t for s in sequences for t in s], dtype=torch.long, device=dev)
        cu = [0]
        for n in lens:
            cu.append(cu[-1] + n)
        cu_t = torch.tensor(cu, dtype=torch.int32)
        pos = torch.cat([torch.arange(n) for n in lens]).to(dev)
        cos, sin = rope_cos_sin(pos, a.head_dim, a.rope_theta, self.dtype)
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
        hidden = self.w["model.embed_tokens.weight"][flat]
        for i in range(a.num_hidden_layers):
            residual = hidden
            h = rms_norm(hidden, self._lw(i, "input_layernorm.weight"), eps)
            q, k, v = self._qkv(i, h)
            q, k = apply_rope(q, k, cos, sin)
            for s_i, slot in enumerate(slots):
                self.k_cache[i][slot, :lens[s_i]] = k[cu[s_i]:cu[s_i + 1]]
                self.v_cache[i][slot, :lens[s_i]] = v[cu[s_i]:cu[s_i + 1]]
            o = fa.flash_attn_varlen_func(q, k, v, cu_t, cu_t, max(lens), max(lens),
                                          causal=True, softmax_scale=self.scaling)
            hidden = residual + F.linear(o.reshape(T, -1), self._lw(i, "self_attn.o_proj.weight"))
            residual = hidden
            h = rms_norm(hidden, self._lw(i, "post_attention_layernorm.weight"), eps)
            hidden = residual + self._mlp(i, h)
        for s_i, slot in enumerate(slots):
            self.seqlens[slot] = lens[s_i]
        hidden = rms_norm(hidden, self.w["model.norm.weight"], eps)
        return hidden[torch.tensor(cu[1:], device=dev) - 1]

    def prefill(self, sequences: list[list[int]], slots: list[int]) -> torch.Tensor:
        """llm.py:116-208 -> logits [n, V]."""
        return F.linear(self.final_hidden_prefill(sequences, slots), self.lm_head)

    def final_hidden_decode(self, tokens: list[int], positions: list[int], slots: list[int]) -> torch.Tensor:
        """model/model.py:279-286 decode branch: [B, H] final-normed hidden."""
        a = self.arch
        eps = a.rms_norm_eps
        ids = torch.tensor(tokens, dtype=torch.long, device=self.device)
        pos = torch.tensor(positions, dtype=torch.long, device=self.device)
        cos, sin = rope_cos_sin(pos, a.head_dim, a.rope_theta, self.dtype)
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
        hidden = self.w["model.embed_tokens.weight"][ids]
        for i in range(a.num_hidden_layers):
            hidden = self.decode_layer(i, hidden, cos, sin, slots)
        for slot in slots:
            self.seqlens[slot] += 1
        return rms_norm(hidden, self.w["model.norm.weight"], eps)

    def rope_rows(self, positions: list[int]):
        """cos / sin of the decode positions, shaped to broadcast over heads."""
        pos = torch.tensor(positions, dtype=torch.long, device=self.device)
        cos, sin = rope_cos_sin(pos, self.arch.head_dim, self.arch.rope_theta, self.dtype)
        return cos.unsqueeze(1), sin.unsqueeze(1)

    def decode_layer(self, i: int, hidden: torch.Tensor, cos, sin, slots: list[int]) -> torch.Tensor:
        """TransformerBlock i on one decode token per row (model/model.py:202-267,
        decode branch :231-241): the new K/V go to position seqlens[slot]
        (not advanced here) and the token attends over seqlens[slot] + 1."""
        eps = self.arch.rms_norm_eps
        B = hidden.shape[0]
        residual = hidden
        h = rms_norm(hidden, self._lw(i, "input_layernorm.weight"), eps)
        q, k, v = self._qkv(i, h)
        q, k = apply_rope(q, k, cos, sin)
        o = torch.empty_like(q)
        for b, slot in enumerate(slots):
            n = int(self.seqlens[slot])
            self.k_cache[i][slot, n] = k[b]
            self.v_cache[i][slot, n] = v[b]
            o[b] = fa.attend(q[b:b + 1], self.k_cache[i][slot, :n + 1],
                             self.v_cache[i][slot, :n + 1], self.scaling, False)[0]
        hidden = residual + F.linear(o.reshape(B, -1), self._lw(i, "self_attn.o_proj.weight"))
        residual = hidden
        h = rms_norm(hidden, self._lw(i, "post_attention_layernorm.weight"), eps)
        return residual + self._mlp(i, h)

    def head(self, hidden: torch.Tensor) -> torch.Tensor:
        """Final norm + lm_head (model/model.py:285-286, :316-318) -> logits."""
        return F.linear(rms_norm(hidden, self.w["model.norm.weight"], self.arch.rms_norm_eps), self.lm_head)

    def decode(self, tokens: list[int], positions: list[int], slots: list[int]) -> torch.Tensor:
        """One decode step -> logits [B, V] (llm.py:210-213)."""
        return F.linear(self.final_hidden_decode(tokens, positions, slots), self.lm_head)

    def clear_slot(self, slot: int):
        """model/model.py:338-341."""
        self.seqlens[slot] = 0


def greedy(logits: torch.Tensor) -> list[int]:
    """llm.py:217-218: argmax over the vocab (first index on ties)."""
    return logits.argmax(dim=-1).tolist()


def run_greedy(oracle: Qwen3Oracle, prompts: list[list[int]], steps: int, slots=None,
               teacher: list[list[int]] | None = None, keep_logits=None):
    """Prefill ``prompts`` then ``steps`` greedy decode steps (the reference's
    loop, llm.py:358-404, with every sequence active until the end).

    Returns tokens [n][steps+1].  ``teacher`` (same shape) forces the fed-back
    tokens, so per-step logits stay comparable after a near-tie flips.
    ``keep_logits`` is a callback ``(step, logits)``."""
    n = len(prompts)
    slots = list(range(n)) if slots is None else slots
    logits = oracle.prefill(prompts, slots)
    if keep_logits:
        keep_logits(0, logits)
    toks = [[t] for t in greedy(logits)]
    pos = [len(p) for p in prompts]
    for s in range(steps):
        feed = [teacher[b][s] if teacher else toks[b][-1] for b in range(n)]
        logits = oracle.decode(feed, pos, slots)
        if keep_logits:
            keep_logits(s + 1, logits)
        for b, t in enumerate(greedy(logits)):
            toks[b].append(t)
        pos = [p + 1 for p in pos]
    return toks
