"""Tensor-parallel linear layers with the reference's interface.

Mirrors yijichar/AWesome_ACceleration model/parallel_layers.py:
constructor arguments, per-rank weight shapes, ``from_linear`` /
``from_fused_qkv`` / ``from_embedding`` slicing and forward return shapes are
the reference's; the forward bodies run the B200 GEMM (``aacc_gemm``) and the
NCCL collectives of ``model.distributed``.

Biases follow the reference: column- and QKV-parallel layers add theirs in
the GEMM (``F.linear(x, weight, bias)``: fused into the B200 GEMM epilogue,
fp32 add before the bf16 rounding), a row-parallel layer adds its bias after
the all-reduce, on TP rank 0 only, the only rank that holds one
(model/parallel_layers.py:163-170, :197-199).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .. import kernels as K
from .distributed import (get_tp_rank, get_tp_world_size, is_distributed, split_tensor_along_dim,
                          tensor_model_parallel_all_gather, tensor_model_parallel_all_reduce)


def _gemm_nd(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    lead = x.shape[:-1]
    if bias is None:
        out = K.gemm(x.reshape(-1, x.shape[-1]).contiguous(), w)
    else:
        out = K.gemm(x.reshape(-1, x.shape[-1]).contiguous(), w, bias=bias)
    return out.view(*lead, w.shape[0])


class ColumnParallelLinear(nn.Module):
    """Y = X A^T with A split by output rows; weight [out/tp, in]
    (model/parallel_layers.py:24-120)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, gather_output: bool = False,
                 skip_bias_add: bool = False):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.gather_output, self.skip_bias_add = gather_output, skip_bias_add
        self.tp_size = get_tp_world_size()
        assert out_features % self.tp_size == 0, \
            f"out_features ({out_features}) must be divisible by tp_size ({self.tp_size})"
        self.out_features_per_partition = out_features // self.tp_size
        self.weight = nn.Parameter(torch.empty(self.out_features_per_partition, in_features))
        if bias:
            self.bias = nn.Parameter(torch.empty(self.out_features_per_partition))
        else:
            self.register_parameter("bias", None)

    def forward(self, input_: torch.Tensor) -> torch.Tensor:
        out = _gemm_nd(input_, self.weight, self.bias)
        if self.gather_output and is_distributed():
            out = tensor_model_parallel_all_gather(out, dim=-1)
        return out

    @classmethod
    def from_linear(cls, linear: nn.Linear, gather_output: bool = False):
        col = cls(linear.in_features, linear.out_features, bias=linear.bias is not None, gather_output=gather_output)
        col.weight.data = split_tensor_along_dim(linear.weight.data, col.tp_size, dim=0)
        if linear.bias is not None:
            col.bias.data = split_tensor_along_dim(linear.bias.data, col.tp_size, dim=0)
        return col


class RowParallelLinear(nn.Module):
    """Y = X A^T with A split by input columns + all-reduce; weight [out, in/tp];
    bias only on TP rank 0 (model/parallel_layers.py:127-231)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, input_is_parallel: bool = True,
                 skip_bias_add: bool = False):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.input_is_parallel, self.skip_bias_add = input_is_parallel, skip_bias_add
        self.tp_size = get_tp_world_size()
        assert in_features % self.tp_size == 0, \
            f"in_features ({in_features}) must be divisible by tp_size ({self.tp_size})"
        self.in_features_per_partition = in_features // self.tp_size
        self.weight = nn.Parameter(torch.empty(out_features, self.in_features_per_partition))
        if bias and get_tp_rank() == 0:
            self.bias = nn.Parameter(torch.empty(out_features))
        else:
            self.register_parameter("bias", None)

    def forward(self, input_: torch.Tensor) -> torch.Tensor:
        if not self.input_is_parallel and is_distributed():
            input_ = split_tensor_along_dim(input_, self.tp_size, dim=-1)
        out = _gemm_nd(input_, self.weight)
        if is_distributed():
            out = tensor_model_parallel_all_reduce(out)
        if self.bias is not None:  # rank 0 only, after the all-reduce (model/parallel_layers.py:197-199)
            out = K.bias_add(out.contiguous(), self.bias)
        return out

    @classmethod
    def from_linear(cls, linear: nn.Linear, input_is_parallel: bool = True):
        row = cls(linear.in_features, linear.out_features, bias=linear.bias is not None,
                  input_is_parallel=input_is_parallel)
        row.weight.data = split_tensor_along_dim(linear.weight.data, row.tp_size, dim=1)
        if linear.bias is not None and get_tp_rank() == 0:
            row.bias.data = linear.bias.data.clone()
        return row


def qkv_rank_rows(num_q_heads: int, num_kv_heads: int, head_dim: int, tp_rank: int, tp_size: int):
    """Row ranges of a fused [Q | K | V] weight owned by one TP rank
    (model/parallel_layers.py:367-389, model/model_tp.py:509-542)."""
    q_size, kv_size = num_q_heads * head_dim, num_kv_heads * head_dim
    qp, kvp = q_size // tp_size, kv_size // tp_size
    q0 = tp_rank * qp
    k0 = q_size + tp_rank * kvp
    v0 = q_size + kv_size + tp_rank * kvp
    return (q0, q0 + qp), (k0, k0 + kvp), (v0, v0 + kvp)


class QKVParallelLinear(nn.Module):
    """Fused QKV split by attention head; weight [(Hq + 2 Hkv) * D / tp, hidden]
    holding this rank's [q | k | v] rows (model/parallel_layers.py:238-400)."""

    def __init__(self, hidden_size: int, num_q_heads: int, num_kv_heads: int, head_dim: int, bias: bool = False):
        super().__init__()
        self.hidden_size, self.num_q_heads, self.num_kv_heads, self.head_dim = \
            hidden_size, num_q_heads, num_kv_heads, head_dim
        self.tp_size = get_tp_world_size()
        assert num_q_heads % self.tp_size == 0, \
            f"num_q_heads ({num_q_heads}) must be divisible by tp_size ({self.tp_size})"
        assert num_kv_heads % self.tp_size == 0, \
            f"num_kv_heads ({num_kv_heads}) must be divisible by tp_size ({self.tp_size})"
        self.num_q_heads_per_partition = num_q_heads // self.tp_size
        self.num_kv_heads_per_partition = num_kv_heads // self.tp_size
        self.q_size = num_q_heads * head_dim
        self.kv_size = num_kv_heads * head_dim
        self.qkv_size = self.q_size + 2 * self.kv_size
        self.q_size_per_partition = self.num_q_heads_per_partition * head_dim
        self.kv_size_per_partition = self.num_kv_heads_per_partition * head_dim
        self.qkv_size_per_partition = self.q_size_per_partition + 2 * self.kv_size_per_partition
        self.weight = nn.Parameter(torch.empty(self.qkv_size_per_partition, hidden_size))
        if bias:
            self.bias = nn.Parameter(torch.empty(self.qkv_size_per_partition))
        else:
            self.register_parameter("bias", None)

    def forward(self, hidden_states: torch.Tensor):
        if hidden_states.dim() not in (2, 3):
            raise ValueError(f"hidden_states must be 2D or 3D, got shape={tuple(hidden_states.shape)}")
        qkv = _gemm_nd(hidden_states, self.weight, self.bias)
        qs, ks = self.q_size_per_partition, self.kv_size_per_partition
        lead = hidden_states.shape[:-1]
        q = qkv[..., :qs].reshape(*lead, self.num_q_heads_per_partition, self.head_dim)
        k = qkv[..., qs:qs + ks].reshape(*lead, self.num_kv_heads_per_partition, self.head_dim)
        v = qkv[..., qs + ks:].reshape(*lead, self.num_kv_heads_per_partition, self.head_dim)
        return q, k, v

    @classmethod
    def from_fused_qkv(cls, qkv_weight: torch.Tensor, qkv_bias: Optional[torch.Tensor], hidden_size: int,
                       num_q_heads: int, num_kv_heads: int, head_dim: int):
        layer = cls(hidden_size, num_q_heads, num_kv_heads, head_dim, bias=qkv_bias is not None)
        (q0, q1), (k0, k1), (v0, v1) = qkv_rank_rows(num_q_heads, num_kv_heads, head_dim, get_tp_rank(),
                                                      get_tp_world_size())
        layer.weight.data = torch.cat([qkv_weight[q0:q1], qkv_weight[k0:k1], qkv_weight[v0:v1]], 0)
        if qkv_bias is not None:
            layer.bias.data = torch.cat([qkv_bias[q0:q1], qkv_bias[k0:k1], qkv_bias[v0:v1]], 0)
        return layer


class VocabParallelEmbedding(nn.Module):
    """Embedding split by vocabulary rows + all-reduce of the masked lookup
    (model/parallel_layers.py:407-488).  The per-rank row range is also the
    vocab shard the B200 lm_head scores under TP."""

    def __init__(self, num_embeddings: int, embedding_dim: int, padding_idx: Optional[int] = None):
        super().__init__()
        self.num_embeddings, self.embedding_dim, self.padding_idx = num_embeddings, embedding_dim, padding_idx
        self.tp_size, self.tp_rank = get_tp_world_size(), get_tp_rank()
        assert num_embeddings % self.tp_size == 0, \
            f"num_embeddings ({num_embeddings}) must be divisible by tp_size ({self.tp_size})"
        self.num_embeddings_per_partition = num_embeddings // self.tp_size
        self.vocab_start_index = self.tp_rank * self.num_embeddings_per_partition
        self.vocab_end_index = self.vocab_start_index + self.num_embeddings_per_partition
        self.weight = nn.Parameter(torch.empty(self.num_embeddings_per_partition, embedding_dim))

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        mask = (input_ids >= self.vocab_start_index) & (input_ids < self.vocab_end_index)
        local = (input_ids - self.vocab_start_index).clamp(0, self.num_embeddings_per_partition - 1)
        out = K.gather_rows(self.weight, local.reshape(-1).contiguous())
        out = out.view(*input_ids.shape, self.embedding_dim) * mask.unsqueeze(-1)
        if is_distributed():
            out = tensor_model_parallel_all_reduce(out)
        return out

    @classmethod
    def from_embedding(cls, embedding: nn.Embedding):
        vp = cls(embedding.num_embeddings, embedding.embedding_dim, padding_idx=embedding.padding_idx)
        vp.weight.data = split_tensor_along_dim(embedding.weight.data, vp.tp_size, dim=0)
        return vp
