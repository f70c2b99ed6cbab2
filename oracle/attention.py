"""CPU restatement of the three flash-attn entry points the reference calls
(test infrastructure).

flash-attn 2 (un-vendored, unpinned by the reference; 2.8.3 installed here)
has no CPU kernels, so the reference cannot run on a CPU as shipped.  These
functions restate its documented semantics (flash_attn/flash_attn_interface.py
docstrings of ``flash_attn_varlen_func``, ``flash_attn_with_kvcache`` and
``flash_attn_func``):

* GQA: query head ``h`` reads KV head ``h // (Hq // Hkv)``.
* causal masks are aligned to the bottom-right corner of the score matrix
  (query ``i`` of ``Lq`` sees keys ``j <= i + Lk - Lq``).
* ``flash_attn_with_kvcache`` first writes ``k``/``v`` into the cache at row
  ``cache_batch_idx[b]``, position ``cache_seqlens[b]``, then attends over the
  first ``cache_seqlens[b] + 1`` cached tokens.  It does not advance
  ``cache_seqlens`` (the reference does that itself, model/model.py:241).

Numerics follow the FlashAttention-2 algorithm: fp32 scores and softmax
statistics; the probabilities are rounded to the input dtype before the PV
product (bf16/fp16 inputs) while the normaliser uses the fp32 probabilities.
"""
from __future__ import annotations

import torch


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
           causal: bool) -> torch.Tensor:
    """q [Lq,Hq,D], k/v [Lk,Hkv,D] -> [Lq,Hq,D] in q.dtype."""
    Lq, Hq, D = q.shape
    Lk, Hkv, _ = k.shape
    G = Hq // Hkv
    qf = q.float()
    kf = k.float().repeat_interleave(G, dim=1)
    vf = v.float().repeat_interleave(G, dim=1)
    s = torch.einsum("qhd,khd->hqk", qf, kf) * scale
    if causal:
        i = torch.arange(Lq, device=q.device).unsqueeze(1)
        j = torch.arange(Lk, device=q.device).unsqueeze(0)
        s = s.masked_fill(j > i + (Lk - Lq), float("-inf"))
    m = s.amax(dim=-1, keepdim=True)
    p = torch.exp(s - m)
    l = p.sum(dim=-1, keepdim=True)
    pv = p.to(q.dtype).float() if q.dtype in (torch.bfloat16, torch.float16) else p
    o = torch.einsum("hqk,khd->qhd", pv, vf) / l.permute(1, 0, 2)
    return o.to(q.dtype)


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                           dropout_p=0.0, softmax_scale=None, causal=False, **_):
    D = q.shape[-1]
    scale = softmax_scale if softmax_scale is not None else D ** -0.5
    out = torch.empty_like(q)
    cq = cu_seqlens_q.tolist()
    ck = cu_seqlens_k.tolist()
    for i in range(len(cq) - 1):
        out[cq[i]:cq[i + 1]] = attend(q[cq[i]:cq[i + 1]], k[ck[i]:ck[i + 1]], v[ck[i]:ck[i + 1]],
                                      scale, causal)
    return out


def flash_attn_with_kvcache(q, k_cache, v_cache, k=None, v=None, rotary_cos=None, rotary_sin=None,
                            cache_seqlens=None, cache_batch_idx=None, cache_leftpad=None,
                            block_table=None, softmax_scale=None, causal=False, **_):
    assert rotary_cos is None and block_table is None and cache_leftpad is None
    B, Sq, Hq, D = q.shape
    scale = softmax_scale if softmax_scale is not None else D ** -0.5
    idx = cache_batch_idx.tolist() if cache_batch_idx is not None else list(range(B))
    lens = cache_seqlens.tolist()
    out = torch.empty_like(q)
    for b in range(B):
        row, n = idx[b], lens[b]
        if k is not None:
            k_cache[row, n:n + k.shape[1]] = k[b]
            v_cache[row, n:n + v.shape[1]] = v[b]
            n = n + k.shape[1]
        out[b] = attend(q[b], k_cache[row, :n], v_cache[row, :n], scale, causal)
    return out


def flash_attn_func(q, k, v, dropout_p=0.0, softmax_scale=None, causal=False, **_):
    D = q.shape[-1]
    scale = softmax_scale if softmax_scale is not None else D ** -0.5
    return torch.stack([attend(q[b], k[b], v[b], scale, causal) for b in range(q.shape[0])])
