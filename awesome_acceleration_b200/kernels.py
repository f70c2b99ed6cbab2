"""Tensor-level wrappers over the C ABI (one call = one or two kernel launches).

Tensors must be CUDA, contiguous and of the documented dtype; every call
launches on the current PyTorch stream, so it composes with CUDA-graph
capture.  Outputs are allocated here only when the caller passes none.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

BF16 = torch.bfloat16


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _lib_():
    return _lib.load()


def _req(t: torch.Tensor, dtype, name: str):
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name}: expected a contiguous CUDA {dtype} tensor, got {t.dtype} "
                         f"{'cuda' if t.is_cuda else 'cpu'} contiguous={t.is_contiguous()}")


# ---------------------------------------------------------------- KV cache
def kv_store(k: torch.Tensor, v: torch.Tensor, slot_mapping: torch.Tensor, k_cache: torch.Tensor,
             v_cache: torch.Tensor) -> None:
    """k/v [T, Hkv, 128] (row-strided views allowed); caches [blocks, Hkv, bs, 128]."""
    nb, hkv, bs, _ = k_cache.shape
    _req(slot_mapping, torch.int64, "slot_mapping")
    _lib.check(_lib_().aacc_kv_store(_p(k), _p(v), k.shape[0], k.stride(0), v.stride(0), _p(slot_mapping),
                                     _p(k_cache), _p(v_cache), nb, hkv, bs, _stream()), "kv_store")


def decode_slot_mapping(rows, seqlens, block_tables, block_size: int, num_blocks: int, out) -> None:
    _lib.check(_lib_().aacc_decode_slot_mapping(_p(rows), _p(seqlens), _p(block_tables), block_tables.shape[1],
                                                block_size, num_blocks, _p(out), rows.shape[0], _stream()),
               "decode_slot_mapping")


def advance_seqlens(rows, seqlens, positions=None) -> None:
    _lib.check(_lib_().aacc_advance_seqlens(_p(rows), _p(seqlens), _p(positions), rows.shape[0], _stream()),
               "advance_seqlens")


def gather_rows(src: torch.Tensor, idx: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty((idx.shape[0],) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
    row_bytes = src[0].numel() * src.element_size()
    _lib.check(_lib_().aacc_gather_rows(_p(src), src.shape[0], row_bytes, _p(idx), idx.shape[0], _p(out),
                                        _stream()), "gather_rows")
    return out


# ---------------------------------------------------------------- attention
def decode_workspace_bytes(batch: int, num_q_heads: int, max_context: int, split_tokens: int = 0) -> int:
    return int(_lib_().aacc_paged_decode_workspace_bytes(batch, num_q_heads, max_context, split_tokens))


def paged_decode_attention(q, k_cache, v_cache, block_tables, rows, seqlens, *, ctx_add: int, scale: float,
                           max_context: int, workspace: torch.Tensor | None, out=None,
                           split_tokens: int = 0) -> torch.Tensor:
    """q [B, Hq, 128] -> out [B, Hq, 128] over seqlens[rows[b]] + ctx_add cached tokens."""
    B, hq, _ = q.shape
    nb, hkv, bs, _ = k_cache.shape
    if out is None:
        out = torch.empty_like(q)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _lib.check(_lib_().aacc_paged_decode_attention(
        _p(q), _p(out), _p(k_cache), _p(v_cache), nb, _p(block_tables), block_tables.shape[1], _p(rows),
        _p(seqlens), ctx_add, B, hq, hkv, bs, scale, split_tokens, max_context, _p(workspace), ws_bytes,
        _stream()), "paged_decode_attention")
    return out


def prefill_attention(q, k_cache, v_cache, block_tables, seq_rows, cu_q, ctx_start, *, max_q_len: int,
                      scale: float, out=None) -> torch.Tensor:
    """q [T, Hq, 128] packed by cu_q -> out [T, Hq, 128] (causal over cached context + chunk)."""
    T, hq, _ = q.shape
    nb, hkv, bs, _ = k_cache.shape
    if out is None:
        out = torch.empty_like(q)
    _lib.check(_lib_().aacc_prefill_attention(
        _p(q), _p(out), T, _p(k_cache), _p(v_cache), nb, _p(block_tables), block_tables.shape[1], _p(seq_rows),
        _p(cu_q), _p(ctx_start), seq_rows.shape[0], max_q_len, hq, hkv, bs, scale, _stream()),
        "prefill_attention")
    return out


# ---------------------------------------------------------------- norms
def rmsnorm(x, w, eps: float, out=None):
    H = x.shape[-1]
    rows = x.numel() // H
    if out is None:
        out = torch.empty_like(x)
    _lib.check(_lib_().aacc_rmsnorm(_p(x), _p(w), _p(out), rows, H, eps, _stream()), "rmsnorm")
    return out


def add_rmsnorm(delta, residual, w, eps: float, out=None):
    """residual <- bf16(residual + delta); returns rmsnorm(residual)."""
    H = residual.shape[-1]
    rows = residual.numel() // H
    if out is None:
        out = torch.empty_like(residual)
    _lib.check(_lib_().aacc_add_rmsnorm(_p(delta), _p(residual), _p(w), _p(out), rows, H, eps, _stream()),
               "add_rmsnorm")
    return out


def embed_rmsnorm(ids, table, w, eps: float, residual_out, out):
    rows = ids.numel()
    V, H = table.shape
    _lib.check(_lib_().aacc_embed_rmsnorm(_p(ids), _p(table), V, _p(residual_out), _p(w), _p(out), rows, H, eps,
                                          _stream()), "embed_rmsnorm")
    return out


# ---------------------------------------------------------------- GEMMs
def gemm(x, w, out=None, bias=None):
    """x [M, K] @ w[N, K]^T (+ bias [N], added in fp32 before the bf16 rounding)."""
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=BF16, device=x.device)
    if bias is None:
        _lib.check(_lib_().aacc_gemm(_p(x), _p(w), _p(out), M, N, K, _stream()), "gemm")
    else:
        _req(bias, BF16, "bias")
        if bias.numel() != N:
            raise ValueError(f"gemm: bias has {bias.numel()} elements, expected {N}")
        _lib.check(_lib_().aacc_gemm_bias(_p(x), _p(w), _p(bias), _p(out), M, N, K, _stream()), "gemm_bias")
    return out


def bias_add(x, bias):
    """x [..., N] <- bf16(x + bias [N]) in place."""
    _req(x, BF16, "x")
    _req(bias, BF16, "bias")
    N = x.shape[-1]
    if bias.numel() != N:
        raise ValueError(f"bias_add: bias has {bias.numel()} elements, expected {N}")
    _lib.check(_lib_().aacc_bias_add(_p(x), _p(bias), x.numel() // N, N, _stream()), "bias_add")
    return x


def pick_splits(M: int, N: int, K: int, sms: int = 148, cap: int = 16, max_elems: int | None = None) -> int:
    """Largest divisor of K/64 (at most `cap`, and with splits*M*N fp32
    partials fitting `max_elems`) that keeps the split-K grid within one wave
    of CTAs (one 128x128 tile per SM) and whose fp32 partials (written, then
    read back) are no more bytes than the weights (splits*M*N*4 <= N*K*2).
    Measured on the cfg2 decode step (M=256): o_proj / down_proj at 4 splits
    beat 8 by 1.0 / 0.6 us per layer; QKV keeps 2."""
    tiles = ((N + 127) // 128) * ((M + 127) // 128)
    nk = K // 64
    best = 1
    for d in range(1, min(nk, cap) + 1):
        if (nk % d == 0 and tiles * d <= sms and (max_elems is None or d * M * N <= max_elems)
                and (d == 1 or 2 * d * M <= K)):
            best = d
    return best


def _check_partial(partial, splits: int, M: int, N: int, what: str):
    """The fp32 partial buffer must hold splits * M * N values (the kernels
    write every one of them; the C ABI cannot see the buffer's size)."""
    _req(partial, torch.float32, f"{what}: partial")
    if partial.numel() < splits * M * N:
        raise ValueError(f"{what}: partial holds {partial.numel()} values, needs {splits} x {M} x {N}")


def gemm_splitk(x, w, partial, splits: int):
    """partial [splits, M, N] fp32 <- split-K partial products of x @ w^T."""
    M, K = x.shape
    N = w.shape[0]
    _check_partial(partial, splits, M, N, "gemm_splitk")
    _lib.check(_lib_().aacc_gemm_splitk(_p(x), _p(w), _p(partial), M, N, K, splits, _stream()), "gemm_splitk")
    return partial


def splitk_add_rmsnorm(partial, splits: int, residual, w, eps: float, out):
    H = residual.shape[-1]
    rows = residual.numel() // H
    _lib.check(_lib_().aacc_splitk_add_rmsnorm(_p(partial), splits, _p(residual), _p(w), _p(out), rows, H, eps,
                                               _stream()), "splitk_add_rmsnorm")
    return out


def splitk_qkv_norm_rope_store(partial, splits: int, q_norm_w, k_norm_w, eps: float, positions, rope_cos_sin,
                               slot_mapping, k_cache, v_cache, num_q_heads: int, q_out):
    M = q_out.shape[0]
    nb, hkv, bs, _ = k_cache.shape
    _lib.check(_lib_().aacc_splitk_qkv_norm_rope_store(
        _p(partial), splits, _p(q_norm_w), _p(k_norm_w), eps, _p(positions), _p(rope_cos_sin),
        rope_cos_sin.shape[0], _p(slot_mapping), _p(q_out), _p(k_cache), _p(v_cache), nb, num_q_heads, hkv, bs, M,
        _stream()), "splitk_qkv_norm_rope_store")
    return q_out


def splitk_silu_mul(partial, splits: int, out):
    M, I = out.shape
    _lib.check(_lib_().aacc_splitk_silu_mul(_p(partial), splits, _p(out), M, I, _stream()), "splitk_silu_mul")
    return out


def splitk_reduce(partial, splits: int, out):
    rows, cols = out.shape
    _lib.check(_lib_().aacc_splitk_reduce(_p(partial), splits, _p(out), rows, cols, _stream()), "splitk_reduce")
    return out


# ---------------------------------------------------------------- small-batch decode projections
SKINNY_MAX_ROWS = 64      # what the kernels take
SKINNY_DEFAULT_ROWS = 32  # batches the engine sends through them
# Batches up to this run the QKV / SiLU epilogues in the GEMM's last split CTAs.  Off: on
# B200 the serial tail of the last CTA cost more than the separate epilogue launch at
# every batch measured (Qwen3-0.6B shapes, B = 1: 30.5 vs 27.4 us per layer).
SKINNY_FUSED_ROWS = 0
SKINNY_TARGET_CTAS = 296      # QKV / gate-up grids: about two CTAs per SM
SKINNY_TARGET_CTAS_ROW = 148  # o / down grids: fewer splits for the norm kernel to sum


def pick_skinny_splits(M: int, N: int, K: int, target: int = 296, max_elems: int | None = None,
                       cap: int = 64) -> int:
    """Split count of the small-batch GEMMs: the largest divisor d <= cap of
    K/64 with (N/128) * d CTAs at most `target` (two per SM by default: a CTA
    takes ~74-98 KB of shared memory), fp32 partials no more than half the
    weight bytes (4 * d * M <= K) and d * M * N fitting `max_elems`; 1 when
    the weight tiles alone reach the target."""
    tiles, nk = N // 128, K // 64
    best = 1
    for d in range(1, min(nk, cap) + 1):
        if (nk % d == 0 and tiles * d <= target and 4 * d * M <= K
                and (max_elems is None or d * M * N <= max_elems)):
            best = d
    return best


def _check_counters(counters, N: int, what: str):
    if counters.dtype != torch.int32 or counters.numel() < N // 128:
        raise ValueError(f"{what}: counters must be int32 with at least {N // 128} entries")


def gemm_skinny_splitk(x, w, partial, splits: int):
    """partial [splits, M, N] fp32 <- split-K partial products of x @ w^T
    (M <= 64 rows; the weights are the MMA's 128-row operand)."""
    M, K = x.shape
    N = w.shape[0]
    _check_partial(partial, splits, M, N, "gemm_skinny_splitk")
    _lib.check(_lib_().aacc_gemm_skinny_splitk(_p(x), _p(w), _p(partial), M, N, K, splits, _stream()),
               "gemm_skinny_splitk")
    return partial


def skinny_qkv_norm_rope_store(x, w_qkv, partial, splits: int, counters, q_norm_w, k_norm_w, eps: float, positions,
                               rope_cos_sin, slot_mapping, k_cache, v_cache, num_q_heads: int, q_out):
    """QKV projection + q/k norm + RoPE + KV store for M <= 64 rows in one
    launch (the epilogue runs in the last split CTA of each head)."""
    M, K = x.shape
    nb, hkv, bs, _ = k_cache.shape
    _check_counters(counters, w_qkv.shape[0], "skinny_qkv_norm_rope_store")
    _check_partial(partial, splits, M, w_qkv.shape[0], "skinny_qkv_norm_rope_store")
    _lib.check(_lib_().aacc_skinny_qkv_norm_rope_store(
        _p(x), _p(w_qkv), _p(partial), splits, _p(counters), _p(q_norm_w), _p(k_norm_w), eps, _p(positions),
        _p(rope_cos_sin), rope_cos_sin.shape[0], _p(slot_mapping), _p(q_out), _p(k_cache), _p(v_cache), nb,
        num_q_heads, hkv, bs, M, K, _stream()), "skinny_qkv_norm_rope_store")
    return q_out


def skinny_silu_mul(x, w_gate_up, partial, splits: int, counters, out):
    """out [M, I] = SiLU(gate) * up for M <= 64 rows in one launch."""
    M, K = x.shape
    I = w_gate_up.shape[0] // 2
    _check_counters(counters, 2 * I, "skinny_silu_mul")
    _check_partial(partial, splits, M, 2 * I, "skinny_silu_mul")
    _lib.check(_lib_().aacc_skinny_silu_mul(_p(x), _p(w_gate_up), _p(partial), splits, _p(counters), _p(out), M, I, K,
                                            _stream()), "skinny_silu_mul")
    return out


def gemm_silu_mul(x, w_gate_up, out=None):
    M, K = x.shape
    I = w_gate_up.shape[0] // 2
    if out is None:
        out = torch.empty((M, I), dtype=BF16, device=x.device)
    _lib.check(_lib_().aacc_gemm_silu_mul(_p(x), _p(w_gate_up), _p(out), M, I, K, _stream()), "gemm_silu_mul")
    return out


def qkv_norm_rope_store(x, w_qkv, q_norm_w, k_norm_w, eps: float, positions, rope_cos_sin, slot_mapping,
                        k_cache, v_cache, num_q_heads: int, q_out=None):
    M, K = x.shape
    nb, hkv, bs, _ = k_cache.shape
    if q_out is None:
        q_out = torch.empty((M, num_q_heads, 128), dtype=BF16, device=x.device)
    _lib.check(_lib_().aacc_qkv_norm_rope_store(
        _p(x), _p(w_qkv), _p(q_norm_w), _p(k_norm_w), eps, _p(positions), _p(rope_cos_sin), rope_cos_sin.shape[0],
        _p(slot_mapping), _p(q_out), _p(k_cache), _p(v_cache), nb, num_q_heads, hkv, bs, M, K, _stream()),
        "qkv_norm_rope_store")
    return q_out


# ---------------------------------------------------------------- decode projections (cluster split-K)
CLUSTER_MAX_ROWS = 256


def gemm_cluster(x, w, out=None, splits: int = 0):
    """bf16 x [M, K] @ w [N, K]^T for a decode batch (M <= 256), K split over a
    thread-block cluster and summed through distributed shared memory."""
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=BF16, device=x.device)
    _lib.check(_lib_().aacc_gemm_cluster(_p(x), _p(w), _p(out), M, N, K, splits, _stream()), "gemm_cluster")
    return out


def gemm_silu_mul_cluster(x, w_gate_up, out=None, splits: int = 0):
    M, K = x.shape
    I = w_gate_up.shape[0] // 2
    if out is None:
        out = torch.empty((M, I), dtype=BF16, device=x.device)
    _lib.check(_lib_().aacc_gemm_silu_mul_cluster(_p(x), _p(w_gate_up), _p(out), M, I, K, splits, _stream()),
               "gemm_silu_mul_cluster")
    return out


def qkv_norm_rope_store_cluster(x, w_qkv, q_norm_w, k_norm_w, eps: float, positions, rope_cos_sin, slot_mapping,
                                k_cache, v_cache, num_q_heads: int, q_out=None, splits: int = 0):
    M, K = x.shape
    nb, hkv, bs, _ = k_cache.shape
    if q_out is None:
        q_out = torch.empty((M, num_q_heads, 128), dtype=BF16, device=x.device)
    _lib.check(_lib_().aacc_qkv_norm_rope_store_cluster(
        _p(x), _p(w_qkv), _p(q_norm_w), _p(k_norm_w), eps, _p(positions), _p(rope_cos_sin), rope_cos_sin.shape[0],
        _p(slot_mapping), _p(q_out), _p(k_cache), _p(v_cache), nb, num_q_heads, hkv, bs, M, K, splits, _stream()),
        "qkv_norm_rope_store_cluster")
    return q_out


def gemm_cluster_plan(M: int, N: int, K: int) -> tuple[int, int, int]:
    """(tile rows / 128, tiles over M, splits) the cluster GEMMs pick for M x N x K on this GPU."""
    mt, mtiles, splits = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _lib.check(_lib_().aacc_gemm_cluster_plan(M, N, K, ctypes.byref(mt), ctypes.byref(mtiles), ctypes.byref(splits)),
               "gemm_cluster_plan")
    return mt.value, mtiles.value, splits.value


def gemm_cluster_capacity(tile_rows_128: int, splits: int) -> int:
    """CTAs of the cluster GEMM with clusters of `splits` that fit on this GPU at once."""
    return int(_lib_().aacc_gemm_cluster_capacity(tile_rows_128, splits))


def lm_head_workspace_bytes(M: int, vocab: int) -> int:
    return int(_lib_().aacc_lm_head_workspace_bytes(M, vocab))


def lm_head_argmax(x, w, tokens, workspace, *, logits=None, best_val=None, vocab_offset: int = 0,
                   temperature=None, seeds=None, counters=None):
    """Next token of each row of x: greedy, or, for rows whose `temperature`
    (fp32 [M]) is > 0, a sample of softmax(bf16(logits / T)) drawn with
    counter-based Gumbel noise keyed by seeds / counters (int64 [M])."""
    M, K = x.shape
    V = w.shape[0]
    if temperature is not None:
        for t, dt, name in ((temperature, torch.float32, "temperature"), (seeds, torch.int64, "seeds"),
                            (counters, torch.int64, "counters")):
            if t is None or t.dtype != dt or t.numel() < M or not t.is_contiguous():
                raise ValueError(f"lm_head_argmax: {name} must be a contiguous {dt} tensor of >= {M} rows")
    _lib.check(_lib_().aacc_lm_head_sample(
        _p(x), _p(w), M, V, K, vocab_offset, _p(temperature), _p(seeds), _p(counters), _p(tokens), _p(best_val),
        _p(logits), _p(workspace), workspace.numel() * workspace.element_size(), _stream()), "lm_head_argmax")
    return tokens


def argmax_rows(logits, tokens=None):
    M, V = logits.shape
    if tokens is None:
        tokens = torch.empty(M, dtype=torch.int64, device=logits.device)
    _lib.check(_lib_().aacc_argmax_rows(_p(logits), M, V, _p(tokens), _stream()), "argmax_rows")
    return tokens


def sample_rows(logits, temperatures, seeds, counters, tokens=None):
    """Temperature sampling over materialised logits [M, V] (per-row host
    temperatures / seeds / counters); rows with temperature 0 take the argmax."""
    M, V = logits.shape
    dev = logits.device
    t = torch.as_tensor(temperatures, dtype=torch.float32).to(dev)
    sc = torch.as_tensor([list(seeds), list(counters)], dtype=torch.int64).to(dev)
    if tokens is None:
        tokens = torch.empty(M, dtype=torch.int64, device=dev)
    _lib.check(_lib_().aacc_sample_rows(_p(logits), M, V, _p(t), _p(sc[0]), _p(sc[1]), _p(tokens), _stream()),
               "sample_rows")
    return tokens


def argmax_merge(cand_val, cand_idx, tokens=None):
    """cand_val/cand_idx [shards, M] -> tokens [M]."""
    S, M = cand_val.shape
    if tokens is None:
        tokens = torch.empty(M, dtype=torch.int64, device=cand_val.device)
    _lib.check(_lib_().aacc_argmax_merge(_p(cand_val), _p(cand_idx), M, S, _p(tokens), _stream()), "argmax_merge")
    return tokens


def argmax_merge_packed(gathered, M: int, tokens):
    """Merge the vocab shards' candidates all-gathered as one int64 buffer
    [shards, 2 M] per rank: ids in [:M], fp32 values in the first M float32
    of [M:2M] (see Qwen3Runtime._argmax) -> tokens [M]."""
    S, W = gathered.shape
    if W != 2 * M or gathered.dtype != torch.int64 or not gathered.is_contiguous():
        raise ValueError("argmax_merge_packed: expected a contiguous int64 [shards, 2 M] buffer")
    vals = gathered.view(torch.float32)  # [S, 4 M]
    _lib.check(_lib_().aacc_argmax_merge_strided(_p(vals[:, 2 * M:]), _p(gathered), M, S, 4 * M, 2 * M, _p(tokens),
                                                 _stream()), "argmax_merge_packed")
    return tokens


def tp_set_peer_wait_ms(ms: int) -> None:
    """How long an exchange waits for a peer before it reports ERR_PEER_TIMEOUT (default 20 s)."""
    _lib.check(_lib_().aacc_tp_set_peer_wait_ms(int(ms)), "tp_set_peer_wait_ms")


def tp_exchange_bytes(world: int, max_rows: int, hidden: int) -> int:
    return int(_lib_().aacc_tp_exchange_bytes(world, max_rows, hidden))


def peer_buffer_alloc(nbytes: int) -> tuple[int, bytes]:
    """Zero-filled dedicated device buffer + its 64-byte CUDA IPC handle (set-up only)."""
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    _lib.check(_lib_().aacc_peer_buffer_alloc(nbytes, ctypes.byref(ptr), handle), "peer_buffer_alloc")
    return ptr.value, handle.raw


def peer_buffer_open(handle: bytes) -> int:
    ptr = ctypes.c_void_p()
    _lib.check(_lib_().aacc_peer_buffer_open(ctypes.create_string_buffer(handle, 64), ctypes.byref(ptr)),
               "peer_buffer_open")
    return ptr.value


def peer_buffer_close(ptr: int) -> None:
    _lib.check(_lib_().aacc_peer_buffer_close(ptr), "peer_buffer_close")


def peer_buffer_free(ptr: int) -> None:
    _lib.check(_lib_().aacc_peer_buffer_free(ptr), "peer_buffer_free")


def tp_allreduce_add_rmsnorm(src, splits: int, buffers, rank: int, max_rows: int, residual, w, eps: float, out,
                             two_shot: bool = False):
    """All-reduce of a RowParallel output over the group's exchange buffers, fused with the
    split-K sum (src fp32 [splits, M, H], or bf16 [M, H] with splits=0), the residual add
    (residual updated in place) and the RMSNorm into `out`."""
    M, H = residual.shape
    world = len(buffers)
    arr = (ctypes.c_void_p * world)(*buffers)
    _lib.check(_lib_().aacc_tp_allreduce_add_rmsnorm(_p(src), splits, arr, world, rank, int(two_shot), max_rows,
                                                     _p(residual), _p(w), _p(out), M, H, eps, _stream()),
               "tp_allreduce_add_rmsnorm")
    return out
