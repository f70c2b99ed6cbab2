"""Per-step Qwen3 hot path on the B200 kernels (prefill + decode).

``Qwen3Runtime`` owns the flat per-layer weight list, the paged KV cache and
the static decode buffers, and drives the C-ABI kernels layer by layer:

  decode step (one token per row, all on device, CUDA-graph captured per
  batch size):
    slot_mapping <- block_tables/seqlens                  (decode_slot_mapping)
    res, x       <- embed[ids], rmsnorm                   (embed_rmsnorm)
    per layer:
      q, K/V->cache <- x @ Wqkv^T, q/k-norm, RoPE          (qkv_norm_rope_store)
      o            <- paged attention over seqlens+1       (paged_decode_attention)
      d            <- o @ Wo^T            [TP: all-reduce]  (gemm)
      res, x       <- res + d, rmsnorm                     (add_rmsnorm)
      a            <- silu(x Wg^T) * (x Wu^T)              (gemm_silu_mul)
      d            <- a @ Wd^T            [TP: all-reduce]  (gemm)
      res, x       <- res + d, next rmsnorm                (add_rmsnorm)
    ids          <- argmax(x @ lm_head^T) [TP: vocab shards + merge]
    seqlens, positions += 1                                (advance_seqlens)

  prefill (packed, chunked): the same layer chain over the chunk's tokens,
  with K/V stored by the QKV epilogue and causal attention over the paged
  cache (prefill_attention), then argmax of the last token of every sequence
  that ends in the chunk.

This is the reference's ``LLM._prefill`` (llm.py:116-208),
``TransformerBlock.forward`` (model/model.py:202-267) and the TP twins
(llm_tp.py:397-517, model/model_tp.py:177-324) restructured around fused
kernels.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from . import kernels as K
from .kv_cache import PagedKVCache


@dataclass
class LayerWeights:
    in_ln: torch.Tensor       # [H]
    wqkv: torch.Tensor        # [(Hq + 2 Hkv) * 128, H]  (this rank's heads)
    q_norm: torch.Tensor      # [128]
    k_norm: torch.Tensor      # [128]
    wo: torch.Tensor          # [H, Hq * 128]
    post_ln: torch.Tensor     # [H]
    w_gate_up: torch.Tensor   # [2 I, H] gate/up interleaved by 64 rows
    wd: torch.Tensor          # [H, I]


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, group: int = 64) -> torch.Tensor:
    """Rows [128j, 128j+64) = gate rows [64j, 64j+64), next 64 = up rows."""
    I, H = gate.shape
    if I % group:
        raise ValueError(f"intermediate size {I} must be a multiple of {group}")
    return torch.stack([gate.view(I // group, group, H), up.view(I // group, group, H)], 1).reshape(2 * I, H)


def rope_table(max_pos: int, head_dim: int, theta: float, device, dtype=torch.bfloat16) -> torch.Tensor:
    """[max_pos][head_dim] = cos[:half] | sin[:half] of the reference's cached
    RoPE table (model/model.py:63, :72-78), built with the same torch ops.

    The reference converts its whole module, the ``inv_freq`` buffer
    included, to the model dtype (``cls(config).to(dtype)``,
    model/model.py:358), so in a bf16 model the positions
    (``arange(seq_len, dtype=inv_freq.dtype)``) and frequencies are bf16 and
    every op rounds to bf16.  Reproducing that keeps K/V bit-exact with it."""
    inv_freq = (1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))).to(dtype).to(device)
    t = torch.arange(max_pos, device=device, dtype=inv_freq.dtype)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    half = head_dim // 2
    return torch.cat([emb.cos().to(dtype)[:, :half], emb.sin().to(dtype)[:, :half]], dim=-1).contiguous()


def _stream():
    return torch.cuda.current_stream().cuda_stream


class PeerExchange:
    """NVLink exchange buffers of one TP group for aacc_tp_allreduce_add_rmsnorm.

    Every rank allocates one dedicated, zero-filled device buffer and maps
    every peer's through CUDA IPC; the handles travel over the group's Gloo
    twin.  All ranks construct it together (it is collective) and only when
    every rank can reach every other rank's GPU peer-to-peer; otherwise
    ``create`` returns None on all ranks and the NCCL path stays in use.
    """

    def __init__(self, rank: int, world: int, cpu_group, max_rows: int, hidden: int, two_shot: bool):
        self.rank, self.world, self.max_rows, self.hidden, self.two_shot = rank, world, max_rows, hidden, two_shot
        self.cpu_group = cpu_group
        self.own, handle = K.peer_buffer_alloc(K.tp_exchange_bytes(world, max_rows, hidden))
        dev = torch.cuda.current_device()
        info = [None] * world
        torch.distributed.all_gather_object(info, (handle, dev), group=cpu_group)
        ok = all(p == rank or torch.cuda.can_device_access_peer(dev, d) for p, (_, d) in enumerate(info))
        oks = [None] * world
        torch.distributed.all_gather_object(oks, ok, group=cpu_group)
        self.ptrs: list[int] = []
        self.usable = all(oks)
        if self.usable:
            self.ptrs = [self.own if p == rank else K.peer_buffer_open(h) for p, (h, _) in enumerate(info)]
        torch.distributed.barrier(group=cpu_group)  # every buffer zeroed and mapped before the first push

    @classmethod
    def create(cls, rank, world, cpu_group, max_rows, hidden, two_shot):
        ex = cls(rank, world, cpu_group, max_rows, hidden, two_shot)
        if not ex.usable:
            ex.close()
            return None
        return ex

    def close(self) -> None:
        """Collective: unmap the peers' buffers, wait for every rank, free our own."""
        if self.own is None:
            return
        torch.cuda.synchronize()
        for p, ptr in enumerate(self.ptrs):
            if p != self.rank:
                K.peer_buffer_close(ptr)
        self.ptrs = []
        torch.distributed.barrier(group=self.cpu_group)
        K.peer_buffer_free(self.own)
        self.own = None


class TPComm:
    """Collective hooks of the tensor-parallel path (identity at TP=1)."""

    def __init__(self, rank: int = 0, size: int = 1, group=None, cpu_group=None):
        self.rank, self.size, self.group, self.cpu_group = rank, size, group, cpu_group
        self.exchange: PeerExchange | None = None

    def all_reduce(self, t: torch.Tensor) -> None:
        if self.size > 1:
            torch.distributed.all_reduce(t, group=self.group)

    def all_gather(self, out: torch.Tensor, t: torch.Tensor) -> None:
        """out [size, n] <- every rank's t [n] (rank order)."""
        torch.distributed.all_gather_into_tensor(out.view(-1), t, group=self.group)

    def enable_peer_exchange(self, max_rows: int, hidden: int) -> None:
        """Set up the NVLink exchange for RowParallel outputs of up to max_rows rows
        (collective over the TP group).  AACC_TP_EXCHANGE=0 keeps NCCL;
        AACC_TP_TWO_SHOT=0 selects the one-shot exchange (two-shot measured faster from 2 ranks up)."""
        if (self.size < 2 or self.size > 8 or self.cpu_group is None or self.exchange is not None
                or os.environ.get("AACC_TP_EXCHANGE", "1") == "0"
                or torch.distributed.get_backend(self.group) != "nccl" or (hidden // 8) % self.size):
            return
        two_shot = os.environ.get("AACC_TP_TWO_SHOT", "1") != "0"
        self.exchange = PeerExchange.create(self.rank, self.size, self.cpu_group, max_rows, hidden, two_shot)

    def allreduce_add_rmsnorm(self, src, splits: int, res, w, eps: float, out) -> bool:
        """res += all_reduce(src) (src: fp32 split-K partials, or bf16 with splits=0), out = rmsnorm(res)
        in one NVLink kernel; False when the exchange is off or M exceeds its capacity."""
        ex = self.exchange
        if ex is None or res.shape[0] > ex.max_rows:
            return False
        K.tp_allreduce_add_rmsnorm(src, splits, ex.ptrs, self.rank, ex.max_rows, res, w, eps, out,
                                   two_shot=ex.two_shot)
        return True

    def close(self) -> None:
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None


class _DecodeBuffers:
    def __init__(self, B: int, H: int, Hq: int, I: int, vocab: int, tp: int, max_context: int, device):
        i64 = dict(dtype=torch.int64, device=device)
        bf = dict(dtype=torch.bfloat16, device=device)
        self.meta = torch.zeros((4, B), **i64)  # ids | positions | rows | sampling seeds
        self.ids, self.pos, self.rows, self.seed = self.meta[0], self.meta[1], self.meta[2], self.meta[3]
        self.temp = torch.zeros(B, dtype=torch.float32, device=device)  # sampling temperature (0 = greedy)
        self.slot_map = torch.zeros(B, **i64)
        self.res = torch.zeros((B, H), **bf)
        self.x = torch.zeros((B, H), **bf)
        self.delta = torch.zeros((B, H), **bf)
        self.q = torch.zeros((B, Hq, 128), **bf)
        self.attn = torch.zeros((B, Hq, 128), **bf)
        self.act = torch.zeros((B, I), **bf)
        ws = K.decode_workspace_bytes(B, Hq, max_context)
        self.attn_ws = torch.zeros(max(ws, 16), dtype=torch.uint8, device=device)  # zeroed merge counters
        self.lm_ws = torch.empty(K.lm_head_workspace_bytes(B, vocab), dtype=torch.uint8, device=device)
        self.best = torch.zeros(B, dtype=torch.float32, device=device)
        self.tok = torch.zeros(B, **i64)
        # split-K fp32 partials of the decode projections (the split count is
        # capped so that splits * B * N fits): 32 MB
        self.part = torch.empty(max(8 << 20, 16 * B * H), dtype=torch.float32, device=device)
        # per-128-row-tile arrival counters of the small-batch GEMMs (zero between launches)
        self.sk_cnt = torch.zeros(4096, dtype=torch.int32, device=device)
        if tp > 1:  # this rank's argmax candidates (ids | fp32 scores) and the all-gathered [tp, 2 B]
            self.cand = torch.zeros(2 * B, **i64)
            self.g_cand = torch.zeros(tp * 2 * B, **i64)


class Qwen3Runtime:
    def __init__(self, *, hidden: int, intermediate: int, num_q_heads: int, num_kv_heads: int, vocab: int,
                 eps: float, layers: list[LayerWeights], embed: torch.Tensor, final_norm: torch.Tensor,
                 lm_head: torch.Tensor, kv: PagedKVCache, rope: torch.Tensor, comm: TPComm | None = None,
                 vocab_offset: int = 0, max_batch: int = 256, use_graphs: bool = True,
                 prefill_chunk_tokens: int = 32768):
        self.comm = comm or TPComm()
        tp = self.comm.size
        self.H, self.eps = hidden, eps
        self.Hq, self.Hkv = num_q_heads // tp, num_kv_heads // tp   # this rank's heads
        self.I = intermediate // tp
        self.vocab = vocab                                          # full vocabulary
        self.vocab_local = lm_head.shape[0]
        self.vocab_offset = vocab_offset
        self.layers, self.embed, self.final_norm, self.lm_head = layers, embed, final_norm, lm_head
        self.kv, self.rope = kv, rope
        self.scale = 128 ** -0.5
        self.max_batch = max_batch
        self.use_graphs = use_graphs
        self.chunk = prefill_chunk_tokens
        self.cluster_gemm = os.environ.get("AACC_CLUSTER_GEMM", "0") == "1"
        self.skinny_rows = int(os.environ.get("AACC_SKINNY_ROWS", str(K.SKINNY_DEFAULT_ROWS)))
        if not self.skinny_shapes_ok(hidden, self.Hq, self.Hkv, self.I):
            self.skinny_rows = 0
        self.skinny_fused_rows = int(os.environ.get("AACC_SKINNY_FUSED_ROWS", str(K.SKINNY_FUSED_ROWS)))
        self.device = embed.device
        self.max_context = kv.max_blocks * kv.block_size
        self.buf = _DecodeBuffers(max_batch, hidden, self.Hq, self.I, self.vocab_local, tp, self.max_context,
                                  self.device)
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_launches: dict[int, int] = {}  # kernels per replay of the batch-B graph
        self.graph_replays = 0
        self.replayed_launches = 0  # kernels run by graph replays (sum over replays of the graph's launches)
        self.h2d_bytes = 0  # host->device bytes staged by this runtime
        self.d2h_bytes = 0
        self._pinned = torch.zeros((4, max_batch), dtype=torch.int64).pin_memory()
        self._pinned_temp = torch.zeros(max_batch, dtype=torch.float32).pin_memory()
        self._tok_host = torch.zeros(max_batch, dtype=torch.int64).pin_memory()
        # two pinned read-back buffers, so a step's tokens can be read while the next step runs
        self._tok_ring = [torch.zeros(max_batch, dtype=torch.int64).pin_memory() for _ in range(2)]
        self._tok_events = [torch.cuda.Event(), torch.cuda.Event()]
        self._tok_err = torch.zeros(2, dtype=torch.int32).pin_memory()  # device error word after each read-back
        self._tok_next = 0
        # TP: RowParallel outputs of decode-sized batches go over NVLink peer memory
        # (one fused kernel) instead of NCCL + separate residual/norm kernels.
        self.comm.enable_peer_exchange(max_batch, hidden)

    # ------------------------------------------------------------------ layers
    @staticmethod
    def skinny_shapes_ok(hidden: int, q_heads: int, kv_heads: int, inter: int) -> bool:
        """The small-batch GEMMs take output widths in whole 128-row weight
        tiles: true for every Qwen3 shape and TP slice of one."""
        return not any(n % 128 for n in (hidden, (q_heads + 2 * kv_heads) * 128, 2 * inter))

    def _splits(self, M, w, part):
        if part is None:
            return 1
        return K.pick_splits(M, w.shape[0], w.shape[1], max_elems=part.numel())

    def _cluster(self, M, part) -> bool:
        """AACC_CLUSTER_GEMM=1 runs decode-sized batches through the cluster
        split-K projections (one launch each, epilogue fused, partials summed
        in distributed shared memory).  The default is split-K through L2 +
        an epilogue kernel, measured faster at every batch from 1 to 256
        (cfg2 shapes: 45.5 vs 51.4 us per layer at B = 256, 33 vs 45 at
        B = 1): the cluster kernel's staging, two cluster barriers and
        remote reduction cost as much latency as the launch they remove."""
        return part is not None and 0 < M <= K.CLUSTER_MAX_ROWS and self.cluster_gemm

    def _skinny(self, M, part) -> bool:
        """Decode batches of at most `skinny_rows` rows (AACC_SKINNY_ROWS)
        run the small-batch GEMMs: weights as the MMA's 128-row operand, a
        third of the shared memory per CTA, so two or three CTAs share an SM
        and a projection's weight stream overlaps the kernel before it.  The
        QKV / SiLU epilogues run in the split-K epilogue kernels, or, for
        batches up to AACC_SKINNY_FUSED_ROWS (default 0: measured slower), in
        the GEMM's last split CTA of each tile."""
        return part is not None and 0 < M <= min(self.skinny_rows, K.SKINNY_MAX_ROWS) and not self.cluster_gemm

    def _skinny_part(self, M, w, part, target):
        N, Kd = w.shape
        sp = K.pick_skinny_splits(M, N, Kd, target=target, max_elems=part.numel())
        return sp, part[:sp * M * N].view(sp, M, N)

    def _qkv(self, i, lw, x, positions, slot_map, q, part):
        """Fused QKV projection + q/k-norm + RoPE + KV store (model/model.py:219-226)."""
        kv = self.kv
        M = x.shape[0]
        if self._skinny(M, part):
            sp, pv = self._skinny_part(M, lw.wqkv, part, K.SKINNY_TARGET_CTAS)
            if M <= self.skinny_fused_rows:
                K.skinny_qkv_norm_rope_store(x, lw.wqkv, pv, sp, self.buf.sk_cnt, lw.q_norm, lw.k_norm, self.eps,
                                             positions, self.rope, slot_map, kv.k[i], kv.v[i], self.Hq, q_out=q)
            else:
                K.gemm_skinny_splitk(x, lw.wqkv, pv, sp)
                K.splitk_qkv_norm_rope_store(pv, sp, lw.q_norm, lw.k_norm, self.eps, positions, self.rope, slot_map,
                                             kv.k[i], kv.v[i], self.Hq, q_out=q)
            return
        if self._cluster(M, part):
            K.qkv_norm_rope_store_cluster(x, lw.wqkv, lw.q_norm, lw.k_norm, self.eps, positions, self.rope, slot_map,
                                          kv.k[i], kv.v[i], self.Hq, q_out=q)
            return
        splits = self._splits(M, lw.wqkv, part)
        if splits > 1:
            N = lw.wqkv.shape[0]
            pv = part[:splits * M * N].view(splits, M, N)
            K.gemm_splitk(x, lw.wqkv, pv, splits)
            K.splitk_qkv_norm_rope_store(pv, splits, lw.q_norm, lw.k_norm, self.eps, positions, self.rope, slot_map,
                                         kv.k[i], kv.v[i], self.Hq, q_out=q)
        else:
            K.qkv_norm_rope_store(x, lw.wqkv, lw.q_norm, lw.k_norm, self.eps, positions, self.rope, slot_map,
                                  kv.k[i], kv.v[i], self.Hq, q_out=q)

    def _gate_up(self, lw, x, act, part):
        """gate/up projection + SiLU-mul (model/model.py:189-190)."""
        M = x.shape[0]
        if self._skinny(M, part):
            sp, pv = self._skinny_part(M, lw.w_gate_up, part, K.SKINNY_TARGET_CTAS)
            if M <= self.skinny_fused_rows:
                K.skinny_silu_mul(x, lw.w_gate_up, pv, sp, self.buf.sk_cnt, act)
            else:
                K.gemm_skinny_splitk(x, lw.w_gate_up, pv, sp)
                K.splitk_silu_mul(pv, sp, act)
            return
        if self._cluster(M, part):
            K.gemm_silu_mul_cluster(x, lw.w_gate_up, out=act)
            return
        splits = self._splits(M, lw.w_gate_up, part)
        if splits > 1:
            N = lw.w_gate_up.shape[0]
            pv = part[:splits * M * N].view(splits, M, N)
            K.gemm_splitk(x, lw.w_gate_up, pv, splits)
            K.splitk_silu_mul(pv, splits, act)
        else:
            K.gemm_silu_mul(x, lw.w_gate_up, out=act)

    def _row_parallel(self, inp, w, delta, res, norm_w, x, part):
        """RowParallel projection + residual add + next RMSNorm.  Decode-sized
        batches use split-K (every SM streams a K slice of the weight) and sum
        the fp32 partials inside the norm kernel; under TP the bf16 partial
        output is all-reduced first (RowParallelLinear, parallel_layers.py:190-195)."""
        M = inp.shape[0]
        # The NVLink exchange only runs inside captured decode graphs: there the
        # ranks replay in step, while eager launches (prefill, capture warm-up)
        # can lag by a host stall, which NCCL's blocking collectives absorb.
        graph = self.comm.size > 1 and torch.cuda.is_current_stream_capturing()
        if self._cluster(M, part):
            K.gemm_cluster(inp, w, out=delta)
            if graph and self.comm.allreduce_add_rmsnorm(delta, 0, res, norm_w, self.eps, x):
                return
            self.comm.all_reduce(delta)
            K.add_rmsnorm(delta, res, norm_w, self.eps, out=x)
            return
        if self._skinny(M, part):
            splits, pv = self._skinny_part(M, w, part, K.SKINNY_TARGET_CTAS_ROW)
            K.gemm_skinny_splitk(inp, w, pv, splits)
        else:
            splits = self._splits(M, w, part)
            pv = part[:splits * M * w.shape[0]].view(splits, M, w.shape[0]) if splits > 1 else None
            if splits > 1:
                K.gemm_splitk(inp, w, pv, splits)
        if pv is not None:
            if self.comm.size == 1:
                K.splitk_add_rmsnorm(pv, splits, res, norm_w, self.eps, out=x)
                return
            if graph and self.comm.allreduce_add_rmsnorm(pv, splits, res, norm_w, self.eps, x):
                return
            K.splitk_reduce(pv, splits, delta)
        else:
            K.gemm(inp, w, out=delta)
            if graph and self.comm.size > 1 and self.comm.allreduce_add_rmsnorm(delta, 0, res, norm_w, self.eps, x):
                return
        self.comm.all_reduce(delta)
        K.add_rmsnorm(delta, res, norm_w, self.eps, out=x)

    def _layer_chain(self, x, res, delta, q, attn, act, attend, positions, slot_map, part=None):
        """All layers for rows already embedded into (res, x); `attend(i, q, out)`
        runs this layer's attention; `part` (fp32 workspace) enables split-K."""
        L = len(self.layers)
        for i, lw in enumerate(self.layers):
            self._qkv(i, lw, x, positions, slot_map, q, part)
            attend(i, q, attn)
            self._row_parallel(attn.view(attn.shape[0], -1), lw.wo, delta, res, lw.post_ln, x, part)
            self._gate_up(lw, x, act, part)
            nxt = self.layers[i + 1].in_ln if i + 1 < L else self.final_norm
            self._row_parallel(act, lw.wd, delta, res, nxt, x, part)

    def _argmax(self, x, tokens, best, ws, logits=None, cand=None, gathered=None, sample=None):
        """Next token of each row of x (greedy, or sampled for rows whose
        temperature in `sample` = (temperature, seeds, counters) is > 0).
        Under TP every rank scores its vocab shard into `cand` (int64 [2 M]:
        global ids in [:M], fp32 scores in the first M float32 of [M:]), ONE
        all-gather collects every rank's candidates into `gathered`
        ([tp, 2 M]) and the merge kernel picks the best (lowest id on ties)."""
        t, sd, ct = sample if sample is not None else (None, None, None)
        if self.comm.size == 1:
            K.lm_head_argmax(x, self.lm_head, tokens, ws, logits=logits, best_val=best,
                             vocab_offset=self.vocab_offset, temperature=t, seeds=sd, counters=ct)
            return
        M = x.shape[0]
        K.lm_head_argmax(x, self.lm_head, cand[:M], ws, logits=logits, best_val=cand[M:].view(torch.float32)[:M],
                         vocab_offset=self.vocab_offset, temperature=t, seeds=sd, counters=ct)
        self.comm.all_gather(gathered, cand)
        K.argmax_merge_packed(gathered, M, tokens)

    # ------------------------------------------------------------------ decode
    def _decode_body(self, B: int, logits=None):
        b = self.buf
        kv = self.kv
        rows, ids, pos = b.rows[:B], b.ids[:B], b.pos[:B]
        K.decode_slot_mapping(rows, kv.seqlens, kv.block_tables, kv.block_size, kv.num_blocks, b.slot_map[:B])
        K.embed_rmsnorm(ids, self.embed, self.layers[0].in_ln, self.eps, b.res[:B], b.x[:B])

        def attend(i, q, out):
            K.paged_decode_attention(q, kv.k[i], kv.v[i], kv.block_tables, rows, kv.seqlens, ctx_add=1,
                                     scale=self.scale, max_context=self.max_context, workspace=b.attn_ws, out=out)

        self._layer_chain(b.x[:B], b.res[:B], b.delta[:B], b.q[:B], b.attn[:B], b.act[:B], attend, pos,
                          b.slot_map[:B], part=b.part)
        t = self.comm.size
        cand = b.cand[:2 * B] if t > 1 else None
        gathered = b.g_cand[:t * 2 * B].view(t, 2 * B) if t > 1 else None
        # sampling counter = position of the input token (advances on device every step)
        self._argmax(b.x[:B], ids, b.best[:B], b.lm_ws, logits=logits, cand=cand, gathered=gathered,
                     sample=(b.temp[:B], b.seed[:B], pos))
        K.advance_seqlens(rows, kv.seqlens, pos)

    def padded_batch(self, B: int) -> int:
        """Rows a decode step of B sequences runs: with CUDA graphs, B rounded
        up to a bucket (a power of two up to 8, a multiple of 8 up to 64, then
        of 32; at most max_batch), so that a batch that shrinks as sequences
        finish replays a few captured graphs instead of capturing one per
        size.  Rows past B are padding (slot index -1): the kernels skip
        their cache reads and writes and the host ignores their tokens."""
        if not self.use_graphs or B <= 0:
            return B
        if B <= 8:
            p = 1 << (B - 1).bit_length()
        elif B <= 64:
            p = (B + 7) // 8 * 8
        else:
            p = (B + 31) // 32 * 32
        return min(p, self.max_batch)

    def load_decode_inputs(self, ids, positions, rows, temperatures=None, seeds=None) -> None:
        """Stage one decode batch (host sequences of ints) into the static
        buffers, padded to padded_batch(len(rows)) rows.  `temperatures` and
        `seeds` (per row; default greedy) select temperature sampling."""
        B = len(rows)
        if B > self.max_batch:
            raise ValueError(f"decode batch {B} exceeds max_batch {self.max_batch}")
        Bp = self.padded_batch(B)
        # The pinned staging buffers may still feed an in-flight copy.
        torch.cuda.current_stream().synchronize()
        p, pt = self._pinned, self._pinned_temp
        p[0, :B] = torch.as_tensor(ids, dtype=torch.int64)
        p[1, :B] = torch.as_tensor(positions, dtype=torch.int64)
        p[2, :B] = torch.as_tensor(rows, dtype=torch.int64)
        p[3, :B] = 0 if seeds is None else torch.as_tensor(seeds, dtype=torch.int64)
        pt[:B] = 0.0 if temperatures is None else torch.as_tensor(temperatures, dtype=torch.float32)
        p[:, B:Bp] = 0
        p[2, B:Bp] = -1
        pt[B:Bp] = 0.0
        self.buf.meta[:, :Bp].copy_(p[:, :Bp], non_blocking=True)
        self.buf.temp[:Bp].copy_(pt[:Bp], non_blocking=True)
        self.h2d_bytes += 4 * Bp * 8 + 4 * Bp

    def load_positions_rows(self, positions, rows) -> None:
        """Stage positions and rows only; the ids are already on the device
        (e.g. the prefill's next tokens copied into buf.ids)."""
        B = len(rows)
        Bp = self.padded_batch(B)
        torch.cuda.current_stream().synchronize()
        p = self._pinned
        p[1, :B] = torch.as_tensor(positions, dtype=torch.int64)
        p[2, :B] = torch.as_tensor(rows, dtype=torch.int64)
        p[1, B:Bp] = 0
        p[2, B:Bp] = -1
        self.buf.meta[1:3, :Bp].copy_(p[1:3, :Bp], non_blocking=True)
        self.buf.temp[:Bp].zero_()  # greedy
        self.h2d_bytes += 2 * Bp * 8

    def reserve_decode(self, rows) -> None:
        """Host block bookkeeping for one decode step of `rows` (new token at
        lengths[row]).  Vectorised: only rows whose new token opens a block
        go through reserve (once every block_size steps)."""
        kv = self.kv
        r = np.asarray(rows, dtype=np.int64)
        need = (kv.lengths[r] + kv.block_size) // kv.block_size  # blocks for lengths + 1 tokens
        for i in np.nonzero(need > kv._nblk[r])[0]:
            kv.reserve(int(r[i]), int(kv.lengths[r[i]]) + 1)
        kv.sync()

    def decode_step(self, rows, logits: torch.Tensor | None = None) -> torch.Tensor:
        """Run one decode step on the staged inputs of `rows` (host list).  The
        next tokens overwrite buf.ids[:B] (device); positions/seqlens advance."""
        B = len(rows)
        self.reserve_decode(rows)
        if logits is not None or not self.use_graphs:
            self._decode_body(B, logits)
        else:
            Bp = self.padded_batch(B)
            g = self._graphs.get(Bp)
            if g is None:
                g = self._capture(Bp)
            g.replay()
            self.graph_replays += 1
            self.replayed_launches += self.graph_launches[Bp]
        self.kv.lengths[np.asarray(rows, dtype=np.int64)] += 1
        return self.buf.ids[:B]

    def capture_buckets(self, max_rows: int | None = None) -> None:
        """Capture the decode graph of every batch bucket up to max_rows ahead
        of a run, so that none is captured while the batch shrinks.  Each
        capture runs one eager step on all-padding rows, which reads and
        writes no sequence state.  Collective under TP: every rank captures
        the same sizes in the same order."""
        if not self.use_graphs:
            return
        top = min(max_rows or self.max_batch, self.max_batch)
        sizes = sorted({self.padded_batch(b) for b in range(1, top + 1)})
        meta, temp = self.buf.meta, self.buf.temp
        saved, saved_t = meta.clone(), temp.clone()
        meta.zero_()
        meta[2].fill_(-1)
        temp.zero_()
        for Bp in sizes:
            if Bp not in self._graphs:
                self._capture(Bp)
        meta.copy_(saved)
        temp.copy_(saved_t)

    def _capture(self, B: int) -> torch.cuda.CUDAGraph:
        # Capturing must not change state: run the body once eagerly on a
        # side stream (warms every kernel), undo its seqlen/position advance,
        # then capture.
        b, kv = self.buf, self.kv
        saved_meta = b.meta[:, :B].clone()
        saved_len = kv.seqlens.clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._decode_body(B)
        torch.cuda.current_stream().wait_stream(s)
        b.meta[:, :B].copy_(saved_meta)
        kv.seqlens.copy_(saved_len)
        g = torch.cuda.CUDAGraph()
        lib = _lib.load()
        n0 = lib.aacc_launch_count()
        with torch.cuda.graph(g):
            self._decode_body(B)
        self.graph_launches[B] = int(lib.aacc_launch_count() - n0)
        b.meta[:, :B].copy_(saved_meta)
        kv.seqlens.copy_(saved_len)
        self._graphs[B] = g
        return g

    def read_tokens(self, B: int) -> list[int]:
        """D2H of the last decode step's tokens (synchronises the stream)."""
        t = self._tok_host[:B]
        t.copy_(self.buf.ids[:B], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        self.d2h_bytes += B * 8
        return t.tolist()

    def copy_tokens_async(self, B: int) -> int:
        """Queue the D2H of the last decode step's tokens into one of two pinned
        buffers, behind that step on the stream (a later step overwriting the
        device ids runs after the copy).  Returns the handle for wait_tokens;
        each buffer is reused every second call."""
        i = self._tok_next
        self._tok_next ^= 1
        self._tok_ring[i][:B].copy_(self.buf.ids[:B], non_blocking=True)
        _lib.check(_lib.load().aacc_get_device_error_async(self._tok_err[i:].data_ptr(), _stream()),
                   "aacc_get_device_error_async")
        self._tok_events[i].record()
        self.d2h_bytes += B * 8
        return i

    def wait_tokens(self, handle: int, B: int) -> list[int]:
        """Tokens of a copy_tokens_async call (waits for that copy only)."""
        self._tok_events[handle].synchronize()
        return self._tok_ring[handle][:B].tolist()

    def token_error(self, handle: int) -> int:
        """The device error word as it stood after that step (after wait_tokens)."""
        return int(self._tok_err[handle])

    # ------------------------------------------------------------------ prefill
    def prefill(self, sequences: list[list[int]], rows: list[int], *, positions: list[list[int]] | None = None,
                store_lengths: list[int] | None = None, all_logits: bool = False, last_logits: bool = False,
                temperatures: list[float] | None = None, seeds: list[int] | None = None):
        """Packed (chunked) prefill of whole prompts into `rows`.

        Returns the next token of every sequence (device int64 [n]): greedy,
        or sampled where `temperatures` (per sequence, with `seeds`) is > 0;
        with ``last_logits`` also the bf16 logits of the last tokens [n, V];
        with ``all_logits`` the logits of every token [T, V] instead (greedy)."""
        kv = self.kv
        n = len(sequences)
        lens = [len(s) for s in sequences]
        if min(lens) <= 0:
            raise ValueError("empty prompt")
        for r, L in zip(rows, lens):
            kv.reserve(r, L)
        kv.sync()
        T = sum(lens)
        dev = self.device
        flat = np.fromiter((t for s in sequences for t in s), dtype=np.int64, count=T)
        if positions is None:
            pos = np.concatenate([np.arange(L, dtype=np.int64) for L in lens])
        else:
            pos = np.concatenate([np.asarray(p, dtype=np.int64) for p in positions])
        smap = np.concatenate([kv.slot_mapping(r, 0, L) for r, L in zip(rows, lens)])
        host = torch.from_numpy(np.stack([flat, pos, smap])).pin_memory()
        meta = host.to(dev, non_blocking=True)
        self.h2d_bytes += host.numel() * 8
        ids_d, pos_d, smap_d = meta[0], meta[1], meta[2]
        tokens = torch.empty(n, dtype=torch.int64, device=dev)
        samp = None
        if temperatures is not None and any(t > 0 for t in temperatures):
            last_pos = [L - 1 for L in lens] if positions is None else [int(p_[-1]) for p_ in positions]
            sh = torch.tensor([list(seeds or [0] * n), last_pos], dtype=torch.int64).pin_memory()
            th = torch.tensor(list(temperatures), dtype=torch.float32).pin_memory()
            sd = sh.to(dev, non_blocking=True)
            samp = (th.to(dev, non_blocking=True), sd[0], sd[1])  # counter = position of the last prompt token
            self.h2d_bytes += sh.numel() * 8 + th.numel() * 4
        V = self.vocab if self.comm.size == 1 else self.vocab_local
        out_logits = None
        if all_logits:
            out_logits = torch.empty((T, V), dtype=torch.bfloat16, device=dev)
        elif last_logits:
            out_logits = torch.empty((n, V), dtype=torch.bfloat16, device=dev)

        # Chunk plan: pieces (seq index, start, end) with at most self.chunk tokens per chunk.
        chunks, cur, cur_tok = [], [], 0
        offs = np.concatenate([[0], np.cumsum(lens)])
        for si, L in enumerate(lens):
            st = 0
            while st < L:
                take = min(L - st, self.chunk - cur_tok)
                cur.append((si, st, st + take))
                cur_tok += take
                st += take
                if cur_tok == self.chunk:
                    chunks.append(cur)
                    cur, cur_tok = [], 0
        if cur:
            chunks.append(cur)

        H = self.H
        maxT = max(sum(e - s for _, s, e in ch) for ch in chunks)
        bf = dict(dtype=torch.bfloat16, device=dev)
        res = torch.empty((maxT, H), **bf)
        x = torch.empty((maxT, H), **bf)
        delta = torch.empty((maxT, H), **bf)
        q = torch.empty((maxT, self.Hq, 128), **bf)
        attn = torch.empty((maxT, self.Hq, 128), **bf)
        act = torch.empty((maxT, self.I), **bf)
        lm_ws = torch.empty(K.lm_head_workspace_bytes(maxT if all_logits else n, self.vocab_local),
                            dtype=torch.uint8, device=dev)
        best = torch.empty(maxT if all_logits else n, dtype=torch.float32, device=dev)
        for ch in chunks:
            t0 = int(offs[ch[0][0]] + ch[0][1])
            Tc = sum(e - s for _, s, e in ch)
            npc = len(ch)
            # Sequences whose last token lies in this chunk: consecutive indices [a, a + m).
            ends = [(si, int(offs[si] + e - 1 - t0)) for si, s, e in ch if e == lens[si]]
            # Per-piece attention metadata: block-table row, query offsets, context before the piece.
            cu = np.zeros(npc + 1, dtype=np.int64)
            cu[1:] = np.cumsum([e - s for _, s, e in ch])
            m64 = np.concatenate([np.asarray([rows[si] for si, _, _ in ch], dtype=np.int64),
                                  np.asarray([r for _, r in ends], dtype=np.int64)])
            m32 = np.concatenate([cu, np.asarray([s for _, s, _ in ch], dtype=np.int64)]).astype(np.int32)
            d64 = torch.from_numpy(m64).pin_memory().to(dev, non_blocking=True)
            d32 = torch.from_numpy(m32).pin_memory().to(dev, non_blocking=True)
            self.h2d_bytes += m64.size * 8 + m32.size * 4
            seq_rows, last_idx = d64[:npc], d64[npc:]
            cu_q, ctx0 = d32[:npc + 1], d32[npc + 1:]
            max_q = max(e - s for _, s, e in ch)
            xs, rs, ds = x[:Tc], res[:Tc], delta[:Tc]
            K.embed_rmsnorm(ids_d[t0:t0 + Tc], self.embed, self.layers[0].in_ln, self.eps, rs, xs)

            def attend(i, qq, out, seq_rows=seq_rows, cu_q=cu_q, ctx0=ctx0, max_q=max_q):
                K.prefill_attention(qq, kv.k[i], kv.v[i], kv.block_tables, seq_rows, cu_q, ctx0, max_q_len=max_q,
                                    scale=self.scale, out=out)

            self._layer_chain(xs, rs, ds, q[:Tc], attn[:Tc], act[:Tc], attend, pos_d[t0:t0 + Tc],
                              smap_d[t0:t0 + Tc])
            if all_logits:
                tk = torch.empty(Tc, dtype=torch.int64, device=dev)
                K.lm_head_argmax(xs, self.lm_head, tk, lm_ws, logits=out_logits[t0:t0 + Tc], best_val=best[:Tc],
                                 vocab_offset=self.vocab_offset)
            elif ends:
                a, m = ends[0][0], len(ends)
                hx = K.gather_rows(xs, last_idx)
                lg = out_logits[a:a + m] if last_logits else None
                sm = None if samp is None else tuple(t[a:a + m] for t in samp)
                if self.comm.size > 1:
                    cand = torch.empty(2 * m, dtype=torch.int64, device=dev)
                    gathered = torch.empty((self.comm.size, 2 * m), dtype=torch.int64, device=dev)
                    self._argmax(hx, tokens[a:a + m], best[a:a + m], lm_ws, logits=lg, cand=cand, gathered=gathered,
                                 sample=sm)
                else:
                    self._argmax(hx, tokens[a:a + m], best[a:a + m], lm_ws, logits=lg, sample=sm)
        if all_logits:
            last = torch.from_numpy(offs[1:] - 1).to(dev)
            K.argmax_rows(K.gather_rows(out_logits, last), tokens)
        kv.set_lengths(rows, store_lengths if store_lengths is not None else lens)
        return (tokens, out_logits) if (all_logits or last_logits) else tokens
