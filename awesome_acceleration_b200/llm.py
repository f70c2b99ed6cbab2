"""Single-GPU continuous-batching engine with the reference's public API.

Mirrors yijichar/AWesome_ACceleration ``llm.py``: ``LLM(model_path,
max_num_seqs, max_seq_len, dtype)``, ``generate`` / ``chat`` returning a
``concurrent.futures.Future`` of ``list[GenerationOutput]``, ``stop``, and
the background ``_inference_loop`` with the same phases (drain queue, assign
lowest free slots, prefill new sequences, one decode step for all active
sequences, stop checks).  ``generate_ids`` takes token ids directly (the
reference only accepts strings; synthetic benchmarks need ids).

The per-step model work runs on the B200 kernels: a packed, chunked prefill
and a CUDA-graph-captured decode step whose greedy argmax is fused into the
lm_head GEMM, so the host only reads back one int64 per sequence per step.
"""
from __future__ import annotations

import bisect
import concurrent.futures
import itertools
import os
import queue
import threading
import time
from dataclasses import dataclass, field

import torch

from .model.model import Qwen3Config, Qwen3ForCausalLM


@dataclass
class GenerationOutput:
    """Result of a single prompt generation (llm.py:15-21)."""
    text: str
    token_ids: list[int]
    prompt_tokens: int = 0
    generated_tokens: int = 0


@dataclass
class _Request:
    """Internal request tracking for continuous batching (llm.py:24-33)."""
    token_ids: list[list[int]]
    max_tokens: int
    temperature: float
    ignore_eos: bool
    future: concurrent.futures.Future
    results: list = field(default_factory=list)
    pending_indices: list = field(default_factory=list)
    seeds: list = field(default_factory=list)  # per prompt: key of its sampling noise (temperature > 0)


_M64 = (1 << 64) - 1


def sampling_seed(base: int, serial: int, index: int) -> int:
    """Seed of prompt `index` of the `serial`-th request of an engine seeded
    with `base` (SplitMix64 output function; a non-negative int64)."""
    z = (base * 0x100000001B3 + serial * 0x10001 + index + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return (z ^ (z >> 31)) & 0x7FFFFFFFFFFFFFFF


def kv_sized_max_seqs(config: Qwen3Config, max_num_seqs: int, max_seq_len: int, reserve_gb: float,
                      device, tp_size: int = 1, prefill_chunk_tokens: int = 0) -> int:
    """The reference's batch sizing from GPU memory (llm.py:58-71, llm_tp.py:160-178):
    KV bytes per token (this rank's heads) against the memory left after a fixed
    reserve.  Called once the weights are on the device, it also keeps the
    memory they already hold and one prefill chunk's activations out of the
    KV budget: the reference's fixed reserve only covers a 0.6B model."""
    torch.cuda.synchronize(device)
    torch.cuda.empty_cache()  # blocks the allocator caches (e.g. weight-init temporaries) are free for the KV pool
    free, total = torch.cuda.mem_get_info(device)
    per_tok = 2 * config.num_key_value_heads * config.head_dim * 2 * config.num_hidden_layers // tp_size
    q_cols = config.num_attention_heads * config.head_dim // tp_size
    act = prefill_chunk_tokens * (3 * config.hidden_size + 2 * q_cols + config.intermediate_size // tp_size) * 2
    reserve = reserve_gb * (1024 ** 3)
    avail = min(total - reserve, free - reserve - act)
    return max(1, min(max_num_seqs, int(avail / per_tok) // max_seq_len))


class LLM:
    """High-throughput Qwen3 engine with continuous batching on one B200."""

    def __init__(self, model_path: str | None = None, max_num_seqs: int = 32, max_seq_len: int = 4096,
                 dtype=torch.bfloat16, *, config: Qwen3Config | None = None, model: Qwen3ForCausalLM | None = None,
                 seed: int = 0, block_size: int = 256, use_cuda_graphs: bool = True,
                 prefill_chunk_tokens: int = 32768, device=None, verbose: bool = False):
        self.device = torch.device(device or "cuda")
        if self.device.type == "cuda" and self.device.index is None:  # pin it: the loop runs in another thread
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        self.max_seq_len = max_seq_len
        self.verbose = verbose
        self.tokenizer = None
        if model is not None:
            self.model = model
            self.config = model.config
        elif model_path is not None and os.path.exists(os.path.join(model_path, "model.safetensors")):
            self.config = Qwen3Config.from_json(os.path.join(model_path, "config.json"))
            self.model = Qwen3ForCausalLM.from_pretrained(model_path, self.config, self.device, dtype)
        else:
            if config is None and model_path is not None:
                config = Qwen3Config.from_json(os.path.join(model_path, "config.json"))
            self.config = config or Qwen3Config()
            self.model = Qwen3ForCausalLM.random_init(self.config, self.device, dtype, seed=seed)
        if model_path is not None and os.path.exists(os.path.join(model_path, "tokenizer_config.json")):
            from transformers import AutoTokenizer
            self.tokenizer = AutoTokenizer.from_pretrained(model_path, trust_remote_code=True)
        self.model.eval()
        self.model.use_cuda_graphs = use_cuda_graphs
        self.model.prefill_chunk_tokens = prefill_chunk_tokens
        self.model.fuse_qkv()  # before sizing: the fused weights are what stays resident
        self.max_num_seqs = kv_sized_max_seqs(self.config, max_num_seqs, max_seq_len, 3.0, self.device,
                                              prefill_chunk_tokens=prefill_chunk_tokens)
        self.model.init_kv_cache(self.max_num_seqs, max_seq_len, self.device, dtype, block_size=block_size)
        self._request_queue: queue.Queue[_Request] = queue.Queue()
        self._base_seed = int(seed)  # sampling noise: one stream per (request, prompt)
        self._serials = itertools.count(1)
        self._loop_running = False
        self._loop_thread = None
        self._loop_error: BaseException | None = None
        self.stats = {"prefill_s": 0.0, "decode_s": 0.0, "decode_steps": 0, "prefill_tokens": 0}
        self._warmup()

    # ----------------------------------------------------------------- internals
    def _warmup(self):
        """One prefill + one decode step on slot 0, then reset (llm.py:102-108)."""
        rt = self.model._rt()
        rt.prefill([[0]], [0])
        rt.load_decode_inputs([0], [1], [0])
        rt.decode_step([0])
        rt.read_tokens(1)
        self.model.clear_all_slots()
        torch.cuda.synchronize(self.device)

    @torch.inference_mode()
    def _prefill(self, sequences: list[list[int]], slot_indices: list[int]) -> torch.Tensor:
        """Packed prefill of `sequences` into `slot_indices` -> last-token logits
        [n, V] (llm.py:116-208)."""
        _, logits = self.model._rt().prefill(sequences, list(slot_indices), last_logits=True)
        return logits

    @torch.inference_mode()
    def _decode_step(self, input_ids: torch.Tensor, positions: torch.Tensor,
                     slot_indices: torch.Tensor) -> torch.Tensor:
        """One decode step -> logits [B, V] (llm.py:210-213)."""
        return self.model(input_ids, positions, slot_indices)[:, 0, :]

    def _sample_tokens(self, logits: torch.Tensor, temperature: float) -> list[int]:
        """Next tokens from materialised logits [B, V] (llm.py:215-219): greedy
        at temperature 0, else softmax(logits / T) sampling with the kernel's
        Gumbel-max draw (fresh seeds from the engine's stream)."""
        from .kernels import argmax_rows, sample_rows
        if temperature == 0:
            return argmax_rows(logits.contiguous()).tolist()
        B = logits.shape[0]
        serial = next(self._serials)
        seeds = [sampling_seed(self._base_seed, serial, i) for i in range(B)]
        return sample_rows(logits.contiguous(), [float(temperature)] * B, seeds, [0] * B).tolist()

    def _ensure_loop(self):
        if self._loop_error is not None:
            raise RuntimeError("inference loop failed") from self._loop_error
        if not self._loop_running:
            self._loop_running = True
            self._loop_thread = threading.Thread(target=self._inference_loop, daemon=True)
            self._loop_thread.start()

    def _submit(self, token_ids, max_tokens, temperature, ignore_eos) -> concurrent.futures.Future:
        if temperature < 0:
            raise ValueError(f"temperature must be >= 0, got {temperature}")
        for t in token_ids:
            if len(t) == 0:
                raise ValueError("empty prompt")
            if len(t) >= self.max_seq_len:
                raise ValueError(f"prompt of {len(t)} tokens does not fit max_seq_len={self.max_seq_len}")
        self._ensure_loop()
        future = concurrent.futures.Future()
        serial = next(self._serials)
        req = _Request(token_ids=[list(map(int, t)) for t in token_ids], max_tokens=max_tokens,
                       temperature=temperature, ignore_eos=ignore_eos, future=future,
                       results=[None] * len(token_ids), pending_indices=list(range(len(token_ids))),
                       seeds=[sampling_seed(self._base_seed, serial, i) for i in range(len(token_ids))])
        self._request_queue.put(req)
        return future

    # ----------------------------------------------------------------- public API
    def generate(self, prompts: list[str], max_tokens: int = 100, temperature: float = 0.0,
                 ignore_eos: bool = False) -> concurrent.futures.Future:
        """Submit text prompts (chat template applied, llm.py:225-264)."""
        if self.tokenizer is None:
            raise RuntimeError("no tokenizer loaded: use generate_ids() with token ids")
        ids = []
        for p in prompts:
            text = self.tokenizer.apply_chat_template([{"role": "user", "content": p}], tokenize=False,
                                                      add_generation_prompt=True)
            ids.append(self.tokenizer.encode(text, add_special_tokens=False))
        return self._submit(ids, max_tokens, temperature, ignore_eos)

    def generate_ids(self, token_ids: list[list[int]], max_tokens: int = 100, temperature: float = 0.0,
                     ignore_eos: bool = False) -> concurrent.futures.Future:
        """Submit prompts as token ids; same semantics as ``generate``."""
        return self._submit(token_ids, max_tokens, temperature, ignore_eos)

    def chat(self, messages: list[dict], max_tokens: int = 100, temperature: float = 0.0,
             ignore_eos: bool = False) -> concurrent.futures.Future:
        """Multi-turn chat generation (llm.py:266-300)."""
        if self.tokenizer is None:
            raise RuntimeError("no tokenizer loaded")
        text = self.tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True)
        return self._submit([self.tokenizer.encode(text, add_special_tokens=False)], max_tokens, temperature,
                            ignore_eos)

    def stop(self, timeout: float = 30.0):
        """Stop the background loop (llm.py:302-309)."""
        if not self._loop_running:
            return
        self._loop_running = False
        if self._loop_thread:
            self._loop_thread.join(timeout=timeout)
            self._loop_thread = None

    def _decode_text(self, tokens: list[int]) -> str:
        return self.tokenizer.decode(tokens, skip_special_tokens=True) if self.tokenizer is not None else ""

    # ----------------------------------------------------------------- loop
    @torch.inference_mode()
    def _inference_loop(self):
        """Continuous batching (llm.py:315-446).  Any exception fails every
        outstanding request's future instead of leaving it unresolved."""
        active: dict[int, list] = {}
        pending: list[_Request] = []
        try:
            if self.device.type == "cuda":  # a new thread starts on device 0: run on the engine's GPU
                torch.cuda.set_device(self.device)
            self._run_loop(active, pending)
        except BaseException as e:  # noqa: BLE001 - propagate to every waiter
            self._loop_error = e
            self._loop_running = False
            seen = set()
            for req in [r for r, *_ in active.values()] + pending:
                if id(req) not in seen and not req.future.done():
                    seen.add(id(req))
                    req.future.set_exception(e)
            while True:
                try:
                    req = self._request_queue.get_nowait()
                except queue.Empty:
                    break
                if not req.future.done():
                    req.future.set_exception(e)

    def _finish(self, req: _Request, idx: int, tokens: list[int]):
        req.results[idx] = GenerationOutput(self._decode_text(tokens), tokens, len(req.token_ids[idx]), len(tokens))
        if all(r is not None for r in req.results):
            req.future.set_result(req.results)

    def _run_loop(self, active: dict, pending: list):
        rt = self.model._rt()
        kv = self.model.kv
        free_slots = list(range(self.max_num_seqs))
        eos = self.config.eos_token_id
        self.model.clear_all_slots()
        staged: list[int] | None = None  # rows whose inputs the device buffers hold
        # Decode steps launched but not read yet: (rows, read-back handle, launch time).  While
        # the host reads step t's tokens and runs the stop checks, step t+1 already runs on the
        # device (the graph takes its ids and positions from step t on the device).
        inflight: list = []
        t_last = time.perf_counter()
        while self._loop_running or pending or active or inflight:
            # Phase 1: drain the queue.
            while True:
                try:
                    pending.append(self._request_queue.get_nowait())
                except queue.Empty:
                    break
            if not pending and not active and not inflight:
                if not self._loop_running:
                    break
                time.sleep(0.001)
                continue
            if not inflight:  # the batch only changes between steps that are all read
                # Phase 2: lowest free slots to pending prompts.
                new_work = []
                for req in list(pending):
                    while req.pending_indices and free_slots:
                        new_work.append((req, req.pending_indices.pop(0), free_slots.pop(0)))
                    if not req.pending_indices:
                        pending.remove(req)
                # Phase 3: prefill.
                if new_work:
                    t0 = time.perf_counter()
                    seqs = [r.token_ids[i] for r, i, _ in new_work]
                    slots = [s for _, _, s in new_work]
                    # per-request temperature (the reference applies the first request's to the whole batch)
                    toks = rt.prefill(seqs, slots, temperatures=[r.temperature for r, _, _ in new_work],
                                      seeds=[r.seeds[i] for r, i, _ in new_work]).tolist()
                    rt.d2h_bytes += 8 * len(toks)
                    self.stats["prefill_s"] += time.perf_counter() - t0
                    self.stats["prefill_tokens"] += sum(len(s) for s in seqs)
                    for (req, idx, slot), tok in zip(new_work, toks):
                        plen = len(req.token_ids[idx])
                        if 1 >= req.max_tokens or (not req.ignore_eos and tok == eos):
                            self._finish(req, idx, [tok])
                            kv.release(slot)
                            bisect.insort(free_slots, slot)
                        else:
                            active[slot] = [req, idx, [tok], plen]
                    staged = None
                if not active:
                    continue
            # Phase 4: decode steps.
            slots = list(active.keys())
            if not inflight:
                if staged != slots:
                    rt.load_decode_inputs([active[s][2][-1] for s in slots], [active[s][3] for s in slots], slots,
                                          temperatures=[active[s][0].temperature for s in slots],
                                          seeds=[active[s][0].seeds[active[s][1]] for s in slots])
                    staged = slots
                inflight.append(self._launch_step(rt, slots))
            # Run one step ahead when that cannot change the batch: no row reaches its
            # max_tokens / max_seq_len limit in the step being read (an EOS stop can still
            # end a row; its extra token is dropped), and no waiting request could take a
            # slot freed by it.
            if (len(inflight) == 1 and inflight[0][0] == slots and not (pending and free_slots)
                    and all(len(st[2]) + 1 < st[0].max_tokens and st[3] + 1 < self.max_seq_len
                            for st in active.values())):
                inflight.append(self._launch_step(rt, slots))
            step_slots, handle, t0 = inflight.pop(0)
            sampled = rt.wait_tokens(handle, len(step_slots))
            now = time.perf_counter()
            self.stats["decode_s"] += now - max(t0, t_last)
            self.stats["decode_steps"] += 1
            t_last = now
            # Phase 5: stop checks (rows that ended at an earlier step are skipped).
            finished = False
            for slot, tok in zip(step_slots, sampled):
                st = active.get(slot)
                if st is None:
                    continue
                st[2].append(tok)
                st[3] += 1
                req = st[0]
                if (len(st[2]) >= req.max_tokens or st[3] >= self.max_seq_len
                        or (not req.ignore_eos and tok == eos)):
                    self._finish(req, st[1], st[2])
                    del active[slot]
                    kv.release(slot)
                    bisect.insort(free_slots, slot)
                    finished = True
            if finished:
                staged = None

    @staticmethod
    def _launch_step(rt, slots):
        """One decode step of `slots` plus the queued read-back of its tokens."""
        t0 = time.perf_counter()
        rt.decode_step(slots)
        return slots, rt.copy_tokens_async(len(slots)), t0
