"""Tensor-parallel / DP x TP engine with the reference's public API.

Mirrors yijichar/AWesome_ACceleration ``llm_tp.py``: ``LLMTP(model_path,
max_num_seqs, max_seq_len, dtype, enable_tp, tp_size)`` run under torchrun,
one process per GPU.  The TP-group leader (tp_rank 0) owns the request queue,
the scheduler and the results; the other ranks run ``serve_worker()`` and
follow pickled control messages over the TP Gloo group (actions ``exit``,
``release``, ``clear_all_slots``, ``prefill_flat``, ``decode``), exactly the
reference's leader/worker protocol (:705-760, :766-984).  DP replicas (world
= dp * tp) each run their own leader and scheduler (:83-120).

Per-step device work: the decode inputs travel as one packed [3, B] int64
NCCL broadcast (ids | positions | rows, llm_tp.py:301-338) and only when the
batch composition changed; the decode step itself (RowParallel all-reduces,
vocab-parallel argmax merge) is one CUDA graph per batch size, so every rank
ends the step with the same next tokens without further messages.
"""
from __future__ import annotations

import bisect
import concurrent.futures
import itertools
import os
import queue
import threading
import time

import torch

from . import _lib
from .llm import GenerationOutput, _Request, kv_sized_max_seqs, sampling_seed
from .model import distributed as D
from .model.model import Qwen3Config, Qwen3ForCausalLM
from .model.model_tp import Qwen3ForCausalLMTP

__all__ = ["LLMTP", "GenerationOutput"]


class LLMTP:
    def __init__(self, model_path: str | None = None, max_num_seqs: int = 32, max_seq_len: int = 1024,
                 dtype=torch.bfloat16, enable_tp: bool = True, tp_size: int = 1, *,
                 config: Qwen3Config | None = None, state_dict: dict | None = None, seed: int = 0,
                 block_size: int = 256, use_cuda_graphs: bool = True, prefill_chunk_tokens: int = 32768,
                 timeout_s: float = 300.0):
        if enable_tp:
            D.init_distributed(tp_size=tp_size, timeout_s=timeout_s)
        self.tp_size = D.get_tp_world_size()
        self.tp_rank = D.get_tp_rank()
        self.dp_size = D.get_dp_world_size()
        self.dp_rank = D.get_dp_rank()
        self.global_rank = D.get_global_rank()
        self.is_tp_leader = D.is_tp_leader()
        self.is_global_rank_0 = D.is_global_rank_0()
        self.is_rank_0 = self.is_tp_leader
        local = int(os.environ.get("LOCAL_RANK", 0))
        self.device = torch.device(f"cuda:{local}")
        self.dtype = dtype
        self.max_seq_len = max_seq_len
        if config is None and model_path is not None:
            config = Qwen3Config.from_json(os.path.join(model_path, "config.json"))
        self.config = config or Qwen3Config()
        tp = self.tp_size > 1
        Model = Qwen3ForCausalLMTP if tp else Qwen3ForCausalLM
        has_ckpt = model_path is not None and os.path.exists(os.path.join(model_path, "model.safetensors"))
        if state_dict is not None:
            if tp:
                self.model = Qwen3ForCausalLMTP.from_state_dict(state_dict, self.config, self.device, dtype)
            else:
                with torch.device("meta"):
                    m = Qwen3ForCausalLM(self.config)
                m = m.to_empty(device=self.device).to(dtype)
                m.load_state_dict({k: v.to(dtype) for k, v in state_dict.items()}, strict=False)
                self.model = m
        elif has_ckpt:
            self.model = Model.from_pretrained(model_path, self.config, self.device, dtype)
        else:
            self.model = Model.random_init(self.config, self.device, dtype, seed=seed)
        self.tokenizer = None
        if self.is_tp_leader and model_path is not None and \
                os.path.exists(os.path.join(model_path, "tokenizer_config.json")):
            from transformers import AutoTokenizer
            self.tokenizer = AutoTokenizer.from_pretrained(model_path, trust_remote_code=True)
        self.model.eval()
        self.model.use_cuda_graphs = use_cuda_graphs
        self.model.prefill_chunk_tokens = prefill_chunk_tokens
        self.model.fuse_qkv()  # before sizing: the fused weights are what stays resident
        self.max_num_seqs = kv_sized_max_seqs(self.config, max_num_seqs, max_seq_len, 15.0, self.device, self.tp_size,
                                              prefill_chunk_tokens)
        if self.tp_size > 1:  # free memory differs a little per GPU; the group must agree on slots and buckets
            n = torch.tensor([self.max_num_seqs], dtype=torch.int64)
            torch.distributed.all_reduce(n, op=torch.distributed.ReduceOp.MIN, group=D.get_tp_cpu_group())
            self.max_num_seqs = int(n.item())
        self.model.init_kv_cache(self.max_num_seqs, max_seq_len, self.device, dtype, block_size=block_size)
        self._bcast = torch.zeros(5 * self.model.max_batch, dtype=torch.int64, device=self.device)
        self._base_seed = int(seed)  # sampling noise: one stream per (request, prompt)
        self._serials = itertools.count(1)
        self._request_queue: queue.Queue | None = queue.Queue() if self.is_tp_leader else None
        self._loop_running = False
        self._loop_thread = None
        self._loop_error: BaseException | None = None
        self.prof = None
        self._barrier()
        self._warmup()
        self._barrier()

    # ----------------------------------------------------------------- helpers
    def _barrier(self):
        if self.tp_size > 1:
            torch.distributed.barrier(group=D.get_tp_cpu_group())

    def _warmup(self):
        rt = self.model._rt()
        rt.prefill([[0]], [0])
        rt.load_decode_inputs([0], [1], [0])
        rt.decode_step([0])
        torch.cuda.synchronize(self.device)
        self.model.clear_all_slots()

    def _stage_decode(self, ids, positions, rows, temperatures=None, seeds=None):
        """Leader: one packed [5, B] NCCL broadcast of ids | positions | rows |
        sampling seeds | temperature bits into every rank's decode buffers
        (llm_tp.py:301-338)."""
        rt = self.model._rt()
        B = rt.padded_batch(len(rows))  # padding rows included
        bc = self._bcast[:5 * B].view(5, B)
        if self.is_tp_leader:
            rt.load_decode_inputs(ids, positions, rows, temperatures, seeds)
            bc[:4].copy_(rt.buf.meta[:, :B])
            bc[4].copy_(rt.buf.temp[:B].view(torch.int32))
        D.broadcast_tensor(self._bcast[:5 * B], src=0)
        if not self.is_tp_leader:
            rt.buf.meta[:, :B].copy_(bc[:4])
            rt.buf.temp[:B].view(torch.int32).copy_(bc[4])

    # ----------------------------------------------------------------- public API (leader)
    def generate(self, prompts: list[str], max_tokens: int = 100, temperature: float = 0.0,
                 ignore_eos: bool = False) -> concurrent.futures.Future:
        assert self.is_tp_leader, "generate() should only be called on the TP-group leader."
        if self.tokenizer is None:
            raise RuntimeError("no tokenizer loaded: use generate_ids() with token ids")
        ids = []
        for p in prompts:
            text = self.tokenizer.apply_chat_template([{"role": "user", "content": p}], tokenize=False,
                                                      add_generation_prompt=True)
            ids.append(self.tokenizer.encode(text, add_special_tokens=False))
        return self.generate_ids(ids, max_tokens, temperature, ignore_eos)

    def generate_ids(self, token_ids: list[list[int]], max_tokens: int = 100, temperature: float = 0.0,
                     ignore_eos: bool = False) -> concurrent.futures.Future:
        assert self.is_tp_leader, "generate_ids() should only be called on the TP-group leader."
        if temperature < 0:
            raise ValueError(f"temperature must be >= 0, got {temperature}")
        for t in token_ids:
            if len(t) == 0 or len(t) >= self.max_seq_len:
                raise ValueError(f"prompt length {len(t)} outside [1, max_seq_len)")
        if self._loop_error is not None:
            raise RuntimeError("inference loop failed") from self._loop_error
        if not self._loop_running:
            self._loop_running = True
            self._loop_thread = threading.Thread(target=self._inference_loop, daemon=True)
            self._loop_thread.start()
        fut = concurrent.futures.Future()
        serial = next(self._serials)
        self._request_queue.put(_Request([list(map(int, t)) for t in token_ids], max_tokens, temperature, ignore_eos,
                                         fut, [None] * len(token_ids), list(range(len(token_ids))),
                                         [sampling_seed(self._base_seed, serial, i) for i in range(len(token_ids))]))
        return fut

    def chat(self, messages: list[dict], max_tokens: int = 100, temperature: float = 0.0,
             ignore_eos: bool = False) -> concurrent.futures.Future:
        assert self.is_tp_leader, "chat() should only be called on the TP-group leader."
        if self.tokenizer is None:
            raise RuntimeError("no tokenizer loaded")
        text = self.tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True)
        return self.generate_ids([self.tokenizer.encode(text, add_special_tokens=False)], max_tokens, temperature,
                                 ignore_eos)

    def stop(self, timeout: float = 30.0):
        """Stop the leader loop; it broadcasts ``exit`` to the workers (llm_tp.py:636-646)."""
        if self.is_tp_leader:
            self._loop_running = False
            if self._loop_thread is not None:
                self._loop_thread.join(timeout=timeout)
                self._loop_thread = None

    def serve_worker(self):
        """Worker ranks: follow the leader's commands until ``exit`` (llm_tp.py:289-295)."""
        assert not self.is_tp_leader, "serve_worker() should only be called on TP worker ranks."
        self._worker_loop()

    # ----------------------------------------------------------------- worker loop
    @torch.inference_mode()
    def _worker_loop(self):
        rt = self.model._rt()
        kv = self.model.kv
        self.model.clear_all_slots()
        rows: list[int] = []
        while True:
            ctl = D.broadcast_object(None, src=0)
            act = ctl["action"]
            if act == "exit":
                break
            if act == "release":
                for s in ctl["slots"]:
                    kv.release(int(s))
            elif act == "clear_all_slots":
                self.model.clear_all_slots()
            elif act == "prefill_flat":
                rt.prefill(ctl["sequences"], ctl["slots"], temperatures=ctl.get("temperatures"), seeds=ctl.get("seeds"))
            elif act == "decode":
                if ctl.get("restage"):
                    rows = ctl["slots"]
                    self._stage_decode(None, None, rows)
                rt.decode_step(rows)
            else:
                raise RuntimeError(f"[Rank {self.tp_rank}] Unknown action: {act}")
        torch.cuda.synchronize(self.device)

    # ----------------------------------------------------------------- leader loop
    @torch.inference_mode()
    def _inference_loop(self):
        if self.device.type == "cuda":  # a new thread starts on device 0: run on this rank's GPU
            torch.cuda.set_device(self.device)
        if not self.is_tp_leader:
            self._worker_loop()
            return
        active: dict[int, list] = {}
        pending: list[_Request] = []
        try:
            self._leader_loop(active, pending)
            if self.tp_size > 1:
                D.broadcast_object({"action": "exit"}, src=0)
        except BaseException as e:  # noqa: BLE001
            self._loop_error = e
            self._loop_running = False
            if self.tp_size > 1:
                try:
                    D.broadcast_object({"action": "exit"}, src=0)
                except Exception:  # noqa: BLE001
                    pass
            for req in {id(r): r for r, *_ in active.values()}.values():
                if not req.future.done():
                    req.future.set_exception(e)
            for req in pending:
                if not req.future.done():
                    req.future.set_exception(e)

    def _send(self, msg):
        if self.tp_size > 1:
            D.broadcast_object(msg, src=0)

    def _finish(self, req, idx, tokens):
        text = self.tokenizer.decode(tokens, skip_special_tokens=True) if self.tokenizer is not None else ""
        req.results[idx] = GenerationOutput(text, tokens, len(req.token_ids[idx]), len(tokens))
        if all(r is not None for r in req.results):
            req.future.set_result(req.results)

    def _leader_loop(self, active, pending):
        rt = self.model._rt()
        kv = self.model.kv
        eos = self.config.eos_token_id
        free_slots = list(range(self.max_num_seqs))
        self.model.clear_all_slots()
        self._send({"action": "clear_all_slots"})
        staged = None
        # Decode steps launched (and sent to the workers) but not read yet: (rows, read-back
        # handle).  While the leader reads step t's tokens, step t+1 already runs on every rank.
        inflight: list = []
        while self._loop_running or pending or active or inflight:
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
                new_work = []
                for req in list(pending):
                    while req.pending_indices and free_slots:
                        new_work.append((req, req.pending_indices.pop(0), free_slots.pop(0)))
                    if not req.pending_indices:
                        pending.remove(req)
                if new_work:
                    seqs = [r.token_ids[i] for r, i, _ in new_work]
                    slots = [s for _, _, s in new_work]
                    temps = [r.temperature for r, _, _ in new_work]  # per request (the reference uses the first's)
                    seeds = [r.seeds[i] for r, i, _ in new_work]
                    self._send({"action": "prefill_flat", "sequences": seqs, "slots": slots, "temperatures": temps,
                                "seeds": seeds})
                    toks = rt.prefill(seqs, slots, temperatures=temps, seeds=seeds).tolist()
                    released = []
                    for (req, idx, slot), tok in zip(new_work, toks):
                        if 1 >= req.max_tokens or (not req.ignore_eos and tok == eos):
                            self._finish(req, idx, [tok])
                            kv.release(slot)
                            released.append(slot)
                            bisect.insort(free_slots, slot)
                        else:
                            active[slot] = [req, idx, [tok], len(req.token_ids[idx])]
                    if released:
                        self._send({"action": "release", "slots": released})
                    staged = None
                if not active:
                    continue
            slots = list(active.keys())
            if not inflight:
                inflight.append(self._launch_decode(rt, slots, staged != slots, active))
                staged = slots
            # Run one step ahead when that cannot change the batch (as LLM._run_loop does).
            if (len(inflight) == 1 and inflight[0][0] == slots and not (pending and free_slots)
                    and all(len(st[2]) + 1 < st[0].max_tokens and st[3] + 1 < self.max_seq_len
                            for st in active.values())):
                inflight.append(self._launch_decode(rt, slots, False, active))
            step_slots, handle = inflight.pop(0)
            sampled = rt.wait_tokens(handle, len(step_slots))
            if self.tp_size > 1 and rt.token_error(handle):
                # a timed-out NVLink exchange leaves the group out of step: stop, do not crawl on
                _lib.raise_on_device_error("TP decode step")
            released = []
            for slot, tok in zip(step_slots, sampled):
                st = active.get(slot)
                if st is None:  # ended at an earlier step; this token came from a step run ahead
                    continue
                st[2].append(tok)
                st[3] += 1
                req = st[0]
                if len(st[2]) >= req.max_tokens or st[3] >= self.max_seq_len or (not req.ignore_eos and tok == eos):
                    self._finish(req, st[1], st[2])
                    del active[slot]
                    kv.release(slot)
                    released.append(slot)
                    bisect.insort(free_slots, slot)
            if released:
                self._send({"action": "release", "slots": released})
                staged = None

    def _launch_decode(self, rt, slots, restage, active):
        """Send one decode step to the workers, stage it if the batch changed, run it
        here and queue the read-back of its tokens."""
        B = len(slots)
        if B > rt.max_batch:  # before the workers are sent into this step's collectives
            raise ValueError(f"decode batch {B} exceeds the runtime's max_batch {rt.max_batch}")
        self._send({"action": "decode", "batch_size": B, "restage": restage, "slots": slots if restage else None})
        if restage:
            self._stage_decode([active[s][2][-1] for s in slots], [active[s][3] for s in slots], slots,
                               [active[s][0].temperature for s in slots],
                               [active[s][0].seeds[active[s][1]] for s in slots])
        rt.decode_step(slots)
        return slots, rt.copy_tokens_async(B)
