#!/usr/bin/env python3
"""Benchmark: Qwen3 greedy generation throughput (output tok/s) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                    [--workload cfg2|cfg4|cfg5|attn|gemm] [--small]

Default workload (cfg2): Qwen3-0.6B architecture, random-init bf16 weights,
256 sequences x 1024 uniform-random prompt tokens, 1024 greedy output tokens
each (EOS ignored), continuous batching, paged KV block 256.  One "step" is
one whole generation job: the packed prefill of all 256 prompts plus 1023
decode steps (256 x 1024 output tokens).

* ``value``: device-timed throughput with the prompts already in HBM and the
  decode loop replaying the captured decode-step graph (next tokens stay on
  the device); CUDA events on the launching stream, max over ranks.
* ``e2e``: the same job through the public API ``LLM.generate_ids`` with
  host token lists in and out (pinned H2D staging each step, a D2H read of
  every step's tokens).
* ``roofline``: the dominant kernel, the paged decode attention, timed with
  CUDA events on the real end-of-job KV state (algorithmic bytes = K+V of
  every context token + q in + o out + block-table reads).
* ``cpu_baseline``: the CPU oracle (a restatement of the reference's own
  PyTorch code path, bf16 on all host cores) over a bounded sample of the
  same workload, prefill and decode timed apart.
* ``tp``: cfg4 (Qwen3-8B, 128 x 2048 in / 512 out) at tensor parallel =
  the whole world, so the 1/2/4/8-GPU runs record the 8B model's TP scaling.

Under torchrun (N>1) every rank runs an independent cfg2 replica (DP, weak
scaling); ``value`` is the total over ranks divided by the slowest rank.
``--impl reference`` times the reference's CPU implementation (the oracle)
on rank 0 only.  ``--workload attn`` is the decode-attention microbenchmark
(B = 256, 16 / 8 heads, contexts U[512, 4096], a 65,536-block pool).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    def __init__(self, device_index: int):
        # nvidia-smi numbering can differ from CUDA's: address the GPU by UUID.
        try:
            self.index = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:  # noqa: BLE001
            self.index = str(device_index)
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        load = [s for s in sm if s > 300] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- workload
def arch_0p6b():
    from awesome_acceleration_b200.model.model import Qwen3Config
    return Qwen3Config()


def make_prompts(n, length, vocab, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n, length), generator=g).tolist()


# DRAM bytes (read + write) per algorithmic byte of the decode attention, from
# one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum of one launch
# of `bench.py --workload attn --small`: 2.484 GB against 2.447 GB
# algorithmic); the traffic of a full-size launch is scaled from it by the
# bytes it must move (traffic grows in proportion to the context streamed).
ATTN_TRAFFIC_PER_ALG_BYTE = 1.015
ATTN_TRAFFIC_SOURCE = "ncu capture of --workload attn --small, scaled by algorithmic bytes"


def attention_bytes(ctx, hq, hkv, bs):
    """Algorithmic bytes of one paged decode-attention launch."""
    ctx = np.asarray(ctx, dtype=np.int64)
    return int(ctx.sum() * hkv * 128 * 2 * 2 + len(ctx) * hq * 128 * 2 * 2
               + np.ceil(ctx / bs).sum() * 4)


class Cfg2:
    def __init__(self, args):
        self.n_seqs = 32 if args.small else 256
        self.prompt = 256 if args.small else 1024
        self.out = 64 if args.small else 1024
        if args.midrun:  # profiler captures: the job's mean decode context, a few steps
            self.prompt, self.out = 1536, 8
        self.seed = 1234 + args.rank


def build_engine(cfg2, device, use_graphs=True):
    from awesome_acceleration_b200.llm import LLM
    cfg = arch_0p6b()
    max_seq_len = cfg2.prompt + cfg2.out + 16
    return LLM(None, max_num_seqs=cfg2.n_seqs, max_seq_len=max_seq_len, config=cfg, seed=cfg2.seed,
               use_cuda_graphs=use_graphs, device=device)


def device_job(llm, prompts, out_tokens, mark=None):
    """One whole job on device: prefill all prompts, then out_tokens-1 decode
    steps replaying the decode graph (tokens stay on device).  `mark`, a CUDA
    event, is recorded between the prefill and the decode loop."""
    rt = llm.model._rt()
    kv = llm.model.kv
    rows = list(range(len(prompts)))
    for r in rows:  # all blocks the job needs, so no table upload mid-loop
        kv.reserve(r, len(prompts[r]) + out_tokens)
    kv.sync()
    first = rt.prefill(prompts, rows)
    rt.buf.ids[:len(rows)].copy_(first)
    if mark is not None:
        mark.record(torch.cuda.current_stream())
    rt.load_positions_rows([len(p) for p in prompts], rows)
    for _ in range(out_tokens - 1):
        rt.decode_step(rows)
    return rows


def reset_job(llm, rows):
    llm.model.kv.clear_all()


def run_cfg2(args, device):
    cfg2 = Cfg2(args)
    torch.manual_seed(0)
    llm = build_engine(cfg2, device)
    vocab = llm.config.vocab_size
    prompts = make_prompts(cfg2.n_seqs, cfg2.prompt, vocab, cfg2.seed)
    from awesome_acceleration_b200 import _lib
    lib = _lib.load()
    rt = llm.model._rt()
    stream = torch.cuda.current_stream()
    # ---- warm-up (also captures the decode graph)
    for _ in range(args.warmup):
        rows = device_job(llm, prompts, cfg2.out)
        torch.cuda.synchronize()
        reset_job(llm, rows)
    _lib.raise_on_device_error("warm-up")
    # ---- timed region: K whole jobs, device-resident inputs
    barrier(args)
    torch.cuda.synchronize()
    launches0 = lib.aacc_launch_count()
    graph_before = rt.graph_replays
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    em = torch.cuda.Event(enable_timing=True)
    elapsed = prefill_s = 0.0
    with ClockSampler(torch.cuda.current_device()) as clk:
        for _ in range(args.steps):
            e0.record(stream)
            rows = device_job(llm, prompts, cfg2.out, mark=em)
            e1.record(stream)
            e1.synchronize()
            elapsed += e0.elapsed_time(e1) / 1e3
            prefill_s += e0.elapsed_time(em) / 1e3
            reset_job(llm, rows)
    torch.cuda.synchronize()
    _lib.raise_on_device_error("timed region")
    eager_launches = lib.aacc_launch_count() - launches0
    replays = rt.graph_replays - graph_before
    launches = eager_launches + replays * rt.graph_launches.get(cfg2.n_seqs, 0)
    t_max = max_over_ranks(args, elapsed)
    out_tok = cfg2.n_seqs * cfg2.out
    value = args.world * out_tok * args.steps / t_max
    if args.profile:  # profiler capture: only the timed jobs run
        return {"metric": "output tok/s", "value": round(value, 1), "unit": "output tok/s",
                "note": "profiler run: not a bench value", "gpu_launches": int(lib.aacc_launch_count() - launches0)}

    # ---- roofline of the dominant kernel (paged decode attention) on the
    # end-of-job KV state: every row at prompt + out - 1 cached tokens.
    rows = device_job(llm, prompts, cfg2.out)
    torch.cuda.synchronize()
    roof = attention_roofline(llm, rows, reps=20)
    reset_job(llm, rows)

    # ---- e2e through the public API (host lists in/out)
    torch.cuda.synchronize()
    barrier(args)
    h2d0, d2h0 = rt.h2d_bytes, rt.d2h_bytes
    e0.record(stream)
    t0 = time.perf_counter()
    res = llm.generate_ids(prompts, max_tokens=cfg2.out, ignore_eos=True).result()
    e1.record(stream)
    e1.synchronize()
    e2e_s = max(e0.elapsed_time(e1) / 1e3, time.perf_counter() - t0)
    h2d = rt.h2d_bytes - h2d0
    d2h = rt.d2h_bytes - d2h0
    gen = sum(r.generated_tokens for r in res)
    assert gen == out_tok, (gen, out_tok)
    e2e_max = max_over_ranks(args, e2e_s)
    llm.stop()
    e2e = {"value": args.world * gen / e2e_max, "unit": "output tok/s",
           "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "api": "LLM.generate_ids"}
    step_ms = t_max / args.steps * 1e3
    line = {
        "metric": "output tok/s (Qwen3-0.6B, 256x1024 in / 1024 out, greedy)",
        "value": round(value, 1), "unit": "output tok/s", "n_gpus": args.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform random token ids, random-init weights)",
        "config": {"workload": "cfg2: Qwen3-0.6B 256 seqs x 1024 prompt / 1024 output, greedy, ignore_eos, "
                               "paged KV block 256" + (" [SMALL]" if args.small else ""),
                   "global_batch": cfg2.n_seqs * args.world, "seq_len": cfg2.prompt + cfg2.out,
                   "parallelism": f"dp{args.world}" if args.world > 1 else "single",
                   "l2": "inputs larger than L2 (KV cache ~60 GB, weights 1.2 GB per step)"},
        "e2e": e2e, "roofline": roof, "gpu_launches": int(launches), "clocks": clk.summary(),
        "phases": phase_summary(cfg2, args.steps, elapsed, prefill_s, llm.config),
    }
    return line


def phase_summary(cfg2, steps, elapsed, prefill_s, cfg):
    """Prefill / decode split of the timed jobs and the whole-job HBM roofline
    (weights + KV bytes of every decode step over the measured copy bandwidth)."""
    pk, kind = peaks()
    decode_s = (elapsed - prefill_s) / steps
    n_dec = cfg2.out - 1
    kv_tok = 2 * cfg.num_hidden_layers * cfg.num_key_value_heads * cfg.head_dim * 2
    w_bytes = weight_bytes(cfg)
    ctx = cfg2.prompt + 1 + np.arange(n_dec)  # tokens attended at each decode step
    dec_bytes = n_dec * w_bytes + cfg2.n_seqs * kv_tok * float(ctx.sum() + n_dec)
    ideal = dec_bytes / (pk["hbm_gbs"] * 1e9)
    return {"prefill_ms": round(prefill_s / steps * 1e3, 1), "decode_ms": round(decode_s * 1e3, 1),
            "decode_ms_per_step": round(decode_s / n_dec * 1e3, 3),
            "decode_tok_per_s": round(cfg2.n_seqs * n_dec / decode_s, 1),
            "decode_hbm_bytes": dec_bytes, "decode_roofline_frac": round(ideal / decode_s, 3),
            "peak_kind": kind}


def attention_roofline(llm, rows, reps=20):
    """Time the paged decode attention alone on the real KV state (layer 0),
    CUDA events on the launching stream."""
    from awesome_acceleration_b200 import kernels as Kk
    rt = llm.model._rt()
    kv = llm.model.kv
    B = len(rows)
    ctx = [int(kv.lengths[r]) + 1 for r in rows]
    q = torch.randn((B, rt.Hq, 128), dtype=torch.bfloat16, device=kv.k.device) / 11.3
    out = torch.empty_like(q)
    rows_d = torch.tensor(rows, dtype=torch.int64, device=kv.k.device)
    stream = torch.cuda.current_stream()
    times = []
    # Rotate over layers so every launch reads cold KV (a layer's K+V exceeds L2).
    for i in range(reps + 3):
        layer = i % kv.num_layers
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        Kk.paged_decode_attention(q, kv.k[layer], kv.v[layer], kv.block_tables, rows_d, kv.seqlens, ctx_add=1,
                                  scale=rt.scale, max_context=rt.max_context, workspace=rt.buf.attn_ws, out=out)
        e1.record(stream)
        e1.synchronize()
        if i >= 3:
            times.append(e0.elapsed_time(e1) / 1e3)
    t = statistics.mean(times)
    byts = attention_bytes(ctx, rt.Hq, rt.Hkv, kv.block_size)
    pk, kind = peaks()
    ach = byts / t / 1e9
    return {"kernel": "paged_decode_kernel (split merge fused)", "bound": "hbm",
            "achieved": round(ach, 1), "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(ach / pk["hbm_gbs"], 3),
            "peak_kind": kind, "traffic": int(byts * ATTN_TRAFFIC_PER_ALG_BYTE), "traffic_source": ATTN_TRAFFIC_SOURCE,
            "bytes_per_launch": byts, "us_per_launch": round(t * 1e6, 2),
            "state": f"B={B}, ctx={min(ctx)}..{max(ctx)}"}


# --------------------------------------------------------------------------- decode-attention microbenchmark
def run_attn(args, device):
    from awesome_acceleration_b200 import _lib, kernels as Kk
    g = torch.Generator().manual_seed(7)
    B, hq, hkv, bs = 256, 16, 8, 256
    nb = 4096 if args.small else 65536
    lo, hi = 512, 4096
    ctx = torch.randint(lo, hi + 1, (B,), generator=g).tolist()
    maxb = (hi + bs - 1) // bs
    perm = torch.randperm(nb, generator=g)
    bt = torch.full((B, maxb), -1, dtype=torch.int32)
    it = 0
    for b, c in enumerate(ctx):
        n = (c + bs - 1) // bs
        bt[b, :n] = perm[it:it + n].int()
        it += n
    kc = torch.empty((nb, hkv, bs, 128), dtype=torch.bfloat16, device=device)
    vc = torch.empty_like(kc)
    kc.normal_()
    vc.normal_()
    q = torch.randn((B, hq, 128), dtype=torch.bfloat16, device=device) / 128 ** 0.5
    seqlens = torch.tensor(ctx, dtype=torch.int32, device=device) - 1
    rows = torch.arange(B, dtype=torch.int64, device=device)
    btd = bt.to(device)
    ws = torch.zeros(Kk.decode_workspace_bytes(B, hq, maxb * bs), dtype=torch.uint8, device=device)
    out = torch.empty_like(q)
    # slot mapping of the new token (1 per sequence) + its store, as in a decode step
    stream = torch.cuda.current_stream()

    def call():
        Kk.paged_decode_attention(q, kc, vc, btd, rows, seqlens, ctx_add=1, scale=128 ** -0.5,
                                  max_context=maxb * bs, workspace=ws, out=out)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    flush = torch.empty(256 * 1024 * 1024 // 2, dtype=torch.bfloat16, device=device)
    times = []
    with ClockSampler(torch.cuda.current_device()) as clk:
        for _ in range(args.steps):
            flush.zero_()  # > L2: every launch reads K/V from HBM
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            call()
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1) / 1e3)
    _lib.raise_on_device_error("attn bench")
    # spot-check: a few output rows against a plain torch fp32 attention over
    # the same paged K/V (the kernel rounds P to bf16 before P.V)
    G = hq // hkv
    check_err = 0.0
    for b in sorted({0, 1, B // 2, B - 1}):
        n = ctx[b]
        blocks = bt[b, :(n + bs - 1) // bs].long().to(device)
        kk = kc[blocks].permute(1, 0, 2, 3).reshape(hkv, -1, 128)[:, :n].float()
        vv = vc[blocks].permute(1, 0, 2, 3).reshape(hkv, -1, 128)[:, :n].float()
        qq = q[b].float().view(hkv, G, 128)
        p = torch.softmax(qq @ kk.transpose(1, 2) * 128 ** -0.5, dim=-1)
        ref = (p @ vv).reshape(hq, 128)
        check_err = max(check_err, (out[b].float() - ref).abs().max().item())
    check_tol = 2e-2
    if not check_err <= check_tol:
        raise RuntimeError(f"attn bench: output rows differ from torch fp32 attention by {check_err:.3g}")
    t = statistics.mean(times)
    byts = attention_bytes(ctx, hq, hkv, bs)
    pk, kind = peaks()
    ach = byts / t / 1e9
    return {"metric": "paged decode-attention HBM GB/s (B=256, Hq16/Hkv8, ctx U[512,4096])",
            "value": round(ach, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t * 1e3, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg3 decode-attention microbenchmark", "pool_blocks": nb,
                       "l2": "flushed between launches",
                       "output_check": {"rows": 4, "vs": "torch fp32 attention", "max_abs_err": round(check_err, 5),
                                        "tol": check_tol}},
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(ach / pk["hbm_gbs"], 3), "traffic": int(byts * ATTN_TRAFFIC_PER_ALG_BYTE),
                         "traffic_source": ATTN_TRAFFIC_SOURCE, "peak_kind": kind},
            "gpu_launches": 2 * args.steps, "clocks": clk.summary()}


# --------------------------------------------------------------------------- HBM ceilings (context for the roofline)
def run_hbm(args, device):
    """Read-only and copy bandwidth of this GPU with library-independent torch
    kernels: an int64 max-reduction over an 8 GB buffer (reads only) and a
    2 GB copy (read + write, the form MEASURED_PEAKS.json's hbm_gbs takes).
    The decode attention reads its KV stream once and writes little, so the
    read-only figure is its practical ceiling."""
    n = (1 if args.small else 4) * 1024 ** 3
    x = torch.empty(n, dtype=torch.bfloat16, device=device)
    x.normal_()
    y = torch.empty(1024 ** 3 // (4 if args.small else 1), dtype=torch.bfloat16, device=device)
    z = torch.empty_like(y)
    stream = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1) / 1e3)
        return statistics.median(ts)

    with ClockSampler(torch.cuda.current_device()) as clk:
        t_read = timed(lambda: x.view(torch.int64).max())
        t_copy = timed(lambda: z.copy_(y))
    read_gbs = x.numel() * 2 / t_read / 1e9
    copy_gbs = 2 * y.numel() * 2 / t_copy / 1e9
    pk, kind = peaks()
    return {"metric": "HBM read-only GB/s (int64 max over 8 GB)", "value": round(read_gbs, 1), "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "HBM ceilings", "copy_gbs": round(copy_gbs, 1), "measured_peak_hbm_gbs": pk["hbm_gbs"],
                       "peak_kind": kind, "l2": "buffers larger than L2"},
            "gpu_launches": 0, "clocks": clk.summary()}


# --------------------------------------------------------------------------- prefill attention (tensor pipe)
def run_prefill_attn(args, device):
    """Causal prefill attention over the paged cache on one packed chunk of
    the cfg2 prefill: 32 sequences x 1024 prompt tokens (32,768 query tokens;
    --prefill-len L packs 32768 / L prompts of L tokens), 16 / 8 heads, block
    256, a permuted block pool.  FLOPs = 4 * 128 * Hq * sum over queries of
    the keys each attends (causal).  AACC_PREFILL_ATTN=mma times the mma.sync
    kernel instead of the tcgen05 one."""
    from awesome_acceleration_b200 import _lib, kernels as Kk
    L = args.prefill_len
    n = (8 if args.small else 32) * 1024 // L
    hq, hkv, bs = 16, 8, 256
    g = torch.Generator().manual_seed(11)
    nb = n * (L // bs) + 8
    perm = torch.randperm(nb, generator=g)
    bt = perm[:n * (L // bs)].view(n, L // bs).int().to(device)
    kc = torch.randn((nb, hkv, bs, 128), generator=g).to(torch.bfloat16).to(device)
    vc = torch.randn((nb, hkv, bs, 128), generator=g).to(torch.bfloat16).to(device)
    q = torch.randn((n * L, hq, 128), generator=g).to(torch.bfloat16).to(device)
    rows = torch.arange(n, dtype=torch.int64, device=device)
    cu = (torch.arange(n + 1, dtype=torch.int32) * L).to(device)
    c0 = torch.zeros(n, dtype=torch.int32, device=device)
    out = torch.empty_like(q)

    def call():
        Kk.prefill_attention(q, kc, vc, bt, rows, cu, c0, max_q_len=L, scale=128 ** -0.5, out=out)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    ts = []
    with ClockSampler(torch.cuda.current_device()) as clk:
        for _ in range(args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            call()
            e1.record(stream)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1) / 1e3)
    _lib.raise_on_device_error("prefill attention")
    t = statistics.median(ts)
    flops = 4 * 128 * hq * n * (L * (L + 1) // 2)
    pk, kind = peaks()
    ach = flops / t / 1e12
    kernel = "mma.sync" if os.environ.get("AACC_PREFILL_ATTN", "").startswith("m") else "tcgen05"
    return {"metric": f"causal prefill attention TFLOP/s ({n} x {L} tokens, 16/8 heads)", "value": round(ach, 1),
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg2 prefill chunk attention", "prompt_len": L, "kernel": kernel,
                       "l2": "q 134 MB + K/V 143 MB > L2"},
            "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(ach / pk["bf16_tflops"], 3), "traffic": None, "peak_kind": kind},
            "gpu_launches": args.steps + args.warmup, "clocks": clk.summary()}


# --------------------------------------------------------------------------- cfg4: Qwen3-8B tensor parallel
QWEN3_8B_KW = dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36, num_attention_heads=32,
                   num_key_value_heads=8, tie_word_embeddings=False)


def weight_bytes(cfg, tp: int = 1) -> float:
    """bf16 bytes of the weights one decode step streams on each rank: every
    layer's QKV, o, gate/up and down projections (sharded over tp) plus the
    lm_head (vocab-sharded over tp; the tied embedding for Qwen3-0.6B)."""
    H, I, D = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    q, kv = cfg.num_attention_heads * D, cfg.num_key_value_heads * D
    layer = H * (q + 2 * kv) + q * H + 2 * I * H + I * H
    return 2.0 * (cfg.num_hidden_layers * layer + cfg.vocab_size * H) / tp


def exchange_us(rt, rows: int, calls: int = 32, reps: int = 5):
    """Device time of one RowParallel exchange call (all-reduce + residual add
    + RMSNorm over NVLink peer memory) on `rows` x hidden bf16 rows: `calls`
    back-to-back calls captured in one CUDA graph, replayed `reps` times by
    every rank of the TP group together.  None without the exchange."""
    ex = rt.comm.exchange
    if ex is None or rows > ex.max_rows:
        return None
    dev = rt.device
    src = torch.zeros((rows, rt.H), dtype=torch.bfloat16, device=dev)
    res = torch.zeros_like(src)
    out = torch.empty_like(src)
    w = torch.ones(rt.H, dtype=torch.bfloat16, device=dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(calls):
                rt.comm.allreduce_add_rmsnorm(src, 0, res, w, rt.eps, out)
    torch.cuda.current_stream().wait_stream(s)
    torch.distributed.barrier(group=rt.comm.cpu_group)
    g.replay()  # warm
    torch.cuda.synchronize()
    torch.distributed.barrier(group=rt.comm.cpu_group)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    e1.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (reps * calls)


def run_cfg4(args, device, steps=None, warmup=None, tp=None):
    """cfg4: Qwen3-8B architecture (random-init bf16), 128 seqs x 2048 prompt
    tokens, 512 greedy outputs, tensor parallel over the torchrun world (TP =
    `tp`, default --tp or the world; DP = world / TP replicas).  Every rank of
    a TP group runs the same device job; each decode step is one CUDA graph
    holding the RowParallel exchanges and the vocab-parallel argmax
    all-gather.  `steps` / `warmup` override --steps / --warmup."""
    from awesome_acceleration_b200 import _lib
    from awesome_acceleration_b200.llm_tp import LLMTP
    from awesome_acceleration_b200.model.model import Qwen3Config
    tp = tp or args.tp or args.world
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    cfg = Qwen3Config(**QWEN3_8B_KW)
    n_seqs, prompt, out = (16, 512, 32) if args.small else (128, 2048, 512)
    llm = LLMTP(None, max_num_seqs=n_seqs, max_seq_len=prompt + out + 16, enable_tp=args.world > 1, tp_size=tp,
                config=cfg, seed=7)
    dp = llm.dp_size
    prompts = make_prompts(n_seqs, prompt, cfg.vocab_size, 4321 + llm.dp_rank)
    lib = _lib.load()
    rt = llm.model._rt()
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        rows = device_job(llm, prompts, out)
        torch.cuda.synchronize()
        reset_job(llm, rows)
    _lib.raise_on_device_error("warm-up")
    barrier(args)
    torch.cuda.synchronize()
    n0, r0 = lib.aacc_launch_count(), rt.graph_replays
    e0, e1, em = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    elapsed = prefill_s = 0.0
    with ClockSampler(torch.cuda.current_device()) as clk:
        for _ in range(steps):
            e0.record(stream)
            rows = device_job(llm, prompts, out, mark=em)
            e1.record(stream)
            e1.synchronize()
            elapsed += e0.elapsed_time(e1) / 1e3
            prefill_s += e0.elapsed_time(em) / 1e3
            reset_job(llm, rows)
    _lib.raise_on_device_error("timed region")
    launches = lib.aacc_launch_count() - n0 + (rt.graph_replays - r0) * rt.graph_launches.get(n_seqs, 0)
    t_max = max_over_ranks(args, elapsed)
    pf_max = max_over_ranks(args, prefill_s)
    value = dp * n_seqs * out * steps / t_max
    ex = rt.comm.exchange
    exchange = "none" if tp == 1 else "nccl" if ex is None else ("nvlink two-shot" if ex.two_shot else "nvlink one-shot")
    ex_us = exchange_us(rt, n_seqs) if tp > 1 else None
    pk, kind = peaks()
    n_dec = out - 1
    kv_tok = 2 * cfg.num_hidden_layers * cfg.num_key_value_heads * cfg.head_dim * 2 // tp
    ctx = prompt + 1 + np.arange(n_dec)
    dec_bytes = n_dec * weight_bytes(cfg, tp) + n_seqs * kv_tok * float(ctx.sum() + n_dec)
    decode_s = (t_max - pf_max) / steps
    llm_stop = getattr(llm, "stop", None)
    if llm_stop:
        llm_stop()
    rt.comm.close()
    return {
        "metric": f"output tok/s (Qwen3-8B, {n_seqs}x{prompt} in / {out} out, greedy, TP{tp} x DP{dp})",
        "value": round(value, 1), "unit": "output tok/s", "n_gpus": args.world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(t_max / steps * 1e3, 2), "higher_is_better": True,
        "scaling": "strong" if dp == 1 else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform random token ids, random-init weights)",
        "config": {"workload": "cfg4: Qwen3-8B TP" + (" [SMALL]" if args.small else ""), "global_batch": n_seqs * dp,
                   "seq_len": prompt + out, "parallelism": f"tp{tp}" + (f"xdp{dp}" if dp > 1 else ""),
                   "l2": "inputs larger than L2", "row_parallel_exchange": exchange},
        "gpu_launches": int(launches), "clocks": clk.summary(),
        "phases": {"prefill_ms": round(pf_max / steps * 1e3, 1), "decode_ms": round(decode_s * 1e3, 1),
                   "decode_ms_per_step": round(decode_s / n_dec * 1e3, 3),
                   "decode_roofline_frac_per_gpu": round(dec_bytes / (pk["hbm_gbs"] * 1e9) / decode_s, 3),
                   "exchange_us_per_call": None if ex_us is None else round(ex_us, 2),
                   "peak_kind": kind},
    }


def tp_block(args, device):
    """cfg4 (Qwen3-8B, 128 x 2048 in / 512 out) at TP = the whole world: one
    warm-up job and two timed jobs, added to the default bench line so that
    the 1/2/4/8-GPU runs record the tensor-parallel scaling of the 8B model
    (the north star's TP target) next to the cfg2 DP replicas."""
    line = run_cfg4(args, device, steps=2, warmup=1, tp=args.world)
    ph = line["phases"]
    return {"workload": "cfg4: Qwen3-8B 128 seqs x 2048 prompt / 512 output, greedy, ignore_eos, paged KV block 256",
            "tp": args.world, "value": line["value"], "unit": "output tok/s", "steps": line["steps"],
            "warmup": line["warmup"], "ms_per_step": line["ms_per_step"], "prefill_ms": ph["prefill_ms"],
            "decode_ms_per_step": ph["decode_ms_per_step"],
            "decode_roofline_frac_per_gpu": ph["decode_roofline_frac_per_gpu"],
            "row_parallel_exchange": line["config"]["row_parallel_exchange"],
            "exchange_us_per_call": ph["exchange_us_per_call"], "gpu_launches": line["gpu_launches"],
            "clocks": line["clocks"], "timing": "CUDA events per job, max over ranks"}


# --------------------------------------------------------------------------- cfg5: Qwen3-32B DP x TP
def run_cfg5(args, device):
    """cfg5: Qwen3-32B architecture (random-init bf16), 512
    requests with prompts ~U[256,4096] and outputs ~U[128,1024] (one request
    per sequence with its own max_tokens), greedy, ignore_eos, through the
    engine's public API: the TP-group leader runs continuous batching, the
    other ranks serve it, and the requests are dealt round-robin over the DP
    replicas (benchmark_tp.py:288-292).  TP = --tp (default: the world).
    The timed region is the whole job through LLMTP.generate_ids (host token
    lists in, host results out), so `value` is already end to end."""
    from awesome_acceleration_b200 import _lib
    from awesome_acceleration_b200.llm_tp import LLMTP
    from awesome_acceleration_b200.model.model import Qwen3Config
    tp = args.tp or args.world
    cfg = Qwen3Config(hidden_size=5120, intermediate_size=25600, num_hidden_layers=64, num_attention_heads=64,
                      num_key_value_heads=8, tie_word_embeddings=False)
    n_req = 64 if args.small else 512
    plo, phi, olo, ohi = (256, 1024, 32, 128) if args.small else (256, 4096, 128, 1024)
    rng = np.random.default_rng(2025)
    plen = rng.integers(plo, phi + 1, n_req)
    olen = rng.integers(olo, ohi + 1, n_req)
    g = torch.Generator().manual_seed(77)
    prompts = [torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist() for n in plen]
    llm = LLMTP(None, max_num_seqs=n_req, max_seq_len=phi + ohi + 16, enable_tp=args.world > 1, tp_size=tp,
                config=cfg, seed=7)
    dp = llm.dp_size
    mine = list(range(llm.dp_rank, n_req, dp))
    rt = llm.model._rt()
    rt.capture_buckets(min(len(mine), llm.max_num_seqs))
    lib = _lib.load()
    elapsed, gen = 0.0, 0
    if llm.is_tp_leader:
        for w in range(args.warmup):  # short jobs: scheduler, prefill and decode paths warm
            futs = [llm.generate_ids([prompts[i][:64]], max_tokens=4 + w, ignore_eos=True) for i in mine[:8]]
            [f.result() for f in futs]
        torch.cuda.synchronize()
        h2d0, d2h0, n0, r0, l0 = (rt.h2d_bytes, rt.d2h_bytes, lib.aacc_launch_count(), rt.graph_replays,
                                  rt.replayed_launches)
        with ClockSampler(torch.cuda.current_device()) as clk:
            for _ in range(args.steps):
                t0 = time.perf_counter()
                futs = [llm.generate_ids([prompts[i]], max_tokens=int(olen[i]), ignore_eos=True) for i in mine]
                outs = [f.result()[0] for f in futs]
                torch.cuda.synchronize()
                elapsed += time.perf_counter() - t0
                gen += sum(o.generated_tokens for o in outs)
        assert gen == args.steps * int(olen[mine].sum()), gen
        h2d, d2h = rt.h2d_bytes - h2d0, rt.d2h_bytes - d2h0
        replays = rt.graph_replays - r0
        launches = lib.aacc_launch_count() - n0 + rt.replayed_launches - l0
        clocks = clk.summary()
        llm.stop()
    else:
        llm.serve_worker()
        h2d = d2h = launches = replays = 0
        clocks = {}
    _lib.raise_on_device_error("cfg5 job")
    t_max = max_over_ranks(args, elapsed)
    total = torch.tensor([gen], dtype=torch.float64, device="cuda")
    if args.world > 1:
        torch.distributed.all_reduce(total)
    value = float(total.item()) / t_max
    return {
        "metric": f"output tok/s (Qwen3-32B, {n_req} requests, prompts U[{plo},{phi}], outputs U[{olo},{ohi}], "
                  f"greedy, TP{tp} x DP{dp})",
        "value": round(value, 1), "unit": "output tok/s", "n_gpus": args.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(t_max / args.steps * 1e3, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform random token ids and lengths, random-init weights)",
        "config": {"workload": "cfg5: Qwen3-32B DP x TP, continuous batching" + (" [SMALL]" if args.small else ""),
                   "global_batch": n_req, "seq_len": phi + ohi, "parallelism": f"tp{tp}" + (f"xdp{dp}" if dp > 1 else ""),
                   "max_num_seqs_per_replica": llm.max_num_seqs, "l2": "inputs larger than L2",
                   "timing": "wall clock around LLMTP.generate_ids on each TP leader, max over ranks"},
        "e2e": {"value": round(value, 1), "unit": "output tok/s", "h2d_bytes_per_step": int(h2d // args.steps),
                "d2h_bytes_per_step": int(d2h // args.steps), "api": "LLMTP.generate_ids",
                "note": "value is itself measured through the public API"},
        "gpu_launches": int(launches), "clocks": clocks, "decode_steps": int(replays),
    }


# --------------------------------------------------------------------------- prefill GEMMs (tensor pipe)
def run_decode_projections(args, device):
    """The decode projections of one layer as the engine runs them at B rows:
    QKV + q/k-norm + RoPE + KV store, o_proj + residual add + RMSNorm,
    gate/up + SiLU, down + residual add + RMSNorm, over layers of distinct
    weights (Qwen3-0.6B shapes: 28 layers, 840 MB; --proj-shapes 8b: Qwen3-8B
    shapes, 8 layers, 3.1 GB; larger than L2 either way, so every layer streams
    its weights from HBM), captured in one CUDA graph per variant:
      * splitk: split-K partials through L2 + epilogue kernels (B > 32);
      * skinny_fused: small-batch GEMMs (weights as the 128-row MMA operand),
        QKV / SiLU epilogues in the same launch (the engine's path up to
        SKINNY_FUSED_ROWS rows); skinny: the same GEMMs with the split-K
        epilogue kernels (the engine's path up to SKINNY_DEFAULT_ROWS); o / down
        partials summed by the norm kernel in both (B <= 64);
      * cluster: cluster split-K kernels (partials in distributed shared
        memory, epilogues fused) + add_rmsnorm (opt-in in the engine).
    Reports us per layer for the whole sequence and for each projection
    alone; `value` and the roofline are the engine's default path at B."""
    from awesome_acceleration_b200 import _lib, kernels as Kk
    from awesome_acceleration_b200.runtime import interleave_gate_up, rope_table
    B = args.batch or (32 if args.small else 256)
    if args.proj_shapes == "8b":
        L, H, I, hq, hkv, bs, model = 8, 4096, 12288, 32, 8, 256, "Qwen3-8B"
    else:
        L, H, I, hq, hkv, bs, model = 28, 1024, 3072, 16, 8, 256, "Qwen3-0.6B"
    g = torch.Generator(device=device).manual_seed(3)

    def rnd(*shape, std=0.02):
        return (torch.randn(shape, generator=g, device=device) * std).to(torch.bfloat16)

    layers = []
    for _ in range(1 if args.hot_weights else L):
        layers.append({"qkv": rnd((hq + 2 * hkv) * 128, H), "o": rnd(H, hq * 128),
                       "gu": interleave_gate_up(rnd(I, H), rnd(I, H)).contiguous(), "d": rnd(H, I),
                       "qn": torch.ones(128, dtype=torch.bfloat16, device=device),
                       "kn": torch.ones(128, dtype=torch.bfloat16, device=device),
                       "ln": torch.ones(H, dtype=torch.bfloat16, device=device)})
    layers = layers * (L // len(layers))  # --hot-weights: one layer's weights L times (L2-resident)
    x, res = rnd(B, H, std=1.0), rnd(B, H, std=1.0)
    attn, act, delta = rnd(B, hq * 128, std=1.0), rnd(B, I, std=1.0), rnd(B, H)
    q = torch.empty((B, hq, 128), dtype=torch.bfloat16, device=device)
    rope = rope_table(4096, 128, 1e6, device)
    pos = torch.randint(0, 4096, (B,), device=device)
    nb = (B + bs - 1) // bs + 1
    kc = torch.zeros((nb, hkv, bs, 128), dtype=torch.bfloat16, device=device)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(nb * bs, device=device)[:B]
    part = torch.empty(max(8 << 20, 16 * B * H), dtype=torch.float32, device=device)
    cnt = torch.zeros(4096, dtype=torch.int32, device=device)

    def pv(M, N, splits):
        return part[:splits * M * N].view(splits, M, N)

    def sk_splits(N, Kd, target):
        return Kk.pick_skinny_splits(B, N, Kd, target=target, max_elems=part.numel())

    def qkv(lw, variant):
        N = lw["qkv"].shape[0]
        if variant == "cluster":
            Kk.qkv_norm_rope_store_cluster(x, lw["qkv"], lw["qn"], lw["kn"], 1e-6, pos, rope, slots, kc, vc, hq,
                                           q_out=q)
            return
        if variant == "skinny_fused":
            sp = sk_splits(N, H, Kk.SKINNY_TARGET_CTAS)
            Kk.skinny_qkv_norm_rope_store(x, lw["qkv"], pv(B, N, sp), sp, cnt, lw["qn"], lw["kn"], 1e-6, pos, rope,
                                          slots, kc, vc, hq, q)
            return
        if variant == "skinny":
            sp = sk_splits(N, H, Kk.SKINNY_TARGET_CTAS)
            Kk.gemm_skinny_splitk(x, lw["qkv"], pv(B, N, sp), sp)
            Kk.splitk_qkv_norm_rope_store(pv(B, N, sp), sp, lw["qn"], lw["kn"], 1e-6, pos, rope, slots, kc, vc, hq, q)
            return
        sp = Kk.pick_splits(B, N, H, max_elems=part.numel())
        if sp > 1:
            Kk.gemm_splitk(x, lw["qkv"], pv(B, N, sp), sp)
            Kk.splitk_qkv_norm_rope_store(pv(B, N, sp), sp, lw["qn"], lw["kn"], 1e-6, pos, rope, slots, kc, vc, hq, q)
        else:
            Kk.qkv_norm_rope_store(x, lw["qkv"], lw["qn"], lw["kn"], 1e-6, pos, rope, slots, kc, vc, hq, q_out=q)

    def row(inp, wt, ln, variant):
        N, Kd = wt.shape
        if variant == "cluster":
            Kk.gemm_cluster(inp, wt, out=delta)
            Kk.add_rmsnorm(delta, res, ln, 1e-6, out=x)
            return
        if variant.startswith("skinny"):
            sp = sk_splits(N, Kd, Kk.SKINNY_TARGET_CTAS_ROW)
            Kk.gemm_skinny_splitk(inp, wt, pv(B, N, sp), sp)
            Kk.splitk_add_rmsnorm(pv(B, N, sp), sp, res, ln, 1e-6, out=x)
            return
        sp = Kk.pick_splits(B, N, Kd, max_elems=part.numel())
        if sp > 1:
            Kk.gemm_splitk(inp, wt, pv(B, N, sp), sp)
            Kk.splitk_add_rmsnorm(pv(B, N, sp), sp, res, ln, 1e-6, out=x)
        else:
            Kk.gemm(inp, wt, out=delta)
            Kk.add_rmsnorm(delta, res, ln, 1e-6, out=x)

    def gate_up(lw, variant):
        if variant == "cluster":
            Kk.gemm_silu_mul_cluster(x, lw["gu"], out=act)
            return
        if variant == "skinny_fused":
            sp = sk_splits(2 * I, H, Kk.SKINNY_TARGET_CTAS)
            Kk.skinny_silu_mul(x, lw["gu"], pv(B, 2 * I, sp), sp, cnt, act)
            return
        if variant == "skinny":
            sp = sk_splits(2 * I, H, Kk.SKINNY_TARGET_CTAS)
            Kk.gemm_skinny_splitk(x, lw["gu"], pv(B, 2 * I, sp), sp)
            Kk.splitk_silu_mul(pv(B, 2 * I, sp), sp, act)
            return
        sp = Kk.pick_splits(B, 2 * I, H, max_elems=part.numel())
        if sp > 1:
            Kk.gemm_splitk(x, lw["gu"], pv(B, 2 * I, sp), sp)
            Kk.splitk_silu_mul(pv(B, 2 * I, sp), sp, act)
        else:
            Kk.gemm_silu_mul(x, lw["gu"], out=act)

    ops = {"qkv": lambda lw, v: qkv(lw, v), "o_norm": lambda lw, v: row(attn, lw["o"], lw["ln"], v),
           "gate_up": lambda lw, v: gate_up(lw, v), "down_norm": lambda lw, v: row(act, lw["d"], lw["ln"], v)}
    seqs = {"layer": list(ops)} | {k: [k] for k in ops}
    variants = (["skinny_fused", "skinny"] if B <= Kk.SKINNY_MAX_ROWS else []) + ["splitk"] + (
        [] if args.no_cluster else ["cluster"])
    engine = ("skinny_fused" if B <= Kk.SKINNY_FUSED_ROWS else "skinny") if B <= Kk.SKINNY_DEFAULT_ROWS else "splitk"
    stream = torch.cuda.current_stream()
    res_us = {}
    pk, kind = peaks()
    with ClockSampler(torch.cuda.current_device()) as clk:
        for variant in variants:
            for name, seq in seqs.items():
                def body():
                    for lw in layers:
                        for op in seq:
                            ops[op](lw, variant)
                body()  # eager warm-up (plans, tensor maps, smem attributes)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                side = torch.cuda.Stream()
                side.wait_stream(stream)
                with torch.cuda.stream(side):
                    with torch.cuda.graph(graph, stream=side):
                        body()
                stream.wait_stream(side)
                for _ in range(args.warmup):
                    graph.replay()
                ts = []
                for _ in range(args.steps):
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    graph.replay()
                    e1.record(stream)
                    e1.synchronize()
                    ts.append(e0.elapsed_time(e1) / 1e3)
                del graph
                res_us[f"{variant}.{name}"] = round(statistics.median(ts) / L * 1e6, 2)
    _lib.raise_on_device_error("decode projections")
    w_layer = 2 * ((hq + 2 * hkv) * 128 * H + H * hq * 128 + 2 * I * H + H * I)
    flops = 2 * B * w_layer / 2
    t = res_us[f"{engine}.layer"] * 1e-6
    by_variant = {v: {"us_per_layer": res_us[f"{v}.layer"],
                      "weight_GBps": round(w_layer / (res_us[f"{v}.layer"] * 1e-6) / 1e9, 1),
                      "frac_of_hbm": round(w_layer / (res_us[f"{v}.layer"] * 1e-6) / 1e9 / pk["hbm_gbs"], 3)}
                  for v in variants}
    cfg = {"workload": f"decode projections of one layer ({model} shapes), " + (
               f"one layer's weights {L} times (L2-resident)" if args.hot_weights
               else f"{L} layers of distinct weights per graph"),
           "engine_path": engine, "per_variant_us": res_us, "per_variant": by_variant,
           "weight_bytes_per_layer": w_layer, "l2": f"weights {L * w_layer / 1e6:.0f} MB > L2"}
    if "skinny" in variants:
        cfg["skinny_rows"] = {"engine_up_to": Kk.SKINNY_DEFAULT_ROWS, "fused_epilogues_up_to": Kk.SKINNY_FUSED_ROWS}
        cfg["skinny_splits"] = {"qkv": sk_splits((hq + 2 * hkv) * 128, H, Kk.SKINNY_TARGET_CTAS),
                                "o": sk_splits(H, hq * 128, Kk.SKINNY_TARGET_CTAS_ROW),
                                "gate_up": sk_splits(2 * I, H, Kk.SKINNY_TARGET_CTAS),
                                "down": sk_splits(H, I, Kk.SKINNY_TARGET_CTAS_ROW)}
    if "cluster" in variants:
        cfg["cluster_plans (mt, m_tiles, splits)"] = {
            "qkv": Kk.gemm_cluster_plan(B, (hq + 2 * hkv) * 128, H), "o": Kk.gemm_cluster_plan(B, H, hq * 128),
            "gate_up": Kk.gemm_cluster_plan(B, 2 * I, H), "down": Kk.gemm_cluster_plan(B, H, I)}
    return {"metric": f"decode projections us per layer ({model} shapes, B={B})", "value": res_us[f"{engine}.layer"],
            "unit": "us per layer", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": cfg,
            "roofline": {"bound": "hbm", "achieved": round(w_layer / t / 1e9, 1), "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": round(w_layer / t / 1e9 / pk["hbm_gbs"], 3), "traffic": None,
                         "peak_kind": kind, "tensor_tflops": round(flops / t / 1e12, 1)},
            "gpu_launches": None, "clocks": clk.summary()}


def run_gemm(args, device):
    """The four cfg2 projections on one prefill chunk (M tokens) or, with
    --decode, on one decode batch (M = 256 rows; weight-bandwidth bound)."""
    if args.decode:
        return run_decode_projections(args, device)
    from awesome_acceleration_b200 import _lib, kernels as Kk
    from awesome_acceleration_b200.runtime import interleave_gate_up
    M = 8192 if args.small else 32768
    H, I, hq, hkv = 1024, 3072, 16, 8
    g = torch.Generator(device=device).manual_seed(3)
    x = torch.randn((M, H), generator=g, device=device).to(torch.bfloat16)
    a = torch.randn((M, I), generator=g, device=device).to(torch.bfloat16)
    xo = torch.randn((M, hq * 128), generator=g, device=device).to(torch.bfloat16)
    w = {n: (torch.randn(s, generator=g, device=device) * 0.02).to(torch.bfloat16) for n, s in
         [("qkv", ((hq + 2 * hkv) * 128, H)), ("o", (H, hq * 128)), ("gu", (2 * I, H)), ("d", (H, I))]}
    w["gu"] = interleave_gate_up(w["gu"][:I], w["gu"][I:]).contiguous()
    ops = {"qkv_proj": (lambda: Kk.gemm(x, w["qkv"]), 2 * M * w["qkv"].shape[0] * H),
           "o_proj": (lambda: Kk.gemm(xo, w["o"]), 2 * M * H * hq * 128),
           "gate_up_silu": (lambda: Kk.gemm_silu_mul(x, w["gu"]), 2 * M * 2 * I * H),
           "down_proj": (lambda: Kk.gemm(a, w["d"]), 2 * M * H * I)}
    stream = torch.cuda.current_stream()
    res = {}
    pk, kind = peaks()
    with ClockSampler(torch.cuda.current_device()) as clk:
        for name, (fn, flops) in ops.items():
            for _ in range(args.warmup):
                fn()
            ts = []
            for _ in range(args.steps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
                e1.synchronize()
                ts.append(e0.elapsed_time(e1) / 1e3)
            t = statistics.mean(ts)
            wbytes = flops // (2 * M) * 2  # weight bytes: N*K bf16
            res[name] = {"us": round(t * 1e6, 1), "tflops": round(flops / t / 1e12, 1),
                         "frac": round(flops / t / 1e12 / pk["bf16_tflops"], 3),
                         "weight_gbs": round(wbytes / t / 1e9, 1)}
    _lib.raise_on_device_error("gemm bench")
    tot_f = sum(f for _, f in ops.values())
    tot_t = sum(r["us"] for r in res.values()) / 1e6
    ach = tot_f / tot_t / 1e12
    return {"metric": f"prefill projection GEMMs TFLOP/s (M={M} tokens, Qwen3-0.6B shapes)", "value": round(ach, 1),
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg2 prefill GEMMs (one chunk)", "per_op": res},
            "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(ach / pk["bf16_tflops"], 3), "traffic": None, "peak_kind": kind},
            "gpu_launches": 4 * (args.steps + args.warmup), "clocks": clk.summary()}


# --------------------------------------------------------------------------- CPU baseline (oracle)
_CPU_ORACLE: dict = {}


def cpu_sample(n_seqs=4, prompt=1024, steps=12, seed=99):
    """The reference's CPU code path (restated by the oracle, bf16, all host
    cores) on a bounded sample of the cfg2 workload: a packed prefill of
    n_seqs prompts of `prompt` tokens, then `steps` greedy decode steps of the
    n_seqs sequences at contexts prompt+1 .. prompt+steps.  The two phases are
    timed apart.  Returns (decode output tok/s, info with both rates)."""
    from oracle.qwen3_oracle import Qwen3Oracle, greedy
    from oracle.weights import QWEN3_0_6B, init_weights
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    key = (n_seqs, prompt, steps, seed)
    if _CPU_ORACLE.get("key") != key:  # weights and caches built once per process
        sd = init_weights(QWEN3_0_6B, seed)
        _CPU_ORACLE.update(key=key, orc=Qwen3Oracle(QWEN3_0_6B, sd, torch.bfloat16, num_slots=n_seqs,
                                                    max_seq_len=prompt + steps + 8))
    orc = _CPU_ORACLE["orc"]
    prompts = make_prompts(n_seqs, prompt, QWEN3_0_6B.vocab_size, seed)
    slots = list(range(n_seqs))
    for s_ in slots:
        orc.clear_slot(s_)
    with torch.inference_mode():
        t0 = time.perf_counter()
        toks = greedy(orc.prefill(prompts, slots))
        t1 = time.perf_counter()
        for s in range(steps):
            toks = greedy(orc.decode(toks, [prompt + s] * n_seqs, slots))
        t2 = time.perf_counter()
    pre, dec = n_seqs * prompt / (t1 - t0), n_seqs * steps / (t2 - t1)
    return dec, {"cores": cores, "prefill_tok_per_s": round(pre, 1), "decode_tok_per_s": round(dec, 3),
                 "sample": f"{n_seqs} seqs x {prompt} prompt tokens: packed prefill ({t1 - t0:.1f} s, "
                           f"{pre:.0f} prompt tok/s) then {steps} greedy decode steps at contexts "
                           f"{prompt + 1}..{prompt + steps} ({t2 - t1:.1f} s); value = decode output tok/s "
                           f"(the phase that produces 1023 of every 1024 output tokens), bf16"}


def cpu_baseline_entry(v, info):
    return {"value": round(v, 3), "unit": "output tok/s", "cores": info["cores"], "kind": "port",
            "phase": "decode", "prefill_tok_per_s": info["prefill_tok_per_s"],
            "decode_tok_per_s": info["decode_tok_per_s"], "sample": info["sample"]}


def run_reference(args):
    vals, infos = [], []
    for i in range(args.warmup + args.steps):
        v, info = cpu_sample()
        if i >= args.warmup:
            vals.append(v)
            infos.append(info)
    v = statistics.mean(vals)
    info = dict(infos[-1], prefill_tok_per_s=round(statistics.mean(x["prefill_tok_per_s"] for x in infos), 1),
                decode_tok_per_s=round(v, 3))
    return {"impl": "reference", "metric": "output tok/s (Qwen3-0.6B, 256x1024 in / 1024 out, greedy)",
            "value": round(v, 3), "unit": "output tok/s", "n_gpus": args.world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg2 (bounded CPU sample: decode phase at context ~1024)", "parallelism": "cpu"},
            "cpu_baseline": cpu_baseline_entry(v, info),
            "e2e": {"value": round(v, 3), "unit": "output tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# --------------------------------------------------------------------------- dist plumbing
def barrier(args):
    if args.world > 1:
        torch.distributed.barrier()


def max_over_ranks(args, x: float) -> float:
    if args.world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="cfg2", choices=["cfg2", "cfg4", "cfg5", "attn", "gemm", "prefill-attn",
                                                             "hbm"])
    ap.add_argument("--tp", type=int, default=0, help="cfg4/cfg5: tensor-parallel size (default: the whole world)")
    ap.add_argument("--small", action="store_true", help="small case for profiler captures")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp-block", action="store_true",
                    help="cfg2: skip the cfg4 (Qwen3-8B) tensor-parallel block at TP = the world")
    ap.add_argument("--decode", action="store_true", help="gemm workload: decode-batch shapes")
    ap.add_argument("--batch", type=int, default=0, help="gemm --decode: batch rows (default 256)")
    ap.add_argument("--prefill-len", type=int, default=1024, choices=[256, 512, 1024, 2048, 4096, 8192],
                    help="prefill-attn: prompt length of the 32,768-token chunk")
    ap.add_argument("--proj-shapes", default="0.6b", choices=["0.6b", "8b"],
                    help="gemm --decode: Qwen3-0.6B (28 layers) or Qwen3-8B (8 layers) projection shapes")
    ap.add_argument("--no-cluster", action="store_true", help="gemm --decode: skip the cluster variant")
    ap.add_argument("--skinny-ctas", type=int, default=0,
                    help="target CTAs of the small-batch QKV / gate-up grids (default: the library's)")
    ap.add_argument("--skinny-ctas-row", type=int, default=0,
                    help="target CTAs of the small-batch o / down grids (default: the library's)")
    ap.add_argument("--hot-weights", action="store_true",
                    help="gemm --decode: reuse one layer's weights (L2-resident) to bound what prefetching could gain")
    ap.add_argument("--midrun", action="store_true",
                    help="cfg2 profiler case: 1536-token prompts (the job's mean decode context), 7 decode steps")
    ap.add_argument("--profile", action="store_true",
                    help="profiler capture: warm-up + timed jobs only (no roofline/e2e/CPU legs)")
    args = ap.parse_args()
    if args.skinny_ctas or args.skinny_ctas_row:
        from awesome_acceleration_b200 import kernels as _k
        _k.SKINNY_TARGET_CTAS = args.skinny_ctas or _k.SKINNY_TARGET_CTAS
        _k.SKINNY_TARGET_CTAS_ROW = args.skinny_ctas_row or _k.SKINNY_TARGET_CTAS_ROW
    args.world = int(os.environ.get("WORLD_SIZE", "1"))
    args.rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if args.world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                             device_id=device)
    try:
        line = {"attn": run_attn, "gemm": run_gemm, "cfg2": run_cfg2, "cfg4": run_cfg4, "cfg5": run_cfg5,
                "prefill-attn": run_prefill_attn, "hbm": run_hbm}[args.workload](args, device)
        if args.workload == "cfg2" and not (args.small or args.profile or args.no_tp_block):
            import gc
            gc.collect()
            torch.cuda.empty_cache()
            line["tp"] = tp_block(args, device)
        if args.world == 1 and args.workload == "cfg2" and not (args.no_cpu_baseline or args.profile):
            v, info = cpu_sample()
            line["cpu_baseline"] = cpu_baseline_entry(v, info)
        if args.rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if args.world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
