#!/usr/bin/env python3
"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the UNMODIFIED reference engine code (yijichar/AWesome_ACceleration
``llm.py`` ``LLM._prefill`` / ``LLM._decode_step`` -> ``model/model.py``) on
the CPU with seeded random-init weights.  flash-attn has no CPU kernels, so
its three entry points are replaced by the restatement in
``oracle/attention.py``; everything else is the reference's own code.

Usage (only where the reference source tree is present):
    python tests/golden/make_golden.py --reference /path/to/reference

Writes ``tests/golden/<case>.npz``.  Each file holds the greedy token stream,
the logits at a fixed subset of vocab ids plus the top-2 logits per step, and
K/V cache samples, all produced by the reference code.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import attention as fa  # noqa: E402
from oracle.weights import QWEN3_0_6B, TINY, TINY_G4, TP8B_2L, init_weights, random_prompts  # noqa: E402

# name: (arch, dtype, seed, norm_jitter, prompt lengths, decode steps, kv layers, kv positions)
CASES = {
    "cfg1_0p6b_fp32": (QWEN3_0_6B, torch.float32, 1234, 0.0, [128] * 4, 32, [0, 27], [0, 1, 127, 128, 159]),
    "cfg1_0p6b_bf16_short": (QWEN3_0_6B, torch.bfloat16, 1234, 0.0, [64, 64], 4, [0, 27], [0, 63, 64, 67]),
    "tiny_fp32_ragged": (TINY, torch.float32, 7, 0.1, [5, 17, 40, 1], 8, [0, 1], [0, 4, 16, 39, 47]),
    "tiny_bf16_ragged": (TINY, torch.bfloat16, 7, 0.1, [5, 17, 40, 1], 8, [0, 1], [0, 4, 16, 39, 47]),
    "tinyg4_bf16": (TINY_G4, torch.bfloat16, 11, 0.1, [33, 300], 6, [0, 1], [0, 255, 256, 299, 305]),
    # Qwen3-0.6B in bf16 at the engine's dtype: 4 x 128 prompt tokens, 64 greedy decode steps.
    "qwen06b_bf16_64": (QWEN3_0_6B, torch.bfloat16, 2024, 0.0, [128] * 4, 64, [0, 27],
                        [0, 127, 128, 191]),
    # Qwen3-8B proportions (hidden 4096, 32 / 8 heads, MLP 12288, untied lm_head), two layers:
    # the tensor-parallel parity case (G = 4 query heads per kv head on every rank at TP 2 / 4).
    "tp8b2l_bf16": (TP8B_2L, torch.bfloat16, 31, 0.1, [96, 33, 128, 7], 32, [0, 1], [0, 6, 32, 95, 127, 150]),
}
N_SUB = 512


def load_reference(ref_root: str):
    # Compile the reference from its .py sources only: never pick up the
    # bytecode shipped in its __pycache__ directories.
    sys.pycache_prefix = os.path.join("/tmp", "aacc_ref_pycache")
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    import flash_attn  # noqa: F401  (imports on CPU; its kernels do not run there)
    import llm as ref_llm
    import model.model as ref_model
    ref_llm.flash_attn_varlen_func = fa.flash_attn_varlen_func
    ref_model.flash_attn_with_kvcache = fa.flash_attn_with_kvcache
    flash_attn.flash_attn_func = fa.flash_attn_func
    return ref_llm, ref_model


def build_engine(ref_llm, ref_model, arch, dtype, sd, num_slots, max_seq_len):
    cfg = ref_model.Qwen3Config(**{k: v for k, v in arch.as_dict().items()
                                   if k in ref_model.Qwen3Config.__annotations__})
    model = ref_model.Qwen3ForCausalLM(cfg).to(dtype)
    missing, unexpected = model.load_state_dict({k: v.to(dtype) for k, v in sd.items()}, strict=False)
    assert not unexpected, unexpected
    model.eval()
    model.fuse_qkv()
    model.init_kv_cache(num_slots, max_seq_len, torch.device("cpu"), dtype)
    # LLM.__init__ needs CUDA and a tokenizer (llm.py:48, :79); _prefill and
    # _decode_step only read these attributes.
    eng = object.__new__(ref_llm.LLM)
    eng.device = torch.device("cpu")
    eng.dtype = dtype
    eng.max_seq_len = max_seq_len
    eng.config = cfg
    eng.model = model
    return eng


@torch.inference_mode()
def run_case(ref_llm, ref_model, name, spec):
    arch, dtype, seed, jitter, lens, steps, kv_layers, kv_pos = spec
    sd = init_weights(arch, seed, norm_jitter=jitter)
    n = len(lens)
    max_seq_len = ((max(lens) + steps + 64) // 64) * 64
    eng = build_engine(ref_llm, ref_model, arch, dtype, sd, n, max_seq_len)
    prompts = [p[:L] for p, L in zip(random_prompts(n, max(lens), arch.vocab_size, seed + 1), lens)]
    slots = list(reversed(range(n)))  # non-identity slot assignment
    g = torch.Generator().manual_seed(seed + 2)
    vocab_idx = torch.randperm(arch.vocab_size, generator=g)[:min(N_SUB, arch.vocab_size)].sort().values
    subs, top_v, top_i, toks = [], [], [], []

    def record(logits):
        lf = logits.float()
        subs.append(lf[:, vocab_idx].numpy())
        tv, ti = lf.topk(2, dim=-1)
        top_v.append(tv.numpy())
        top_i.append(ti.numpy())
        toks.append(logits.argmax(dim=-1).numpy())

    logits = eng._prefill(prompts, slots)
    record(logits)
    positions = torch.tensor([[L] for L in lens], dtype=torch.long)
    for _ in range(steps):
        ids = torch.tensor(toks[-1], dtype=torch.long).unsqueeze(1)
        logits = eng._decode_step(ids, positions, torch.tensor(slots, dtype=torch.long))
        record(logits)
        positions = positions + 1
    kk, vv = [], []
    for li in kv_layers:
        attn = eng.model.model.layers[li].self_attn
        kk.append(torch.stack([attn._kv_cache[s][kv_pos] for s in slots]).float().numpy())
        vv.append(torch.stack([attn._v_cache[s][kv_pos] for s in slots]).float().numpy())
    seqlens = eng.model.model.layers[0].self_attn._cache_seqlens
    out = dict(
        tokens=np.stack(toks, 1).astype(np.int64),  # [n, steps+1]
        logits_sub=np.stack(subs, 0),              # [steps+1, n, N_SUB]
        top2_val=np.stack(top_v, 0), top2_idx=np.stack(top_i, 0).astype(np.int64),
        vocab_idx=vocab_idx.numpy().astype(np.int64),
        kv_k=np.stack(kk), kv_v=np.stack(vv),       # [layers, n, pos, Hkv, D]
        kv_layers=np.array(kv_layers), kv_pos=np.array(kv_pos),
        prompts=np.array([p + [-1] * (max(lens) - len(p)) for p in prompts], dtype=np.int64),
        lens=np.array(lens), slots=np.array(slots),
        seqlens=np.array([int(seqlens[s]) for s in slots]),
        seed=seed, norm_jitter=jitter, steps=steps, max_seq_len=max_seq_len,
        dtype=str(dtype).replace("torch.", ""), arch=json.dumps(arch.as_dict()),
    )
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **out)
    print(f"{name}: wrote {path}  tokens[0][:8]={out['tokens'][0][:8].tolist()}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AACC_REFERENCE"),
                    help="checkout of the reference project (or set AACC_REFERENCE)")
    ap.add_argument("--cases", nargs="*", default=list(CASES))
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference <path to the reference checkout> or set AACC_REFERENCE")
    torch.set_num_threads(os.cpu_count() or 8)
    ref_llm, ref_model = load_reference(args.reference)
    for name in args.cases:
        run_case(ref_llm, ref_model, name, CASES[name])


if __name__ == "__main__":
    main()
