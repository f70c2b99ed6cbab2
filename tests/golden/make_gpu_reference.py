#!/usr/bin/env python3
"""Run the reference's PyTorch path on a GPU for a golden case (test infrastructure).

The golden vectors in this folder come from the reference engine run on a
CPU.  Two bf16 implementations that sum in different orders drift apart by a
few bf16 ulps over 28 layers, so this script records the same computation
done by cuBLAS on the GPU: the oracle (``oracle/qwen3_oracle.py``, the
reference's ``LLM._prefill`` / ``LLM._decode_step`` restated op for op, and
pinned to the reference's own CPU run) executed on ``cuda`` with eager bf16
ops, as the reference runs them (flash-attn replaced by the oracle's fp32
attention restatement).  The decode steps are teacher-forced with the CPU
golden's token stream, so every step's logits compare position for position
with the CPU golden and with the B200 kernels.

Usage (on a machine with a CUDA GPU):
    python tests/golden/make_gpu_reference.py [--cases qwen06b_bf16_64] [--out DIR]

Writes ``<out>/<case>_gpuref.npz`` with the CPU golden's fields
``tokens`` (this run's argmax), ``logits_sub``, ``top2_val``, ``top2_idx``
plus ``gpu_name`` and ``torch_version``.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.qwen3_oracle import Qwen3Oracle  # noqa: E402
from oracle.weights import Qwen3Arch, init_weights  # noqa: E402


@torch.inference_mode()
def run_case(name: str, out_dir: str) -> str:
    z = np.load(os.path.join(HERE, f"{name}.npz"))
    arch = Qwen3Arch(**json.loads(str(z["arch"])))
    dtype = getattr(torch, str(z["dtype"]))
    sd = init_weights(arch, int(z["seed"]), norm_jitter=float(z["norm_jitter"]))
    lens = z["lens"].tolist()
    prompts = [z["prompts"][i][:L].tolist() for i, L in enumerate(lens)]
    slots = z["slots"].tolist()
    orc = Qwen3Oracle(arch, sd, dtype, num_slots=len(lens), max_seq_len=int(z["max_seq_len"]), device="cuda")
    del sd
    vi = torch.from_numpy(z["vocab_idx"]).cuda()
    subs, tv_, ti_, toks = [], [], [], []

    def record(lg):
        lf = lg.float()
        subs.append(lf[:, vi].cpu().numpy())
        tv, ti = lf.topk(2, dim=-1)
        tv_.append(tv.cpu().numpy())
        ti_.append(ti.cpu().numpy())
        toks.append(lg.argmax(-1).cpu().numpy())

    record(orc.prefill(prompts, slots))
    pos = list(lens)
    for s in range(int(z["steps"])):
        record(orc.decode(z["tokens"][:, s].tolist(), pos, slots))
        pos = [p + 1 for p in pos]
    path = os.path.join(out_dir, f"{name}_gpuref.npz")
    np.savez_compressed(path, tokens=np.stack(toks, 1).astype(np.int64), logits_sub=np.stack(subs, 0),
                        top2_val=np.stack(tv_, 0), top2_idx=np.stack(ti_, 0).astype(np.int64),
                        gpu_name=torch.cuda.get_device_name(), torch_version=torch.__version__)
    err = np.abs(np.stack(subs, 0) - z["logits_sub"]).max(axis=(1, 2))
    print(f"{name}: wrote {path}; max |gpu - cpu| logits per step: max {err.max():.4f}, "
          f"steps over 2e-2: {int((err > 2e-2).sum())} of {len(err)}")
    return path


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--cases", nargs="*", default=["qwen06b_bf16_64"])
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    if not torch.cuda.is_available():
        ap.error("needs a CUDA GPU")
    os.makedirs(a.out, exist_ok=True)
    for n in a.cases:
        run_case(n, a.out)


if __name__ == "__main__":
    main()
