"""End-to-end parity of the B200 model against the reference's golden vectors
and the bf16 CPU oracle (prefill + teacher-forced decode, greedy streams)."""
import numpy as np
import pytest
import torch

from conftest import build_model, load_golden
from oracle.qwen3_oracle import Qwen3Oracle, run_greedy
from oracle.weights import TINY, Qwen3Arch, init_weights, random_prompts

pytestmark = pytest.mark.gpu
TOL = 2e-2  # logits max-abs, bf16
# The golden vectors come from the reference run on a CPU.  At the 0.6B size
# (28 layers, |logit| up to ~3.1, bf16 ulp 0.0156) the reference's own
# PyTorch path on the B200 (cuBLAS, eager bf16) differs from that CPU run by
# up to 0.035 max-abs on the same weights and inputs (measured), i.e. >2e-2
# is bf16 accumulation order, not an algorithmic difference.  The full-size
# goldens are therefore checked at 2.5 bf16 ulps of the largest logit.
TOL_BY_CASE = {"cfg1_0p6b_bf16_short": 4e-2}


def check_step(step, lg_mine, toks_mine, g, tol=TOL):
    """Logits within tol on the golden vocab subset; argmax equal unless the
    reference itself has a near-tie at that step."""
    vi = torch.from_numpy(g["vocab_idx"])
    sub = lg_mine.float().cpu()[:, vi].numpy()
    err = np.abs(sub - g["logits_sub"][step]).max()
    assert err <= tol, f"step {step}: logits max-abs {err:.4f} > {tol}"
    ref_tok = g["tokens"][:, step]
    for b, t in enumerate(toks_mine.tolist()):
        if t != ref_tok[b]:
            top1, top2 = g["top2_val"][step][b]
            assert top1 - top2 <= 2 * tol, f"step {step} row {b}: token {t} != {ref_tok[b]} (gap {top1 - top2})"
    return err, int((toks_mine.cpu().numpy() != ref_tok).sum())


@pytest.mark.parametrize("name", ["tiny_bf16_ragged", "tinyg4_bf16", "cfg1_0p6b_bf16_short"])
def test_model_vs_reference_golden(cuda, name):
    g = load_golden(name)
    arch = Qwen3Arch(**g["arch"])
    sd = init_weights(arch, int(g["seed"]), norm_jitter=float(g["norm_jitter"]))
    lens = g["lens"].tolist()
    prompts = [g["prompts"][i][:L].tolist() for i, L in enumerate(lens)]
    slots = g["slots"].tolist()
    m = build_model(arch, sd, len(lens), int(g["max_seq_len"]), cuda)
    rt = m._rt()
    tol = TOL_BY_CASE.get(name, TOL)
    toks, lg = rt.prefill(prompts, slots, last_logits=True)
    errs, flips = [], 0
    e, f = check_step(0, lg, toks, g, tol)
    errs.append(e)
    flips += f
    pos = list(lens)
    for s in range(int(g["steps"])):
        feed = g["tokens"][:, s].tolist()  # teacher forcing with the reference's stream
        rt.load_decode_inputs(feed, pos, slots)
        lgd = torch.empty((len(slots), arch.vocab_size), dtype=torch.bfloat16, device=cuda)
        out = rt.decode_step(slots, logits=lgd)
        e, f = check_step(s + 1, lgd, out.clone(), g, tol)
        errs.append(e)
        flips += f
        pos = [p + 1 for p in pos]
    from awesome_acceleration_b200 import _lib
    assert _lib.device_error() == 0
    # KV cache samples vs the reference (K/V go through the QKV GEMM, so equal up to bf16 rounding).
    for li, layer in enumerate(g["kv_layers"].tolist()):
        for i, slot in enumerate(slots):
            n = int(g["seqlens"][i])
            kk, vv = m.kv.gather(layer, slot, n)
            kp = [p for p in g["kv_pos"].tolist() if p < n]
            idx = [g["kv_pos"].tolist().index(p) for p in kp]
            assert (kk.cpu()[kp].float().numpy() - g["kv_k"][li, i][idx]).__abs__().max() <= 0.1
            assert (vv.cpu()[kp].float().numpy() - g["kv_v"][li, i][idx]).__abs__().max() <= 0.05
    print(f"{name}: max logits err per step {np.round(errs, 4).tolist()}, argmax flips at near-ties: {flips}")


def test_decode_graph_equals_eager(cuda):
    arch = TINY
    sd = init_weights(arch, 3, norm_jitter=0.1)
    prompts = random_prompts(5, 70, arch.vocab_size, 4)
    prompts = [p[:n] for p, n in zip(prompts, [70, 3, 33, 64, 65])]
    outs = []
    for graphs in (False, True):
        m = build_model(arch, sd, 5, 256, cuda, use_cuda_graphs=graphs)
        rt = m._rt()
        rows = [4, 2, 0, 1, 3]
        first = rt.prefill(prompts, rows).tolist()
        rt.load_decode_inputs(first, [len(p) for p in prompts], rows)
        seq = [first]
        for _ in range(12):
            rt.decode_step(rows)
            seq.append(rt.read_tokens(5))
        outs.append(seq)
    assert outs[0] == outs[1]


def test_chunked_prefill_equals_whole(cuda):
    arch = TINY
    sd = init_weights(arch, 5, norm_jitter=0.1)
    prompts = [p[:n] for p, n in zip(random_prompts(3, 600, arch.vocab_size, 6), [600, 257, 90])]
    res = []
    for chunk in (1 << 20, 256, 100):
        m = build_model(arch, sd, 3, 1024, cuda, prefill_chunk_tokens=chunk)
        tok, lg = m._rt().prefill(prompts, [0, 1, 2], last_logits=True)
        res.append((tok.cpu(), lg.float().cpu()))
    for tok, lg in res[1:]:
        assert torch.equal(tok, res[0][0])
        assert (lg - res[0][1]).abs().max().item() <= 1e-2


def test_greedy_stream_vs_bf16_oracle(cuda):
    """Free-running greedy streams against the bf16 CPU oracle (same rounding
    points as the reference): identical until a reference-side near-tie."""
    arch = TINY
    sd = init_weights(arch, 9, norm_jitter=0.1)
    lens = [12, 40, 7, 128]
    prompts = [p[:n] for p, n in zip(random_prompts(4, 128, arch.vocab_size, 10), lens)]
    steps = 24
    orc = Qwen3Oracle(arch, sd, torch.bfloat16, num_slots=4, max_seq_len=256)
    gaps = []

    def keep(step, lg):
        tv = lg.float().topk(2, dim=-1).values
        gaps.append((tv[:, 0] - tv[:, 1]).tolist())

    ref = run_greedy(orc, prompts, steps, keep_logits=keep)
    m = build_model(arch, sd, 4, 256, cuda)
    rt = m._rt()
    rows = [0, 1, 2, 3]
    first = rt.prefill(prompts, rows).tolist()
    mine = [[t] for t in first]
    rt.load_decode_inputs(first, lens, rows)
    for _ in range(steps):
        rt.decode_step(rows)
        for b, t in enumerate(rt.read_tokens(4)):
            mine[b].append(t)
    for b in range(4):
        for s in range(steps + 1):
            if mine[b][s] != ref[b][s]:
                assert gaps[s][b] <= 2 * TOL, f"row {b} diverged at step {s} without a near-tie"
                break
