"""Pin the CPU oracle to golden vectors produced by the reference's own code
(tests/golden/make_golden.py runs llm.py _prefill/_decode_step)."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle.qwen3_oracle import Qwen3Oracle
from oracle.weights import Qwen3Arch, init_weights

CASES = ["tiny_fp32_ragged", "tiny_bf16_ragged", "tinyg4_bf16", "cfg1_0p6b_bf16_short", "cfg1_0p6b_fp32",
         "qwen06b_bf16_64", "tp8b2l_bf16"]


def run_oracle_on_golden(g: dict):
    arch = Qwen3Arch(**g["arch"])
    dtype = torch.float32 if g["dtype"] == "float32" else torch.bfloat16
    sd = init_weights(arch, int(g["seed"]), norm_jitter=float(g["norm_jitter"]))
    lens = g["lens"].tolist()
    prompts = [g["prompts"][i][:L].tolist() for i, L in enumerate(lens)]
    slots = g["slots"].tolist()
    orc = Qwen3Oracle(arch, sd, dtype, num_slots=len(lens), max_seq_len=int(g["max_seq_len"]))
    logits = [orc.prefill(prompts, slots)]
    toks = [logits[-1].argmax(-1)]
    pos = list(lens)
    for _ in range(int(g["steps"])):
        logits.append(orc.decode(toks[-1].tolist(), pos, slots))
        toks.append(logits[-1].argmax(-1))
        pos = [p + 1 for p in pos]
    return orc, logits, torch.stack(toks, 1)


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference(name):
    torch.set_num_threads(8)
    g = load_golden(name)
    orc, logits, toks = run_oracle_on_golden(g)
    tol = 1e-4 if g["dtype"] == "float32" else 2e-2
    # Greedy streams identical for every step the reference produced.
    assert np.array_equal(toks.numpy(), g["tokens"]), "greedy stream differs from the reference"
    vi = torch.from_numpy(g["vocab_idx"])
    for s, lg in enumerate(logits):
        sub = lg.float()[:, vi].numpy()
        err = np.abs(sub - g["logits_sub"][s]).max()
        assert err <= tol, f"step {s}: logits max-abs {err} > {tol}"
        tv, ti = lg.float().topk(2, dim=-1)
        assert np.abs(tv.numpy() - g["top2_val"][s]).max() <= tol
    # KV cache samples at (layer, slot, pos) — bit-exact.
    slots = g["slots"].tolist()
    for li, layer in enumerate(g["kv_layers"].tolist()):
        for i, slot in enumerate(slots):
            k = orc.k_cache[layer][slot][torch.from_numpy(g["kv_pos"])].float().numpy()
            v = orc.v_cache[layer][slot][torch.from_numpy(g["kv_pos"])].float().numpy()
            assert np.array_equal(k, g["kv_k"][li, i]), f"K cache layer {layer} slot {slot}"
            assert np.array_equal(v, g["kv_v"][li, i]), f"V cache layer {layer} slot {slot}"
    assert [int(orc.seqlens[s]) for s in slots] == g["seqlens"].tolist()


def test_paged_slot_restatement():
    """Block-table slot mapping equals the reference's flat index under an
    identity block layout and is a bijection under a permuted one."""
    from oracle.qwen3_oracle import paged_slot
    bs, max_seq_len, nslots = 256, 1024, 5
    per = max_seq_len // bs
    ident = [[s * per + j for j in range(per)] for s in range(nslots)]
    for s in range(nslots):
        for p in (0, 1, 255, 256, 257, 1023):
            assert paged_slot(ident[s], p, bs) == s * max_seq_len + p  # llm.py:139-140
    rng = np.random.default_rng(0)
    perm = rng.permutation(nslots * per).reshape(nslots, per)
    seen = {paged_slot(perm[s], p, bs) for s in range(nslots) for p in range(max_seq_len)}
    assert len(seen) == nslots * max_seq_len


@pytest.mark.parametrize("name", ["qwen06b_bf16_64", "tp8b2l_bf16"])
def test_reference_cross_device_spread(name):
    """The committed cuBLAS run of the reference path (make_gpu_reference.py,
    teacher-forced with the CPU golden's tokens) against the reference's own
    CPU run: the same computation on two devices differs by a few bf16 ulps of
    the row's largest logit at every step, which is why the B200 path's
    end-to-end logits are held to this spread (and each op to 2e-2)."""
    from conftest import bf16_ulp, load_gpuref
    g, r = load_golden(name), load_gpuref(name)
    assert r is not None, f"{name}_gpuref.npz missing"
    assert r["logits_sub"].shape == g["logits_sub"].shape
    err = np.abs(r["logits_sub"] - g["logits_sub"])
    row_ulp = bf16_ulp(np.abs(g["logits_sub"]).max(axis=2, keepdims=True))
    print(f"{name}: cuBLAS vs CPU reference logits max-abs {err.max():.4f}, rms {np.sqrt((err ** 2).mean()):.4f}, "
          f"{(err / row_ulp).max():.1f} ulps of the row maximum; greedy top-1 agreement "
          f"{(r['top2_idx'][..., 0] == g['top2_idx'][..., 0]).mean():.3f}")
    assert 0.02 < err.max() < 0.1  # recorded spread (bf16 drift, not a different algorithm)
    assert (r["top2_idx"][..., 0] == g["top2_idx"][..., 0]).mean() >= 0.95
