"""Engine-level behaviour on the GPU: the reference's LLM API (continuous
batching, stop rules, futures), checkpoint loading from safetensors, and the
KV export/import used for prefill/decode disaggregation."""
import json
import os

import pytest
import torch

from oracle.qwen3_oracle import Qwen3Oracle, run_greedy
from oracle.weights import TINY, init_weights, random_prompts

pytestmark = pytest.mark.gpu


def _cfg():
    from awesome_acceleration_b200.model.model import Qwen3Config
    return Qwen3Config(**{k: v for k, v in TINY.as_dict().items() if k in Qwen3Config.__annotations__})


def _model(sd, slots=4, max_seq_len=256):
    from awesome_acceleration_b200.model.model import Qwen3ForCausalLM
    with torch.device("meta"):
        m = Qwen3ForCausalLM(_cfg())
    m = m.to_empty(device="cuda").to(torch.bfloat16)
    m.load_state_dict({k: v.to(torch.bfloat16) for k, v in sd.items()}, strict=False)
    return m


def test_llm_generate_ids_continuous_batching(cuda):
    """More prompts than slots, ragged lengths, per-request max_tokens: every
    future resolves with the reference's GenerationOutput fields, and each
    stream equals the same prompt run alone (batch composition must not
    change results beyond argmax near-ties)."""
    from awesome_acceleration_b200.llm import LLM
    sd = init_weights(TINY, 40, norm_jitter=0.1)
    llm = LLM(model=_model(sd), max_num_seqs=3, max_seq_len=200)
    prompts = [p[:n] for p, n in zip(random_prompts(7, 60, TINY.vocab_size, 41), [60, 1, 13, 33, 2, 59, 20])]
    f1 = llm.generate_ids(prompts[:4], max_tokens=10, ignore_eos=True)
    f2 = llm.generate_ids(prompts[4:], max_tokens=5, ignore_eos=True)
    r1, r2 = f1.result(timeout=120), f2.result(timeout=120)
    assert [o.generated_tokens for o in r1] == [10] * 4 and [o.generated_tokens for o in r2] == [5] * 3
    assert [o.prompt_tokens for o in r1 + r2] == [len(p) for p in prompts]
    alone = llm.generate_ids([prompts[2]], max_tokens=10, ignore_eos=True).result(timeout=60)[0]
    assert alone.token_ids == r1[2].token_ids
    llm.stop()


def test_llm_stops_on_eos_and_max_seq_len(cuda):
    from awesome_acceleration_b200.llm import LLM
    sd = init_weights(TINY, 42, norm_jitter=0.1)
    llm = LLM(model=_model(sd), max_num_seqs=2, max_seq_len=70)
    prompt = random_prompts(1, 60, TINY.vocab_size, 43)[0]
    # pos >= max_seq_len stops generation (llm.py:417): 60-token prompt, limit 70:
    # the prefill token plus decode steps at positions 60..69 -> 11 tokens
    out = llm.generate_ids([prompt], max_tokens=100, ignore_eos=True).result(timeout=60)[0]
    assert out.generated_tokens == 11
    # EOS: make the first generated token the EOS id and check the stop
    # (the loop reads the EOS id when it starts; stop it first)
    first = out.token_ids[0]
    llm.stop()
    llm.config.eos_token_id = first
    out2 = llm.generate_ids([prompt], max_tokens=100, ignore_eos=False).result(timeout=60)[0]
    assert out2.token_ids == [first]
    with pytest.raises(ValueError):
        llm.generate_ids([prompt], temperature=-0.7)
    with pytest.raises(ValueError):
        llm.generate_ids([[]])
    llm.stop()


def test_llm_failure_resolves_futures(cuda):
    """A failing step fails every outstanding future (the reference leaves
    them unresolved, llm.py:315-446)."""
    from awesome_acceleration_b200.llm import LLM
    sd = init_weights(TINY, 44, norm_jitter=0.1)
    llm = LLM(model=_model(sd), max_num_seqs=2, max_seq_len=128)
    rt = llm.model._rt()

    def boom(*a, **k):
        raise RuntimeError("injected host-side failure")

    rt.decode_step = boom
    fut = llm.generate_ids([[1, 2, 3], [4, 5]], max_tokens=5, ignore_eos=True)
    with pytest.raises(RuntimeError, match="injected"):
        fut.result(timeout=60)
    with pytest.raises(RuntimeError):
        llm.generate_ids([[1]], max_tokens=2)


def test_from_pretrained_safetensors(cuda, tmp_path):
    """LLM(model_path) loads config.json + model.safetensors (model/model.py:353-384)
    and produces the same tokens as the in-memory state dict."""
    from safetensors.torch import save_file

    from awesome_acceleration_b200.llm import LLM
    sd = init_weights(TINY, 45, norm_jitter=0.1)
    save_file({k: v.to(torch.bfloat16).contiguous() for k, v in sd.items()}, str(tmp_path / "model.safetensors"))
    with open(tmp_path / "config.json", "w") as f:
        json.dump(TINY.as_dict(), f)
    a = LLM(str(tmp_path), max_num_seqs=2, max_seq_len=128)
    b = LLM(model=_model(sd), max_num_seqs=2, max_seq_len=128)
    prompts = [[3, 1, 4, 1, 5], [9, 2, 6]]
    ra = a.generate_ids(prompts, max_tokens=6, ignore_eos=True).result(timeout=60)
    rb = b.generate_ids(prompts, max_tokens=6, ignore_eos=True).result(timeout=60)
    assert [o.token_ids for o in ra] == [o.token_ids for o in rb]
    a.stop()
    b.stop()


def test_export_import_request_kv(cuda):
    """KV of a prefilled sequence exported from one slot and imported into
    another continues decoding exactly like the original
    (model/model.py:156-177, :386-401)."""
    sd = init_weights(TINY, 46, norm_jitter=0.1)
    m = _model(sd)
    m.fuse_qkv()
    m.init_kv_cache(4, 256, "cuda", torch.bfloat16)
    rt = m._rt()
    prompt = random_prompts(1, 300, TINY.vocab_size, 47)[0][:200]
    tok = rt.prefill([prompt], [0]).tolist()
    payload = m.export_request_kv(0, len(prompt))
    assert len(payload["layers"]) == TINY.num_hidden_layers
    assert payload["layers"][0]["k"].shape == (len(prompt), TINY.num_key_value_heads, 128)
    m.import_request_kv(3, payload, len(prompt))
    for s in range(2):
        k0, v0 = m.kv.gather(s, 0, len(prompt))
        k3, v3 = m.kv.gather(s, 3, len(prompt))
        assert torch.equal(k0, k3) and torch.equal(v0, v3)
    # device-resident hand-off (no host round trip): export to a GPU, import into slot 2
    dev_payload = m.export_request_kv(0, len(prompt), device="cuda")
    assert dev_payload["layers"][0]["k"].is_cuda
    m.import_request_kv(2, dev_payload, len(prompt))
    k2, v2 = m.kv.gather(1, 2, len(prompt))
    k0, v0 = m.kv.gather(1, 0, len(prompt))
    assert torch.equal(k0, k2) and torch.equal(v0, v2)
    outs = []
    for row in (0, 3):
        rt.load_decode_inputs(tok, [len(prompt)], [row])
        seq = []
        for _ in range(4):
            rt.decode_step([row])
            seq.append(rt.read_tokens(1)[0])
        outs.append(seq)
    assert outs[0] == outs[1]


def test_bucketed_decode_graphs_match_eager(cuda):
    """Per-request max_tokens make the decode batch shrink step by step; with
    CUDA graphs the runtime pads it to a bucket (padding rows have slot -1)
    and replays a few graphs.  Every stream must equal the eager run, which
    uses the exact batch size."""
    from awesome_acceleration_b200.llm import LLM
    sd = init_weights(TINY, 44, norm_jitter=0.1)
    lens = [60, 1, 13, 33, 2, 59, 20, 41, 7, 18, 50]
    prompts = [p[:n] for p, n in zip(random_prompts(len(lens), 60, TINY.vocab_size, 45), lens)]
    max_toks = [3, 17, 1, 9, 12, 5, 20, 2, 14, 8, 11]
    runs = []
    for graphs in (False, True):
        llm = LLM(model=_model(sd), max_num_seqs=10, max_seq_len=200, use_cuda_graphs=graphs)
        futs = [llm.generate_ids([p], max_tokens=t, ignore_eos=True) for p, t in zip(prompts, max_toks)]
        outs = [f.result(timeout=120)[0] for f in futs]
        assert [o.generated_tokens for o in outs] == max_toks
        runs.append([o.token_ids for o in outs])
        rt = llm.model._rt()
        if graphs:
            assert set(rt._graphs) <= {1, 2, 4, 8, 10}, sorted(rt._graphs)  # 9-10 rows: capped at max_batch
        llm.stop()
    assert runs[0] == runs[1]


def test_llm_temperature_sampling(cuda):
    """temperature > 0 through the engine (llm.py:215-219): reproducible for a
    given engine seed and request order, identical with and without CUDA
    graphs, different from greedy and from another seed, and a
    temperature-0 request in the same batch keeps its greedy stream."""
    from awesome_acceleration_b200.llm import LLM
    sd = init_weights(TINY, 46, norm_jitter=0.1)
    prompts = [p[:n] for p, n in zip(random_prompts(4, 40, TINY.vocab_size, 47), [40, 9, 23, 31])]
    runs = []
    for graphs in (True, False, True):
        llm = LLM(model=_model(sd), max_num_seqs=4, max_seq_len=128, seed=5, use_cuda_graphs=graphs)
        hot = llm.generate_ids(prompts[:3], max_tokens=16, temperature=1.5, ignore_eos=True)
        cold = llm.generate_ids(prompts[3:], max_tokens=16, temperature=0.0, ignore_eos=True)
        runs.append(([o.token_ids for o in hot.result(timeout=120)], cold.result(timeout=120)[0].token_ids))
        llm.stop()
    assert runs[0] == runs[1] == runs[2]
    llm = LLM(model=_model(sd), max_num_seqs=4, max_seq_len=128, seed=5)
    greedy = llm.generate_ids(prompts, max_tokens=16, ignore_eos=True).result(timeout=120)
    llm.stop()
    other = LLM(model=_model(sd), max_num_seqs=4, max_seq_len=128, seed=6)
    resampled = other.generate_ids(prompts[:3], max_tokens=16, temperature=1.5, ignore_eos=True).result(timeout=120)
    other.stop()
    assert runs[0][1] == greedy[3].token_ids
    assert runs[0][0] != [o.token_ids for o in greedy[:3]]
    assert runs[0][0] != [o.token_ids for o in resampled]
