"""Tensor parallelism on >= 2 GPUs (NCCL + the NVLink exchange): the TP model
against the reference's golden vectors (Qwen3-8B layer shapes, two layers,
tests/golden/tp8b2l_bf16.npz) at TP = 2 / 4 / 8, the LLMTP leader/worker
engine, and the exchange kernel against an exact rank-order sum."""
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
TP_RMS_MARGIN = 1.5


def _ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, fn, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        q.put((rank, fn(rank, world, *args), None))
    except BaseException:  # noqa: BLE001
        q.put((rank, None, traceback.format_exc()))
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def run_ranks(world, fn, *args, timeout=300):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, fn, args)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(world):
        r, val, err = q.get(timeout=timeout)
        assert err is None, f"rank {r}:\n{err}"
        out[r] = val
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def _prompts():
    from oracle.weights import TINY, random_prompts
    return [p[:n] for p, n in zip(random_prompts(4, 90, TINY.vocab_size, 31), [90, 7, 40, 64])]


def _tp_golden_case(rank, world):
    """One rank of the TP model on the 8B-shaped golden: teacher-forced
    logits (shards gathered) at every step, then the free-running greedy
    stream through the captured decode graphs (RowParallel outputs over the
    NVLink exchange, vocab-parallel argmax)."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), here]
    import numpy as np
    from conftest import load_golden
    from test_parity_gpu import free_running
    from awesome_acceleration_b200 import _lib
    from awesome_acceleration_b200.model import distributed as D
    from awesome_acceleration_b200.model.model import Qwen3Config
    from awesome_acceleration_b200.model.model_tp import Qwen3ForCausalLMTP
    from oracle.weights import Qwen3Arch, init_weights
    D.init_distributed(world, timeout_s=300)
    dev = torch.device("cuda", rank)
    g = load_golden("tp8b2l_bf16")
    arch = Qwen3Arch(**g["arch"])
    cfg = Qwen3Config(**{k: v for k, v in arch.as_dict().items() if k in Qwen3Config.__annotations__})
    sd = init_weights(arch, int(g["seed"]), norm_jitter=float(g["norm_jitter"]))
    m = Qwen3ForCausalLMTP.from_state_dict(sd, cfg, dev)
    del sd
    m.fuse_qkv()
    lens = g["lens"].tolist()
    prompts = [g["prompts"][i][:L].tolist() for i, L in enumerate(lens)]
    slots = g["slots"].tolist()
    m.init_kv_cache(len(lens), int(g["max_seq_len"]), dev, torch.bfloat16)
    rt = m._rt()
    vi = torch.from_numpy(g["vocab_idx"]).to(dev)

    def full(shard):
        return D.tensor_model_parallel_all_gather(shard.contiguous(), dim=-1)

    _, lg = rt.prefill(prompts, slots, last_logits=True)
    subs = [full(lg).float()[:, vi].cpu().numpy()]
    pos = list(lens)
    for s in range(int(g["steps"])):
        rt.load_decode_inputs(g["tokens"][:, s].tolist(), pos, slots)
        shard = torch.empty((len(slots), rt.vocab_local), dtype=torch.bfloat16, device=dev)
        rt.decode_step(slots, logits=shard)
        subs.append(full(shard).float()[:, vi].cpu().numpy())
        pos = [p + 1 for p in pos]
    mine = np.stack(subs)
    m.kv.clear_all()
    near = free_running(m, g, prompts, lens, slots)
    exchange = rt.comm.exchange is not None
    assert _lib.device_error() == 0
    err = np.abs(mine - g["logits_sub"])
    return float(err.max()), float(np.sqrt((err ** 2).mean())), int((err <= 2e-2).sum()), err.size, near, exchange


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_vs_reference_golden(cuda, world):
    """TP = world on the Qwen3-8B layer shapes (32 / 8 heads: 4 query heads per
    kv head on every rank, hidden 4096, untied vocab-parallel lm_head): logits
    within the reference's own CPU-vs-cuBLAS spread at every step, and the
    free-running greedy stream equal to the reference's except at its near-ties."""
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    from test_parity_gpu import SPREAD_MARGIN, TOL, reference_spread
    res = run_ranks(world, _tp_golden_case, timeout=900)
    ref_mx, ref_rms = reference_spread("tp8b2l_bf16")
    mx, rms, within, total, near, exchange = res[0]
    for r in range(1, world):
        assert res[r][4] == near, f"rank {r} saw a different greedy stream"
    print(f"\nTP={world} (NVLink exchange: {exchange}): logits max-abs {mx:.4f}, rms {rms:.4f} (reference's own "
          f"spread {ref_mx:.4f} / {ref_rms:.4f}); {within} of {total} logits within {TOL}; "
          f"{len(near)} reference near-tie steps {near}")
    assert exchange, "the NVLink exchange was not set up"
    # Each rank rounds its RowParallel partial output to bf16 before the
    # all-reduce, as the reference's TP path does (F.linear in bf16, then
    # all_reduce, model/parallel_layers.py:191-195): one more rounding per
    # projection than the single-GPU run the spread was measured on, hence
    # the wider rms margin.
    assert mx <= max(TOL, SPREAD_MARGIN * ref_mx) and rms <= TP_RMS_MARGIN * ref_rms


def _llmtp_engine(rank, world):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from awesome_acceleration_b200.llm_tp import LLMTP
    from awesome_acceleration_b200.model.model import Qwen3Config
    from oracle.weights import TINY, init_weights
    cfg = Qwen3Config(**{k: v for k, v in TINY.as_dict().items() if k in Qwen3Config.__annotations__})
    llm = LLMTP(None, max_num_seqs=3, max_seq_len=256, enable_tp=True, tp_size=world, config=cfg,
                state_dict=init_weights(TINY, 30, norm_jitter=0.1))
    if not llm.is_tp_leader:
        llm.serve_worker()
        return None
    prompts = _prompts() + [[5, 6, 7], [9] * 20]  # more prompts than slots: continuous batching
    outs = llm.generate_ids(prompts, max_tokens=9, ignore_eos=True).result(timeout=240)
    # temperature sampling across the TP group: the vocab shards' perturbed scores merge to one draw
    hot = llm.generate_ids(prompts[:2], max_tokens=6, temperature=1.2, ignore_eos=True).result(timeout=240)
    llm.stop()
    assert [len(o.token_ids) for o in hot] == [6, 6]
    return [o.token_ids for o in outs], [o.generated_tokens for o in outs]


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
def test_llmtp_engine_two_ranks(cuda):
    res = run_ranks(2, _llmtp_engine)
    toks, gen = res[0]
    assert gen == [9] * 6
    assert all(len(t) == 9 for t in toks)


def _exchange_case(rank, world):
    """The NVLink exchange kernel against NCCL: all-gather every rank's bf16
    output, sum in fp32 in rank order, round, then the add+RMSNorm kernel."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    from awesome_acceleration_b200 import _lib
    from awesome_acceleration_b200 import kernels as K
    from awesome_acceleration_b200.model import distributed as D
    from awesome_acceleration_b200.runtime import TPComm
    D.init_distributed(world, timeout_s=120)
    dev = torch.device("cuda", rank)
    bad = []
    for hidden in (1024, 4096):
        comm = TPComm(rank, world, D.get_tp_group(), D.get_tp_cpu_group())
        comm.enable_peer_exchange(256, hidden)
        assert comm.exchange is not None
        w = (1 + 0.1 * torch.randn(hidden, generator=torch.Generator().manual_seed(7))).bfloat16().to(dev)
        step = 0
        for two_shot in (False, True):
            comm.exchange.two_shot = two_shot
            for M, splits in ((1, 0), (37, 3), (128, 8), (256, 2), (200, 0)):
                step += 1
                g = torch.Generator().manual_seed(1000 * step + rank)
                if splits:
                    src = torch.randn(splits, M, hidden, generator=g).to(dev)
                    mine = torch.empty(M, hidden, dtype=torch.bfloat16, device=dev)
                    K.splitk_reduce(src, splits, mine)
                else:
                    src = torch.randn(M, hidden, generator=g).bfloat16().to(dev)
                    mine = src.clone()
                res0 = torch.randn(M, hidden, generator=torch.Generator().manual_seed(step)).bfloat16().to(dev)
                # reference: exact fp32 sum in rank order of the all-gathered outputs
                allv = torch.empty(world, M, hidden, dtype=torch.bfloat16, device=dev)
                dist.all_gather_into_tensor(allv.view(-1), mine.view(-1), group=D.get_tp_group())
                acc = torch.zeros(M, hidden, dtype=torch.float32, device=dev)
                for p in range(world):
                    acc += allv[p].float()
                delta = acc.bfloat16()
                res_ref, y_ref = res0.clone(), torch.empty_like(res0)
                K.add_rmsnorm(delta, res_ref, w, 1e-6, out=y_ref)
                if world == 2:  # NCCL's bf16 sum of two ranks is the same rounding
                    nc = mine.clone()
                    dist.all_reduce(nc, group=D.get_tp_group())
                    if not torch.equal(nc, delta):
                        bad.append(("nccl", hidden, two_shot, M, splits))
                res, y = res0.clone(), torch.empty_like(res0)
                assert comm.allreduce_add_rmsnorm(src, splits, res, w, 1e-6, y)
                torch.cuda.synchronize()
                if not (torch.equal(res, res_ref) and torch.equal(y, y_ref)):
                    bad.append((hidden, two_shot, M, splits, (res.float() - res_ref.float()).abs().max().item(),
                                (y.float() - y_ref.float()).abs().max().item()))
        # graph replays keep the ranks' call counters in step
        M = 64
        src = torch.zeros(4, M, hidden, device=dev)
        res, y = torch.zeros(M, hidden, dtype=torch.bfloat16, device=dev), torch.empty(M, hidden, dtype=torch.bfloat16,
                                                                                     device=dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                comm.allreduce_add_rmsnorm(src, 4, res, w, 1e-6, y)
        torch.cuda.current_stream().wait_stream(s)
        for it in range(5):
            g = torch.Generator().manual_seed(50 + it + 100 * rank)
            src.copy_(torch.randn(4, M, hidden, generator=g))
            res.copy_(torch.randn(M, hidden, generator=torch.Generator().manual_seed(it)).bfloat16())
            res0 = res.clone()
            graph.replay()
            torch.cuda.synchronize()
            mine = torch.empty(M, hidden, dtype=torch.bfloat16, device=dev)
            K.splitk_reduce(src, 4, mine)
            allv = torch.empty(world, M, hidden, dtype=torch.bfloat16, device=dev)
            dist.all_gather_into_tensor(allv.view(-1), mine.view(-1), group=D.get_tp_group())
            acc = torch.zeros(M, hidden, dtype=torch.float32, device=dev)
            for p in range(world):
                acc += allv[p].float()
            res_ref, y_ref = res0.clone(), torch.empty_like(res0)
            K.add_rmsnorm(acc.bfloat16(), res_ref, w, 1e-6, out=y_ref)
            if not (torch.equal(res, res_ref) and torch.equal(y, y_ref)):
                bad.append(("graph", hidden, it))
        del graph
        assert _lib.device_error() == 0
        comm.close()
    return bad


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_exchange_kernel(cuda, world):
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    res = run_ranks(world, _exchange_case)
    for r in range(world):
        assert res[r] == [], f"rank {r}: {res[r]}"
