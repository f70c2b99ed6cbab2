"""Tensor parallelism on >= 2 GPUs (NCCL): the TP model and the LLMTP
leader/worker engine against the single-GPU path on the same weights."""
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


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


def _tp_model_stream(rank, world, steps):
    """Prefill + decode on the TP model; returns tokens and last-step logits."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from awesome_acceleration_b200.model import distributed as D
    from awesome_acceleration_b200.model.model import Qwen3Config
    from awesome_acceleration_b200.model.model_tp import Qwen3ForCausalLMTP
    from oracle.weights import TINY, init_weights
    D.init_distributed(world, timeout_s=120)
    dev = torch.device("cuda", rank)
    cfg = Qwen3Config(**{k: v for k, v in TINY.as_dict().items() if k in Qwen3Config.__annotations__})
    sd = init_weights(TINY, 30, norm_jitter=0.1)
    m = Qwen3ForCausalLMTP.from_state_dict(sd, cfg, dev)
    m.fuse_qkv()
    m.init_kv_cache(4, 256, dev, torch.bfloat16)
    rt = m._rt()
    prompts = _prompts()
    rows = [0, 1, 2, 3]
    toks = rt.prefill(prompts, rows).tolist()
    seq = [toks]
    rt.load_decode_inputs(toks, [len(p) for p in prompts], rows)
    for _ in range(steps):
        rt.decode_step(rows)
        seq.append(rt.read_tokens(4))
    # one more step with materialised (gathered) logits through forward()
    ids = torch.tensor([[t] for t in seq[-1]], device=dev)
    pos = torch.tensor([[len(p) + steps] for p in prompts], device=dev)
    logits = m(ids, pos, torch.tensor(rows, device=dev))[:, 0].float().cpu()
    return seq, logits


def _single_stream(steps):
    from awesome_acceleration_b200.model.model import Qwen3Config, Qwen3ForCausalLM
    from oracle.weights import TINY, init_weights
    dev = torch.device("cuda", 0)
    cfg = Qwen3Config(**{k: v for k, v in TINY.as_dict().items() if k in Qwen3Config.__annotations__})
    sd = init_weights(TINY, 30, norm_jitter=0.1)
    with torch.device("meta"):
        m = Qwen3ForCausalLM(cfg)
    m = m.to_empty(device=dev).to(torch.bfloat16)
    m.load_state_dict({k: v.to(torch.bfloat16) for k, v in sd.items()}, strict=False)
    m.fuse_qkv()
    m.init_kv_cache(4, 256, dev, torch.bfloat16)
    rt = m._rt()
    prompts = _prompts()
    rows = [0, 1, 2, 3]
    toks = rt.prefill(prompts, rows).tolist()
    seq = [toks]
    rt.load_decode_inputs(toks, [len(p) for p in prompts], rows)
    for _ in range(steps):
        rt.decode_step(rows)
        seq.append(rt.read_tokens(4))
    ids = torch.tensor([[t] for t in seq[-1]], device=dev)
    pos = torch.tensor([[len(p) + steps] for p in prompts], device=dev)
    logits = m(ids, pos, torch.tensor(rows, device=dev))[:, 0].float().cpu()
    return seq, logits


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
def test_tp2_matches_single_gpu(cuda):
    steps = 12
    tp = run_ranks(2, _tp_model_stream, steps)
    assert tp[0][0] == tp[1][0], "TP ranks disagree on the greedy stream"
    assert torch.equal(tp[0][1], tp[1][1]), "TP ranks disagree on the gathered logits"
    single_seq, single_logits = _single_stream(steps)
    err = (tp[0][1] - single_logits).abs().max().item()
    assert err <= 2e-2, f"TP=2 logits differ from TP=1 by {err}"
    # Greedy streams agree until a near-tie (the all-reduce sums partial
    # products in a different order than the single-GPU GEMM).
    same = sum(a == b for a, b in zip(tp[0][0], single_seq))
    assert same >= len(single_seq) // 2, (tp[0][0], single_seq)


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
