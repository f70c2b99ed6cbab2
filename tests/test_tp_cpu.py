"""Multi-rank host logic of the TP path on CPU ranks (Gloo): process-group
layout, weight sharding of the parallel layers, the RowParallel all-reduce
placement, vocab-parallel argmax candidates, the leader/worker control
protocol and failure propagation.  No GPU: the GEMM is replaced by a CPU
matmul inside the test processes only."""
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run(rank, world, port, fn, q, *args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        fn(rank, world, *args)
        q.put((rank, None))
    except BaseException:  # noqa: BLE001
        q.put((rank, traceback.format_exc()))
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def spawn(world, fn, *args, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, fn, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, err = q.get(timeout=timeout)
        results[r] = err
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


# ---------------------------------------------------------------------------- workers
def _groups(rank, world, tp):
    from awesome_acceleration_b200.model import distributed as D
    D.init_distributed(tp, backend="gloo", timeout_s=30)
    assert D.get_tp_world_size() == tp and D.get_dp_world_size() == world // tp
    assert D.get_tp_rank() == rank % tp and D.get_dp_rank() == rank // tp
    assert D.get_tp_leader_global_rank() == (rank // tp) * tp
    assert D.is_tp_leader() == (rank % tp == 0) and D.is_global_rank_0() == (rank == 0)
    # The TP group sums over consecutive ranks, the DP group over strided ranks.
    import torch.distributed as dist
    t = torch.tensor([float(rank)])
    dist.all_reduce(t, group=D.get_tp_group())
    base = (rank // tp) * tp
    assert t.item() == sum(range(base, base + tp))
    t = torch.tensor([float(rank)])
    dist.all_reduce(t, group=D.get_dp_group())
    assert t.item() == sum(range(rank % tp, world, tp))
    obj = D.broadcast_object({"leader": rank} if D.is_tp_leader() else None, src=0)
    assert obj == {"leader": base}


def _layers(rank, world):
    from awesome_acceleration_b200 import kernels
    from awesome_acceleration_b200.model import distributed as D
    from awesome_acceleration_b200.model import parallel_layers as PL
    D.init_distributed(world, backend="gloo", timeout_s=30)
    # CPU stand-ins for the GEMM and the bias add (test only)
    kernels.gemm = lambda x, w, out=None, bias=None: (x.float() @ w.float().t()
                                                      + (0 if bias is None else bias.float())).to(x.dtype)
    kernels.bias_add = lambda x, b: x.add_(b)
    g = torch.Generator().manual_seed(0)
    H, I, Hq, Hkv, Dh = 64, 96, 4, 2, 16
    lin = torch.nn.Linear(H, I, bias=False)
    lin.weight.data = torch.randn((I, H), generator=g)
    col = PL.ColumnParallelLinear.from_linear(lin)
    assert col.weight.shape == (I // world, H)
    assert torch.equal(col.weight, lin.weight[rank * I // world:(rank + 1) * I // world])
    down = torch.nn.Linear(I, H, bias=False)
    down.weight.data = torch.randn((H, I), generator=g)
    row = PL.RowParallelLinear.from_linear(down)
    assert row.weight.shape == (H, I // world)
    x = torch.randn((3, 5, I), generator=g)
    xs = x[..., rank * I // world:(rank + 1) * I // world].contiguous()
    y = row(xs)  # partial matmul + all-reduce over the TP group
    assert torch.allclose(y, x @ down.weight.t(), atol=1e-4)
    # biases (model/parallel_layers.py:82, :163-170, :197-199): a column shard adds its slice of
    # the bias in the GEMM; a row-parallel layer keeps its bias on rank 0 only and adds it
    # after the all-reduce, so only rank 0's output carries it
    lin_b = torch.nn.Linear(H, I, bias=True)
    lin_b.weight.data, lin_b.bias.data = torch.randn((I, H), generator=g), torch.randn(I, generator=g)
    col_b = PL.ColumnParallelLinear.from_linear(lin_b)
    sl = slice(rank * I // world, (rank + 1) * I // world)
    assert torch.equal(col_b.bias, lin_b.bias[sl])
    xh = torch.randn((6, H), generator=g)
    assert torch.allclose(col_b(xh), xh @ lin_b.weight[sl].t() + lin_b.bias[sl], atol=1e-4)
    down_b = torch.nn.Linear(I, H, bias=True)
    down_b.weight.data, down_b.bias.data = torch.randn((H, I), generator=g), torch.randn(H, generator=g)
    row_b = PL.RowParallelLinear.from_linear(down_b)
    assert (row_b.bias is not None) == (rank == 0)
    y = row_b(xs)
    exp = x @ down_b.weight.t() + (down_b.bias if rank == 0 else 0)
    assert torch.allclose(y, exp, atol=1e-4)
    full = torch.randn(((Hq + 2 * Hkv) * Dh, H), generator=g)
    fb = torch.randn((Hq + 2 * Hkv) * Dh, generator=g)
    qkv_b = PL.QKVParallelLinear.from_fused_qkv(full, fb, H, Hq, Hkv, Dh)
    qr, kr = Hq // world * Dh, Hkv // world * Dh
    exp_b = torch.cat([fb[rank * qr:(rank + 1) * qr], fb[Hq * Dh + rank * kr:Hq * Dh + (rank + 1) * kr],
                       fb[(Hq + Hkv) * Dh + rank * kr:(Hq + Hkv) * Dh + (rank + 1) * kr]])
    assert torch.equal(qkv_b.bias, exp_b)
    qb, kb, vb = qkv_b(xh)
    assert torch.allclose(torch.cat([qb.flatten(1), kb.flatten(1), vb.flatten(1)], 1),
                          xh @ qkv_b.weight.t() + exp_b, atol=1e-4)
    qkv = PL.QKVParallelLinear.from_fused_qkv(full, None, H, Hq, Hkv, Dh)
    qr, kr = Hq // world * Dh, Hkv // world * Dh
    exp = torch.cat([full[rank * qr:(rank + 1) * qr], full[Hq * Dh + rank * kr:Hq * Dh + (rank + 1) * kr],
                     full[(Hq + Hkv) * Dh + rank * kr:(Hq + Hkv) * Dh + (rank + 1) * kr]])
    assert torch.equal(qkv.weight, exp)
    q, k, v = qkv(torch.randn((7, H), generator=g))
    assert q.shape == (7, Hq // world, Dh) and k.shape == v.shape == (7, Hkv // world, Dh)
    q, k, v = qkv(torch.randn((2, 3, H), generator=g))
    assert q.shape == (2, 3, Hq // world, Dh)
    with pytest.raises(ValueError):
        qkv(torch.randn(H))


def _vocab_argmax(rank, world):
    """Every rank scores its vocab shard; gathering (max, id) candidates and
    taking the highest value (lowest id on ties) equals the global argmax."""
    import torch.distributed as dist
    from awesome_acceleration_b200.model import distributed as D
    D.init_distributed(world, backend="gloo", timeout_s=30)
    g = torch.Generator().manual_seed(1)
    B, V = 6, 40
    logits = torch.randint(-3, 4, (B, V), generator=g).float()  # many ties
    shard = V // world
    local = logits[:, rank * shard:(rank + 1) * shard]
    val, idx = local.max(-1)  # torch.max returns the first index of the max
    idx = idx + rank * shard
    gv = torch.empty((world, B))
    gi = torch.empty((world, B), dtype=torch.int64)
    dist.all_gather_into_tensor(gv.view(-1), val)
    dist.all_gather_into_tensor(gi.view(-1), idx)
    best = gv.max(0).values
    cand = torch.where(gv == best, gi, torch.full_like(gi, 1 << 40))
    assert torch.equal(cand.min(0).values, logits.argmax(-1))


def _exit_propagates(rank, world):
    """A worker that dies between steps turns the leader's next control
    broadcast into an error within the process-group timeout (no hang)."""
    import time
    from awesome_acceleration_b200.model import distributed as D
    D.init_distributed(world, backend="gloo", timeout_s=5)
    if rank == 1:
        os._exit(0)  # dies without joining the next collective
    time.sleep(0.5)
    t0 = time.time()
    with pytest.raises(Exception):
        D.broadcast_object({"action": "decode", "batch_size": 1}, src=0)
        D.broadcast_object({"action": "decode", "batch_size": 1}, src=0)
    assert time.time() - t0 < 60


def _engine_protocol(rank, world, n_req, slots, seed, capacity=None):
    """LLMTP's own leader / worker loops on CPU ranks, over a stand-in runtime
    that logs every step it is told to run (and joins a Gloo collective at
    each, as the real one joins NCCL): a continuous-batching job with more
    requests than slots, ragged prompts, per-request max_tokens and
    temperatures must take every rank through the same steps, in the same
    order, and finish every request.  With `capacity` below `slots` the
    runtime cannot stage a full batch: the leader must fail its requests
    before it sends the oversized step, and the workers must leave cleanly
    instead of waiting inside that step's broadcast."""
    import itertools
    import queue
    import random
    import torch.distributed as dist
    from awesome_acceleration_b200 import llm_tp
    from awesome_acceleration_b200.model import distributed as D
    from awesome_acceleration_b200.runtime import Qwen3Runtime
    D.init_distributed(world, backend="gloo", timeout_s=30)
    log = []

    class KV:
        def __init__(self):
            self.lengths = {}

        def reserve(self, r, n):
            assert n <= 4096

        def release(self, r):
            self.lengths.pop(r, None)

    class Buf:
        meta = torch.zeros((4, slots), dtype=torch.int64)
        temp = torch.zeros(slots, dtype=torch.float32)

    class RT:
        max_batch, use_graphs, buf = capacity or slots, True, Buf()
        padded_batch = Qwen3Runtime.padded_batch

        def load_decode_inputs(self, ids, positions, rows, temperatures=None, seeds=None):
            B, Bp = len(rows), self.padded_batch(len(rows))
            m = self.buf.meta
            m[:, :Bp] = 0
            m[2, :Bp] = -1
            m[0, :B], m[1, :B], m[2, :B] = torch.tensor(ids), torch.tensor(positions), torch.tensor(rows)
            m[3, :B] = torch.tensor(seeds or [0] * B)
            self.buf.temp[:Bp] = 0
            self.buf.temp[:B] = torch.tensor(temperatures or [0.0] * B)

        def prefill(self, seqs, rows, temperatures=None, seeds=None):
            log.append(("prefill", tuple(rows), tuple(len(q) for q in seqs), tuple(temperatures or ()),
                        tuple(seeds or ())))
            dist.all_reduce(torch.ones(1), group=D.get_tp_group())
            for r, q in zip(rows, seqs):
                kv.lengths[r] = len(q)
            return torch.tensor([(sum(q) + len(q)) % 997 for q in seqs])

        def decode_step(self, rows):
            B, Bp = len(rows), self.padded_batch(len(rows))
            m = self.buf.meta
            log.append(("decode", Bp, tuple(m[2, :Bp].tolist()), tuple(m[1, :B].tolist()), tuple(m[3, :B].tolist()),
                        tuple(self.buf.temp[:B].tolist())))
            dist.all_reduce(torch.ones(1), group=D.get_tp_group())
            m[0, :B] = (m[0, :B] * 31 + m[1, :B]) % 997
            m[1, :B] += 1
            for r in rows:
                kv.lengths[r] += 1

        def read_tokens(self, B):
            return self.buf.meta[0, :B].tolist()

        snaps, unread, most_unread = [], 0, 0

        def copy_tokens_async(self, B):
            RT.snaps.append(self.buf.meta[0, :B].tolist())
            RT.unread += 1
            RT.most_unread = max(RT.most_unread, RT.unread)
            return len(RT.snaps) - 1

        def wait_tokens(self, handle, B):
            RT.unread -= 1
            return RT.snaps[handle][:B]

        def token_error(self, handle):
            return 0

    kv, rt = KV(), RT()

    class Model:
        max_batch = slots

        def __init__(self):
            self.kv = kv

        def _rt(self):
            return rt

        def clear_all_slots(self):
            kv.lengths.clear()

    torch.cuda.synchronize = lambda *a, **k: None  # this process has no GPU work to wait for
    llm_tp._lib.raise_on_device_error = lambda *a, **k: None  # nor a device error word
    eng = llm_tp.LLMTP.__new__(llm_tp.LLMTP)
    eng.device = torch.device("cpu")
    eng.model, eng.max_num_seqs, eng.max_seq_len = Model(), slots, 4096
    eng.config = type("C", (), {"eos_token_id": -1})()
    eng.tp_size, eng.tp_rank, eng.is_tp_leader = world, rank, rank == 0
    eng._bcast = torch.zeros(5 * slots, dtype=torch.int64)
    eng._request_queue = queue.Queue() if rank == 0 else None
    eng._loop_running, eng._loop_thread, eng._loop_error, eng.tokenizer = False, None, None, None
    eng._base_seed, eng._serials = 3, itertools.count(1)
    if rank == 0:
        rnd = random.Random(seed)
        reqs = [([rnd.randrange(1000) for _ in range(rnd.randint(1, 60))], rnd.choice([1, 2, 5, 9, 17, 30]),
                 rnd.choice([0.0, 0.0, 0.7])) for _ in range(n_req)]
        futs = [eng.generate_ids([p], max_tokens=m, temperature=t, ignore_eos=True) for p, m, t in reqs]
        if capacity:
            errs = []
            for f in futs:
                try:
                    f.result(timeout=60)
                except ValueError as e:
                    errs.append(e)
            eng.stop()
            assert errs and "max_batch" in str(errs[0]), errs
            assert isinstance(eng._loop_error, ValueError)
        else:
            outs = [f.result(timeout=60)[0] for f in futs]
            eng.stop()
            assert [o.generated_tokens for o in outs] == [m for _, m, _ in reqs]
            assert eng._loop_error is None, eng._loop_error
    else:
        eng.serve_worker()
    logs = [None] * world
    dist.all_gather_object(logs, log, group=D.get_tp_cpu_group())
    assert all(lg == logs[0] for lg in logs), "ranks ran different step sequences"
    if capacity:
        assert all(e[0] != "decode" or e[1] <= capacity for e in logs[0])
        return
    assert any(e[0] == "decode" and e[1] != len([r for r in e[2] if r >= 0]) for e in logs[0])  # padded buckets ran
    if rank == 0:
        assert RT.most_unread == 2  # a step was run ahead while the previous one was read


def _fused_weights_held_once(rank, world):
    """After fuse_qkv a TP rank keeps one copy of its weights: the interleaved
    gate/up (the separate gate/up released) and its own vocab shard of an
    untied lm_head (the full matrix released)."""
    import dataclasses
    from awesome_acceleration_b200.model import distributed as D
    from awesome_acceleration_b200.model.model import Qwen3Config
    from awesome_acceleration_b200.model.model_tp import Qwen3ForCausalLMTP
    from awesome_acceleration_b200.runtime import interleave_gate_up
    from oracle.weights import TINY
    D.init_distributed(world, backend="gloo", timeout_s=30)
    arch = dataclasses.replace(TINY, tie_word_embeddings=False)
    cfg = Qwen3Config(**{k: v for k, v in arch.as_dict().items() if k in Qwen3Config.__annotations__})
    torch.manual_seed(0)
    m = Qwen3ForCausalLMTP(cfg)
    with torch.no_grad():
        for prm in m.parameters():  # parallel layers allocate with torch.empty
            prm.normal_()
    full = m.lm_head.weight.detach().clone()
    gates = [(l.mlp.gate_proj.weight.detach().clone(), l.mlp.up_proj.weight.detach().clone()) for l in m.model.layers]
    m.fuse_qkv()
    V = cfg.vocab_size // world
    assert torch.equal(m._lm_shard, full[rank * V:(rank + 1) * V])
    assert m.lm_head.weight.numel() == 0
    for l, (g, u) in zip(m.model.layers, gates):
        assert torch.equal(l.mlp._gate_up, interleave_gate_up(g, u))
        assert l.mlp.gate_proj.weight.numel() == 0 and l.mlp.up_proj.weight.numel() == 0
    m.fuse_qkv()  # a second call changes nothing
    assert torch.equal(m._lm_shard, full[rank * V:(rank + 1) * V])


# ---------------------------------------------------------------------------- tests
@pytest.mark.parametrize("world,tp", [(2, 2), (4, 2), (4, 4)])
def test_process_groups(world, tp):
    res = spawn(world, _groups, tp)
    assert all(v is None for v in res.values()), res


def test_parallel_layer_sharding_and_row_allreduce():
    res = spawn(2, _layers)
    assert all(v is None for v in res.values()), res


def test_vocab_parallel_argmax_candidates():
    res = spawn(2, _vocab_argmax)
    assert all(v is None for v in res.values()), res


def test_dead_worker_raises_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, 2, port, _exit_propagates, q)) for r in range(2)]
    for p in procs:
        p.start()
    r, err = q.get(timeout=120)
    assert r == 0 and err is None, err
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()


@pytest.mark.parametrize("world,n_req,slots", [(2, 40, 12), (3, 90, 40)])
def test_llmtp_leader_worker_protocol(world, n_req, slots):
    res = spawn(world, _engine_protocol, n_req, slots, world * 1000 + n_req)
    assert all(v is None for v in res.values()), res


def test_llmtp_oversized_decode_batch_fails_without_stranding_workers():
    res = spawn(2, _engine_protocol, 40, 12, 7, 8)
    assert all(v is None for v in res.values()), res


def test_fused_weights_held_once_on_tp_ranks():
    res = spawn(2, _fused_weights_held_once)
    assert all(v is None for v in res.values()), res
