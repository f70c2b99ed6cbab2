"""LLM's continuous-batching loop on the CPU, over a stand-in runtime whose
'device' produces each row's next token from that row's own last token and
position.  Checks the scheduler host path (llm.py:315-446): admission of more
requests than slots, per-request max_tokens, EOS and max_seq_len stops, and
the decode step kept in flight behind the one being read, against the token
streams the rows must produce."""
import itertools
import queue

import torch

from awesome_acceleration_b200.llm import LLM
from awesome_acceleration_b200.runtime import Qwen3Runtime

V, EOS = 97, 7


def _first(prompt):
    return (sum(prompt) * 13 + len(prompt)) % V


def _next(tok, pos):
    return (tok * 31 + pos * 17 + 5) % V


class _KV:
    def __init__(self):
        self.lengths = {}

    def release(self, r):
        self.lengths.pop(r, None)


class _Runtime:
    """Device state per row (last token, position); steps run immediately."""

    def __init__(self, max_batch, log):
        self.max_batch, self.use_graphs, self.log = max_batch, True, log
        self.ids, self.pos, self.rows = {}, {}, []
        self.snaps, self.d2h_bytes, self.kv = [], 0, _KV()
        self.unread, self.most_unread = 0, 0

    padded_batch = Qwen3Runtime.padded_batch

    def prefill(self, seqs, rows, temperatures=None, seeds=None):
        out = []
        for r, q in zip(rows, seqs):
            self.kv.lengths[r] = len(q)
            out.append(_first(q))
        return torch.tensor(out)

    def load_decode_inputs(self, ids, positions, rows, temperatures=None, seeds=None):
        self.rows = list(rows)
        for r, t, p in zip(rows, ids, positions):
            self.ids[r], self.pos[r] = t, p

    def decode_step(self, rows):
        assert list(rows) == self.rows, "a step ran on rows the device was not staged with"
        for r in rows:
            assert r in self.kv.lengths, f"decode step on released row {r}"
            self.ids[r] = _next(self.ids[r], self.pos[r])
            self.pos[r] += 1
        self.log.append(len(rows))

    def copy_tokens_async(self, B):
        self.snaps.append([self.ids[r] for r in self.rows[:B]])
        self.unread += 1
        self.most_unread = max(self.most_unread, self.unread)
        return len(self.snaps) - 1

    def wait_tokens(self, handle, B):
        self.unread -= 1
        return self.snaps[handle][:B]


def _engine(slots, max_seq_len):
    log = []
    rt = _Runtime(slots, log)

    class Model:
        kv = rt.kv

        def _rt(self):
            return rt

        def clear_all_slots(self):
            rt.kv.lengths.clear()

    eng = LLM.__new__(LLM)
    eng.model, eng.config = Model(), type("C", (), {"eos_token_id": EOS})()
    eng.device = torch.device("cpu")
    eng.max_num_seqs, eng.max_seq_len, eng.tokenizer = slots, max_seq_len, None
    eng._request_queue, eng._loop_running, eng._loop_thread, eng._loop_error = queue.Queue(), False, None, None
    eng._base_seed, eng._serials = 0, itertools.count(1)
    eng.stats = {"prefill_s": 0.0, "decode_s": 0.0, "decode_steps": 0, "prefill_tokens": 0}
    return eng, log


def _expected(prompt, max_tokens, ignore_eos, max_seq_len):
    toks, pos = [_first(prompt)], len(prompt)
    while not (len(toks) >= max_tokens or (not ignore_eos and toks[-1] == EOS)):
        if pos >= max_seq_len:
            break
        toks.append(_next(toks[-1], pos))
        pos += 1
    return toks


def _run(n_req, slots, max_seq_len, seed):
    import random
    rnd = random.Random(seed)
    eng, log = _engine(slots, max_seq_len)
    reqs = [([rnd.randrange(V) for _ in range(rnd.randint(1, 40))], rnd.choice([1, 2, 3, 8, 20, 45, 80]),
             rnd.random() < 0.5) for _ in range(n_req)]
    futs = [eng.generate_ids([p], max_tokens=m, ignore_eos=e) for p, m, e in reqs]
    outs = [f.result(timeout=60)[0] for f in futs]
    eng.stop()
    assert eng._loop_error is None
    for (p, m, e), o in zip(reqs, outs):
        assert o.token_ids == _expected(p, m, e, max_seq_len), (p, m, e)
    return log


def test_engine_loop_streams_and_stops():
    for seed in range(6):
        _run(n_req=30, slots=8, max_seq_len=64, seed=seed)


def test_engine_loop_runs_ahead_when_the_batch_is_stable():
    eng, log = _engine(4, 4096)
    prompts = [[1, 2, 3], [4], [5, 6], [7, 8, 9, 10]]
    futs = eng.generate_ids(prompts, max_tokens=50, ignore_eos=True)
    outs = futs.result(timeout=60)
    eng.stop()
    assert [o.token_ids for o in outs] == [_expected(p, 50, True, 4096) for p in prompts]
    assert sum(log) == 4 * 49  # no extra decode step: the last one is not run ahead
    assert eng.model._rt().most_unread == 2  # a step was in flight while the previous one was read
