"""Prefill / decode disaggregation across processes: a request's KV exported
by one process through CUDA IPC (export_request_kv_ipc) and imported by
another into its own paged cache (import_request_kv_ipc) continues decoding
exactly like the original (the reference's export/import, model/model.py:
156-177, :386-401, which it ships through host shared memory,
pd/kv_connector_shm.py:97-209).  Runs with both processes on one GPU, and
across two GPUs (read over NVLink) where the box has them."""
import os
import sys
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
STEPS = 12


def _ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _engine(dev):
    sys.path[:0] = [os.path.dirname(HERE), HERE]
    from conftest import build_model
    from oracle.weights import TINY, init_weights
    return build_model(TINY, init_weights(TINY, 61, norm_jitter=0.1), 4, 512, torch.device("cuda", dev))


def _prompt():
    from oracle.weights import TINY, random_prompts
    return random_prompts(1, 300, TINY.vocab_size, 62)[0][:257]


def _decode(rt, first, length, row):
    rt.load_decode_inputs([first], [length], [row])
    seq = [first]
    for _ in range(STEPS):
        rt.decode_step([row])
        seq.append(rt.read_tokens(1)[0])
    return seq


def _prefill_side(dev, q_ticket, q_ack, q_res):
    try:
        torch.cuda.set_device(dev)
        m = _engine(dev)
        rt = m._rt()
        prompt = _prompt()
        first = rt.prefill([prompt], [0]).tolist()[0]
        ticket, owner = m.export_request_kv_ipc(0, len(prompt))
        q_ticket.put((ticket, first))
        seq = _decode(rt, first, len(prompt), 0)  # the original keeps decoding in its own cache
        q_ack.get(timeout=240)                     # the importer is done reading the buffer
        owner.release()
        from awesome_acceleration_b200 import _lib
        q_res.put(("prefill", seq, _lib.device_error(), None))
    except BaseException:  # noqa: BLE001
        q_res.put(("prefill", None, None, traceback.format_exc()))


def _decode_side(dev, q_ticket, q_ack, q_res):
    try:
        torch.cuda.set_device(dev)
        m = _engine(dev)
        rt = m._rt()
        ticket, first = q_ticket.get(timeout=240)
        m.import_request_kv_ipc(2, ticket)
        q_ack.put("done")
        assert int(m.kv.lengths[2]) == ticket.seqlen == ticket.length
        seq = _decode(rt, first, ticket.length, 2)
        from awesome_acceleration_b200 import _lib
        q_res.put(("decode", seq, _lib.device_error(), None))
    except BaseException:  # noqa: BLE001
        q_res.put(("decode", None, None, traceback.format_exc()))


@pytest.mark.parametrize("devices", [(0, 0), (0, 1)])
def test_kv_handoff_between_processes(cuda, devices):
    if _ngpu() <= max(devices):
        pytest.skip(f"needs {max(devices) + 1} GPUs")
    ctx = mp.get_context("spawn")
    q_ticket, q_ack, q_res = ctx.Queue(), ctx.Queue(), ctx.Queue()
    ps = [ctx.Process(target=_prefill_side, args=(devices[0], q_ticket, q_ack, q_res)),
          ctx.Process(target=_decode_side, args=(devices[1], q_ticket, q_ack, q_res))]
    for p in ps:
        p.start()
    out = {}
    for _ in range(2):
        who, seq, err, tb = q_res.get(timeout=300)
        assert tb is None, f"{who} side:\n{tb}"
        assert err == 0, f"{who} side: device error {err}"
        out[who] = seq
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert out["decode"] == out["prefill"], out
