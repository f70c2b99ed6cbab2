"""Host-side routing of the decode projections (Qwen3Runtime._qkv, _gate_up,
_row_parallel): which kernels a decode batch of M rows runs and with what
split counts, for one GPU and under tensor parallelism, checked on the CPU
against a recording stand-in for the kernel module (no GPU, no kernels)."""
from __future__ import annotations

import types

import pytest
import torch

from awesome_acceleration_b200 import kernels as realK
from awesome_acceleration_b200 import runtime as R

H, I, HQ, HKV = 1024, 3072, 16, 8  # Qwen3-0.6B


class Recorder:
    """The kernels module's constants and planners, with every launch recorded."""

    def __init__(self):
        self.calls = []
        for name in ("SKINNY_MAX_ROWS", "SKINNY_DEFAULT_ROWS", "SKINNY_FUSED_ROWS", "SKINNY_TARGET_CTAS",
                     "SKINNY_TARGET_CTAS_ROW", "CLUSTER_MAX_ROWS", "pick_splits", "pick_skinny_splits"):
            setattr(self, name, getattr(realK, name))

    def __getattr__(self, name):
        def launch(*args, **kw):
            splits = [a for a in args if isinstance(a, int) and not isinstance(a, bool)]
            self.calls.append((name, splits[0] if splits else None))
        return launch


def fake_runtime(tp=1, skinny_rows=32, fused_rows=0, cluster=False, graph_exchange=False):
    rt = types.SimpleNamespace(eps=1e-6, rope=None, Hq=HQ // tp, skinny_rows=skinny_rows, skinny_fused_rows=fused_rows,
                               cluster_gemm=cluster)
    rt.kv = types.SimpleNamespace(k=[None], v=[None])
    rt.buf = types.SimpleNamespace(sk_cnt=None)
    exchanged = []

    def allreduce_add_rmsnorm(src, splits, res, w, eps, out):
        exchanged.append(splits)
        return graph_exchange

    rt.comm = types.SimpleNamespace(size=tp, allreduce_add_rmsnorm=allreduce_add_rmsnorm,
                                    all_reduce=lambda t: exchanged.append("nccl"))
    for m in ("_skinny", "_skinny_part", "_splits", "_cluster", "_qkv", "_gate_up", "_row_parallel"):
        setattr(rt, m, types.MethodType(getattr(R.Qwen3Runtime, m), rt))
    rt.exchanged = exchanged
    return rt


def layer(tp=1):
    hq, hkv, inter = HQ // tp, HKV // tp, I // tp
    return types.SimpleNamespace(wqkv=torch.empty(((hq + 2 * hkv) * 128, H)), q_norm=None, k_norm=None,
                                 w_gate_up=torch.empty((2 * inter, H)), wo=torch.empty((H, hq * 128)),
                                 wd=torch.empty((H, inter)))


def run_layer(rt, M, tp=1, capturing=False, monkeypatch=None):
    lw = layer(tp)
    part = torch.empty(max(8 << 20, 16 * 256 * H))
    x = torch.empty((M, H))
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: capturing)
    rt._qkv(0, lw, x, None, None, None, part)
    rt._gate_up(lw, x, None, part)
    rt._row_parallel(torch.empty((M, I // tp)), lw.wd, None, None, None, x, part)
    return lw


@pytest.fixture
def rec(monkeypatch):
    r = Recorder()
    monkeypatch.setattr(R, "K", r)
    return r


@pytest.mark.parametrize("M", [1, 8, 32])
def test_small_batches_take_the_small_batch_gemms_with_epilogue_kernels(rec, monkeypatch, M):
    rt = fake_runtime()
    run_layer(rt, M, monkeypatch=monkeypatch)
    sk = realK.pick_skinny_splits
    qkv = sk(M, (HQ + 2 * HKV) * 128, H, target=realK.SKINNY_TARGET_CTAS, max_elems=max(8 << 20, 16 * 256 * H))
    gu = sk(M, 2 * I, H, target=realK.SKINNY_TARGET_CTAS, max_elems=max(8 << 20, 16 * 256 * H))
    dn = sk(M, H, I, target=realK.SKINNY_TARGET_CTAS_ROW, max_elems=max(8 << 20, 16 * 256 * H))
    assert rec.calls == [("gemm_skinny_splitk", qkv), ("splitk_qkv_norm_rope_store", qkv),
                         ("gemm_skinny_splitk", gu), ("splitk_silu_mul", gu),
                         ("gemm_skinny_splitk", dn), ("splitk_add_rmsnorm", dn)]


@pytest.mark.parametrize("M", [33, 256])
def test_larger_batches_take_split_k(rec, monkeypatch, M):
    rt = fake_runtime()
    run_layer(rt, M, monkeypatch=monkeypatch)
    names = [c[0] for c in rec.calls]
    assert "gemm_skinny_splitk" not in names
    assert names[-1] in ("splitk_add_rmsnorm", "add_rmsnorm")
    assert names[0] in ("gemm_splitk", "qkv_norm_rope_store")


def test_fused_epilogues_are_opt_in(rec, monkeypatch):
    rt = fake_runtime(fused_rows=4)
    run_layer(rt, 2, monkeypatch=monkeypatch)
    names = [c[0] for c in rec.calls]
    assert names[:2] == ["skinny_qkv_norm_rope_store", "skinny_silu_mul"]
    rec.calls.clear()
    run_layer(rt, 5, monkeypatch=monkeypatch)  # above the opt-in bound: epilogue kernels again
    assert [c[0] for c in rec.calls][:2] == ["gemm_skinny_splitk", "splitk_qkv_norm_rope_store"]


def test_small_batch_partials_feed_the_tp_exchange_inside_graphs(rec, monkeypatch):
    rt = fake_runtime(tp=2, graph_exchange=True)
    run_layer(rt, 4, tp=2, capturing=True, monkeypatch=monkeypatch)
    sk = realK.pick_skinny_splits(4, H, I // 2, target=realK.SKINNY_TARGET_CTAS_ROW,
                                  max_elems=max(8 << 20, 16 * 256 * H))
    assert rec.calls[-1] == ("gemm_skinny_splitk", sk)  # no norm kernel: the exchange applies it
    assert rt.exchanged == [sk] and 1 <= sk <= 64
    # eager (not capturing): partials reduced, NCCL all-reduce, then the norm
    rec.calls.clear()
    rt.exchanged.clear()
    run_layer(rt, 4, tp=2, capturing=False, monkeypatch=monkeypatch)
    assert [c[0] for c in rec.calls][-3:] == ["gemm_skinny_splitk", "splitk_reduce", "add_rmsnorm"]
    assert rt.exchanged == ["nccl"]


def test_cluster_path_overrides_small_batch(rec, monkeypatch):
    rt = fake_runtime(cluster=True)
    run_layer(rt, 4, monkeypatch=monkeypatch)
    assert [c[0] for c in rec.calls][:2] == ["qkv_norm_rope_store_cluster", "gemm_silu_mul_cluster"]


def test_shape_guard():
    ok = R.Qwen3Runtime.skinny_shapes_ok
    assert ok(1024, 16, 8, 3072) and ok(4096, 4, 1, 1536) and ok(5120, 8, 1, 3200)  # 0.6B, 8B TP8, 32B TP8
    assert not ok(1000, 16, 8, 3072) and not ok(1024, 16, 8, 3000)
