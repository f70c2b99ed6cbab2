"""The allocation-free decode-attention entry point.

aacc_paged_decode_attention_noalloc serves callers that cannot allocate
device memory (e.g. plugins under a host runtime that owns every device
allocation, or services with a fixed device footprint after start-up): it
keeps its scratch in a static array inside the library instead of taking a
caller workspace.  This file is collected last so that a failure here leaves
every other test already run; it passes alone in a fresh process too.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _case(seed, dev):
    g = torch.Generator().manual_seed(seed)
    B, G, hkv, bs = 16, 2, 4, 256
    hq = G * hkv
    ctx = [1, 63, 64, 65, 255, 256, 257, 700, 1000, 1500, 2049, 333, 5, 128, 1999, 2048]
    need = [(c + bs - 1) // bs for c in ctx]
    nb = sum(need) + 3
    mb = max(need)
    perm = torch.randperm(nb, generator=g).tolist()
    bt = torch.full((B, mb), -1, dtype=torch.int32)
    it = 0
    for i, n in enumerate(need):
        bt[i, :n] = torch.tensor(perm[it:it + n], dtype=torch.int32)
        it += n
    kc = torch.randn((nb, hkv, bs, 128), generator=g).to(BF).to(dev)
    vc = torch.randn((nb, hkv, bs, 128), generator=g).to(BF).to(dev)
    q = (torch.randn((B, hq, 128), generator=g) / math.sqrt(128)).to(BF).to(dev)
    seqlens = (torch.tensor(ctx, dtype=torch.int32) - 1).to(dev)
    rows = torch.arange(B, dtype=torch.int64, device=dev)
    return dict(q=q, kc=kc, vc=vc, bt=bt.to(dev), rows=rows, seqlens=seqlens, B=B, hq=hq, hkv=hkv, bs=bs, nb=nb,
                max_ctx=mb * bs)


def _with_workspace(lib, c, out, stream):
    ws_bytes = lib.aacc_paged_decode_workspace_bytes(c["B"], c["hq"], c["max_ctx"], 0)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=out.device)
    rc = lib.aacc_paged_decode_attention(
        c["q"].data_ptr(), out.data_ptr(), c["kc"].data_ptr(), c["vc"].data_ptr(), c["nb"], c["bt"].data_ptr(),
        c["bt"].shape[1], c["rows"].data_ptr(), c["seqlens"].data_ptr(), 1, c["B"], c["hq"], c["hkv"], c["bs"],
        128 ** -0.5, 0, c["max_ctx"], ws.data_ptr(), ws_bytes, stream)
    assert rc == 0, lib.aacc_last_error()


def _noalloc(lib, c, out, stream):
    return lib.aacc_paged_decode_attention_noalloc(
        c["q"].data_ptr(), out.data_ptr(), c["kc"].data_ptr(), c["vc"].data_ptr(), c["nb"], c["bt"].data_ptr(),
        c["bt"].shape[1], c["rows"].data_ptr(), c["seqlens"].data_ptr(), 1, c["B"], c["hq"], c["hkv"], c["bs"],
        128 ** -0.5, 0, c["max_ctx"], stream)


def test_noalloc_decode_attention_matches_workspace_entry_point(cuda):
    from awesome_acceleration_b200 import _lib
    lib = _lib.load()  # the C ABI through ctypes
    assert lib.aacc_paged_decode_noalloc_capacity_bytes() == 16 << 20
    stream = torch.cuda.current_stream().cuda_stream
    _lib.clear_device_error()
    for seed in (0, 1):  # two calls in a row: the second reuses the scratch the first left behind
        c = _case(seed, cuda)
        ref = torch.empty_like(c["q"])
        _with_workspace(lib, c, ref, stream)
        out = torch.full_like(c["q"], float("nan"))
        rc = _noalloc(lib, c, out, stream)
        assert rc == 0, lib.aacc_last_error()
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        # Same kernel and split plan: the outputs agree within the attention tests' tolerance (in fact exactly).
        assert (out.float() - ref.float()).abs().max().item() <= 2e-2
        assert torch.equal(out, ref)


def test_noalloc_rejects_plans_beyond_the_static_scratch(cuda):
    from awesome_acceleration_b200 import _lib
    lib = _lib.load()
    c = _case(2, cuda)
    out = torch.empty_like(c["q"])
    # 4096 rows x 64 q heads x 8 splits of 512 tokens need far more than 16 MiB:
    # rejected on the host before anything is launched.
    rc = lib.aacc_paged_decode_attention_noalloc(
        c["q"].data_ptr(), out.data_ptr(), c["kc"].data_ptr(), c["vc"].data_ptr(), c["nb"], c["bt"].data_ptr(),
        c["bt"].shape[1], c["rows"].data_ptr(), c["seqlens"].data_ptr(), 1, 4096, 64, 8, c["bs"], 128 ** -0.5, 512,
        4096, torch.cuda.current_stream().cuda_stream)
    assert rc == 1  # AACC_ERR_INVALID
    assert b"static scratch" in lib.aacc_last_error()
