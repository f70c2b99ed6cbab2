"""Per-kernel parity of the sm_100a kernels against the CPU oracle, called
through the C ABI (awesome_acceleration_b200.kernels -> libaacc_b200.so)."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle.attention import attend
from oracle.qwen3_oracle import apply_rope, rms_norm, rope_cos_sin

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def K():
    from awesome_acceleration_b200 import kernels
    return kernels


def dev_err():
    from awesome_acceleration_b200 import _lib
    return _lib.device_error()


def clear_err():
    from awesome_acceleration_b200 import _lib
    _lib.clear_device_error()


def rand_pool(nb, hkv, bs, gen, dev):
    k = torch.randn((nb, hkv, bs, 128), generator=gen).to(BF).to(dev)
    v = torch.randn((nb, hkv, bs, 128), generator=gen).to(BF).to(dev)
    return k, v


def block_tables_for(ctx, bs, nb, gen, max_blocks=None):
    need = [(c + bs - 1) // bs for c in ctx]
    mb = max_blocks or max(need)
    perm = torch.randperm(nb, generator=gen).tolist()
    assert sum(need) <= nb
    bt = torch.full((len(ctx), mb), -1, dtype=torch.int32)
    it = 0
    for i, n in enumerate(need):
        bt[i, :n] = torch.tensor(perm[it:it + n], dtype=torch.int32)
        it += n
    return bt


def gather_kv(pool, bt_row, length, bs):
    pos = torch.arange(length)
    blk = bt_row.long()[pos // bs]
    return pool[blk, :, pos % bs]  # [length, Hkv, 128]


# --------------------------------------------------------------------------- KV store
def test_kv_store_bit_exact(cuda):
    g = torch.Generator().manual_seed(0)
    nb, hkv, bs, T = 12, 4, 64, 300
    kc = torch.full((nb, hkv, bs, 128), 7.0, dtype=BF, device=cuda)
    vc = torch.full((nb, hkv, bs, 128), -3.0, dtype=BF, device=cuda)
    k = torch.randn((T, hkv * 128 + 64), generator=g).to(BF)  # row stride > row width
    v = torch.randn((T, hkv * 128), generator=g).to(BF)
    slots = torch.randperm(nb * bs, generator=g)[:T]
    slots[::17] = -1  # skipped rows
    clear_err()
    K().kv_store(k.to(cuda)[:, :hkv * 128], v.to(cuda), slots.to(cuda), kc, vc)
    torch.cuda.synchronize()
    assert dev_err() == 0
    kc_h, vc_h = kc.cpu(), vc.cpu()
    written = torch.zeros(nb * bs, dtype=torch.bool)
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        written[s] = True
        assert torch.equal(kc_h[s // bs, :, s % bs], k[t, :hkv * 128].view(hkv, 128))
        assert torch.equal(vc_h[s // bs, :, s % bs], v[t].view(hkv, 128))
    untouched = (~written).nonzero().flatten()
    assert (kc_h.permute(0, 2, 1, 3).reshape(nb * bs, -1)[untouched] == 7.0).all()
    assert (vc_h.permute(0, 2, 1, 3).reshape(nb * bs, -1)[untouched] == -3.0).all()


def test_kv_store_rejects_out_of_pool_slot(cuda):
    nb, hkv, bs = 2, 1, 64
    kc = torch.zeros((nb, hkv, bs, 128), dtype=BF, device=cuda)
    vc = torch.zeros_like(kc)
    k = torch.ones((2, 128), dtype=BF, device=cuda)
    slots = torch.tensor([5, nb * bs + 3], dtype=torch.int64, device=cuda)
    clear_err()
    K().kv_store(k, k, slots, kc, vc)
    torch.cuda.synchronize()
    assert dev_err() & 2  # ERR_SLOT_OOB, access skipped
    assert kc.float().sum().item() == 128.0
    clear_err()


def test_decode_slot_mapping_and_advance(cuda):
    bs, nb = 64, 16
    g = torch.Generator().manual_seed(1)
    ctx = [1, 63, 64, 65, 200]
    bt = block_tables_for([c + 1 for c in ctx], bs, nb, g, max_blocks=6)
    rows = torch.tensor([4, 0, 2, 1, 3], dtype=torch.int64)
    seqlens = torch.zeros(5, dtype=torch.int32)
    for b, r in enumerate(rows.tolist()):
        seqlens[r] = ctx[b]
    bt_rows = torch.full((5, 6), -1, dtype=torch.int32)
    for b, r in enumerate(rows.tolist()):
        bt_rows[r] = bt[b]
    out = torch.empty(5, dtype=torch.int64, device=cuda)
    sl = seqlens.to(cuda)
    pos = torch.arange(5, dtype=torch.int64, device=cuda)
    K().decode_slot_mapping(rows.to(cuda), sl, bt_rows.to(cuda), bs, nb, out)
    K().advance_seqlens(rows.to(cuda), sl, pos)
    torch.cuda.synchronize()
    for b, r in enumerate(rows.tolist()):
        n = ctx[b]
        assert int(out[b]) == int(bt_rows[r, n // bs]) * bs + n % bs
        assert int(sl[r]) == n + 1
    assert pos.tolist() == [1, 2, 3, 4, 5]


# --------------------------------------------------------------------------- decode attention
@pytest.mark.parametrize("G,hkv", [(1, 2), (2, 8), (4, 2), (8, 1)])
def test_paged_decode_attention(cuda, G, hkv):
    g = torch.Generator().manual_seed(10 + G)
    bs = 256
    ctx = [1, 2, 63, 64, 65, 255, 256, 257, 511, 1000, 2049, 4096]
    B = len(ctx)
    hq = G * hkv
    need = sum((c + bs - 1) // bs for c in ctx)
    nb = need + 7
    kp, vp = rand_pool(nb, hkv, bs, g, "cpu")
    bt = block_tables_for(ctx, bs, nb, g)
    rows = torch.randperm(B, generator=g)  # rows are a permutation of the batch
    bt_rows = torch.full_like(bt, -1)
    seqlens = torch.zeros(B, dtype=torch.int32)
    for b in range(B):
        bt_rows[rows[b]] = bt[b]
        seqlens[rows[b]] = ctx[b] - 1  # ctx_add = 1: attend over seqlens + 1
    q = (torch.randn((B, hq, 128), generator=g) / math.sqrt(128)).to(BF)
    scale = 128 ** -0.5
    max_ctx = bt.shape[1] * bs
    ws = torch.zeros(K().decode_workspace_bytes(B, hq, max_ctx, 64), dtype=torch.uint8, device=cuda)
    clear_err()
    for split in (0, 64, 512):
        out = K().paged_decode_attention(q.to(cuda), kp.to(cuda), vp.to(cuda), bt_rows.to(cuda),
                                         rows.to(cuda), seqlens.to(cuda), ctx_add=1, scale=scale,
                                         max_context=max_ctx, workspace=ws, split_tokens=split)
        torch.cuda.synchronize()
        assert dev_err() == 0
        out = out.cpu().float()
        for b in range(B):
            kk = gather_kv(kp, bt[b], ctx[b], bs)
            vv = gather_kv(vp, bt[b], ctx[b], bs)
            ref = attend(q[b:b + 1], kk, vv, scale, False)[0].float()
            err = (out[b] - ref).abs().max().item()
            assert err <= 2e-2, f"split {split} row {b} ctx {ctx[b]}: max-abs {err}"


# --------------------------------------------------------------------------- prefill attention
@pytest.mark.parametrize("G,hkv", [(2, 2), (4, 2), (1, 3), (8, 1)])
def test_prefill_attention_chunked(cuda, G, hkv):
    g = torch.Generator().manual_seed(20 + G)
    bs = 256
    # (context already cached, query chunk length)
    pieces = [(0, 1), (0, 5), (0, 64), (0, 130), (100, 30), (256, 257), (500, 64), (0, 700)]
    S = len(pieces)
    hq = G * hkv
    tot = [c + n for c, n in pieces]
    nb = sum((t + bs - 1) // bs for t in tot) + 3
    kp, vp = rand_pool(nb, hkv, bs, g, "cpu")
    bt = block_tables_for(tot, bs, nb, g)
    T = sum(n for _, n in pieces)
    q = (torch.randn((T, hq, 128), generator=g)).to(BF)
    cu = torch.tensor([0] + np.cumsum([n for _, n in pieces]).tolist(), dtype=torch.int32)
    ctx0 = torch.tensor([c for c, _ in pieces], dtype=torch.int32)
    rows = torch.arange(S, dtype=torch.int64)
    scale = 128 ** -0.5
    clear_err()
    out = K().prefill_attention(q.to(cuda), kp.to(cuda), vp.to(cuda), bt.to(cuda), rows.to(cuda), cu.to(cuda),
                                ctx0.to(cuda), max_q_len=max(n for _, n in pieces), scale=scale)
    torch.cuda.synchronize()
    assert dev_err() == 0
    out = out.cpu().float()
    for s, (c, n) in enumerate(pieces):
        kk = gather_kv(kp, bt[s], c + n, bs)
        vv = gather_kv(vp, bt[s], c + n, bs)
        ref = attend(q[cu[s]:cu[s + 1]], kk, vv, scale, True).float()
        err = (out[cu[s]:cu[s + 1]] - ref).abs().max().item()
        assert err <= 2e-2, f"piece {s} ({c},{n}): max-abs {err}"


# --------------------------------------------------------------------------- norms
@pytest.mark.parametrize("H", [1024, 4096, 5120])
def test_rmsnorm_family(cuda, H):
    g = torch.Generator().manual_seed(H)
    T, eps = 37, 1e-6
    x = (torch.randn((T, H), generator=g) * 3).to(BF)
    d = torch.randn((T, H), generator=g).to(BF)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(BF)
    y = K().rmsnorm(x.to(cuda), w.to(cuda), eps).cpu()
    ref = rms_norm(x, w, eps)
    assert (y.float() - ref.float()).abs().max().item() <= 2 ** -6 * 4  # <= 1 bf16 ulp at |y| < 4
    assert (y == ref).float().mean().item() > 0.999
    res = x.to(cuda).clone()
    y2 = K().add_rmsnorm(d.to(cuda), res, w.to(cuda), eps).cpu()
    r_ref = x + d
    assert torch.equal(res.cpu(), r_ref)
    ref2 = rms_norm(r_ref, w, eps)
    assert (y2 == ref2).float().mean().item() > 0.999
    V = 1000
    table = torch.randn((V, H), generator=g).to(BF)
    ids = torch.randint(0, V, (T,), generator=g)
    res3 = torch.empty((T, H), dtype=BF, device=cuda)
    y3 = torch.empty((T, H), dtype=BF, device=cuda)
    K().embed_rmsnorm(ids.to(cuda), table.to(cuda), w.to(cuda), eps, res3, y3)
    assert torch.equal(res3.cpu(), table[ids])
    assert (y3.cpu() == rms_norm(table[ids], w, eps)).float().mean().item() > 0.999


# --------------------------------------------------------------------------- GEMMs
def bf16_linear_ref(x, w):
    return (x.float() @ w.float().t())


@pytest.mark.parametrize("M", [1, 5, 128, 129, 256, 300, 1111])
@pytest.mark.parametrize("N,Kd", [(1024, 2048), (384, 1024), (4096, 64)])
def test_gemm(cuda, M, N, Kd):
    g = torch.Generator().manual_seed(M * 7 + N)
    x = torch.randn((M, Kd), generator=g).to(BF)
    w = (torch.randn((N, Kd), generator=g) * 0.02).to(BF)
    out = K().gemm(x.to(cuda), w.to(cuda)).cpu().float()
    ref = bf16_linear_ref(x, w)
    err = (out - ref).abs().max().item()
    tol = 1e-2 * ref.abs().max().item() + 1e-3
    assert err <= tol, f"max-abs {err} > {tol}"


@pytest.mark.parametrize("M,N,Kd", [(1, 1024, 2048), (32, 1024, 3072), (200, 1024, 2048), (256, 512, 512)])
def test_splitk_gemm_add_rmsnorm(cuda, M, N, Kd):
    """Split-K partials summed by splitk_reduce / splitk_add_rmsnorm equal the
    unsplit GEMM followed by add_rmsnorm (up to fp32 summation order)."""
    g = torch.Generator().manual_seed(M + N + Kd)
    x = torch.randn((M, Kd), generator=g).to(BF).to(cuda)
    w = (torch.randn((N, Kd), generator=g) * 0.02).to(BF).to(cuda)
    res0 = torch.randn((M, N), generator=g).to(BF).to(cuda)
    nw = (1 + 0.1 * torch.randn(N, generator=g)).to(BF).to(cuda)
    splits = max(2, K().pick_splits(M, N, Kd))  # exercise split-K even where the heuristic picks 1
    part = torch.empty((splits, M, N), dtype=torch.float32, device=cuda)
    K().gemm_splitk(x, w, part, splits)
    ref_f32 = x.float() @ w.float().t()
    assert (part.sum(0) - ref_f32).abs().max().item() <= 1e-3 * ref_f32.abs().max().item() + 1e-4
    delta = torch.empty((M, N), dtype=BF, device=cuda)
    K().splitk_reduce(part, splits, delta)
    acc = part[0].clone()
    for s in range(1, splits):  # the kernels sum the partials in split order
        acc += part[s]
    assert torch.equal(delta, acc.to(BF))
    res = res0.clone()
    y = torch.empty_like(res)
    K().splitk_add_rmsnorm(part, splits, res, nw, 1e-6, out=y)
    res_ref = res0.clone()
    y_ref = K().add_rmsnorm(delta, res_ref, nw, 1e-6)
    assert torch.equal(res, res_ref) and torch.equal(y, y_ref)


@pytest.mark.parametrize("M", [1, 32, 256])
def test_splitk_qkv_and_silu_epilogues(cuda, M):
    """Split-K QKV / SiLU epilogues agree with the fused single-pass GEMM
    epilogues (same rounding points; only the fp32 summation order differs)."""
    from awesome_acceleration_b200.runtime import interleave_gate_up, rope_table
    g = torch.Generator().manual_seed(100 + M)
    H, I, hq, hkv, bs, eps = 1024, 3072, 16, 8, 256, 1e-6
    x = torch.randn((M, H), generator=g).to(BF).to(cuda)
    wqkv = (torch.randn(((hq + 2 * hkv) * 128, H), generator=g) * 0.05).to(BF).to(cuda)
    qn = (1 + 0.1 * torch.randn(128, generator=g)).to(BF).to(cuda)
    kn = (1 + 0.1 * torch.randn(128, generator=g)).to(BF).to(cuda)
    pos = torch.randint(0, 3000, (M,), generator=g).to(cuda)
    nb = 2
    slots = torch.randperm(nb * bs, generator=g)[:M].to(cuda)
    table = rope_table(4096, 128, 1e6, cuda)
    caches = [torch.zeros((nb, hkv, bs, 128), dtype=BF, device=cuda) for _ in range(4)]
    q1 = K().qkv_norm_rope_store(x, wqkv, qn, kn, eps, pos, table, slots, caches[0], caches[1], hq)
    N = wqkv.shape[0]
    splits = max(2, K().pick_splits(M, N, H))
    part = torch.empty((splits, M, N), dtype=torch.float32, device=cuda)
    K().gemm_splitk(x, wqkv, part, splits)
    q2 = torch.empty_like(q1)
    K().splitk_qkv_norm_rope_store(part, splits, qn, kn, eps, pos, table, slots, caches[2], caches[3], hq, q_out=q2)
    for a, b in ((q1, q2), (caches[0], caches[2]), (caches[1], caches[3])):
        assert (a.float() - b.float()).abs().max().item() <= 0.07
        assert (a == b).float().mean().item() > 0.97
    wgu = interleave_gate_up((torch.randn((I, H), generator=g) * 0.05).to(BF),
                             (torch.randn((I, H), generator=g) * 0.05).to(BF)).contiguous().to(cuda)
    a1 = K().gemm_silu_mul(x, wgu)
    s2 = K().pick_splits(M, 2 * I, H)
    part2 = torch.empty((s2, M, 2 * I), dtype=torch.float32, device=cuda)
    K().gemm_splitk(x, wgu, part2, s2)
    a2 = torch.empty_like(a1)
    K().splitk_silu_mul(part2, s2, a2)
    mag = torch.maximum(a1.float().abs(), a2.float().abs())
    # a 1-ulp difference in gate or up moves the product by at most 2 bf16 ulps
    assert ((a1.float() - a2.float()).abs() <= mag * 2 ** -6 + 1e-3).all()
    assert (a1 == a2).float().mean().item() > 0.97


@pytest.mark.parametrize("M", [3, 256, 700])
def test_gemm_silu_mul(cuda, M):
    from awesome_acceleration_b200.runtime import interleave_gate_up
    g = torch.Generator().manual_seed(M)
    H, I = 1024, 3072
    x = torch.randn((M, H), generator=g).to(BF)
    wg = (torch.randn((I, H), generator=g) * 0.05).to(BF)
    wu = (torch.randn((I, H), generator=g) * 0.05).to(BF)
    wgu = interleave_gate_up(wg, wu).contiguous()
    out = K().gemm_silu_mul(x.to(cuda), wgu.to(cuda)).cpu().float()
    ref = (F.silu(F.linear(x, wg)) * F.linear(x, wu)).float()  # reference rounding points (bf16 eager)
    err = (out - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-3, err


@pytest.mark.parametrize("M,hq,hkv", [(1, 16, 8), (40, 16, 8), (260, 8, 2), (1300, 4, 2)])
def test_qkv_norm_rope_store(cuda, M, hq, hkv):
    g = torch.Generator().manual_seed(M + hq)
    H, bs, eps = 1024, 256, 1e-6
    x = torch.randn((M, H), generator=g).to(BF)
    wqkv = (torch.randn(((hq + 2 * hkv) * 128, H), generator=g) * 0.05).to(BF)
    qn = (1 + 0.1 * torch.randn(128, generator=g)).to(BF)
    kn = (1 + 0.1 * torch.randn(128, generator=g)).to(BF)
    pos = torch.randint(0, 5000, (M,), generator=g)
    nb = (M + bs - 1) // bs + 2
    slots = torch.randperm(nb * bs, generator=g)[:M]
    from awesome_acceleration_b200.runtime import rope_table
    table = rope_table(8192, 128, 1e6, cuda)
    kc = torch.zeros((nb, hkv, bs, 128), dtype=BF, device=cuda)
    vc = torch.zeros_like(kc)
    clear_err()
    q = K().qkv_norm_rope_store(x.to(cuda), wqkv.to(cuda), qn.to(cuda), kn.to(cuda), eps, pos.to(cuda), table,
                                slots.to(cuda), kc, vc, hq)
    torch.cuda.synchronize()
    assert dev_err() == 0
    # Oracle chain: F.linear -> q/k RMSNorm -> RoPE (reference rounding points).
    qkv = F.linear(x, wqkv)
    qr = rms_norm(qkv[:, :hq * 128].view(M, hq, 128), qn, eps)
    kr = rms_norm(qkv[:, hq * 128:(hq + hkv) * 128].view(M, hkv, 128), kn, eps)
    vr = qkv[:, (hq + hkv) * 128:].view(M, hkv, 128)
    cos, sin = rope_cos_sin(pos, 128, 1e6, BF)
    qr, kr = apply_rope(qr, kr, cos.unsqueeze(1), sin.unsqueeze(1))
    assert (q.cpu().float() - qr.float()).abs().max().item() <= 0.1
    assert (q.cpu() == qr).float().mean().item() > 0.95
    kc_h, vc_h = kc.cpu(), vc.cpu()
    ks = kc_h[slots // bs, :, slots % bs]
    vs = vc_h[slots // bs, :, slots % bs]
    assert (ks.float() - kr.float()).abs().max().item() <= 0.1
    assert (ks == kr).float().mean().item() > 0.95
    # V is the bf16-rounded projection itself: equal up to one bf16 ulp.
    mag = torch.maximum(vs.float().abs(), vr.float().abs())
    assert ((vs.float() - vr.float()).abs() <= mag * 2 ** -7 + 1e-6).all()


@pytest.mark.parametrize("M,V", [(1, 151936), (7, 4096), (256, 151936), (300, 18992)])
def test_lm_head_argmax(cuda, M, V):
    g = torch.Generator().manual_seed(M + V)
    H = 1024
    x = torch.randn((M, H), generator=g).to(BF)
    w = (torch.randn((V, H), generator=g) * 0.02).to(BF)
    tokens = torch.empty(M, dtype=torch.int64, device=cuda)
    best = torch.empty(M, dtype=torch.float32, device=cuda)
    logits = torch.empty((M, V), dtype=BF, device=cuda)
    ws = torch.empty(K().lm_head_workspace_bytes(M, V), dtype=torch.uint8, device=cuda)
    K().lm_head_argmax(x.to(cuda), w.to(cuda), tokens, ws, logits=logits, best_val=best, vocab_offset=0)
    torch.cuda.synchronize()
    lg = logits.cpu()
    # Fused argmax agrees exactly with torch.argmax over the kernel's own bf16 logits.
    assert torch.equal(tokens.cpu(), lg.argmax(-1))
    assert torch.equal(best.cpu(), lg.float().max(-1).values)
    # And the logits agree with a CPU bf16 linear within bf16 tolerance.
    ref = F.linear(x, w).float()
    assert (lg.float() - ref).abs().max().item() <= 2e-2
    t2 = K().argmax_rows(logits)
    assert torch.equal(t2.cpu(), tokens.cpu())


@pytest.mark.parametrize("M,N,Kd", [(1, 1024, 1024), (77, 384, 256), (300, 3072, 1024)])
def test_gemm_bias_and_bias_add(cuda, M, N, Kd):
    """Fused-bias GEMM (fp32 add before the rounding, F.linear(x, w, b)) and the
    RowParallel post-all-reduce bias add (bf16(out + b))."""
    g = torch.Generator().manual_seed(M + N)
    x = torch.randn((M, Kd), generator=g).to(BF)
    w = (torch.randn((N, Kd), generator=g) * 0.05).to(BF)
    b = torch.randn(N, generator=g).to(BF)
    out = K().gemm(x.to(cuda), w.to(cuda), bias=b.to(cuda))
    ref = (x.float() @ w.float().t() + b.float())
    err = (out.cpu().float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, err
    y = torch.randn((M, N), generator=g).to(BF)
    yd = y.to(cuda)
    K().bias_add(yd, b.to(cuda))
    assert torch.equal(yd.cpu(), (y.float() + b.float()).to(BF))


def test_argmax_merge_ties_lowest_index(cuda):
    val = torch.tensor([[1.0, 5.0], [3.0, 5.0], [3.0, 2.0]], device=cuda)      # [shards=3, M=2]
    idx = torch.tensor([[10, 7], [20, 3], [5, 1]], dtype=torch.int64, device=cuda)
    out = K().argmax_merge(val, idx)
    assert out.tolist() == [5, 3]
    # the TP path's packed layout: one int64 buffer per shard, ids | fp32 values
    S, M = val.shape
    packed = torch.zeros((S, 2 * M), dtype=torch.int64, device=cuda)
    packed[:, :M] = idx
    packed.view(torch.float32)[:, 2 * M:3 * M] = val
    assert K().argmax_merge_packed(packed, M, torch.empty(M, dtype=torch.int64, device=cuda)).tolist() == [5, 3]


@pytest.mark.parametrize("M,V", [(300, 1000), (64, 151936)])
def test_lm_head_temperature_sampling(cuda, M, V):
    """Gumbel-max temperature sampling fused into the lm_head: row by row the
    oracle's draw over the kernel's own bf16 logits, greedy at T = 0, the same
    as sample_rows over materialised logits, and split over vocab shards the
    (score, id) merge gives the same tokens."""
    from oracle.sampling import sample
    g = torch.Generator().manual_seed(V)
    H = 1024
    x = torch.randn((M, H), generator=g).to(BF).to(cuda)
    w = (torch.randn((V, H), generator=g) * 0.05).to(BF).to(cuda)
    temp = torch.tensor([0.0 if i % 5 == 0 else 0.3 + (i % 7) * 0.25 for i in range(M)], device=cuda)
    seeds = torch.arange(M, dtype=torch.int64, device=cuda) * 7919 + 11
    ctr = torch.arange(M, dtype=torch.int64, device=cuda) % 13
    ws = torch.empty(K().lm_head_workspace_bytes(M, V), dtype=torch.uint8, device=cuda)
    tok = torch.empty(M, dtype=torch.int64, device=cuda)
    best = torch.empty(M, dtype=torch.float32, device=cuda)
    logits = torch.empty((M, V), dtype=BF, device=cuda)
    K().lm_head_argmax(x, w, tok, ws, logits=logits, best_val=best, temperature=temp, seeds=seeds, counters=ctr)
    torch.cuda.synchronize()
    lg = logits.float().cpu().numpy()
    ref = sample(lg, temp.cpu().numpy(), seeds.cpu().numpy(), ctr.cpu().numpy())
    same = (tok.cpu().numpy() == ref).mean()
    assert same >= 0.995, same  # device and numpy logf may differ in the last bit at near-ties
    greedy = temp.cpu() == 0
    assert torch.equal(tok.cpu()[greedy], logits.cpu()[greedy].argmax(-1))
    # the materialised-logits kernel draws the same noise
    t2 = K().sample_rows(logits, temp.cpu().tolist(), seeds.cpu().tolist(), ctr.cpu().tolist())
    assert torch.equal(t2.cpu(), tok.cpu())
    # vocab-parallel: two shards + merge == one pass over the whole vocabulary
    half = (V // 2 + 127) // 128 * 128
    cv = torch.empty((2, M), dtype=torch.float32, device=cuda)
    ci = torch.empty((2, M), dtype=torch.int64, device=cuda)
    for s, (a, b) in enumerate(((0, half), (half, V))):
        wsb = torch.empty(K().lm_head_workspace_bytes(M, b - a), dtype=torch.uint8, device=cuda)
        K().lm_head_argmax(x, w[a:b].contiguous(), ci[s], wsb, best_val=cv[s], vocab_offset=a, temperature=temp,
                           seeds=seeds, counters=ctr)
    merged = K().argmax_merge(cv, ci)
    assert torch.equal(merged.cpu(), tok.cpu())
    # same inputs, same draw
    tok2 = torch.empty_like(tok)
    K().lm_head_argmax(x, w, tok2, ws, temperature=temp, seeds=seeds, counters=ctr)
    assert torch.equal(tok2.cpu(), tok.cpu())


def test_temperature_sampling_distribution(cuda):
    """4096 draws of one row against softmax(bf16(logits / T))."""
    from oracle.sampling import reference_probs
    V, H, M, T = 256, 256, 4096, 0.8
    g = torch.Generator().manual_seed(5)
    w = (torch.randn((V, H), generator=g) * 0.15).to(BF).to(cuda)
    x = torch.randn((1, H), generator=g).to(BF).to(cuda).expand(M, H).contiguous()
    ws = torch.empty(K().lm_head_workspace_bytes(M, V), dtype=torch.uint8, device=cuda)
    tok = torch.empty(M, dtype=torch.int64, device=cuda)
    logits = torch.empty((M, V), dtype=BF, device=cuda)
    K().lm_head_argmax(x, w, tok, ws, logits=logits, temperature=torch.full((M,), T, device=cuda),
                       seeds=torch.arange(M, dtype=torch.int64, device=cuda),
                       counters=torch.zeros(M, dtype=torch.int64, device=cuda))
    torch.cuda.synchronize()
    p = reference_probs(logits[0].float().cpu().numpy(), T)
    emp = np.bincount(tok.cpu().numpy(), minlength=V) / M
    tv = 0.5 * np.abs(emp - p).sum()
    assert tv < 0.08, tv  # TV of 4096 draws from the right distribution stays well below this


def test_tp_exchange_wait_runs_out_and_poisons(cuda):
    """A peer that never arrives, on one GPU and without a fault: the 'peer'
    of a two-rank exchange is a second local buffer nothing writes into.  The
    bounded wait runs out, sets the device error word and poisons this rank's
    buffer; the next call then skips its waits and returns at once."""
    import time
    H, M, max_rows = 1024, 4, 8
    nbytes = K().tp_exchange_bytes(2, max_rows, H)
    own = torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
    ghost = torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
    src = torch.randn(M, H, device=cuda).to(BF)
    res = torch.randn(M, H, device=cuda).to(BF)
    w = torch.ones(H, dtype=BF, device=cuda)
    y = torch.empty_like(res)
    bufs = [own.data_ptr(), ghost.data_ptr()]
    clear_err()
    K().tp_set_peer_wait_ms(200)
    try:
        torch.cuda.synchronize()
        t0 = time.time()
        K().tp_allreduce_add_rmsnorm(src, 0, bufs, 0, max_rows, res, w, 1e-6, y, two_shot=True)
        torch.cuda.synchronize()
        t1 = time.time()
        assert dev_err() & 64
        assert own[8192:8196].view(torch.int32).item() == 1  # poisoned
        clear_err()
        K().tp_allreduce_add_rmsnorm(src, 0, bufs, 0, max_rows, res, w, 1e-6, y, two_shot=True)
        torch.cuda.synchronize()
        t2 = time.time()
        assert 0.15 <= t1 - t0 < 10, t1 - t0
        assert t2 - t1 < 0.15, t2 - t1  # a poisoned buffer does not wait
        assert dev_err() == 0
    finally:
        K().tp_set_peer_wait_ms(20000)
        clear_err()


# --------------------------------------------------------------------------- cluster split-K decode projections
@pytest.mark.parametrize("M", [1, 37, 128, 129, 256])
def test_cluster_gemms_equal_splitk_path(cuda, M):
    """The cluster split-K kernels (partials summed in distributed shared memory,
    epilogue fused) equal gemm_splitk + the split-K epilogue kernels bit for
    bit at the same split count, for the QKV (norm + RoPE + KV store), SiLU
    and bf16-store epilogues; the automatic plan stays within bf16 tolerance
    of the unsplit GEMM."""
    from awesome_acceleration_b200.runtime import interleave_gate_up, rope_table
    g = torch.Generator().manual_seed(M)
    H, I, hq, hkv, bs = 1024, 3072, 16, 8, 256
    x = torch.randn((M, H), generator=g).to(BF).to(cuda)
    a = torch.randn((M, I), generator=g).to(BF).to(cuda)
    w = {n: (torch.randn(sh, generator=g) * 0.02).to(BF).to(cuda) for n, sh in
         [("qkv", ((hq + 2 * hkv) * 128, H)), ("o", (H, hq * 128)), ("d", (H, I)), ("g", (I, H)), ("u", (I, H))]}
    wgu = interleave_gate_up(w["g"], w["u"]).contiguous()
    qn = (1 + 0.1 * torch.randn(128, generator=g)).to(BF).to(cuda)
    kn = (1 + 0.1 * torch.randn(128, generator=g)).to(BF).to(cuda)
    rope = rope_table(4096, 128, 1e6, cuda)
    pos = torch.randint(0, 4096, (M,), generator=g).to(cuda)
    nb = (M + bs - 1) // bs + 2
    slots = torch.randperm(nb * bs, generator=g)[:M].to(cuda)
    part = torch.empty(16 * M * 6144, dtype=torch.float32, device=cuda)
    clear_err()
    for splits in (1, 2, 4, 8):
        # bf16 store (o / down)
        for wt, inp in ((w["o"], a[:, :hq * 128].contiguous()), (w["d"], a)):
            N, Kd = wt.shape
            pv = part[:splits * M * N].view(splits, M, N)
            K().gemm_splitk(inp, wt, pv, splits)
            ref = torch.empty((M, N), dtype=BF, device=cuda)
            K().splitk_reduce(pv, splits, ref)
            out = K().gemm_cluster(inp, wt, splits=splits)
            assert torch.equal(out, ref), f"store M={M} N={N} K={Kd} splits={splits}"
        # SiLU-mul
        pv = part[:splits * M * 2 * I].view(splits, M, 2 * I)
        K().gemm_splitk(x, wgu, pv, splits)
        ref = torch.empty((M, I), dtype=BF, device=cuda)
        K().splitk_silu_mul(pv, splits, ref)
        out = K().gemm_silu_mul_cluster(x, wgu, splits=splits)
        assert torch.equal(out, ref), f"silu M={M} splits={splits}"
        # QKV + q/k norm + RoPE + KV store
        N = w["qkv"].shape[0]
        pv = part[:splits * M * N].view(splits, M, N)
        caches = []
        for fused in (False, True):
            kc = torch.zeros((nb, hkv, bs, 128), dtype=BF, device=cuda)
            vc = torch.zeros_like(kc)
            q = torch.zeros((M, hq, 128), dtype=BF, device=cuda)
            if fused:
                K().qkv_norm_rope_store_cluster(x, w["qkv"], qn, kn, 1e-6, pos, rope, slots, kc, vc, hq, q_out=q,
                                                splits=splits)
            else:
                K().gemm_splitk(x, w["qkv"], pv, splits)
                K().splitk_qkv_norm_rope_store(pv, splits, qn, kn, 1e-6, pos, rope, slots, kc, vc, hq, q)
            caches.append((q, kc, vc))
        for t0, t1 in zip(*caches):
            assert torch.equal(t0, t1), f"qkv M={M} splits={splits}"
    torch.cuda.synchronize()
    assert dev_err() == 0
    # automatic plan against the unsplit tcgen05 GEMM
    plan = K().gemm_cluster_plan(M, H, I)
    out = K().gemm_cluster(a, w["d"])
    ref = K().gemm(a, w["d"])
    err = (out.float() - ref.float()).abs().max().item()
    assert err <= 1e-2 * ref.float().abs().max().item() + 1e-3, (plan, err)
    caps = {(mt, s): K().gemm_cluster_capacity(mt, s) for mt in (1, 2) for s in (1, 2, 3, 4, 6, 8, 16)}
    print(f"M={M}: plans qkv {K().gemm_cluster_plan(M, 4096, H)}, gate/up {K().gemm_cluster_plan(M, 2 * I, H)}, "
          f"o {K().gemm_cluster_plan(M, H, 2048)}, down {plan}; resident CTAs per (tile rows/128, splits) {caps}")


@pytest.mark.parametrize("M", [1, 5, 16, 17, 33, 64])
def test_skinny_gemms(cuda, M):
    """Small-batch GEMMs (weights as the MMA's 128-row operand): the split-K
    partials agree with the general split-K kernel's and sum to torch's fp32
    product; the fused QKV (norm + RoPE + KV store) and SiLU forms equal
    gemm_skinny_splitk + the split-K epilogue kernels bit for bit (same
    partials, same epilogue arithmetic), launch after launch; the arrival
    counters are zero after every launch."""
    from awesome_acceleration_b200.runtime import interleave_gate_up, rope_table
    g = torch.Generator().manual_seed(1000 + M)
    H, I, hq, hkv, bs = 1024, 3072, 16, 8, 256
    x = torch.randn((M, H), generator=g).to(BF).to(cuda)
    a = torch.randn((M, I), generator=g).to(BF).to(cuda)
    w = {n: (torch.randn(sh, generator=g) * 0.02).to(BF).to(cuda) for n, sh in
         [("qkv", ((hq + 2 * hkv) * 128, H)), ("d", (H, I)), ("g", (I, H)), ("u", (I, H))]}
    wgu = interleave_gate_up(w["g"], w["u"]).contiguous()
    qn = (1 + 0.1 * torch.randn(128, generator=g)).to(BF).to(cuda)
    kn = (1 + 0.1 * torch.randn(128, generator=g)).to(BF).to(cuda)
    rope = rope_table(4096, 128, 1e6, cuda)
    pos = torch.randint(0, 4096, (M,), generator=g).to(cuda)
    nb = (M + bs - 1) // bs + 2
    slots = torch.randperm(nb * bs, generator=g)[:M].to(cuda)
    part = torch.empty(48 * M * 6144, dtype=torch.float32, device=cuda)
    part2 = torch.empty_like(part)
    cnt = torch.zeros(1024, dtype=torch.int32, device=cuda)
    clear_err()
    exact = {}
    for wt, inp in ((w["d"], a), (w["qkv"], x), (wgu, x)):
        N, Kd = wt.shape
        ref = inp.float() @ wt.float().t()
        for splits in sorted({1, 2, 4, K().pick_skinny_splits(M, N, Kd)}):
            if (Kd // 64) % splits:
                continue
            pv = part[:splits * M * N].view(splits, M, N)
            K().gemm_skinny_splitk(inp, wt, pv, splits)
            pg = part2[:splits * M * N].view(splits, M, N)
            K().gemm_splitk(inp, wt, pg, splits)
            torch.cuda.synchronize()
            d = (pv - pg).abs().max().item()
            exact[(N, splits)] = d == 0
            assert d <= 1e-5 * pg.abs().max().item() + 1e-6, (N, splits, d)
            err = (pv.sum(0) - ref).abs().max().item()
            assert err <= 1e-3 * ref.abs().max().item() + 1e-4, (N, splits, err)
    # fused epilogues against the separate epilogue kernels on the same partials
    N = w["qkv"].shape[0]
    for splits in sorted({1, 4, K().pick_skinny_splits(M, N, H)}):
        pv = part[:splits * M * N].view(splits, M, N)
        outs = []
        for fused in (False, True, True):  # the second fused launch reuses the counters
            kc = torch.zeros((nb, hkv, bs, 128), dtype=BF, device=cuda)
            vc = torch.zeros_like(kc)
            q = torch.zeros((M, hq, 128), dtype=BF, device=cuda)
            if fused:
                K().skinny_qkv_norm_rope_store(x, w["qkv"], pv, splits, cnt, qn, kn, 1e-6, pos, rope, slots, kc, vc,
                                               hq, q_out=q)
            else:
                K().gemm_skinny_splitk(x, w["qkv"], pv, splits)
                K().splitk_qkv_norm_rope_store(pv, splits, qn, kn, 1e-6, pos, rope, slots, kc, vc, hq, q)
            outs.append((q, kc, vc))
        for o in outs[1:]:
            for t0, t1 in zip(outs[0], o):
                assert torch.equal(t0, t1), f"qkv M={M} splits={splits}"
        torch.cuda.synchronize()
        assert int(cnt.abs().sum().item()) == 0
    N = 2 * I
    for splits in sorted({1, 4, K().pick_skinny_splits(M, N, H)}):
        pv = part[:splits * M * N].view(splits, M, N)
        K().gemm_skinny_splitk(x, wgu, pv, splits)
        ref = torch.empty((M, I), dtype=BF, device=cuda)
        K().splitk_silu_mul(pv, splits, ref)
        for _ in range(2):
            out = torch.full((M, I), float("nan"), dtype=BF, device=cuda)
            K().skinny_silu_mul(x, wgu, pv, splits, cnt, out)
            assert torch.equal(out, ref), f"silu M={M} splits={splits}"
        torch.cuda.synchronize()
        assert int(cnt.abs().sum().item()) == 0
    assert dev_err() == 0
    print(f"M={M}: skinny partials bit-equal to the general split-K kernel's: {exact}")


def test_skinny_gemm_rejects_bad_shapes(cuda):
    """Shapes the small-batch kernels do not take are refused before launch."""
    x = torch.zeros((65, 1024), dtype=BF, device=cuda)
    w = torch.zeros((1024, 1024), dtype=BF, device=cuda)
    part = torch.zeros(65 * 1024 * 16, dtype=torch.float32, device=cuda)
    with pytest.raises(RuntimeError):
        K().gemm_skinny_splitk(x, w, part, 1)  # 65 rows
    with pytest.raises(RuntimeError):
        K().gemm_skinny_splitk(x[:4], w, part, 3)  # 3 does not divide 16 slabs
    with pytest.raises(RuntimeError):
        K().gemm_skinny_splitk(x[:4], w[:1000], part, 1)  # N not a multiple of 128


@pytest.mark.parametrize("M", [300, 450])
def test_gemm_splitk_rows_over_256(cuda, M):
    """Decode batches above 256 rows (the engine's batch holds every KV slot,
    ~450 for Qwen3-32B at TP4) take the 256-row tiles; their split-K partials
    sum to torch's fp32 product."""
    g = torch.Generator().manual_seed(M)
    for N, Kd in ((1024, 2048), (5120, 2048)):
        x = torch.randn((M, Kd), generator=g).to(BF).to(cuda)
        w = (torch.randn((N, Kd), generator=g) * 0.02).to(BF).to(cuda)
        ref = x.float() @ w.float().t()
        for splits in (1, 2, 4):
            part = torch.empty((splits, M, N), dtype=torch.float32, device=cuda)
            K().gemm_splitk(x, w, part, splits)
            err = (part.sum(0) - ref).abs().max().item()
            assert err <= 1e-3 * ref.abs().max().item() + 1e-4, (N, splits, err)
