"""Row-wise operators around the hot path (GPUOps.rms / addScale / normRope / geluMul /
geluPle / pleMix, the tied bf16 head and the greedy pick) against the oracle's
formulas, through the C ABI."""
import ctypes as C
import importlib
import math

import numpy as np
import pytest
import torch

from conftest import bf16_round, max_rel

pytestmark = pytest.mark.gpu

mo = importlib.import_module("oracle.model_oracle")
L = importlib.import_module("gemma4-js_b200._lib")


def P(t):
    return C.c_void_p(t.data_ptr())


def g(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


def test_rms_and_add_scale(ctx):
    x = torch.randn((5, 1536), device="cuda", generator=g(1)) * 3
    sc = torch.rand(1536, device="cuda", generator=g(2)) + 0.5
    out = torch.empty_like(x)
    L.call("g4_rms", ctx.handle, P(x), P(sc), 5, 1536, C.c_float(1e-6), P(out), 0)
    ref = mo.rms(x.cpu().numpy(), sc.cpu().numpy(), 1e-6)
    assert max_rel(out.cpu().numpy(), ref) < 1e-5
    outb = torch.empty((5, 1536), dtype=torch.bfloat16, device="cuda")
    L.call("g4_rms", ctx.handle, P(x), None, 5, 1536, C.c_float(1e-6), P(outb), 1)
    assert max_rel(outb.float().cpu().numpy(), mo.rms(x.cpu().numpy(), None, 1e-6)) < 5e-3
    y = torch.empty_like(x)
    L.call("g4_add_scale", ctx.handle, P(x), P(out), C.c_longlong(x.numel()), C.c_float(0.75), P(y))
    assert torch.allclose(y, (x + out) * 0.75)


def test_post_norm_add(ctx):
    h = torch.randn((3, 1536), device="cuda", generator=g(3))
    y = torch.randn((3, 1536), device="cuda", generator=g(4)) * 5
    wp = torch.rand(1536, device="cuda", generator=g(5)) + 0.5
    wn = torch.rand(1536, device="cuda", generator=g(6)) + 0.5
    x = torch.empty((3, 1536), dtype=torch.bfloat16, device="cuda")
    h0 = h.cpu().numpy()
    L.call("g4_post_norm_add", ctx.handle, P(h), P(y), 1536, P(wp), C.c_float(0.8), P(wn), 3, 1536, C.c_float(1e-6), P(x))
    hr = (h0 + mo.rms(y.cpu().numpy(), wp.cpu().numpy(), 1e-6)) * np.float32(0.8)
    assert max_rel(h.cpu().numpy(), hr) < 1e-5
    assert max_rel(x.float().cpu().numpy(), mo.rms(hr, wn.cpu().numpy(), 1e-6)) < 5e-3


@pytest.mark.parametrize("hd,angles,base", [(256, 128, 10000.0), (512, 64, 1000000.0), (64, 32, 10000.0)])
def test_qkv_post_norm_rope_and_append(ctx, hd, angles, base):
    H, rows, cap = 8, 3, 40
    y = torch.randn((rows, (H + 2) * hd), device="cuda", generator=g(hd))
    qn = torch.rand(hd, device="cuda", generator=g(7)) * 0.5 + 0.2
    kn = torch.rand(hd, device="cuda", generator=g(8)) * 0.5 + 0.2
    q = torch.empty((rows, H, hd), dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros((2 * cap, hd), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros((2 * cap, hd), dtype=torch.bfloat16, device="cuda")
    seq_pos = torch.tensor([0, 21], dtype=torch.int32, device="cuda")
    rmap = L.G4Rows(seq_pos.data_ptr(), 1, rows, 0)  # sequence 1, positions 21..23
    L.call("g4_qkv_post", ctx.handle, P(y), (H + 2) * hd, H, hd, 1, P(qn), P(kn), C.c_float(1e-6), angles,
           C.c_float(base), C.byref(rmap), rows, P(q), P(kc), P(vc), cap)
    yn = y.cpu().numpy()
    pos = np.arange(21, 24)
    qr = mo.norm_rope(yn[:, :H * hd].reshape(rows, H, hd), qn.cpu().numpy(), pos, angles, base, 1e-6)
    kr = mo.norm_rope(yn[:, H * hd:(H + 1) * hd], kn.cpu().numpy(), pos, angles, base, 1e-6)
    vr = mo.rms(yn[:, (H + 1) * hd:], None, 1e-6)
    assert max_rel(q.float().cpu().numpy(), qr) < 5e-3
    assert max_rel(kc[cap + 21:cap + 24].float().cpu().numpy(), kr) < 5e-3
    assert max_rel(vc[cap + 21:cap + 24].float().cpu().numpy(), vr) < 5e-3
    assert float(kc[:cap + 21].abs().sum()) == 0.0  # nothing written outside the three slots


def test_gelu_mul_and_gelu_ple(ctx):
    rows, inter = 4, 6144
    gu = torch.randn((rows, 2 * inter), device="cuda", generator=g(9)) * 4
    out = torch.empty((rows, inter), dtype=torch.bfloat16, device="cuda")
    L.call("g4_gelu_mul", ctx.handle, P(gu), rows, inter, P(out))
    gn = gu.cpu().numpy()
    assert max_rel(out.float().cpu().numpy(), mo.gelu(gn[:, :inter]) * gn[:, inter:]) < 5e-3
    pg = torch.randn((rows, 256), device="cuda", generator=g(10)) * 30  # exercises the +-10 clamp
    pl = torch.randn((rows, 35, 256), device="cuda", generator=g(11))
    o2 = torch.empty((rows, 256), dtype=torch.bfloat16, device="cuda")
    L.call("g4_gelu_ple", ctx.handle, P(pg), P(pl), 7, 35, 256, rows, P(o2))
    ref = mo.gelu(pg.cpu().numpy()) * pl.cpu().numpy()[:, 7, :]
    assert max_rel(o2.float().cpu().numpy(), ref) < 5e-3


def test_ple_mix(ctx):
    rows = 3
    proj = torch.randn((rows, 35 * 256), device="cuda", generator=g(12)) * 10
    norm = torch.rand(256, device="cuda", generator=g(13)) + 0.5
    tok = torch.randn((rows, 35 * 256), device="cuda", generator=g(14)) * 0.05
    out = torch.empty_like(proj)
    L.call("g4_ple_mix", ctx.handle, P(proj), C.c_float(1 / math.sqrt(1536)), P(norm), P(tok), rows, 35, 256,
           C.c_float(1e-6), P(out))
    p = proj.cpu().numpy().reshape(rows, 35, 256) * np.float32(1 / math.sqrt(1536))
    ref = (mo.rms(p, norm.cpu().numpy(), 1e-6) + tok.cpu().numpy().reshape(rows, 35, 256) * 16) * np.float32(0.7071067811865476)
    assert max_rel(out.cpu().numpy().reshape(rows, 35, 256), ref) < 1e-5


@pytest.mark.parametrize("M", [1, 3, 16, 40])
def test_dense_head_and_argmax(rt, ctx, M):
    model = importlib.import_module("gemma4-js_b200.model")
    V, K = 20000, 1536
    E = (torch.randn((V, K), device="cuda", generator=g(15)) * 0.05).to(torch.bfloat16)
    d = model.Dense(ctx, E)
    x = torch.randn((M, K), device="cuda", generator=g(M)).to(torch.bfloat16)
    logits = torch.empty((M, V), dtype=torch.float32, device="cuda")
    L.call("g4_dense_matmul", ctx.handle, d.handle, P(x), M, P(logits))
    ref = x.float() @ E.float().T
    assert max_rel(logits.cpu().numpy(), ref.cpu().numpy()) < 1e-4
    ids = torch.empty(M, dtype=torch.int32, device="cuda")
    vals = torch.empty(M, dtype=torch.float32, device="cuda")
    logits[0, 123] = 1e4          # a clear winner, capped to ~30
    logits[0, 7] = float("nan")  # skipped like the reference's non-finite check
    L.call("g4_softcap_argmax", ctx.handle, P(logits), M, V, C.c_float(30.0), P(ids), P(vals))
    capped = torch.tanh(logits / 30) * 30
    capped = torch.nan_to_num(capped, nan=-float("inf"))
    assert ids.tolist() == capped.argmax(dim=1).int().tolist()
    assert abs(float(vals[0]) - 30.0) < 1e-4
    ctx.check_device()


def test_argmax_ties_pick_lowest_index(ctx):
    logits = torch.zeros((2, 9000), device="cuda")
    logits[0, [17, 4100, 8999]] = 5.0
    logits[1, [8999, 300]] = 2.0
    ids = torch.empty(2, dtype=torch.int32, device="cuda")
    L.call("g4_softcap_argmax", ctx.handle, P(logits), 2, 9000, C.c_float(30.0), P(ids), None)
    assert ids.tolist() == [17, 300]


def test_embed(ctx):
    E = (torch.randn((1000, 1536), device="cuda", generator=g(16)) * 0.05).to(torch.bfloat16)
    ids = torch.tensor([5, 999, 0], dtype=torch.int32, device="cuda")
    h = torch.empty((3, 1536), device="cuda")
    x = torch.empty((3, 1536), dtype=torch.bfloat16, device="cuda")
    L.call("g4_embed", ctx.handle, P(E), 1000, 1536, P(ids), 3, C.c_float(math.sqrt(1536)), P(h), P(x))
    ref = E[ids.long()].float() * np.float32(math.sqrt(1536))
    assert torch.equal(h, ref)
    assert torch.equal(x, ref.to(torch.bfloat16))


@pytest.mark.parametrize("M,K,N", [(256, 6144, 1536), (256, 1536, 2560), (40, 1536, 256), (8, 1536, 1536)])
def test_planes_consumers_match_the_summed_linear(rt, ctx, M, K, N):
    """g4_linear_w4a16_planes + the *_planes operators give the same bits as the linear's
    f32 output fed to the plain operators (split K, one plane, and the GEMV)."""
    gen = g(M + K + N)
    packed = torch.randint(-2**31, 2**31 - 1, (N, K // 8), device="cuda", dtype=torch.int32, generator=gen)
    sc = torch.randn((N, K // 32), device="cuda", generator=gen).abs_().mul_(0.02).to(torch.bfloat16)
    lin = rt.W4Linear(ctx, packed, sc)
    x = torch.randn((M, K), device="cuda", generator=gen).to(torch.bfloat16)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    L.call("g4_linear_w4a16", ctx.handle, lin.handle, P(x), M, P(y), 0)
    # post_norm_add
    h0 = torch.randn((M, N), device="cuda", generator=gen)
    wp = torch.rand(N, device="cuda", generator=gen) + 0.5
    wn = torch.rand(N, device="cuda", generator=gen) + 0.5
    h1, h2 = h0.clone(), h0.clone()
    x1 = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    x2 = torch.empty_like(x1)
    L.call("g4_post_norm_add", ctx.handle, P(h1), P(y), N, P(wp), C.c_float(0.9), P(wn), M, N, C.c_float(1e-6), P(x1))
    pl = L.G4Planes()
    L.call("g4_linear_w4a16_planes", ctx.handle, lin.handle, P(x), M, C.byref(pl))
    L.call("g4_post_norm_add_planes", ctx.handle, P(h2), C.byref(pl), P(wp), C.c_float(0.9), P(wn), M, N,
           C.c_float(1e-6), P(x2))
    assert torch.equal(h1, h2) and torch.equal(x1, x2)
    # gelu_mul over [gate | up] halves
    inter = N // 2
    a1 = torch.empty((M, inter), dtype=torch.bfloat16, device="cuda")
    a2 = torch.empty_like(a1)
    L.call("g4_gelu_mul", ctx.handle, P(y), M, inter, P(a1))
    L.call("g4_linear_w4a16_planes", ctx.handle, lin.handle, P(x), M, C.byref(pl))
    L.call("g4_gelu_mul_planes", ctx.handle, C.byref(pl), M, inter, P(a2))
    assert torch.equal(a1, a2)
    # gelu_ple over the first 256 columns as the gate of layer 1 of 3
    dim = 256 if N >= 256 else N
    per = torch.randn((M, 3, dim), device="cuda", generator=gen)
    yg = y[:, :dim].contiguous()
    b1 = torch.empty((M, dim), dtype=torch.bfloat16, device="cuda")
    b2 = torch.empty_like(b1)
    L.call("g4_gelu_ple", ctx.handle, P(yg), P(per), 1, 3, dim, M, P(b1))
    L.call("g4_linear_w4a16_planes", ctx.handle, lin.handle, P(x), M, C.byref(pl))
    pl_g = L.G4Planes(pl.base, pl.count, pl.stride, pl.ld)  # the gate reads columns 0..dim-1 of each row
    L.call("g4_gelu_ple_planes", ctx.handle, C.byref(pl_g), P(per), 1, 3, dim, M, P(b2))
    assert torch.equal(b1, b2)
    ctx.check_device()


@pytest.mark.parametrize("hd", [256, 512])
def test_qkv_post_planes_match_the_summed_linear(rt, ctx, hd):
    """g4_qkv_post_planes over the split-K planes of the qkv linear gives the bits of
    g4_qkv_post over the linear's summed output (the planes are added in slice order)."""
    H, M, K, cap = 8, 40, 1536, 64
    N = (H + 2) * hd
    gen = torch.Generator(device="cuda").manual_seed(hd)
    packed = torch.randint(-2**31, 2**31 - 1, (N, K // 8), device="cuda", dtype=torch.int32, generator=gen)
    sc = torch.randn((N, K // 32), device="cuda", generator=gen).abs_().mul_(0.02).to(torch.bfloat16)
    lin = rt.W4Linear(ctx, packed, sc)
    x = torch.randn((M, K), device="cuda", generator=gen).to(torch.bfloat16)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    L.call("g4_linear_w4a16", ctx.handle, lin.handle, P(x), M, P(y), 0)
    qn = torch.rand(hd, device="cuda", generator=gen) + 0.5
    kn = torch.rand(hd, device="cuda", generator=gen) + 0.5
    seq_pos = torch.tensor([7], dtype=torch.int32, device="cuda")
    rmap = L.G4Rows(seq_pos.data_ptr(), 0, M, 0)
    outs = []
    for planes in (False, True):
        q = torch.empty((M, H, hd), dtype=torch.bfloat16, device="cuda")
        kc = torch.zeros((cap, hd), dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros((cap, hd), dtype=torch.bfloat16, device="cuda")
        args = (H, hd, 1, P(qn), P(kn), C.c_float(1e-6), hd // 4, C.c_float(1e6), C.byref(rmap), M, P(q), P(kc), P(vc), cap)
        if planes:
            pl = L.G4Planes()
            L.call("g4_linear_w4a16_planes", ctx.handle, lin.handle, P(x), M, C.byref(pl))
            assert pl.count > 1
            L.call("g4_qkv_post_planes", ctx.handle, C.byref(pl), *args)
        else:
            L.call("g4_qkv_post", ctx.handle, P(y), N, *args)
        outs.append((q, kc, vc))
    ctx.check_device()
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("M", [1, 17, 40, 300])
@pytest.mark.parametrize("cap", [30.0, 0.0, 0.05])  # 0.05: most logits saturate, ties everywhere
def test_dense_argmax_fused_matches_two_pass(rt, ctx, M, cap):
    """g4_dense_argmax (logits tiles + softcap + greedy pick in one kernel) against
    g4_dense_matmul + g4_softcap_argmax: the same bits above 16 rows (the same tensor-core
    accumulation order), the torch fp32 pick within rounding below."""
    model = importlib.import_module("gemma4-js_b200.model")
    V, K = 20000, 1536  # 79 vocabulary tiles, the last one partial
    E = (torch.randn((V, K), device="cuda", generator=g(21)) * 0.05).to(torch.bfloat16)
    d = model.Dense(ctx, E)
    x = torch.randn((M, K), device="cuda", generator=g(22 + M)).to(torch.bfloat16)
    ids2 = torch.empty(M, dtype=torch.int32, device="cuda")
    vals2 = torch.empty(M, dtype=torch.float32, device="cuda")
    L.call("g4_dense_argmax", ctx.handle, d.handle, P(x), M, C.c_float(cap), P(ids2), P(vals2))
    ctx.check_device()
    if M > 16:
        logits = torch.empty((M, V), dtype=torch.float32, device="cuda")
        L.call("g4_dense_matmul", ctx.handle, d.handle, P(x), M, P(logits))
        ids1 = torch.empty(M, dtype=torch.int32, device="cuda")
        vals1 = torch.empty(M, dtype=torch.float32, device="cuda")
        L.call("g4_softcap_argmax", ctx.handle, P(logits), M, V, C.c_float(cap), P(ids1), P(vals1))
        assert torch.equal(ids1, ids2) and torch.equal(vals1, vals2)
    else:
        ref = x.float() @ E.float().T
        capped = torch.tanh(ref / cap) * cap if cap > 0 else ref
        best = capped.max(dim=1).values
        picked = capped.gather(1, ids2.long().unsqueeze(1)).squeeze(1)
        assert torch.all(best - picked < 1e-3)
        assert torch.allclose(vals2, best, atol=1e-3)


@pytest.mark.parametrize("M,K,inter", [(256, 1536, 6144), (40, 512, 1024), (3, 512, 1024), (300, 256, 512),
                                      (1, 1536, 6144), (16, 1536, 6144), (8, 2048, 1024), (5, 256, 512),
                                      (2, 4096, 1024)])
def test_geglu_fused_linear_matches_linear_then_gelu_mul(rt, ctx, M, K, inter):
    """g4_linear_w4a16_geglu on the interleaved rows gives the same bits as the linear on
    [gate; up] (f32) followed by g4_gelu_mul: fused epilogue (unsplit tiles), planes +
    GeGLU pass (split K), and below 17 rows the GEMV computing each gate tile with its up
    tile in one CTA (K up to 2048; K = 4096 takes the GEMV + GeGLU pass)."""
    model = importlib.import_module("gemma4-js_b200.model")
    gen = g(M + K + inter)
    N = 2 * inter
    packed = torch.randint(-2**31, 2**31 - 1, (N, K // 8), device="cuda", dtype=torch.int32, generator=gen)
    sc = torch.randn((N, K // 32), device="cuda", generator=gen).abs_().mul_(0.02).to(torch.bfloat16)
    lin = rt.W4Linear(ctx, packed, sc)
    lin_i = rt.W4Linear(ctx, model.interleave_geglu(packed, inter), model.interleave_geglu(sc, inter))
    x = torch.randn((M, K), device="cuda", generator=gen).to(torch.bfloat16)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    L.call("g4_linear_w4a16", ctx.handle, lin.handle, P(x), M, P(y), 0)
    a1 = torch.empty((M, inter), dtype=torch.bfloat16, device="cuda")
    L.call("g4_gelu_mul", ctx.handle, P(y), M, inter, P(a1))
    a2 = torch.empty_like(a1)
    L.call("g4_linear_w4a16_geglu", ctx.handle, lin_i.handle, P(x), M, P(a2))
    ctx.check_device()
    assert torch.equal(a1, a2)


def test_fused_head_pick_matches_oracle_softcap_and_tie_rule(rt, ctx, oracle):
    """head_argmax_kernel against the reference's pick computed on the host: f32 softcap
    tanh(raw / 30) * 30, then the lowest index of the largest capped value
    (gemma4-webgpu.js:465-478, topK gpu-runtime.js:1396-1425).  The raw logits are exact
    (one-hot activations times bf16-exact table entries), so only the softcap and the tie
    rule are under test.  Planted cases per row: exact ties of the maximum at several
    indices; saturated logits (raw >= 600, where the capped value is exactly 30.0 for every
    raw) with the largest raw at a higher index than a smaller saturated one; and a
    near-cap maximum (raw 80.5 against 80.0) that must stay distinct.  The kernel computes
    the softcap only when a raw maximum improves, which equals this rule for a
    non-decreasing softcap."""
    model = importlib.import_module("gemma4-js_b200.model")
    M, V, K = 24, 20000, 1536  # M > 16: the fused tcgen05 head
    rng = np.random.default_rng(77)
    E = (np.round(rng.uniform(-40, 40, (V, K)) * 4) / 4).astype(np.float32)  # multiples of 0.25: bf16-exact
    expect = []
    for m in range(M):
        col = E[:, m]
        kind = m % 4
        if kind == 0:    # exact ties of the maximum
            idx = np.sort(rng.choice(V, 3, replace=False))
            col[idx] = 64.0
        elif kind == 1:  # saturated: raw 600 at a low index, raw 1024 and 2048 later: capped 30.0 for all
            idx = np.sort(rng.choice(V, 3, replace=False))
            col[idx[0]], col[idx[1]], col[idx[2]] = 600.0, 1024.0, 2048.0
        elif kind == 2:  # near the cap but distinct
            idx = np.sort(rng.choice(V, 2, replace=False))
            col[idx[0]], col[idx[1]] = 80.0, 80.5
        capped = np.tanh(col / np.float32(30.0)).astype(np.float32) * np.float32(30.0)
        expect.append(int(np.argmax(capped)))   # numpy argmax: the lowest index of the maximum
    assert np.array_equal(bf16_round(E), E)
    d = model.Dense(ctx, torch.from_numpy(oracle.f32_to_bf16_bits(E).view(np.int16)).cuda().view(torch.bfloat16))
    x = np.zeros((M, K), np.float32)
    x[np.arange(M), np.arange(M)] = 1.0     # raw[m, r] = E[r, m] exactly
    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    ids = torch.empty(M, dtype=torch.int32, device="cuda")
    vals = torch.empty(M, dtype=torch.float32, device="cuda")
    L.call("g4_dense_argmax", ctx.handle, d.handle, P(xt), M, C.c_float(30.0), P(ids), P(vals))
    ctx.check_device()
    assert ids.cpu().tolist() == expect
    ref_vals = np.array([np.tanh(E[expect[m], m] / np.float32(30.0)) * np.float32(30.0) for m in range(M)], np.float32)
    assert np.allclose(vals.cpu().numpy(), ref_vals, rtol=2e-6, atol=0)


@pytest.mark.parametrize("M,K,N", [(1, 1536, 256), (5, 1536, 256), (16, 512, 256), (40, 1536, 256), (3, 4096, 512)])
def test_linear_gelu_ple_matches_planes_then_gelu_ple(rt, ctx, M, K, N):
    """g4_linear_w4a16_gelu_ple (GELU_PLE in the GEMV epilogue up to 16 rows, planes + the
    GELU_PLE pass above) gives the bits of g4_linear_w4a16_planes + g4_gelu_ple_planes."""
    gen = g(M + K + N)
    layers, layer = 35, 7
    packed = torch.randint(-2**31, 2**31 - 1, (N, K // 8), device="cuda", dtype=torch.int32, generator=gen)
    sc = torch.randn((N, K // 32), device="cuda", generator=gen).abs_().mul_(0.02).to(torch.bfloat16)
    lin = rt.W4Linear(ctx, packed, sc)
    x = torch.randn((M, K), device="cuda", generator=gen).to(torch.bfloat16)
    per_layer = torch.randn((M, layers * N), device="cuda", generator=gen)
    pl = L.G4Planes()
    L.call("g4_linear_w4a16_planes", ctx.handle, lin.handle, P(x), M, C.byref(pl))
    a1 = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    L.call("g4_gelu_ple_planes", ctx.handle, C.byref(pl), P(per_layer), layer, layers, N, M, P(a1))
    a2 = torch.empty_like(a1)
    L.call("g4_linear_w4a16_gelu_ple", ctx.handle, lin.handle, P(x), M, P(per_layer), layer, layers, P(a2))
    ctx.check_device()
    assert torch.equal(a1, a2)
    assert float(a2.float().abs().sum()) > 0
