"""The reference's f32 buffer convention at the C ABI (GPUOps.w4 and GPUOps.attention take
and return f32 buffers, custom-webgpu/gpu-runtime.js:1316-1324, :1357-1365).

g4_linear_w4a16_f32 and g4_attention_f32 take f32 inputs as the reference's model graph
holds them (not pre-rounded to bf16) and are compared with the oracle's f32 arithmetic
on those unrounded inputs (tolerance: max|y - ref| / max|ref| <= 1e-2).  They must also
equal the bf16 entry points fed RNE-rounded inputs bit for bit, and g4_convert must be
bit-identical to roundFloat32ToBF16 (official-w4a16.js:34-48) on special values too.
"""
import ctypes as C
import importlib

import numpy as np
import pytest
import torch

from conftest import bf16_round, max_rel
from test_linear_gpu import make_weights

pytestmark = pytest.mark.gpu

L = importlib.import_module("gemma4-js_b200._lib")
TOL = 1e-2


def P(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.parametrize("M,K,N", [(1, 1536, 6144), (5, 512, 384), (16, 2048, 264), (40, 512, 384),
                                   (300, 256, 1536)])
def test_linear_f32_matches_oracle_on_unrounded_x(rt, ctx, ops, oracle, M, K, N):
    packed, scales = make_weights(oracle, K, N, M + K + N)
    lin = rt.W4Linear(ctx, packed, scales)
    x = np.random.default_rng(M * 7 + K).standard_normal((M, K)).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    L.call("g4_linear_w4a16_f32", ctx.handle, lin.handle, P(xt), M, P(y))
    ctx.check_device()
    ref = oracle.linear_w4a16(x, packed, scales, nthreads=8)  # f32 x, exact f32 weights
    assert max_rel(y.cpu().numpy(), ref) < TOL
    y2 = ops.w4(lin, xt.to(torch.bfloat16), M, out_dtype=torch.float32)
    assert torch.equal(y, y2)


@pytest.mark.parametrize("rows,keylen,sliding", [(1, 700, False), (3, 700, True), (1, 4096, False)])
def test_attention_f32_matches_oracle_on_unrounded_q(rt, ctx, ops, oracle, rows, keylen, sliding):
    hd = 256
    rng = np.random.default_rng(rows + keylen)
    k = rng.standard_normal((keylen, hd)).astype(np.float32) * 0.3
    v = rng.standard_normal((keylen, hd)).astype(np.float32)
    q = (rng.standard_normal((rows, 8, hd)) * 0.3).astype(np.float32)
    cache = rt.KVCache(ctx, hd, keylen)
    cache.append(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), keylen, 0)  # f32 rows, as KVCache.append
    out = torch.full((rows, 8, hd), float("nan"), dtype=torch.float32, device="cuda")
    qt = torch.from_numpy(q).cuda()
    L.call("g4_attention_f32", ctx.handle, P(qt), cache.handle, rows, 8, hd, keylen, keylen - rows, int(sliding), 512,
           P(out))
    ctx.check_device()
    ref = oracle.attention(q, k, v, keylen - rows, sliding, 512)  # the reference's f32 q, K and V
    assert max_rel(out.cpu().numpy(), ref) < TOL
    o2 = ops.attention(qt.to(torch.bfloat16), cache, rows, 8, hd, keylen, keylen - rows, sliding, 512)
    assert torch.equal(out, o2.float())


def test_convert_is_the_reference_rounding(rt, ctx, oracle):
    rng = np.random.default_rng(5)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 3.0e38, -3.4e38, 1.0, 1.00390625,
                        1.01171875, 65504.0], np.float32)
    halfway = (np.arange(1, 200, dtype=np.uint32) << 16 | 0x8000).view(np.float32)  # ties to even
    x = np.concatenate([special, halfway, rng.standard_normal(100003).astype(np.float32) * 1e3])
    n = x.size
    src = torch.from_numpy(x).cuda()
    b = torch.empty(n, dtype=torch.int16, device="cuda")
    L.call("g4_convert", ctx.handle, P(src), 0, P(b), 1, n)
    f = torch.empty(n, dtype=torch.float32, device="cuda")
    L.call("g4_convert", ctx.handle, P(b), 1, P(f), 0, n)
    b2 = torch.empty(n, dtype=torch.int16, device="cuda")
    L.call("g4_convert", ctx.handle, P(b), 1, P(b2), 1, n)
    ctx.check_device()
    bits = b.cpu().numpy().view(np.uint16)
    assert np.array_equal(bits, oracle.f32_to_bf16_bits(x))
    assert np.array_equal(f.cpu().numpy().view(np.uint32), bits.astype(np.uint32) << 16)
    assert torch.equal(b, b2)
    with pytest.raises(L.G4Error):
        L.call("g4_convert", ctx.handle, P(src), 0, P(b), 7, n)


# ---- the rest of GPUOps in the reference's own form (f32 buffers in and out), each against
# the oracle's restatement of its WGSL shader (oracle/model_oracle.py).

def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def test_gpuops_elementwise_and_norms_match_the_shaders(rt, ctx, ops):
    mo = importlib.import_module("oracle.model_oracle")
    rng = np.random.default_rng(9)
    rows, width = 5, 1536
    x = rng.standard_normal((rows, width)).astype(np.float32) * 3
    sc = (1 + 0.1 * rng.standard_normal(width)).astype(np.float32)
    assert max_rel(ops.rms(_t(x), rows, width, _t(sc)).cpu().numpy().reshape(rows, width), mo.rms(x, sc, 1e-6)) < 1e-5
    assert max_rel(ops.rms(_t(x), rows, width).cpu().numpy().reshape(rows, width), mo.rms(x, None, 1e-6)) < 1e-5
    a, b = x.reshape(-1), rng.standard_normal(rows * width).astype(np.float32)
    assert torch.equal(ops.addScale(_t(a), _t(b), a.size, 0.75).cpu(), torch.from_numpy((a + b) * np.float32(0.75)))
    assert torch.equal(ops.scale(_t(a), a.size, -1.5).cpu(), torch.from_numpy(a * np.float32(-1.5)))
    gate = rng.standard_normal(4096).astype(np.float32) * 4
    gate[:4] = [1e4, -1e4, 0.0, 30.0]  # the +-10 clamp of the tanh argument
    up = rng.standard_normal(4096).astype(np.float32)
    assert max_rel(ops.geluMul(_t(gate), _t(up), gate.size).cpu().numpy(), mo.gelu(gate) * up) < 1e-5
    g2 = rng.standard_normal((3, 256)).astype(np.float32)
    ple = rng.standard_normal((3, 35, 256)).astype(np.float32)
    for layer in (0, 17, 34):
        got = ops.geluPle(_t(g2), _t(ple), 3, layer).cpu().numpy().reshape(3, 256)
        assert max_rel(got, mo.gelu(g2) * ple[:, layer, :]) < 1e-5
    ctx.check_device()


@pytest.mark.parametrize("hd,prop,base,pos0", [(256, 1.0, 10000.0, 0), (256, 1.0, 10000.0, 4093), (512, 0.25, 1e6, 77)])
def test_gpuops_norm_rope_matches_the_shader(rt, ctx, ops, hd, prop, base, pos0):
    mo = importlib.import_module("oracle.model_oracle")
    rng = np.random.default_rng(hd + pos0)
    rows, heads = 3, 8
    x = rng.standard_normal((rows, heads, hd)).astype(np.float32)
    sc = (0.3 * (1 + 0.1 * rng.standard_normal(hd))).astype(np.float32)
    got = ops.normRope(_t(x), rows, heads, hd, pos0, _t(sc), prop, base).cpu().numpy().reshape(rows, heads, hd)
    ref = mo.norm_rope(x, sc, pos0 + np.arange(rows), int(prop * hd / 2), base, 1e-6)
    # theta = pos / base^(2i/hd) in f32 as the shader: one ulp of theta (2.4e-4 rad at 4095)
    # between CUDA's powf and numpy's f32 power moves sin/cos by as much
    tol = 1e-4 + 4 * np.spacing(np.float32(pos0 + rows))
    assert max_rel(got, ref) < tol
    ctx.check_device()


def test_gpuops_ple_mix_and_head_softcap(rt, ctx, ops, oracle):
    mo = importlib.import_module("oracle.model_oracle")
    model = importlib.import_module("gemma4-js_b200.model")
    rng = np.random.default_rng(3)
    rows = 4
    proj = rng.standard_normal((rows, 35, 256)).astype(np.float32)
    norm = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    tok = rng.standard_normal((rows, 35, 256)).astype(np.float32) * 0.05
    got = ops.pleMix(_t(proj), _t(norm), _t(tok), rows).cpu().numpy().reshape(rows, 35, 256)
    ref = (mo.rms(proj, norm, 1e-6) + tok * np.float32(16.0)) * np.float32(0.7071067811865476)
    assert max_rel(got, ref) < 1e-5
    # headChunk = bf16 tied head + softcap 30 over every vocabulary row at once
    V, K = 3000, 1536
    E = (rng.standard_normal((V, K)) * 0.05).astype(np.float32)
    Eb = bf16_round(E)
    d = model.Dense(ctx, torch.from_numpy(oracle.f32_to_bf16_bits(E).view(np.int16)).cuda().view(torch.bfloat16))
    xh = bf16_round(rng.standard_normal((1, K)).astype(np.float32) * 2)
    logits = torch.empty((1, V), dtype=torch.float32, device="cuda")
    L.call("g4_dense_matmul", ctx.handle, d.handle, P(_t(xh).to(torch.bfloat16)), 1, P(logits))
    L.call("g4_softcap", ctx.handle, P(logits), V, C.c_float(30.0))
    ctx.check_device()
    ref = np.tanh((xh @ Eb.T) / np.float32(30.0)) * np.float32(30.0)
    assert max_rel(logits.cpu().numpy(), ref) < 1e-4
