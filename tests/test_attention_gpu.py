"""GQA decode attention and the bf16 KV cache on the GPU, against the oracle (1e-2)."""
import numpy as np
import pytest
import torch

from conftest import bf16_round, max_rel

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _case(rt, ctx, ops, oracle, hd, keylen, rows, sliding, window=512, heads=8, seed=0, cap=None):
    rng = np.random.default_rng(seed + keylen * 3 + rows)
    k = bf16_round(rng.standard_normal((keylen, hd)).astype(np.float32))
    v = bf16_round(rng.standard_normal((keylen, hd)).astype(np.float32))
    q = bf16_round((rng.standard_normal((rows, heads, hd)) * (0.25 / np.sqrt(hd / 64))).astype(np.float32))
    cache = rt.KVCache(ctx, hd, cap or keylen + 8)
    kt = torch.from_numpy(k).to(torch.bfloat16).cuda()
    vt = torch.from_numpy(v).to(torch.bfloat16).cuda()
    # append in two pieces like prefill then decode
    cut = max(0, keylen - rows)
    if cut:
        cache.append(kt[:cut], vt[:cut], cut, 0)
    cache.append(kt[cut:], vt[cut:], keylen - cut, cut)
    assert cache.length == keylen
    qt = torch.from_numpy(q).to(torch.bfloat16).cuda()
    out = ops.attention(qt, cache, rows, heads, hd, keylen, keylen - rows, sliding, window)
    ctx.check_device()
    ref = oracle.attention(q, k, v, keylen - rows, sliding, window)
    return out.float().cpu().numpy(), ref


@pytest.mark.parametrize("keylen", [1, 2, 15, 64, 65, 511, 512, 513, 1000, 2176, 4352])
@pytest.mark.parametrize("sliding", [False, True])
def test_decode_hd256(rt, ctx, ops, oracle, keylen, sliding):
    out, ref = _case(rt, ctx, ops, oracle, 256, keylen, 1, sliding)
    assert max_rel(out, ref) < TOL


@pytest.mark.parametrize("rows", [2, 5, 64])
@pytest.mark.parametrize("sliding", [False, True])
def test_multi_row_hd256(rt, ctx, ops, oracle, rows, sliding):
    out, ref = _case(rt, ctx, ops, oracle, 256, 700, rows, sliding)
    assert max_rel(out, ref) < TOL


@pytest.mark.parametrize("hd,keylen", [(512, 1), (512, 700), (64, 300), (128, 1500)])
def test_other_head_dims(rt, ctx, ops, oracle, hd, keylen):
    out, ref = _case(rt, ctx, ops, oracle, hd, keylen, 1, False)
    assert max_rel(out, ref) < TOL


def test_small_window_and_fewer_heads(rt, ctx, ops, oracle):
    out, ref = _case(rt, ctx, ops, oracle, 256, 300, 3, True, window=17, heads=5)
    assert max_rel(out, ref) < TOL


def test_kv_append_rules(rt, ctx, g4, oracle):
    cache = rt.KVCache(ctx, 256, 16)
    k = torch.randn(4, 256, device="cuda")
    v = torch.randn(4, 256, device="cuda")
    with pytest.raises(g4.G4Error, match="KV append position 3 != cache length 0"):
        cache.append(k, v, 4, 3)
    cache.append(k, v, 4, 0)  # f32 input is rounded to nearest-even bf16
    kc, vc = cache.tensors()
    exp = oracle.f32_to_bf16_bits(k.cpu().numpy()).view(np.int16)
    assert np.array_equal(kc[:4].cpu().view(torch.int16).numpy(), exp)
    with pytest.raises(g4.G4Error, match="KV cache capacity 16 exceeded"):
        cache.append(torch.zeros(13, 256, device="cuda"), torch.zeros(13, 256, device="cuda"), 13, 4)
    cache.reset()
    assert cache.length == 0


def test_attention_argument_errors(rt, ctx, ops, g4):
    cache = rt.KVCache(ctx, 256, 32)
    cache.append(torch.zeros(8, 256, device="cuda", dtype=torch.bfloat16),
                 torch.zeros(8, 256, device="cuda", dtype=torch.bfloat16), 8, 0)
    q = torch.zeros(1, 8, 256, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(g4.G4Error, match="keylen"):
        ops.attention(q, cache, 1, 8, 256, 9, 8, False, 512)
    with pytest.raises(g4.G4Error, match="query positions"):
        ops.attention(q, cache, 1, 8, 256, 8, 8, False, 512)
    with pytest.raises(g4.G4Error, match="heads"):
        ops.attention(torch.zeros(1, 16, 256, device="cuda", dtype=torch.bfloat16), cache, 1, 16, 256, 8, 7, False, 512)


@pytest.mark.parametrize("nseq,sliding", [(40, True), (40, False), (64, True), (64, False), (160, True), (160, False),
                                          (300, True)])
def test_attention_rows_batched(rt, ctx, oracle, nseq, sliding):
    """g4_attention_rows: one decode row for each of nseq independent sequences at their own
    device-side positions in one cache object (sequence s at rows s * stride).  40 rows:
    keys split over CTAs + combine; 64: one CTA per row; above the SM count: two CTAs per
    SM on the sliding layers."""
    import ctypes as C
    from importlib import import_module
    L = import_module("gemma4-js_b200._lib")
    hd, heads, stride, window = 256, 8, 1100, 512
    rng = np.random.default_rng(nseq * 7 + int(sliding))
    cache = rt.KVCache(ctx, hd, nseq * stride)
    k = bf16_round((rng.standard_normal((nseq * stride, hd)) * 0.3).astype(np.float32))
    v = bf16_round(rng.standard_normal((nseq * stride, hd)).astype(np.float32))
    cache.append(torch.from_numpy(k).to(torch.bfloat16).cuda(), torch.from_numpy(v).to(torch.bfloat16).cuda(),
                 nseq * stride, 0)
    pos = rng.integers(0, stride, nseq).astype(np.int32)
    pos[:3] = [0, stride - 1, window]
    q = bf16_round((rng.standard_normal((nseq, heads, hd)) * 0.25).astype(np.float32))
    qd = torch.from_numpy(q).to(torch.bfloat16).cuda()
    posd = torch.from_numpy(pos).cuda()
    out = torch.empty_like(qd)
    rmap = L.G4Rows(posd.data_ptr(), 0, 1, 0)
    L.call("g4_attention_rows", ctx.handle, C.c_void_p(qd.data_ptr()), cache.handle, nseq, heads, hd, C.byref(rmap),
           stride, int(sliding), window, C.c_void_p(out.data_ptr()))
    ctx.check_device()
    got = out.float().cpu().numpy()
    for s in range(nseq):
        p, r0 = int(pos[s]), s * stride
        ref = oracle.attention(q[s:s + 1], k[r0:r0 + p + 1], v[r0:r0 + p + 1], p, sliding, window)
        assert max_rel(got[s:s + 1], ref) < TOL, s
