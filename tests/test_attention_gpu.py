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


# ------------------------------------------------------------ ring KV caches --
# g4_kv_create_ring keeps each sequence's last `ring` positions (slot = position % ring,
# the first 16384/hd slots repeated after the ring), as the Node reference trims its
# sliding-layer caches (node-reference/src/attention.js:299-305).  The attention reads the
# same key tiles in the same order as from a linear cache, so the results must be equal
# bit for bit, and within the 1e-2 tolerance of the oracle over the full history.

def _ring_len(hd, window, rows):
    return max(window + rows - 1, 16384 // hd)


@pytest.mark.parametrize("hd,window,chunk", [(256, 100, 1), (256, 40, 7), (512, 50, 3), (64, 300, 5), (128, 130, 1)])
def test_ring_cache_matches_linear_and_oracle(rt, ctx, ops, oracle, hd, window, chunk):
    """Positions appended chunk by chunk until the ring has wrapped several times; after
    every chunk the chunk's rows attend (sliding) on a ring cache and on a linear one."""
    ring = _ring_len(hd, window, chunk)
    total = 3 * ring + 37
    rng = np.random.default_rng(hd + window + chunk)
    k = bf16_round((rng.standard_normal((total, hd)) * 0.3).astype(np.float32))
    v = bf16_round(rng.standard_normal((total, hd)).astype(np.float32))
    ringc = rt.KVCache(ctx, hd, total, ring=ring)
    assert (ringc.ring, ringc.seq_rows, ringc.rows) == (ring, ring + 16384 // hd, ring + 16384 // hd)
    lin = rt.KVCache(ctx, hd, total)
    kt, vt = torch.from_numpy(k).to(torch.bfloat16).cuda(), torch.from_numpy(v).to(torch.bfloat16).cuda()
    start, n_checked = 0, 0
    while start < total:
        rows = min(chunk, total - start)
        src_k, src_v = kt[start:start + rows], vt[start:start + rows]
        if (start // chunk) % 3 == 1:  # f32 rows are rounded to bf16 by the append
            src_k, src_v = src_k.float(), src_v.float()
        ringc.append(src_k, src_v, rows, start)
        lin.append(src_k, src_v, rows, start)
        q = bf16_round((rng.standard_normal((rows, 8, hd)) * 0.25).astype(np.float32))
        qt = torch.from_numpy(q).to(torch.bfloat16).cuda()
        keylen = start + rows
        a = ops.attention(qt, ringc, rows, 8, hd, keylen, start, True, window)
        b = ops.attention(qt, lin, rows, 8, hd, keylen, start, True, window)
        assert torch.equal(a, b), f"ring and linear caches differ at positions {start}..{keylen - 1}"
        if n_checked < 6 and (start // chunk) % 11 == 5:
            ref = oracle.attention(q, k[:keylen], v[:keylen], start, True, window)
            assert max_rel(a.float().cpu().numpy(), ref) < TOL
            n_checked += 1
        start = keylen
    ctx.check_device()
    assert ringc.length == total and n_checked > 0
    # the storage holds the last `ring` positions in their slots and the mirrored rows
    ks, _ = ringc.tensors()
    ks = ks.cpu()
    for p in range(total - ring, total):
        assert torch.equal(ks[p % ring], kt[p].cpu()), p
    for sl in range(16384 // hd):
        assert torch.equal(ks[ring + sl], ks[sl]), sl


def _ring_storage(k, v, pos, ring, mirror):
    """Host image of a batched ring cache: sequence s's position p at row s*(ring+mirror) + p % ring
    for its last `ring` positions, then the mirror rows."""
    nseq, _, hd = k.shape
    rows = ring + mirror
    ks = np.zeros((nseq * rows, hd), np.float32)
    vs = np.zeros((nseq * rows, hd), np.float32)
    for s in range(nseq):
        for p in range(max(0, int(pos[s]) + 1 - ring), int(pos[s]) + 1):
            ks[s * rows + p % ring] = k[s, p]
            vs[s * rows + p % ring] = v[s, p]
        ks[s * rows + ring:s * rows + rows] = ks[s * rows:s * rows + mirror]
        vs[s * rows + ring:s * rows + rows] = vs[s * rows:s * rows + mirror]
    return ks, vs


def _upload(cache, ks, vs):
    import ctypes as C
    from importlib import import_module
    L = import_module("gemma4-js_b200._lib")
    kp, vp = C.c_void_p(), C.c_void_p()
    L.call("g4_kv_buffers", cache.handle, C.byref(kp), C.byref(vp))
    cudart = C.CDLL("libcudart.so.12")
    cudart.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    for dst, src in ((kp, ks), (vp, vs)):
        t = torch.from_numpy(src).to(torch.bfloat16).cuda()
        torch.cuda.synchronize()
        assert cudart.cudaMemcpy(dst, C.c_void_p(t.data_ptr()), t.numel() * 2, 3) == 0


@pytest.mark.parametrize("nseq", [24, 200])
def test_ring_cache_attention_rows(rt, ctx, oracle, nseq):
    """g4_attention_rows over a batched ring cache (one decode row per sequence, positions on
    the device, many of them past the ring) equals the same call over a linear cache."""
    import ctypes as C
    from importlib import import_module
    L = import_module("gemma4-js_b200._lib")
    hd, heads, cap, window = 256, 8, 1500, 512
    ring = _ring_len(hd, window, 1)
    mirror = 16384 // hd
    rng = np.random.default_rng(nseq)
    k = bf16_round((rng.standard_normal((nseq, cap, hd)) * 0.3).astype(np.float32))
    v = bf16_round(rng.standard_normal((nseq, cap, hd)).astype(np.float32))
    pos = rng.integers(0, cap, nseq).astype(np.int32)
    pos[:4] = [0, ring - 1, ring, cap - 1]
    ringc = rt.KVCache(ctx, hd, cap, ring=ring, nseq=nseq)
    assert ringc.rows == nseq * (ring + mirror)
    _upload(ringc, *_ring_storage(k, v, pos, ring, mirror))
    lin = rt.KVCache(ctx, hd, nseq * cap)
    _upload(lin, k.reshape(-1, hd), v.reshape(-1, hd))
    q = bf16_round((rng.standard_normal((nseq, heads, hd)) * 0.25).astype(np.float32))
    qd = torch.from_numpy(q).to(torch.bfloat16).cuda()
    posd = torch.from_numpy(pos).cuda()
    rmap = L.G4Rows(posd.data_ptr(), 0, 1, 0)
    outs = []
    for cache, stride in ((ringc, ringc.seq_rows), (lin, cap)):
        out = torch.empty_like(qd)
        L.call("g4_attention_rows", ctx.handle, C.c_void_p(qd.data_ptr()), cache.handle, nseq, heads, hd,
               C.byref(rmap), stride, 1, window, C.c_void_p(out.data_ptr()))
        outs.append(out)
    ctx.check_device()
    assert torch.equal(outs[0], outs[1])
    got = outs[0].float().cpu().numpy()
    for s in range(0, nseq, max(1, nseq // 12)):
        p = int(pos[s])
        ref = oracle.attention(q[s:s + 1], k[s, :p + 1], v[s, :p + 1], p, True, window)
        assert max_rel(got[s:s + 1], ref) < TOL, s


def test_ring_cache_qkv_post_kv_writes_slots_and_mirror(rt, ctx, g4):
    """g4_qkv_post_kv into a ring cache writes each row's K/V at its sequence's slot
    position % ring (and the mirror row below 16384/hd) with the values g4_qkv_post_planes
    writes into a linear cache at the position itself."""
    import ctypes as C
    from importlib import import_module
    L = import_module("gemma4-js_b200._lib")
    hd, heads, nseq, cap, ring = 256, 8, 6, 400, 80
    mirror = 16384 // hd
    width = (heads + 2) * hd
    y = torch.randn((nseq, width), device="cuda")
    qn = torch.rand(hd, device="cuda") + 0.5
    kn = torch.rand(hd, device="cuda") + 0.5
    pos = torch.tensor([0, 5, 63, 64, 79, 333], dtype=torch.int32, device="cuda")
    rmap = L.G4Rows(pos.data_ptr(), 0, 1, 0)
    pl = L.G4Planes(y.data_ptr(), 1, 0, width)
    ringc = rt.KVCache(ctx, hd, cap, ring=ring, nseq=nseq)
    lin = rt.KVCache(ctx, hd, nseq * cap)
    kp, vp = C.c_void_p(), C.c_void_p()
    L.call("g4_kv_buffers", lin.handle, C.byref(kp), C.byref(vp))
    q1 = torch.empty((nseq, heads, hd), dtype=torch.bfloat16, device="cuda")
    q2 = torch.empty_like(q1)
    L.call("g4_qkv_post_planes", ctx.handle, C.byref(pl), heads, hd, 1, C.c_void_p(qn.data_ptr()),
           C.c_void_p(kn.data_ptr()), C.c_float(1e-6), 64, C.c_float(10000.0), C.byref(rmap), nseq,
           C.c_void_p(q1.data_ptr()), kp, vp, cap)
    L.call("g4_qkv_post_kv", ctx.handle, C.byref(pl), heads, hd, C.c_void_p(qn.data_ptr()),
           C.c_void_p(kn.data_ptr()), C.c_float(1e-6), 64, C.c_float(10000.0), C.byref(rmap), nseq,
           C.c_void_p(q2.data_ptr()), ringc.handle)
    ctx.check_device()
    assert torch.equal(q1, q2)
    (lk, lv), (rk, rv) = lin.tensors(), ringc.tensors()
    for s, p in enumerate(pos.tolist()):
        base = s * (ring + mirror)
        assert torch.equal(rk[base + p % ring], lk[s * cap + p]) and torch.equal(rv[base + p % ring], lv[s * cap + p])
        if p % ring < mirror:
            assert torch.equal(rk[base + ring + p % ring], lk[s * cap + p])
    # a position at the capacity writes nothing and raises the device error word
    bad = torch.tensor([cap], dtype=torch.int32, device="cuda")
    bmap = L.G4Rows(bad.data_ptr(), 0, 1, 0)
    L.call("g4_qkv_post_kv", ctx.handle, C.byref(pl), heads, hd, C.c_void_p(qn.data_ptr()),
           C.c_void_p(kn.data_ptr()), C.c_float(1e-6), 64, C.c_float(10000.0), C.byref(bmap), 1,
           C.c_void_p(q2.data_ptr()), ringc.handle)
    with pytest.raises(g4.G4Error):
        ctx.check_device()
    assert torch.equal(ringc.tensors()[0], rk)


def test_ring_cache_argument_errors(rt, ctx, ops, g4):
    import ctypes as C
    from importlib import import_module
    L = import_module("gemma4-js_b200._lib")
    with pytest.raises(g4.G4Error, match="ring of 32 slots"):
        rt.KVCache(ctx, 256, 1000, ring=32)
    ringc = rt.KVCache(ctx, 256, 1000, ring=100)
    z = torch.zeros(20, 256, device="cuda", dtype=torch.bfloat16)
    ringc.append(z, z, 20, 0)
    q = torch.zeros(2, 8, 256, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(g4.G4Error, match="sliding-window attention only"):
        ops.attention(q, ringc, 2, 8, 256, 20, 18, False, 512)
    with pytest.raises(g4.G4Error, match="need 101 ring slots"):
        ops.attention(q, ringc, 2, 8, 256, 20, 18, True, 100)
    ops.attention(q, ringc, 2, 8, 256, 20, 18, True, 99)
    multi = rt.KVCache(ctx, 256, 1000, ring=100, nseq=3)
    with pytest.raises(g4.G4Error, match="ring cache of 3 sequences"):
        multi.append(z, z, 20, 0)
    posd = torch.zeros(3, dtype=torch.int32, device="cuda")
    rmap = L.G4Rows(posd.data_ptr(), 0, 1, 0)
    out = torch.empty(3, 8, 256, device="cuda", dtype=torch.bfloat16)
    qq = torch.zeros(3, 8, 256, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(g4.G4Error, match="seq_stride"):
        L.call("g4_attention_rows", ctx.handle, C.c_void_p(qq.data_ptr()), multi.handle, 3, 8, 256, C.byref(rmap),
               100, 1, 64, C.c_void_p(out.data_ptr()))
    ctx.check_device()
