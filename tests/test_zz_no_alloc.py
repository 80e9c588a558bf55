"""g4_attention_noalloc: attention for callers that cannot allocate device memory.

Hosts that give all device memory to their own pool, or serving loops that cannot take
cudaMalloc's implicit device synchronisation, cannot let g4_attention grow its
workspace.  g4_attention_noalloc keeps the split-KV partials in one fixed device array
inside the library instead.  These tests call it through the C ABI and compare it with
g4_attention on two calls in a row (both split the key range, so the fixed array is
used), then check that a split too large for the array is refused with a clear error.
This file is collected last, so a failure here does not hide the other tests.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import bf16_round, max_rel

pytestmark = pytest.mark.gpu

TOL = 1e-2  # the attention tolerance of the other GPU tests (max|y - ref| / max|ref|)


def _cache(rt, ctx, hd, keylen, seed):
    rng = np.random.default_rng(seed)
    cache = rt.KVCache(ctx, hd, keylen)
    k = torch.from_numpy(bf16_round(rng.standard_normal((keylen, hd)).astype(np.float32))).to(torch.bfloat16).cuda()
    v = torch.from_numpy(bf16_round(rng.standard_normal((keylen, hd)).astype(np.float32))).to(torch.bfloat16).cuda()
    cache.append(k, v, keylen, 0)
    return cache, rng, k.float().cpu().numpy(), v.float().cpu().numpy()


def _noalloc(g4, ctx, q, cache, rows, heads, hd, keylen, qpos0, sliding, window):
    out = torch.full((rows, heads, hd), float("nan"), dtype=torch.bfloat16, device="cuda")
    st = g4.load().g4_attention_noalloc(ctx.handle, C.c_void_p(q.data_ptr()), cache.handle, rows, heads, hd,
                                        keylen, qpos0, int(sliding), window, C.c_void_p(out.data_ptr()))
    return st, out


def test_noalloc_matches_g4_attention_on_two_calls(rt, ctx, ops, g4, oracle):
    """Two calls in a row (the second reuses the array the first wrote), each split over
    CTAs: the same bits as g4_attention (same kernels, same split plan) and within the
    attention tolerance of the oracle."""
    for hd, keylen, rows, sliding, seed in [(256, 4000, 1, False, 1), (256, 2000, 3, True, 2)]:
        cache, rng, k, v = _cache(rt, ctx, hd, keylen, seed)
        qf = bf16_round((rng.standard_normal((rows, 8, hd)) * 0.1).astype(np.float32))
        q = torch.from_numpy(qf).to(torch.bfloat16).cuda()
        ref = ops.attention(q, cache, rows, 8, hd, keylen, keylen - rows, sliding, 512)
        st, out = _noalloc(g4, ctx, q, cache, rows, 8, hd, keylen, keylen - rows, sliding, 512)
        assert st == 0, g4.load().g4_last_error_string()
        ctx.check_device()
        assert not torch.isnan(out.float()).any()
        assert torch.equal(out, ref)
        expect = oracle.attention(qf, k, v, keylen - rows, sliding, 512)
        assert max_rel(out.float().cpu().numpy(), expect) < TOL


def test_noalloc_rejects_a_split_larger_than_its_array(rt, ctx, g4):
    """rows = 2 x SMs - 1 query rows without a row map split every row's keys in two (the
    split rule gives each SM two CTAs), which needs rows x 2 x 8 x (hd + 2) x 4 B of
    partials: more than the 8 MiB array at hd 512 on any GPU with at least 128 SMs."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    hd, keylen = 512, 1024
    rows = 2 * sms - 1
    need = rows * 2 * 8 * (hd + 2) * 4 + 256
    if need <= 8 << 20:
        pytest.skip(f"{sms} SMs: this split fits the 8 MiB array")
    cache, rng, _, _ = _cache(rt, ctx, hd, keylen, 3)
    q = torch.zeros((rows, 8, hd), dtype=torch.bfloat16, device="cuda")
    st, _ = _noalloc(g4, ctx, q, cache, rows, 8, hd, keylen, keylen - rows, False, 512)
    assert st == -6  # G4_ERR_RANGE
    msg = g4.load().g4_last_error_string().decode()
    assert "scratch" in msg and "8388608" in msg and str(need) in msg
