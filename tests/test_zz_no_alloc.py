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
    return cache, rng


def _noalloc(g4, ctx, q, cache, rows, heads, hd, keylen, qpos0, sliding, window):
    out = torch.full((rows, heads, hd), float("nan"), dtype=torch.bfloat16, device="cuda")
    st = g4.load().g4_attention_noalloc(ctx.handle, C.c_void_p(q.data_ptr()), cache.handle, rows, heads, hd,
                                        keylen, qpos0, int(sliding), window, C.c_void_p(out.data_ptr()))
    return st, out


def test_noalloc_matches_g4_attention_on_two_calls(rt, ctx, ops, g4):
    for hd, keylen, rows, sliding, seed in [(256, 4000, 1, False, 1), (256, 2000, 3, True, 2)]:
        cache, rng = _cache(rt, ctx, hd, keylen, seed)
        q = torch.from_numpy(bf16_round((rng.standard_normal((rows, 8, hd)) * 0.1).astype(np.float32)))
        q = q.to(torch.bfloat16).cuda()
        ref = ops.attention(q, cache, rows, 8, hd, keylen, keylen - rows, sliding, 512)
        st, out = _noalloc(g4, ctx, q, cache, rows, 8, hd, keylen, keylen - rows, sliding, 512)
        assert st == 0, g4.load().g4_last_error_string()
        ctx.check_device()
        assert not torch.isnan(out.float()).any()
        assert max_rel(out.float().cpu().numpy(), ref.float().cpu().numpy()) < TOL


def test_noalloc_rejects_a_split_larger_than_its_array(rt, ctx, g4):
    hd, keylen, rows = 512, 1024, 290  # 290 rows x 2 splits x 8 x 514 x 4 B > 8 MiB
    cache, rng = _cache(rt, ctx, hd, keylen, 3)
    q = torch.zeros((rows, 8, hd), dtype=torch.bfloat16, device="cuda")
    st, _ = _noalloc(g4, ctx, q, cache, rows, 8, hd, keylen, keylen - rows, False, 512)
    assert st == -6  # G4_ERR_RANGE
    msg = g4.load().g4_last_error_string().decode()
    assert "scratch" in msg and "8388608" in msg
