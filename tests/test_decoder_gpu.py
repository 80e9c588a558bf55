"""The persistent batch-1 decoder (g4_decoder_step): one greedy decode step of one sequence in
one cooperative launch (one CTA per SM, grid barriers between the phases of every layer).

Checked against the whole-model oracle with the reference's exact f32 weights
(official-w4a16.js:95) and greedy rule (gemma4-webgpu.js:441-480), teacher-forced so every
step is a fresh decision point, with the tolerance rule of test_serving_parity_gpu (the
capped logit at the GPU's pick within 2% of max|logit|; a different pick only inside the
oracle's own top-2 margin).  Also: the same picks as the op-by-op path, bitwise replay in a
CUDA graph, one kernel launch per step, and a position past the cache reported through the
device error word instead of a hang.
"""
import importlib

import numpy as np
import pytest
import torch

from test_serving_parity_gpu import FULL_KW, MAX_TIE_FRAC, Tally

pytestmark = pytest.mark.gpu

model = importlib.import_module("gemma4-js_b200.model")
mo = importlib.import_module("oracle.model_oracle")


def small_cfg(**kw):
    base = dict(hidden=512, layers=5, vocab=4096, intermediate=1024, intermediate_late=1024, window=16)
    base.update(kw)
    return model.ModelConfig().small(**base)


def _teacher_forced(gpu, orc, prompt, forced, tally, tag):
    g_id = gpu.prefill(0, prompt)
    o_id, capped = orc.forward(prompt)
    tally.check(f"{tag} prefill", g_id, float(gpu.buf["val"][0].item()), o_id, capped)
    picks = []
    for step, tok in enumerate(forced):
        ids = torch.tensor([int(tok)], dtype=torch.int32, device="cuda")
        g_id = int(gpu.decode_step(ids_dev=ids, batch=1)[0].item())
        o_id, capped = orc.forward([int(tok)])
        tally.check(f"{tag} step {step}", g_id, float(gpu.buf["val"][0].item()), o_id, capped)
        picks.append(g_id)
    return picks


@pytest.mark.parametrize("cfg_kw,seed", [(dict(), 41), (dict(window=100), 42)])
def test_persistent_decoder_matches_exact_oracle(rt, ctx, cfg_kw, seed):
    """40 teacher-forced steps after a 24-token prompt (windows of 16 and 100 keys: the sliding
    layers drop history), every pick and capped logit checked; one launch per step."""
    cfg = small_cfg(**cfg_kw)
    w = model.random_weights(cfg, seed=seed, **FULL_KW)
    rng = np.random.default_rng(seed)
    prompt = [int(t) for t in rng.integers(0, cfg.vocab, 24)]
    forced = rng.integers(0, cfg.vocab, 40)
    gpu = model.Gemma4Model(ctx, cfg, w, max_batch=1, max_seq=80, max_rows=32, persistent=True)
    assert gpu.decoder() is not None
    orc = mo.OracleModel(cfg, w, max_seq=80, gemm_rows=mo.EXACT)
    tally = Tally()
    n0 = rt.launch_count()
    _teacher_forced(gpu, orc, prompt, forced[:1], tally, "warm")
    n1 = rt.launch_count()
    _teacher_forced_rest = forced[1:]
    for step, tok in enumerate(_teacher_forced_rest):
        ids = torch.tensor([int(tok)], dtype=torch.int32, device="cuda")
        g_id = int(gpu.decode_step(ids_dev=ids, batch=1)[0].item())
        o_id, capped = orc.forward([int(tok)])
        tally.check(f"step {step + 1}", g_id, float(gpu.buf["val"][0].item()), o_id, capped)
    ctx.check_device()
    launches = rt.launch_count() - n1
    assert launches == len(_teacher_forced_rest), f"{launches} launches for {len(_teacher_forced_rest)} steps"
    assert n1 > n0
    print(f"persistent: {tally.checked} picks, ties {tally.ties}, worst value error {tally.worst_val:.2e}")
    assert len(tally.ties) <= max(1, int(MAX_TIE_FRAC * tally.checked))


def test_persistent_decoder_reference_spec(rt, ctx):
    """The checkpoint's own layer spec at small width: head dim 512 + rope 1e6 / 0.25 on global
    layers, wider MLP late, KV-shared layers that read another layer's cache."""
    cfg = model.ModelConfig.reference_spec().small(hidden=512, layers=7, vocab=4096, intermediate=1024,
                                                   intermediate_late=2048, first_shared=5, window=16)
    w = model.random_weights(cfg, seed=43, **FULL_KW)
    rng = np.random.default_rng(43)
    prompt = [int(t) for t in rng.integers(0, cfg.vocab, 20)]
    forced = rng.integers(0, cfg.vocab, 24)
    gpu = model.Gemma4Model(ctx, cfg, w, max_batch=1, max_seq=64, max_rows=32, persistent=True)
    assert gpu.decoder() is not None
    orc = mo.OracleModel(cfg, w, max_seq=64, gemm_rows=mo.EXACT)
    tally = Tally()
    _teacher_forced(gpu, orc, prompt, forced, tally, "ref-spec")
    ctx.check_device()
    print(f"reference spec: {tally.checked} picks, ties {tally.ties}, worst value error {tally.worst_val:.2e}")
    assert len(tally.ties) <= max(1, int(MAX_TIE_FRAC * tally.checked))


def test_persistent_decoder_agrees_with_op_path(rt, ctx):
    """The persistent step and the op-by-op step (the same operators as ~200 launches) give
    the same picks and capped logits within summation-order noise on the same inputs."""
    cfg = small_cfg()
    w = model.random_weights(cfg, seed=44, **FULL_KW)
    rng = np.random.default_rng(44)
    prompt = [int(t) for t in rng.integers(0, cfg.vocab, 12)]
    forced = rng.integers(0, cfg.vocab, 32)
    out = {}
    for persistent in (True, False):
        gpu = model.Gemma4Model(ctx, cfg, w, max_batch=1, max_seq=64, max_rows=16, persistent=persistent)
        assert (gpu.decoder() is not None) == persistent
        gpu.prefill(0, prompt)
        picks, vals = [], []
        for tok in forced:
            ids = torch.tensor([int(tok)], dtype=torch.int32, device="cuda")
            picks.append(int(gpu.decode_step(ids_dev=ids, batch=1)[0].item()))
            vals.append(float(gpu.buf["val"][0].item()))
        out[persistent] = (picks, np.array(vals))
        ctx.check_device()
    (pa, va), (pb, vb) = out[True], out[False]
    scale = np.abs(vb).max()
    assert np.abs(va - vb).max() <= 0.01 * scale
    assert sum(a != b for a, b in zip(pa, pb)) <= 1


def test_persistent_graph_replay_is_bitwise_eager(rt, ctx):
    """The step is deterministic (fixed reduction orders, no atomics on values): 20 replays of a
    captured step give the ids and values of 20 eager steps bit for bit."""
    cfg = small_cfg()
    w = model.random_weights(cfg, seed=45, **FULL_KW)
    prompt = [3, 1, 4, 1, 5, 9, 2, 6]
    res = []
    for graph in (False, True):
        m = model.Gemma4Model(ctx, cfg, w, max_batch=1, max_seq=64, max_rows=16, persistent=True)
        first = m.prefill(0, prompt)
        m.buf["next"][0] = first
        ids, vals = [], []
        if graph:
            m.capture_decode(batch=1)
        for _ in range(20):
            nxt = m.replay_decode() if graph else m.decode_step(batch=1)
            ids.append(int(nxt[0].item()))
            vals.append(float(m.buf["val"][0].item()))
        torch.cuda.synchronize()
        assert int(m.seq_pos[0].item()) == len(prompt) + 20
        res.append((ids, vals))
        m.close()
    assert res[0] == res[1]
    ctx.check_device()


def test_persistent_decoder_position_past_cache_is_reported(rt, ctx):
    """A step at a position past the cache is refused on the device (G4_ERR_DEVICE through the
    error word, next id 0, nothing written, no barrier entered), and the decoder keeps working."""
    cfg = small_cfg()
    w = model.random_weights(cfg, seed=46, **FULL_KW)
    m = model.Gemma4Model(ctx, cfg, w, max_batch=1, max_seq=32, max_rows=16, persistent=True)
    m.prefill(0, [7, 8, 9])
    good = m.seq_pos.clone()
    m.seq_pos[0] = 32
    m.decode_step(ids_dev=torch.tensor([5], dtype=torch.int32, device="cuda"), batch=1)
    with pytest.raises(model.G4Error) as ei:
        ctx.check_device()
    assert ei.value.status == -7
    assert int(m.buf["next"][0].item()) == 0 and int(m.seq_pos[0].item()) == 32
    m.seq_pos.copy_(good)
    nxt = m.decode_step(ids_dev=torch.tensor([5], dtype=torch.int32, device="cuda"), batch=1)
    ctx.check_device()
    assert 0 <= int(nxt[0].item()) < cfg.vocab and int(m.seq_pos[0].item()) == int(good[0].item()) + 1


def test_unsupported_shapes_fall_back_to_the_operators(rt, ctx):
    """hidden 320 is outside the persistent decoder's range (a multiple of 256 is required):
    the model decodes through the operators instead."""
    cfg = small_cfg(hidden=320)
    w = model.random_weights(cfg, seed=47, **FULL_KW)
    m = model.Gemma4Model(ctx, cfg, w, max_batch=1, max_seq=32, max_rows=16, persistent=True)
    assert m.decoder() is None
    m.prefill(0, [1, 2, 3])
    nxt = m.decode_step(ids_dev=torch.tensor([4], dtype=torch.int32, device="cuda"), batch=1)
    ctx.check_device()
    assert 0 <= int(nxt[0].item()) < cfg.vocab
