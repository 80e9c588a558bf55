"""Replica serving on 2 GPUs (skipped with fewer): each rank decodes its block of the
batch on its own GPU and the NCCL-gathered token ids equal a single-GPU decode of the
whole batch, step by step.  Sequences are independent and each row's arithmetic does not
depend on the batch it shares (the decode GEMV and the attention work row by row), so the
ids must match exactly."""
import importlib
import os
import queue
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

B, STEPS, SEED = 8, 6, 31


def _cfg(model):
    return model.ModelConfig().small(hidden=512, layers=5, vocab=4096, intermediate=1024, intermediate_late=1024,
                                     window=16)


def _prompts():
    rng = np.random.default_rng(SEED)
    return [list(rng.integers(0, 4096, 3 + s)) for s in range(B)]


def _decode(model, ctx, cfg, seqs):
    """Prefill each sequence of `seqs` then STEPS batched greedy steps; ids [STEPS + 1][len(seqs)]."""
    w = model.random_weights(cfg, seed=SEED, embed_sigma=0.03, embed_tail=0.5)
    m = model.Gemma4Model(ctx, cfg, w, max_batch=len(seqs), max_seq=64, max_rows=16)
    first = [m.prefill(i, p) for i, p in enumerate(seqs)]
    cur = torch.tensor(first, dtype=torch.int32, device=ctx.torch_device)
    out = [first]
    for _ in range(STEPS):
        cur = m.decode_step(ids_dev=cur, batch=len(seqs)).clone()
        out.append(cur.tolist())
    return out, m


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        rt = importlib.import_module("gemma4-js_b200.runtime")
        model = importlib.import_module("gemma4-js_b200.model")
        serving = importlib.import_module("gemma4-js_b200.serving")
        dist = serving.init_process_group("nccl", timeout_s=60.0, device=torch.device("cuda", rank))
        ctx = rt.Context(rank)
        cfg = _cfg(model)
        start, count = serving.partition(B, world, rank)
        local, _ = _decode(model, ctx, cfg, _prompts()[start:start + count])
        g = serving.TokenGather(dist, B, torch.device("cuda", rank))
        gathered = [g.gather(torch.tensor(row, dtype=torch.int32, device="cuda")).tolist() for row in local]
        ctx.check_device()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", gathered))
    except Exception as e:  # reported to the test, never a hang
        q.put((rank, "exception", repr(e)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_replicas_gather_the_single_gpu_ids():
    rt = importlib.import_module("gemma4-js_b200.runtime")
    model = importlib.import_module("gemma4-js_b200.model")
    ref, _ = _decode(model, rt.Context(0), _cfg(model), _prompts())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = []
    for _ in range(2):
        try:
            res.append(q.get(timeout=600))
        except queue.Empty:
            break
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    assert len(res) == 2 and all(r[1] == "ok" for r in res), res
    for _, _, gathered in res:
        assert gathered == ref
