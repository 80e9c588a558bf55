"""CPU tests of the replica serving logic: partitioning, the token-id gather over a
world-size-2 gloo group, and failure detection when a rank dies (no GPU involved)."""
import importlib
import os
import queue
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

serving = importlib.import_module("gemma4-js_b200.serving")


def test_partition_is_contiguous_and_complete():
    for total in (0, 1, 7, 256):
        for world in (1, 2, 3, 4, 8):
            spans = [serving.partition(total, world, r) for r in range(world)]
            assert sum(c for _, c in spans) == total
            pos = 0
            for s, c in spans:
                assert s == pos
                pos += c
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
    assert serving.partition(256, 8, 3) == (96, 32)
    with pytest.raises(ValueError):
        serving.partition(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _put_and_exit(q, msg):
    """Leaves without the process group's shutdown, after the queue's feeder thread has
    handed msg to the pipe (os._exit would otherwise drop it)."""
    q.put(msg)
    q.close()
    q.join_thread()
    os._exit(0)


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        dist = serving.init_process_group("gloo", timeout_s=5.0)
        total = 7
        start, count = serving.partition(total, world, rank)
        g = serving.TokenGather(dist, total, "cpu")
        if mode == "ok":
            for step in range(3):
                local = torch.arange(start, start + count, dtype=torch.int32) * 10 + step
                out = g.gather(local)
                q.put((rank, step, out.tolist()))
            dist.barrier()
            dist.destroy_process_group()
        elif mode == "heartbeat":  # rank 1 leaves after step 1; rank 0 learns it on the host
            from torch.distributed import distributed_c10d as c10d
            hb = serving.StepHeartbeat(c10d._get_default_store(), rank, world, timeout_s=1.5)
            local = torch.arange(start, start + count, dtype=torch.int32)
            for step in range(3):
                t0 = time.time()
                try:
                    hb.enter(step)
                except serving.RankFailure as e:
                    _put_and_exit(q, (rank, "failure", step, time.time() - t0, str(e)))
                g.gather(local)
                if rank == 1 and step == 1:
                    _put_and_exit(q, (rank, "left", step, 0.0, ""))
            _put_and_exit(q, (rank, "no-failure", 3, 0.0, ""))
        else:  # rank 1 leaves between steps; rank 0 must get an error, not hang
            local = torch.arange(start, start + count, dtype=torch.int32)
            g.gather(local)
            if rank == 1:
                _put_and_exit(q, (rank, "left", None))
            t0 = time.time()
            try:
                g.gather(local)
                msg = (rank, "no-error", time.time() - t0)
            except Exception:  # the process group reports the dead peer
                msg = (rank, "error", time.time() - t0)
            _put_and_exit(q, msg)
    except Exception as e:
        q.put((rank, "exception", repr(e)))


def _run(mode, world=2, wait=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(wait)
    for p in procs:
        if p.is_alive():
            p.kill()
    out = []
    while True:
        try:
            out.append(q.get(timeout=2.0))
        except queue.Empty:
            return out


def test_token_gather_two_ranks():
    res = _run("ok")
    got = {(r, s): v for r, s, v in res}
    for step in range(3):
        expect = [i * 10 + step for i in range(7)]
        assert got[(0, step)] == expect
        assert got[(1, step)] == expect


def test_dead_rank_surfaces_as_an_error():
    res = _run("dead")
    r0 = [x for x in res if x[0] == 0]
    assert r0 and r0[0][1] == "error", res
    assert r0[0][2] < 30.0  # bounded by the process-group timeout, not a hang


def test_heartbeat_reports_a_rank_that_left_between_steps():
    """Rank 1 leaves after step 1: rank 0's entry into step 2 names it within the
    heartbeat limit (1.5 s), on the host, before any collective of step 2 is enqueued."""
    res = _run("heartbeat")
    r0 = [x for x in res if x[0] == 0]
    assert r0 and r0[0][1] == "failure" and r0[0][2] == 2, res
    assert r0[0][3] < 10.0 and "[1]" in r0[0][4]
    assert any(x[0] == 1 and x[1] == "left" for x in res)
