"""Host-side failure detection (peers.py) on CPU ranks (gloo, world size 2), the tensor-parallel block's step loop with
a CPU matmul in place of the rung's GEMMs.  The failures are made on the host: a rank that raises between steps and
says so, a rank that exits without a word, a rank that passes the gate and then never joins the collective.  The
surviving rank must end with the right error in bounded time, never hang."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import peers
import tp_mlp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _reduce_scatter_gloo(out, inp):
    full = inp.clone()
    dist.all_reduce(full, op=dist.ReduceOp.SUM)
    rows = out.shape[0]
    out.copy_(full[dist.get_rank() * rows:(dist.get_rank() + 1) * rows])


def _leave(q, item, code):
    """Reports, flushes the queue (its feeder thread dies with os._exit) and leaves without any teardown."""
    q.put(item)
    q.close()
    q.join_thread()
    os._exit(code)


def _worker(rank, world, port, mode, q):
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=20))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    watch = peers.PeerWatch(store, rank, world, gate_timeout_s=3.0)
    g = torch.Generator().manual_seed(3)
    M, hidden, f = 16, 32, 48
    X = (torch.rand(M, hidden, generator=g) * 2 - 1).half()
    W1 = ((torch.rand(hidden, 2 * f, generator=g) * 2 - 1) / hidden ** 0.5).half()
    W2 = ((torch.rand(f, hidden, generator=g) * 2 - 1) / f ** 0.5).half()
    blk = tp_mlp.TPMLP(tp_mlp.shard_gateup(W1, rank, world), tp_mlp.shard_down(W2, rank, world), rank, world,
                       lambda A, B: (A.float() @ B.float()).to(A.dtype), lambda A, B: A.float() @ B.float(),
                       _reduce_scatter_gloo)
    t0 = time.monotonic()
    outcome = "finished"
    try:
        for step in range(5):
            if rank == 1 and step == 2:
                if mode == "raise":
                    try:
                        raise ValueError("injected host failure")
                    except ValueError as e:
                        watch.fail(f"step {step}: {e}")
                        _leave(q, (rank, "left", 0.0), 1)
                if mode == "vanish":
                    _leave(q, (rank, "left", 0.0), 0)
            watch.gate(step)
            if rank == 1 and step == 2 and mode == "skip_collective":
                _leave(q, (rank, "left", 0.0), 0)
            blk.forward(X)
    except peers.PeerFailed as e:
        outcome = f"PeerFailed: {e}"
    except peers.PeerTimeout as e:
        outcome = f"PeerTimeout: {e}"
    except RuntimeError as e:  # the process group's timeout, or the peer's closed connection
        outcome = f"collective: {type(e).__name__}"
    _leave(q, (rank, outcome, time.monotonic() - t0), 0)  # no teardown collective with a rank that is gone


def _run(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
            pytest.fail(f"rank process {p.pid} still running after 90 s ({mode})")
    return dict((r, (o, t)) for r, o, t in (q.get(timeout=5) for _ in range(world)))


def test_a_rank_that_fails_and_says_so_stops_the_others_at_the_next_gate():
    res = _run("raise")
    outcome, secs = res[0]
    assert outcome.startswith("PeerFailed: rank 1: step 2: injected host failure"), outcome
    assert secs < 20


def test_a_rank_that_vanishes_ends_the_others_gate_with_a_timeout():
    res = _run("vanish")
    outcome, secs = res[0]
    assert outcome.startswith("PeerTimeout"), outcome
    assert secs < 20


def test_a_rank_that_skips_the_collective_ends_it_with_an_error():
    res = _run("skip_collective")
    outcome, secs = res[0]
    assert outcome.startswith("collective:") or outcome.startswith("PeerTimeout"), outcome
    assert secs < 30


def test_every_rank_finishes_when_none_fails():
    res = _run("none")
    assert res[0][0] == "finished" and res[1][0] == "finished"
