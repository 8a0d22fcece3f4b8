"""Host-side failure detection (peers.py) on two GPUs: the tensor-parallel block through the rung's GEMMs and an NCCL
reduce-scatter, two ranks as child processes, NVLS off.  A rank leaves only between steps, with none of its kernels or
collectives in flight (it synchronises first): once after posting its failure, once without a word.  The other rank
must learn of it at its next gate, before it launches anything, and end with PeerFailed or PeerTimeout in bounded
time.  No GPU kernel is made to fault, trap or hang.  Skipped with fewer than two GPUs."""
import datetime
import os
import socket
import time

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _leave(q, item, code):
    q.put(item)
    q.close()
    q.join_thread()
    os._exit(code)  # no teardown collective with a rank that is gone; exit ends this process's context


def _worker(rank, world, port, mode, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist

    import bwgemm
    import peers
    import tp_mlp

    torch.cuda.set_device(rank)
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("nccl", store=store, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20),
                            device_id=torch.device("cuda", rank))
    watch = peers.PeerWatch(store, rank, world, gate_timeout_s=5.0)
    g = torch.Generator(device="cuda").manual_seed(11)
    M, hidden, f = 256, 512, 1024
    X = ((torch.rand((M, hidden), generator=g, device="cuda") * 2 - 1)).half()
    W1 = ((torch.rand((hidden, 2 * f), generator=g, device="cuda") * 2 - 1) / hidden ** 0.5).half()
    W2 = ((torch.rand((f, hidden), generator=g, device="cuda") * 2 - 1) / f ** 0.5).half()
    blk = tp_mlp.TPMLP(tp_mlp.shard_gateup_interleaved(W1, rank, world), tp_mlp.shard_down(W2, rank, world), rank,
                       world, bwgemm.gemm, bwgemm.gemm_f32out, tp_mlp.nccl_reduce_scatter,
                       gemm_swiglu=bwgemm.gemm_swiglu)
    t0 = time.monotonic()
    outcome = "finished"
    try:
        for step in range(5):
            if rank == 1 and step == 2:
                torch.cuda.synchronize()  # nothing of this rank in flight when it leaves
                if mode == "raise":
                    watch.fail(f"step {step}: injected host failure")
                    _leave(q, (rank, "left", 0.0), 1)
                _leave(q, (rank, "left", 0.0), 0)
            watch.gate(step)
            blk.forward(X)
            torch.cuda.synchronize()
    except peers.PeerFailed as e:
        outcome = f"PeerFailed: {e}"
    except peers.PeerTimeout as e:
        outcome = f"PeerTimeout: {e}"
    _leave(q, (rank, outcome, time.monotonic() - t0), 0)


@pytest.mark.parametrize("mode", ["raise", "vanish"])
def test_a_failed_rank_stops_the_other_at_its_gate_on_two_gpus(mode):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
            pytest.fail(f"rank process {p.pid} still running after 180 s ({mode})")
    res = dict((r, (o, t)) for r, o, t in (q.get(timeout=5) for _ in range(world)))
    outcome, secs = res[0]
    if mode == "raise":
        assert outcome.startswith("PeerFailed: rank 1: step 2: injected host failure"), outcome
    else:
        assert outcome.startswith("PeerTimeout"), outcome
    assert secs < 60
