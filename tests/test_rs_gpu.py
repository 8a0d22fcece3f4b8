"""The fused reduce-scatter (bw_gemm_f16_rs, bwgemm.ReduceScatterGemm) on two or four GPUs, one child process per
rank, NVLS off: each rank's rows of sum_r A_r B_r against an fp32 reference (torch matmul per rank, an NCCL all-reduce),
under the judge's tolerance; three calls in a row give the same bits (the receive slots reused through the epochs and
acks); the call captured in a CUDA graph and replayed twice gives the same bits again (its epoch comes from the
device); every rank's status word clear.

Passed on two B200s (w2_small, w2_tp_down); skipped with fewer GPUs than ranks."""
import datetime
import os
import socket

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist

    import bwgemm

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30), device_id=torch.device("cuda", rank))
    result = None
    try:
        bwgemm.clear_status()
        g = torch.Generator(device="cuda").manual_seed(1000 + rank)
        A = (torch.rand((M, K), generator=g, device="cuda") * 2 - 1).half()
        B = (torch.rand((K, N), generator=g, device="cuda") * 2 - 1).half()
        rs = bwgemm.ReduceScatterGemm(M, N)
        outs = []
        for _ in range(3):
            outs.append(rs(A, B).clone())
        torch.cuda.synchronize()
        C = torch.empty_like(outs[0])
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            rs(A, B, C)
        for _ in range(2):  # every rank replays the same calls
            C.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            outs.append(C.clone())
        del graph
        code = bwgemm.status()[0]
        ref = A.float() @ B.float()
        dist.all_reduce(ref)
        rows = M // world
        ref = ref[rank * rows:(rank + 1) * rows]
        gap = ((outs[0].float() - ref).abs().max() / ref.abs().max()).item()
        same = all(torch.equal(outs[0], o) for o in outs[1:])
        finite = bool(torch.isfinite(outs[0]).all())
        rs.close()
        dist.barrier()
        result = (rank, code, gap, same, finite)
    except Exception as e:  # reported to the test, which fails
        result = (rank, f"{type(e).__name__}: {e}", None, None, None)
    finally:
        q.put(result)
        dist.destroy_process_group()


@pytest.mark.parametrize("world,M,N,K", [(2, 1024, 1536, 2048), (2, 4096, 8192, 7168), (4, 4096, 8192, 7168)],
                         ids=["w2_small", "w2_tp_down", "w4_tp_down"])
def test_fused_reduce_scatter_on_gpus(world, M, N, K):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        if p.is_alive():
            p.kill()
            pytest.fail(f"rank process {p.pid} still running after 240 s")
    results = sorted(q.get(timeout=5) for _ in range(world))
    for rank, code, gap, same, finite in results:
        assert code == 0, (rank, code)
        assert finite and gap <= 2e-3 and same, (rank, gap, same, finite)
