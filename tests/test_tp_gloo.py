"""The tensor-parallel MLP block's sharding and collective on CPU ranks (gloo, world size 2), a CPU matmul standing in
for the rung's GEMMs: the block computed over 2 ranks equals the block computed whole."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import tp_mlp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gemm(A, B):
    return (A.float() @ B.float()).to(A.dtype)


def _gemm_f32(A, B):
    return A.float() @ B.float()


def _reduce_scatter_gloo(out, inp):
    """sum over ranks, this rank's rows (all_reduce then a slice: gloo has no reduce-scatter)"""
    full = inp.clone()
    dist.all_reduce(full, op=dist.ReduceOp.SUM)
    rows = out.shape[0]
    out.copy_(full[dist.get_rank() * rows:(dist.get_rank() + 1) * rows])


def _gemm_rs_gloo(A, B):
    """A CPU stand-in for the fused down + reduce-scatter (bw_gemm_f16_rs): this rank's rows of sum_r A_r B_r, fp16."""
    P = A.float() @ B.float()
    out = torch.empty((P.shape[0] // dist.get_world_size(), P.shape[1]), dtype=torch.float32)
    _reduce_scatter_gloo(out, P)
    return out.to(A.dtype)


def _reference(X, W1, W2):
    f = W2.shape[0]
    H = _gemm(X, W1)
    A = (torch.nn.functional.silu(H[:, :f].float()) * H[:, f:].float()).to(X.dtype)
    return (A.float() @ W2.float())


def _worker(rank, world, port, M, hidden, f, q, mode="unfused"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(5)
        X = (torch.rand(M, hidden, generator=g) * 2 - 1).half()
        W1 = ((torch.rand(hidden, 2 * f, generator=g) * 2 - 1) / hidden ** 0.5).half()
        W2 = ((torch.rand(f, hidden, generator=g) * 2 - 1) / f ** 0.5).half()
        if mode != "unfused":  # the interleaved layout, a CPU stand-in for the fused GEMM
            blk = tp_mlp.TPMLP(tp_mlp.shard_gateup_interleaved(W1, rank, world, group=16),
                               tp_mlp.shard_down(W2, rank, world), rank, world, _gemm,
                               None if mode == "fused_rs" else _gemm_f32,
                               None if mode == "fused_rs" else _reduce_scatter_gloo,
                               gemm_swiglu=lambda A, W: tp_mlp.swiglu_reference(A, W, group=16),
                               gemm_rs=_gemm_rs_gloo if mode == "fused_rs" else None)
        else:
            blk = tp_mlp.TPMLP(tp_mlp.shard_gateup(W1, rank, world), tp_mlp.shard_down(W2, rank, world), rank,
                               world, _gemm, _gemm_f32, _reduce_scatter_gloo)
        Y = blk.forward(X)
        ref = _reference(X, W1, W2)[rank * (M // world):(rank + 1) * (M // world)]
        err = (Y.float() - ref).abs().max().item()
        q.put((rank, tuple(Y.shape), err, ref.abs().max().item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["unfused", "fused", "fused_rs"])
@pytest.mark.parametrize("world", [2])
def test_tp_mlp_over_two_cpu_ranks_equals_the_whole_block(world, mode):
    """unfused: gateup, the activation, down in fp32 and a reduce-scatter; fused: the activation in the gateup GEMM;
    fused_rs: also down and the reduce-scatter in one call (no separate collective)."""
    M, hidden, f = 32, 64, 96
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, hidden, f, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = sorted(q.get(timeout=5) for _ in range(world))
    for rank, shape, err, ref_max in results:
        assert shape == (M // world, hidden)
        assert err <= 4e-3 * ref_max + 1e-3, (rank, err, ref_max)  # fp16 roundings of H (unfused) and Y


def test_shards_cover_the_weights_once():
    hidden, f, world = 8, 12, 3
    W1 = torch.arange(hidden * 2 * f, dtype=torch.float32).reshape(hidden, 2 * f)
    W2 = torch.arange(f * hidden, dtype=torch.float32).reshape(f, hidden)
    cols = torch.cat([tp_mlp.shard_gateup(W1, r, world) for r in range(world)], dim=1)
    # every gate column and every up column exactly once, gate shard before up shard on each rank
    assert sorted(cols[0].tolist()) == sorted(W1[0].tolist())
    assert tp_mlp.shard_gateup(W1, 1, world)[0, :f // world].tolist() == W1[0, 4:8].tolist()
    assert tp_mlp.shard_gateup(W1, 1, world)[0, f // world:].tolist() == W1[0, f + 4:f + 8].tolist()
    assert torch.equal(torch.cat([tp_mlp.shard_down(W2, r, world) for r in range(world)]), W2)
    with pytest.raises(ValueError):
        tp_mlp.shard_down(W2, 0, 5)


def test_flops():
    assert tp_mlp.TPMLP.flops(2048, 8192, 28672) == 2.0 * 2048 * 8192 * 57344 + 2.0 * 2048 * 28672 * 8192
