"""The tensor-parallel MLP block over the rung's GEMM: the multi-GPU form of the path (the B200 configs' block of a
Llama-3-70B layer: hidden 8192, MLP 28672, gate and up concatenated into one 8192 x 57344 weight).

Megatron-style, one rank per GPU, p ranks:
  gateup (column-parallel, no communication): rank r holds W1_r = [gate columns of shard r | up columns of shard r]
      (hidden x 2 F/p), H_r = X W1_r in fp16 through the rung's GEMM;
  activation: A_r = silu(H_r[:, :F/p]) * H_r[:, F/p:]  (SwiGLU, on the rank's own shard, no communication), or
      fused into the gateup GEMM's epilogue (bw_gemm_f16_swiglu, W1_r in the layout of shard_gateup_interleaved):
      then H_r is never written;
  down (row-parallel): P_r = A_r W2_r with W2_r = rows [r F/p, (r+1) F/p) of W2 (F x hidden), in fp32 through the
      rung's fp32-output GEMM (bw_gemm_f16_f32out);
  reduce-scatter (NCCL, sum, fp32): rank r receives rows [r M/p, (r+1) M/p) of Y = sum_r P_r, then rounds them to fp16;
      or down and the reduce-scatter in one kernel per rank (bwgemm.ReduceScatterGemm: the partial tiles of the other
      ranks' rows pushed into their memory, each rank summing its own rows' partials in rank order), no NCCL call.

The GEMMs are parameters so that the sharding and the collective can be tested on CPU ranks (gloo) with a CPU matmul
in their place; on the GPU they are the rung's (bwgemm.gemm, bwgemm.gemm_f32out).
"""
import torch
import torch.nn.functional as F


def shard_gateup(W1, rank, world):
    """The rank's columns of the concatenated [gate | up] weight (hidden x 2F): gate shard then up shard."""
    two_f = W1.shape[1]
    f = two_f // 2
    if f % world:
        raise ValueError(f"MLP width {f} does not split over {world} ranks")
    fs = f // world
    gate = W1[:, rank * fs:(rank + 1) * fs]
    up = W1[:, f + rank * fs:f + (rank + 1) * fs]
    return torch.cat([gate, up], dim=1).contiguous()


def shard_gateup_interleaved(W1, rank, world, group=128):
    """The rank's gateup shard laid out for the fused activation (bw_gemm_f16_swiglu): groups of `group` gate columns
    each followed by the matching `group` up columns (a one-time permutation of the weight's columns)."""
    W = shard_gateup(W1, rank, world)
    fs = W.shape[1] // 2
    if fs % group:
        raise ValueError(f"the shard's MLP width {fs} is not a multiple of {group}")
    parts = []
    for g in range(0, fs, group):
        parts.append(W[:, g:g + group])
        parts.append(W[:, fs + g:fs + g + group])
    return torch.cat(parts, dim=1).contiguous()


def swiglu_reference(X, W_interleaved, group=128):
    """What the fused GEMM computes, on any device: silu(gate) * up from fp32 sums, the activation in fp16."""
    H = X.float() @ W_interleaved.float()
    n = H.shape[1]
    idx = torch.arange(n, device=H.device).reshape(-1, 2 * group)
    gate, up = H[:, idx[:, :group].reshape(-1)], H[:, idx[:, group:].reshape(-1)]
    return (F.silu(gate) * up).to(X.dtype)


def shard_down(W2, rank, world):
    """The rank's rows of the down weight (F x hidden)."""
    f = W2.shape[0]
    if f % world:
        raise ValueError(f"MLP width {f} does not split over {world} ranks")
    fs = f // world
    return W2[rank * fs:(rank + 1) * fs].contiguous()


class TPMLP:
    """One rank's part of the block.  W1_r, W2_r: this rank's shards (fp16).  gemm(A, B) -> fp16 C = A B;
    gemm_f32(A, B) -> fp32 C = A B; reduce_scatter(out, inp) sums inp over the ranks into out (this rank's rows)."""

    def __init__(self, W1_r, W2_r, rank, world, gemm, gemm_f32, reduce_scatter=None, gemm_swiglu=None,
                 gemm_rs=None):
        """gemm_swiglu(A, W1_r) -> the activation directly (W1_r then in the interleaved layout of
        shard_gateup_interleaved): the gateup GEMM with the activation in its epilogue.  gemm_rs(A, W2_r) -> this
        rank's rows of the block's output in fp16: down and the reduce-scatter fused (in place of gemm_f32 and
        reduce_scatter)."""
        self.W1, self.W2 = W1_r, W2_r
        self.rank, self.world = rank, world
        self.gemm, self.gemm_f32, self.gemm_swiglu, self.gemm_rs = gemm, gemm_f32, gemm_swiglu, gemm_rs
        self.reduce_scatter = reduce_scatter
        self.fs = W2_r.shape[0]
        if W1_r.shape[1] != 2 * self.fs:
            raise ValueError("gateup shard and down shard disagree on the MLP width")

    def forward(self, X):
        M = X.shape[0]
        if M % self.world:
            raise ValueError(f"{M} tokens do not split over {self.world} ranks")
        if self.gemm_swiglu is not None:
            A = self.gemm_swiglu(X, self.W1)                       # M x F/p, fp16, fused
        else:
            H = self.gemm(X, self.W1)                              # M x 2F/p, fp16
            A = (F.silu(H[:, :self.fs].float()) * H[:, self.fs:].float()).to(X.dtype).contiguous()
        if self.gemm_rs is not None and self.world > 1:
            return self.gemm_rs(A, self.W2)                        # M/p x hidden, fp16, reduced across the ranks
        P = self.gemm_f32(A, self.W2)                              # M x hidden, fp32 partial sums
        if self.world == 1:
            return P.to(X.dtype)
        out = torch.empty((M // self.world, P.shape[1]), dtype=torch.float32, device=P.device)
        self.reduce_scatter(out, P)                                # sum over ranks, this rank's rows
        return out.to(X.dtype)

    @staticmethod
    def flops(M, hidden, f):
        """FLOPs of the whole block (all ranks): the gateup and down GEMMs."""
        return 2.0 * M * hidden * (2 * f) + 2.0 * M * f * hidden


def nccl_reduce_scatter(out, inp):
    import torch.distributed as dist

    dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.SUM)
