#!/usr/bin/env python
"""bench.py -- throughput of the Blackwell rung's GEMM (C = A B, fp16 in, fp32 accumulate, fp16 out) on B200.

One step = one GEMM over one batch of synthetic inputs (seeded uniform [-1, 1) fp16, the value distribution of the
judge's fill, judge/judge.cu:127-134), three input sets rotating as in the judge (so the working set, 3 x (A + B),
is larger than the 126 MB L2 and no flush is needed).

Default workload (N = 1): BASELINE config 1, M x N x K = 4608 x 5632 x 8192, TFLOP/s.  With --gpus N (torchrun, one
rank per GPU) each rank computes its own column shard of a wider GEMM (the column-parallel split of a Megatron MLP:
N = 5632 per rank, no communication): weak scaling, value = all ranks' FLOPs / the slowest rank's device time.

Printed (rank 0, one JSON line): value (device time, inputs resident in HBM), e2e (the same through the public API
with host buffers: pinned host -> device copies of A and B and the device -> host read of C inside the timed region;
`value` with the copies of neighbouring steps overlapping each GEMM as a serving loop runs them, `serial_value` with
everything in order on one stream),
roofline (the kernel against the measured cuBLAS peak), cpu_baseline (the fp64 oracle on a bounded sample of rows,
all host threads), clocks sampled through NVML during the timed region, gpu_launches.  The default line also holds,
at N = 1: sweep (the judge's 17 B200 shapes timed against torch.matmul, cuBLAS, in CUDA graphs, with the geometric
mean of the time ratios; --sweep-shapes a,b,... times only those; --ab-lib <build> adds a third arm, another build of
the library, interleaved with the other two), sustained (config 1 back to back for --sustained-seconds, under the
power cap) and decode (the four weights at M = 1 to 64, GB/s against the measured HBM copy
bandwidth); at every N: tp_mlp (BASELINE config 4 over the job's ranks, with NCCL's reduce-scatter) and, at N > 1,
tp_mlp_fused_rs (the same with bw_gemm_f16_rs); and a headline record repeating the main figures.  --no-sweep,
--no-decode, --no-sustained, --no-tp, --no-e2e and --no-cpu leave parts out.

--impl reference: the reference's CPU path (its fp64 i-k-j GEMM, restated in oracle/oracle.c; the reference's GPU
harness needs its judge, which needs CUDA 13) timed on the host cores on the same workload, in bounded row samples.

--workload tp_mlp: the tensor-parallel MLP block of gemm-ladder_b200/tp_mlp.py over the ranks
(--tp-m tokens, 8192 or 2048; --tp-unfused for the activation as separate torch ops; --tp-fused-rs for down and the
reduce-scatter in one kernel per rank, bw_gemm_f16_rs), total work fixed: strong scaling.  --shape MxNxK times any
shape in place of the workload.  --profile-arm {ours,cublas}: one call of either arm inside an NVTX range "timed" (3
warm-up calls before it), no JSON line: the command for ncu's --nvtx-include.  BWGEMM_LIB=libbwgemm_next.so runs any
of these on the library with the options not yet measured (gemm-ladder_b200/build.py --next); config.library says
which library a line comes from.
"""
import argparse
import datetime
import json
import math
import os
import re
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "gemm-ladder_b200")
for _p in (ROOT, PKG, os.path.join(ROOT, "tests")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

WORKLOADS = {
    "tp_mlp": None,  # the tensor-parallel MLP block (gateup + down + reduce-scatter), --tp-m tokens
    "config1": (4608, 5632, 8192),
    "ladder": (8192, 8192, 8192),
    "ladder_4096": (4096, 6144, 8192),
}
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config1")
    ap.add_argument("--shape", default=None, help="MxNxK in place of the workload (profiling a shape)")
    ap.add_argument("--variant", type=int, default=0)
    ap.add_argument("--tp-m", type=int, default=8192, help="tokens of the tp_mlp workload (2048 or 8192)")
    ap.add_argument("--tp-unfused", action="store_true", help="tp_mlp: the activation as separate torch ops")
    ap.add_argument("--tp-fused-rs", action="store_true",
                    help="tp_mlp: down and the reduce-scatter in one kernel per rank (bw_gemm_f16_rs), no NCCL call")
    ap.add_argument("--sweep", action="store_true",
                    help="time the judge's 17 shapes against cuBLAS (on by default for the 1-GPU config1 run)")
    ap.add_argument("--no-sweep", action="store_true", help="leave the 17-shape sweep out of the default run")
    ap.add_argument("--sweep-shapes", default=None,
                    help="--sweep: only these shapes (comma-separated names of the set, or MxNxK)")
    ap.add_argument("--no-decode", action="store_true", help="leave the decode block (config 3) out")
    ap.add_argument("--no-sustained", action="store_true", help="leave the sustained config-1 run out")
    ap.add_argument("--no-tp", action="store_true", help="leave the tensor-parallel MLP sub-record (config 4) out")
    ap.add_argument("--sustained-seconds", type=float, default=3.0)
    ap.add_argument("--ab-lib", default=None,
                    help="--sweep: also time another build of the library, from gemm-ladder_b200/lib/ (e.g. "
                         "libbwgemm_next.so), interleaved with the two arms in the same process")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--profile-arm", choices=["ours", "cublas"], default=None,
                    help="for ncu: 3 warm-up calls, then one call in an NVTX range named 'timed', and exit")
    return ap.parse_args()


def profile_call(args):
    """One call of an arm at the workload, for `ncu --nvtx --nvtx-include timed/` (no timing, no JSON line)."""
    import torch

    import bwgemm

    torch.cuda.set_device(0)
    M, N, K = WORKLOADS[args.workload]
    A, B = make_sets(M, N, K, seed=1)
    C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    if args.profile_arm == "cublas":
        call = lambda i: torch.matmul(A[i % 3], B[i % 3], out=C)  # noqa: E731
    else:
        call = lambda i: bwgemm.gemm(A[i % 3], B[i % 3], C, variant=args.variant)  # noqa: E731
    for i in range(3):
        call(i)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("timed")
    call(3)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(workload):
    """DRAM bytes per launch of the GEMM kernel at this workload, from the committed ncu summary (or None)."""
    path = os.path.join(ROOT, "profiles", f"gemm_kernel_{workload}.md")
    try:
        with open(path) as f:
            m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


# ------------------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """NVML samples of the SM clock and the clock-event reasons while the timed region runs."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, device_index):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = self._handle(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None

    def _handle(self, device_index):
        import torch

        nv = self._nv
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            return nv.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(device_index)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._h is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------------------ distributed
def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        # a short timeout: a rank that never joins a collective ends it with an error, not a hang
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def dist_max(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    import torch

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


# ------------------------------------------------------------------------------------------------------ our arm
def make_sets(M, N, K, seed, sets=3):
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    A = [(torch.rand((M, K), generator=g, device="cuda") * 2 - 1).half() for _ in range(sets)]
    B = [(torch.rand((K, N), generator=g, device="cuda") * 2 - 1).half() for _ in range(sets)]
    return A, B


def cpu_baseline(M, N, K, seconds):
    """The fp64 oracle (oracle/oracle.c, the reference's i-k-j loop) on a bounded sample of rows, all host threads."""
    import numpy as np

    from oracle import oracle

    threads = os.cpu_count() or 1
    rows0 = min(M, max(threads, 8))
    A, B = oracle.judge_inputs(rows0, N, K)
    t0 = time.perf_counter()
    oracle.gemm_f64(A, B, threads=threads)
    t = time.perf_counter() - t0
    rows = int(min(M, max(rows0, rows0 * seconds / max(t, 1e-6))))
    rows = max(threads, rows // threads * threads) if rows >= threads else rows
    A, B = oracle.judge_inputs(rows, N, K)
    t0 = time.perf_counter()
    oracle.gemm_f64(A, B, threads=threads)
    t = time.perf_counter() - t0
    # the loop as the reference runs it, one thread, on its own CPU case (its LCG inputs)
    A0, B0 = oracle.lcg_inputs(256, 256, 512)
    t1 = time.perf_counter()
    oracle.gemm_f64(A0, B0, threads=1)
    t1 = time.perf_counter() - t1
    del np
    return {"value": 2.0 * rows * N * K / t / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of {M} rows of {M}x{N}x{K}, fp64 i-k-j oracle (oracle/oracle.c), {t:.1f} s",
            "single_thread_config0": {"gflops": round(2.0 * 256 * 256 * 512 / t1 / 1e9, 3), "seconds": round(t1, 4),
                                      "shape": "256x256x512", "cores": 1}}


def sweep(args, stream_runs=3):
    """The judge's 17 shapes (+ BASELINE's ladder variants): ours and torch.matmul (cuBLAS), CUDA graphs of G calls
    on 3 rotating input sets, interleaved rounds, median; ratio = cuBLAS time / ours (the judge's ratio).  With a third
    arm (--ab-lib) 4 rounds, each arm first in two of them and last in the other two.  --sweep-shapes: only the named
    shapes (a name of the set, or MxNxK); the geomean then only if all 17 were run."""
    import ctypes

    import torch

    import bwgemm
    from shapes import CONFIG1, JUDGE_B200, LADDER_4096

    other = None  # the other build of the library (--ab-lib), bound on its own
    if args.ab_lib:
        other = ctypes.CDLL(os.path.join(PKG, "lib", args.ab_lib))
        other.bw_gemm_f16_variant.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p, ctypes.c_int]
        other.bw_gemm_f16_variant.restype = ctypes.c_int

    def call_other(A, B, C):
        M, K = A.shape
        N = B.shape[1]
        rc = other.bw_gemm_f16_variant(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K,
                                       torch.cuda.current_stream().cuda_stream, args.variant)
        if rc:
            raise RuntimeError(f"{args.ab_lib}: status {rc}")

    arms = ("ours", "cublas") + (("other",) if other else ())
    if other:
        stream_runs = 4
    shapes = list(JUDGE_B200) + [LADDER_4096, CONFIG1]
    if args.sweep_shapes:
        known = {n: (n, M, N, K) for n, M, N, K in shapes}
        shapes = []
        for w in args.sweep_shapes.split(","):
            if w in known:
                shapes.append(known[w])
            else:
                M, N, K = map(int, w.lower().split("x"))
                shapes.append((w, M, N, K))
    out = {}
    ratios = []
    for name, M, N, K in shapes:
        A, B = make_sets(M, N, K, seed=M * 7 + N)
        C = torch.empty((M, N), dtype=torch.float16, device="cuda")
        flops = 2.0 * M * N * K
        G = max(3, min(60, int(20e-3 / max(flops / 1.2e15, 5e-6))))
        bwgemm.gemm(A[0], B[0], C, variant=args.variant)  # the first call of a shape (workspace)
        torch.matmul(A[0], B[0], out=C)
        if other:
            call_other(A[0], B[0], C)
        torch.cuda.synchronize()
        graphs = {}
        for arm in arms:
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    for i in range(G):
                        if arm == "ours":
                            bwgemm.gemm(A[i % 3], B[i % 3], C, variant=args.variant)
                        elif arm == "other":
                            call_other(A[i % 3], B[i % 3], C)
                        else:
                            torch.matmul(A[i % 3], B[i % 3], out=C)
            torch.cuda.synchronize()
            graphs[arm] = g
        times = {arm: [] for arm in arms}
        # rounds alternate the arms' order (4 rounds: forward, reversed, reversed, forward)
        flips = (0, 1, 1, 0) if stream_runs == 4 else [r % 2 for r in range(stream_runs)]
        for rnd in range(stream_runs):
            for arm in (arms[::-1] if flips[rnd] else arms):
                g = graphs[arm]
                g.replay()  # warm-up
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                reps = max(1, int(0.15 / max(G * flops / 1.2e15, 1e-5)))
                e0.record()
                for _ in range(reps):
                    g.replay()
                e1.record()
                torch.cuda.synchronize()
                times[arm].append(e0.elapsed_time(e1) / 1e3 / (reps * G))
        t_ours, t_cub = statistics.median(times["ours"]), statistics.median(times["cublas"])
        ratio = t_cub / t_ours
        ratios.append(ratio)
        bytes_alg = 2.0 * (M * K + K * N + M * N)
        out[name] = {"M": M, "N": N, "K": K, "us": round(t_ours * 1e6, 2), "cublas_us": round(t_cub * 1e6, 2),
                     "ratio": round(ratio, 4), "tflops": round(flops / t_ours / 1e12, 1),
                     "gbs": round(bytes_alg / t_ours / 1e9, 1)}
        if other:
            t_other = statistics.median(times["other"])
            out[name].update({"other_us": round(t_other * 1e6, 2), "other_ratio": round(t_cub / t_other, 4)})
        del graphs, A, B, C
        torch.cuda.empty_cache()
    every = all(n in out for n, *_ in JUDGE_B200)

    def geomean(key):
        if not every:
            return None
        v = [out[n][key] for n, *_ in JUDGE_B200]
        return round(math.exp(sum(map(math.log, v)) / len(v)), 4)

    res = {"shapes": out, "geomean_ratio_vs_cublas_17": geomean("ratio"),
           "reference": "torch.matmul fp16 (cuBLAS heuristic), CUDA graphs, 3 rotating input sets"}
    if other:
        res.update({"other_library": args.ab_lib, "other_geomean_ratio_vs_cublas_17": geomean("other_ratio")})
    return res


def tp_mlp_measure(args, rank, world, local, fused_rs=False, steps=None, warmup=None, e2e=True, tp_m=None):
    """BASELINE config 4 on the process group's ranks (tp_mlp.py): the block's device time per step (max over ranks),
    the same block without its collective (gateup + down's fp32 partials only, this rank's compute: max over ranks),
    and the collective's exposed time, the difference.  Every rank calls it; returns rank 0's record (others: None)."""
    import torch

    import bwgemm
    import tp_mlp

    steps = args.steps if steps is None else steps
    warmup = max(3, args.warmup if warmup is None else warmup)
    M, hidden, f = (args.tp_m if tp_m is None else tp_m), 8192, 28672
    gx = torch.Generator(device="cuda")
    gx.manual_seed(7)  # the same tokens on every rank
    X = (torch.rand((M, hidden), generator=gx, device="cuda") * 2 - 1).half()
    gw = torch.Generator(device="cuda")
    gw.manual_seed(100 + rank)  # this rank's shards (synthetic weights, scaled to keep the activations in range)
    W1 = ((torch.rand((hidden, 2 * f // world), generator=gw, device="cuda") * 2 - 1) / hidden ** 0.5).half()
    W2 = ((torch.rand((f // world, hidden), generator=gw, device="cuda") * 2 - 1) / f ** 0.5).half()
    # (random shards: the interleaved gate / up layout of the fused activation needs no permutation here)
    rs = bwgemm.ReduceScatterGemm(M, hidden) if fused_rs and world > 1 else None
    blk = tp_mlp.TPMLP(W1, W2, rank, world, bwgemm.gemm, bwgemm.gemm_f32out,
                       tp_mlp.nccl_reduce_scatter if world > 1 else None,
                       gemm_swiglu=None if args.tp_unfused else bwgemm.gemm_swiglu, gemm_rs=rs)
    stream = torch.cuda.current_stream()
    watch = None
    if world > 1:  # host-side failure detection at the phase boundaries (peers.py), outside the timed region
        import peers

        watch = peers.PeerWatch.from_default_group(gate_timeout_s=120.0)
    try:
        if watch:
            watch.gate()
        for _ in range(warmup):
            blk.forward(X)
        if watch:
            watch.gate()
    except Exception as e:
        if watch and not isinstance(e, (peers.PeerFailed, peers.PeerTimeout)):
            watch.fail(f"{type(e).__name__}: {e}")
        raise
    # the same block without its collective: this rank's GEMMs alone (the activation fused or not, as above), timed
    # before and after the block (the mean of the two, so that a clock that drifts under the power cap between the
    # loops does not show as collective time)
    def local_step():
        Act = bwgemm.gemm_swiglu(X, blk.W1) if not args.tp_unfused else None
        if Act is None:
            H = bwgemm.gemm(X, blk.W1)
            Act = (torch.nn.functional.silu(H[:, :blk.fs].float()) * H[:, blk.fs:].float()).half()
        return bwgemm.gemm_f32out(Act, blk.W2)

    def timed(fn, n):
        barrier(world)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(n):
            fn()
        g1.record(stream)
        barrier(world)
        return dist_max(g0.elapsed_time(g1) / 1e3, world)

    for _ in range(2):
        local_step()
    t_local0 = timed(local_step, steps)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(world)
        e0.record(stream)
        for _ in range(steps):
            Y = blk.forward(X)
        e1.record(stream)
        barrier(world)
    t = dist_max(e0.elapsed_time(e1) / 1e3, world)
    del Y
    t_local = 0.5 * (t_local0 + timed(local_step, steps))
    # the NCCL form's collective alone, on this rank's fp32 partials (the fused form has none to time apart)
    t_coll = None
    if world > 1 and rs is None:
        P = local_step()
        out = torch.empty((M // world, P.shape[1]), dtype=torch.float32, device=P.device)
        t_coll = timed(lambda: tp_mlp.nccl_reduce_scatter(out, P), steps)
        del P, out
    flops = tp_mlp.TPMLP.flops(M, hidden, f)
    te = None
    if e2e:  # end to end: the tokens from pinned host memory, this rank's rows of the result back
        hX = torch.empty((M, hidden), dtype=torch.float16, pin_memory=True)
        hX.copy_(X)
        hY = torch.empty((M // world, hidden), dtype=torch.float16, pin_memory=True)
        steps_e2e = max(3, min(steps, 10))
        barrier(world)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(steps_e2e):
            X.copy_(hX, non_blocking=True)
            hY.copy_(blk.forward(X), non_blocking=True)
        f1.record(stream)
        barrier(world)
        te = dist_max(f0.elapsed_time(f1) / 1e3, world)
    code = bwgemm.status()[0]
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        if rs is not None:
            torch.cuda.synchronize()
            rs.close()
            dist.barrier()
    del blk, X, W1, W2
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    step_ms, local_ms = t / steps * 1e3, t_local / steps * 1e3
    rec = {"M": M, "hidden": hidden, "mlp": f, "parallelism": f"tp{world}", "tflops": round(flops * steps / t / 1e12, 2),
           "ms_per_step": round(step_ms, 4), "steps": steps,
           "local_ms_per_step": round(local_ms, 4),
           "collective_alone_ms": round(t_coll / steps * 1e3, 4) if t_coll else None,
           "exposed_collective_ms": round(step_ms - local_ms, 4) if world > 1 else 0.0,
           "exposed_share": round((step_ms - local_ms) / step_ms, 4) if world > 1 else 0.0,
           "activation": "separate torch ops" if args.tp_unfused else "fused in the gateup epilogue",
           "collective": ("fused: partial tiles pushed into the owners' memory in the down GEMM's kernel"
                          if rs is not None else "NCCL reduce-scatter of fp32 partials") if world > 1 else "none",
           "clocks": clk.summary(), "device_status": code}
    if te is not None:
        rec["e2e"] = {"value": round(flops * steps_e2e / te / 1e12, 2), "unit": "TFLOP/s",
                      "h2d_bytes_per_step": M * hidden * 2, "d2h_bytes_per_step": M // world * hidden * 2}
    return rec


def graph_time(calls, G, seconds=0.1, rounds=3):
    """Seconds per call of `calls(i)` (i = 0 .. G-1), captured in a CUDA graph of G calls on a side stream and replayed
    for about `seconds` per round; the median of `rounds`, on CUDA events."""
    import torch

    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            for i in range(G):
                calls(i)
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    one = max(e0.elapsed_time(e1) / 1e3, 1e-6)
    reps = max(1, int(seconds / one))
    times = []
    for _ in range(rounds):
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / 1e3 / (reps * G))
    del g
    return statistics.median(times)


def decode(args, hbm_gbs):
    """the four weights of a Llama-3-70B layer at M = 1, 8, 16, 32, 64 tokens, through the rung
    (bw_gemm_f16 serves any M), against torch.matmul (cuBLAS); CUDA graphs on 3 rotating input sets (every weight's
    three copies exceed the 126 MB L2).  Bound by HBM: GB/s = 2 (MK + KN + MN) bytes per call over its time, and the
    fraction of the measured copy bandwidth."""
    import torch

    import bwgemm
    from shapes import DECODE_M, DECODE_WEIGHTS

    out = {}
    for wname, N, K in DECODE_WEIGHTS:
        Bs = make_sets(1, N, K, seed=N + K)[1]
        for M in DECODE_M:
            As = make_sets(M, 1, K, seed=M)[0]
            C = torch.empty((M, N), dtype=torch.float16, device="cuda")
            bwgemm.gemm(As[0], Bs[0], C)
            torch.matmul(As[0], Bs[0], out=C)
            torch.cuda.synchronize()
            G = 30
            t = graph_time(lambda i: bwgemm.gemm(As[i % 3], Bs[i % 3], C), G)
            tc = graph_time(lambda i: torch.matmul(As[i % 3], Bs[i % 3], out=C), G)
            gbs = 2.0 * (M * K + K * N + M * N) / t / 1e9
            out[f"{wname}_m{M}"] = {"M": M, "N": N, "K": K, "us": round(t * 1e6, 2), "gbs": round(gbs, 1),
                                    "frac_hbm": round(gbs / hbm_gbs, 4), "cublas_us": round(tc * 1e6, 2),
                                    "ratio_vs_cublas": round(tc / t, 4)}
            del As, C
        del Bs
        torch.cuda.empty_cache()
    fr = [v["frac_hbm"] for v in out.values()]
    return {"shapes": out, "hbm_gbs_peak": hbm_gbs, "min_frac_hbm": min(fr),
            "geomean_frac_hbm": round(math.exp(sum(map(math.log, fr)) / len(fr)), 4),
            "reference": "torch.matmul fp16 (cuBLAS heuristic); CUDA graphs of 30 calls, 3 rotating input sets"}


def sustained(args, A, B, C, local, seconds):
    """Config 1 back to back for `seconds` (the step of a long run under the 1 kW power cap, not the driver's short
    burst): TFLOP/s on CUDA events over the whole window, with the SM clock sampled during it."""
    import torch

    import bwgemm

    M, K = A[0].shape
    N = B[0].shape[1]
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(20):
        bwgemm.gemm(A[i % 3], B[i % 3], C)
    e1.record(stream)
    torch.cuda.synchronize()
    n = max(20, int(seconds / (e0.elapsed_time(e1) / 1e3 / 20)))
    with ClockSampler(local) as clk:
        e0.record(stream)
        for i in range(n):
            bwgemm.gemm(A[i % 3], B[i % 3], C)
        e1.record(stream)
        torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3
    return {"value": round(2.0 * M * N * K * n / t / 1e12, 2), "unit": "TFLOP/s", "calls": n,
            "seconds": round(t, 3), "ms_per_call": round(t / n * 1e3, 5), "clocks": clk.summary()}


def run_tp_mlp(args):
    """the MLP block of a Llama-3-70B layer (hidden 8192, MLP 28672) over the GPUs, Megatron
    tensor parallelism: gateup column-parallel and down row-parallel through the rung's GEMMs, the fp32 partials of
    down reduced by an NCCL reduce-scatter (tp_mlp.py), or down and the reduce-scatter fused (--tp-fused-rs).  Total
    work fixed: strong scaling."""
    import bwgemm

    rank, world, local = dist_setup(args)
    rec = tp_mlp_measure(args, rank, world, local, fused_rs=args.tp_fused_rs)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({
            "metric": "TFLOP/s of the tensor-parallel MLP block (gateup + down + reduce-scatter), BASELINE config 4",
            "value": rec["tflops"], "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": rec["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
            "data": "synthetic: seeded uniform tokens and weights",
            "config": {"workload": f"tp_mlp M={rec['M']} hidden={rec['hidden']} mlp={rec['mlp']}", "M": rec["M"],
                       "parallelism": f"tp{world}", "activation": rec["activation"],
                       "library": os.path.basename(bwgemm.LIB_PATH), "collective": rec["collective"]},
            "clocks": rec["clocks"], "gpu_launches": 2 * args.steps, "device_status": rec["device_status"],
            "local_ms_per_step": rec["local_ms_per_step"], "exposed_collective_ms": rec["exposed_collective_ms"],
            "e2e": rec.get("e2e"),
        }), flush=True)


def e2e_pipelined(bwgemm, hA, hB, dA, dB, C0, steps):
    """Device seconds of `steps` GEMMs fed from pinned host buffers, pipelined over two device slots: on a copy stream
    the host -> device copies of step i's A and B (after the GEMM that last read the slot), on the compute stream the
    GEMM (after those copies and after the device -> host copy that last read the slot's C), on a second copy stream
    the device -> host copy of its C.  The timed region opens on the compute stream before the first copy and closes
    after both copy streams have drained into it."""
    import torch

    st = torch.cuda.current_stream()
    cs, ds = torch.cuda.Stream(), torch.cuda.Stream()
    dC = [C0, torch.empty_like(C0)]
    hC = [torch.empty(C0.shape, dtype=C0.dtype, pin_memory=True) for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]   # the slot's inputs are on the device
    ev_mm = [torch.cuda.Event() for _ in range(2)]   # the slot's GEMM is done: inputs free, C ready
    ev_out = [torch.cuda.Event() for _ in range(2)]  # the slot's C is on the host: C free

    def run(n, start):
        cs.wait_event(start)
        ds.wait_event(start)
        for i in range(n):
            j = i % 2
            with torch.cuda.stream(cs):
                if i >= 2:
                    cs.wait_event(ev_mm[j])
                dA[j].copy_(hA, non_blocking=True)
                dB[j].copy_(hB, non_blocking=True)
                ev_in[j].record(cs)
            st.wait_event(ev_in[j])
            if i >= 2:
                st.wait_event(ev_out[j])
            bwgemm.gemm(dA[j], dB[j], dC[j], stream=st)
            ev_mm[j].record(st)
            with torch.cuda.stream(ds):
                ds.wait_event(ev_mm[j])
                hC[j].copy_(dC[j], non_blocking=True)
                ev_out[j].record(ds)
        st.wait_stream(cs)
        st.wait_stream(ds)

    torch.cuda.synchronize()
    s0 = torch.cuda.Event()
    s0.record(st)
    run(2, s0)  # warm-up of the three streams
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(st)
    run(steps, f0)
    f1.record(st)
    f1.synchronize()
    torch.cuda.synchronize()
    return f0.elapsed_time(f1) / 1e3


def run_ours(args):
    import torch

    import bwgemm

    rank, world, local = dist_setup(args)
    M, N, K = WORKLOADS[args.workload]
    flops_rank = 2.0 * M * N * K
    A, B = make_sets(M, N, K, seed=1234 + rank)
    C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    stream = torch.cuda.current_stream()
    for i in range(max(3, args.warmup)):
        bwgemm.gemm(A[i % 3], B[i % 3], C, variant=args.variant)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(world)
        e0.record(stream)
        for i in range(args.steps):
            bwgemm.gemm(A[i % 3], B[i % 3], C, variant=args.variant)
        e1.record(stream)
        barrier(world)
    t_rank = e0.elapsed_time(e1) / 1e3
    t = dist_max(t_rank, world)
    code = bwgemm.status()[0]
    value = flops_rank * world * args.steps / t / 1e12
    ms_per_step = t / args.steps * 1e3

    # end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        hA = torch.empty((M, K), dtype=torch.float16, pin_memory=True)
        hB = torch.empty((K, N), dtype=torch.float16, pin_memory=True)
        hC = torch.empty((M, N), dtype=torch.float16, pin_memory=True)
        hA.copy_(A[0])
        hB.copy_(B[0])
        dA, dB = A[1], B[1]
        steps_e2e = max(3, min(args.steps, 20))
        for _ in range(2):
            dA.copy_(hA, non_blocking=True)
            dB.copy_(hB, non_blocking=True)
            bwgemm.gemm(dA, dB, C)
            hC.copy_(C, non_blocking=True)
        barrier(world)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(steps_e2e):
            dA.copy_(hA, non_blocking=True)
            dB.copy_(hB, non_blocking=True)
            bwgemm.gemm(dA, dB, C)
            hC.copy_(C, non_blocking=True)
        f1.record(stream)
        barrier(world)
        te = dist_max(f0.elapsed_time(f1) / 1e3, world)
        serial = round(flops_rank * world * steps_e2e / te / 1e12, 2)
        e2e = {"value": serial, "unit": "TFLOP/s",
               "h2d_bytes_per_step": (M * K + K * N) * 2, "d2h_bytes_per_step": M * N * 2,
               "steps": steps_e2e, "path": "bwgemm.gemm (ctypes -> bw_gemm_f16) with pinned host buffers, "
                                           "copies and GEMM in order on one stream"}
        # the same steps pipelined as a serving loop runs them: step i + 1's inputs come in on one copy stream and
        # step i - 1's C goes out on another while step i's GEMM runs (host -> device and device -> host use their own
        # copy engines); every step still moves all its bytes inside the timed region
        barrier(world)
        tp_rank, err = math.inf, "failed on another rank"
        try:
            tp_rank = e2e_pipelined(bwgemm, hA, hB, [A[1], A[2]], [B[1], B[2]], C, steps_e2e)
        except Exception as exc:  # the in-order number above stands
            err = f"{type(exc).__name__}: {exc}"[:200]
        tp = dist_max(tp_rank, world)  # every rank joins, whatever happened on it
        if math.isfinite(tp):
            h2d_gbs = (M * K + K * N) * 2 * steps_e2e / tp / 1e9  # each rank's host -> device rate over the steps
            e2e.update({"value": round(flops_rank * world * steps_e2e / tp / 1e12, 2), "serial_value": serial,
                        "path": "bwgemm.gemm (ctypes -> bw_gemm_f16) with pinned host buffers; step i + 1's "
                                "host -> device copies and step i - 1's device -> host copy overlap step i's GEMM "
                                "(three streams, two device slots)",
                        "h2d_gbs_per_rank": round(h2d_gbs, 1),
                        "bound": ("host -> device copies (the GEMM takes %.0f%% of a step): the ranks share the host's "
                                  "pinned-memory bandwidth" % (100.0 * t / args.steps / (tp / steps_e2e)))
                                 if t / args.steps < 0.8 * tp / steps_e2e else "the GEMM"})
        else:
            e2e["pipelined_error"] = err

    pk, pk_kind = peaks()
    achieved = flops_rank / (t_rank / args.steps) / 1e12
    traffic = profile_traffic(args.workload)
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["bf16_tflops"], 4), "traffic": traffic,
                "peak_kind": f"{pk_kind}: dense 16-bit GEMM (cuBLAS bf16 8192^3, burst)",
                "algorithmic_bytes_per_launch": (M * K + K * N + M * N) * 2}
    result = {
        "metric": "TFLOP/s of C = A.B (fp16 in, fp32 accumulate, fp16 out), BASELINE config 1",
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 (fp32 accumulate)", "data": "synthetic: seeded uniform [-1, 1) fp16",
        "config": {"workload": f"{args.workload} {M}x{N}x{K}" + (f" per rank (column shards, N total {N * world})"
                                                                  if world > 1 else ""),
                   "M": M, "N": N, "K": K, "variant": args.variant, "library": os.path.basename(bwgemm.LIB_PATH),
                   "l2": "3 rotating input sets (%.0f MB) > 126 MB L2, no flush" % (3 * (M * K + K * N) * 2 / 1e6),
                   "parallelism": f"column shards x{world}, no collective" if world > 1 else "1 GPU"},
        "clocks": clk.summary(), "gpu_launches": args.steps, "device_status": code,
        "roofline": roofline, "e2e": e2e,
    }
    default_run = args.workload == "config1" and args.variant == 0
    if world == 1 and default_run and not args.no_sustained:
        result["sustained"] = sustained(args, A, B, C, local, args.sustained_seconds)
    if rank == 0 and world == 1 and not args.no_cpu:
        result["cpu_baseline"] = cpu_baseline(M, N, K, args.cpu_seconds)
    del A, B
    torch.cuda.empty_cache()
    if world == 1 and (args.sweep or (default_run and not args.no_sweep)):
        result["sweep"] = sweep(args)
    if world == 1 and default_run and not args.no_decode:
        result["decode"] = decode(args, pk["hbm_gbs"])
    if default_run and not args.no_tp:
        # BASELINE config 4 at every N: the row-parallel collective the column shards above never exercise
        tp = tp_mlp_measure(args, rank, world, local, fused_rs=False, steps=min(args.steps, 20), e2e=False)
        if rank == 0:
            result["tp_mlp"] = tp
        if world > 1:  # the same block with down and the reduce-scatter in one kernel per rank (bw_gemm_f16_rs)
            tpf = tp_mlp_measure(args, rank, world, local, fused_rs=True, steps=min(args.steps, 20), e2e=False)
            if rank == 0:
                result["tp_mlp_fused_rs"] = tpf
    if rank == 0:
        head = {}
        if "sweep" in result:
            head["geomean_ratio_vs_cublas_17"] = result["sweep"]["geomean_ratio_vs_cublas_17"]
        if "sustained" in result:
            head["sustained_tflops"] = result["sustained"]["value"]
        if "decode" in result:
            head["decode_min_frac_hbm"] = result["decode"]["min_frac_hbm"]
        if "tp_mlp" in result:
            head["tp_mlp_tflops"] = result["tp_mlp"]["tflops"]
        if "tp_mlp_fused_rs" in result:
            head["tp_mlp_fused_rs_tflops"] = result["tp_mlp_fused_rs"]["tflops"]
        result["headline"] = head
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


# ------------------------------------------------------------------------------------------------------ reference arm
def run_reference(args):
    """The reference's CPU GEMM path on the host cores, in bounded row samples of the same workload."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle import oracle

    # tp_mlp: the block's gateup GEMM (M x 57344 x 8192) stands for it on the host
    M, N, K = WORKLOADS[args.workload] if args.workload != "tp_mlp" else (args.tp_m, 57344, 8192)
    threads = os.cpu_count() or 1
    budget = 90.0  # seconds for warm-up + timed steps
    per_step = budget / max(1, args.steps + args.warmup)
    rows0 = min(M, threads)
    A, B = oracle.judge_inputs(rows0, N, K)
    t0 = time.perf_counter()
    oracle.gemm_f64(A, B, threads=threads)
    rate = rows0 / max(time.perf_counter() - t0, 1e-6)  # rows per second
    rows = int(max(1, min(M, rate * per_step)))
    A, B = oracle.judge_inputs(rows, N, K)
    for _ in range(args.warmup):
        oracle.gemm_f64(A, B, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.gemm_f64(A, B, threads=threads)
    t = time.perf_counter() - t0
    value = 2.0 * rows * N * K * args.steps / t / 1e12
    sample = f"{rows} of {M} rows of {M}x{N}x{K} per step, fp64 i-k-j (oracle/oracle.c restating hopper/verif.cu:171-178)"
    print(json.dumps({
        "impl": "reference", "metric": "TFLOP/s of C = A.B (fp16 in, fp32 accumulate, fp16 out), BASELINE config 1",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f64 accumulate of fp16 inputs", "data": "synthetic: the judge's fill",
        "config": {"workload": f"{args.workload} {M}x{N}x{K}", "M": M, "N": N, "K": K},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse()
    if args.shape:
        M, N, K = (int(x) for x in args.shape.lower().split("x"))
        WORKLOADS[args.shape] = (M, N, K)
        args.workload = args.shape
    if args.profile_arm:
        profile_call(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "tp_mlp":
        run_tp_mlp(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
