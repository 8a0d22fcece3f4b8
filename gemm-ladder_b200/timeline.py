"""Per-block timeline of one launch of the rung's kernel, from the library built with the timeline compiled in
(``python gemm-ladder_b200/build.py --trace`` -> lib/libbwgemm_trace.so).  Needs a GPU.

    python gemm-ladder_b200/timeline.py MxNxK[:variant] [...]   [--dump] [--next]

For each shape: 5 calls, then one timed call whose per-block %globaltimer stamps are read back (bw_trace_read).
Printed, relative to the earliest block's entry: set-up done, the MMA issuer's first full stage and last commit, the
epilogue's end, the exit (min / p10 / median / p90 / max over the blocks); the MMA issuer's waits for full stages and
for a free accumulator; and, by kind of each block's last segment (a whole tile, a split tile's writer, or its
reducer), when its accumulator was ready, when it decided, and when its reduction copied and summed the partials.
--dump adds the raw stamps of the 8 slowest blocks.  --next times the library with the options not yet measured
(build.py --next), the timeline compiled in (lib/libbwgemm_next_trace.so).

The stamps (csrc/gemm_kernel.cuh, BW_TRACE_AT / BW_TRACE_VAL), per block:
  0 entry, 1 set-up done, 2 first full stage, 3 last MMA commit, 4 epilogue done, 5 exit, 6 the last segment's
  accumulator ready, 7 split decision, 8 kind | partials << 8 | segment << 16, 9 reduction start, 10 partials copied,
  11 partials summed, 12 ns waiting on full stages, 13 ns waiting on a free accumulator, 14 K-blocks issued.
"""
import ctypes
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import bwgemm  # noqa: E402
import build  # noqa: E402

SLOTS = 16
KINDS = {0: "whole", 1: "reducer", 2: "reducer (fast)", 3: "writer"}


def load(next_options=False):
    lib = ctypes.CDLL(build.build(trace=True, next_options=next_options))
    vp, i = ctypes.c_void_p, ctypes.c_int
    lib.bw_gemm_plan.argtypes = [i, i, i, i, i, ctypes.POINTER(bwgemm.Plan)]
    lib.bw_gemm_plan.restype = i
    lib.bw_gemm_f16_variant.argtypes = [vp, vp, vp, i, i, i, vp, i]
    lib.bw_gemm_f16_variant.restype = i
    lib.bw_trace_read.argtypes = [ctypes.POINTER(ctypes.c_ulonglong), i]
    lib.bw_trace_read.restype = i
    return lib


def timeline(lib, M, N, K, variant=0, dump=False):
    A = (torch.rand(M, K, device="cuda") * 2 - 1).half()
    B = (torch.rand(K, N, device="cuda") * 2 - 1).half()
    C = torch.empty(M, N, device="cuda", dtype=torch.float16)
    q = bwgemm.Plan()  # the rule of the library being timed
    bwgemm.check(lib.bw_gemm_plan(M, N, K, torch.cuda.get_device_properties(0).multi_processor_count, variant,
                                  ctypes.byref(q)))
    plan = q.as_dict()
    call = lambda: lib.bw_gemm_f16_variant(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, None, variant)  # noqa
    for _ in range(5):
        if call():
            raise RuntimeError(bwgemm.lib().bw_last_error_string().decode())
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    call()
    e1.record()
    torch.cuda.synchronize()
    g = plan["grid"]
    buf = (ctypes.c_ulonglong * (g * SLOTS))()
    if lib.bw_trace_read(buf, g):
        raise RuntimeError("bw_trace_read failed")
    raw = np.array(buf, dtype=np.uint64).reshape(g, SLOTS)
    t0 = raw[:, 0].astype(np.float64).min()
    rel = lambda k: (raw[:, k].astype(np.float64) - t0) / 1e3  # noqa: E731  us after the first entry
    print(f"{M}x{N}x{K} v{variant}: event {e0.elapsed_time(e1) * 1e3:.1f} us, grid {g}, kernel {plan['kernel']}, "
          f"bn {plan['bn']}, whole tiles {plan['dp_tiles']}, split tiles {plan['sk_tiles']} "
          f"(splits {plan['splits']}, ksplit {plan['ksplit']})")
    kind = raw[:, 8] & 0xFF
    for kd, name in KINDS.items():
        sel = kind == kd
        if not sel.any():
            continue
        line = f"   last segment {name:15s} n={sel.sum():3d}: accumulator ready med {np.median(rel(6)[sel]):7.2f}"
        if kd:  # only split segments stamp the decision
            line += f" | decided {np.median(rel(7)[sel]):7.2f}"
        if kd in (1, 2):
            line += f" | copied {np.median(rel(10)[sel]):7.2f} | summed {np.median(rel(11)[sel]):7.2f}"
        line += f" | epilogue done med {np.median(rel(4)[sel]):7.2f} max {rel(4)[sel].max():7.2f} us"
        print(line)
    mma = raw[:, 14] > 0  # the blocks whose thread issued MMAs (a pair's leader; every block otherwise)
    if mma.any():
        span = (raw[mma, 3].astype(np.float64) - raw[mma, 2].astype(np.float64)) / 1e3
        wf, wa, nk = raw[mma, 12] / 1e3, raw[mma, 13] / 1e3, raw[mma, 14].astype(np.float64)
        print(f"   MMA issuer: mainloop med {np.median(span):7.2f} us; waits on full stages med {np.median(wf):6.2f} us "
              f"({np.median(wf / span) * 100:.1f} %), on a free accumulator med {np.median(wa):5.2f} us; "
              f"{np.median(nk):.0f} K-blocks, {np.median(span / nk) * 1e3:.0f} ns each")
    for k, name in [(1, "set-up done"), (2, "first stage"), (3, "last MMA"), (4, "epilogue done"), (5, "exit")]:
        col = rel(k)
        if k in (2, 3):  # only MMA-issuing blocks stamp these
            col = col[mma]
        q = np.percentile(col, [0, 10, 50, 90, 100])
        print(f"   {name:14s} min {q[0]:7.2f}  p10 {q[1]:7.2f}  med {q[2]:7.2f}  p90 {q[3]:7.2f}  max {q[4]:7.2f} us")
    if dump:
        for b in np.argsort(-rel(4))[:8]:
            print(f"   block {b:3d}: " + " ".join(f"{rel(k)[b]:8.2f}" for k in range(6)) +
                  f" | kind {KINDS.get(int(kind[b]), '?')}, partials {int(raw[b, 8] >> 8) & 0xFF}")


def main(argv):
    dump = "--dump" in argv
    specs = [a for a in argv if not a.startswith("--")]
    if not specs:
        print(__doc__)
        return 2
    torch.cuda.set_device(0)
    lib = load("--next" in argv)
    for spec in specs:
        shape, _, var = spec.partition(":")
        M, N, K = (int(x) for x in shape.lower().split("x"))
        timeline(lib, M, N, K, int(var or 0), dump)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
