"""Generate the golden fixtures that pin the oracle to the reference (test infrastructure).

Runs the reference's own Hopper host emulator (oracle/_ref/emu_dump, built by ``make -f oracle/ref.mk emu_dump`` from
the reference's hopper/emu/emu.cpp where it lies) for a few of its step-7 kernels at shapes each kernel takes, on the
emulator's own inputs (LCG seed 7, hopper/emu/emu.cpp:2568-2570), and keeps, per case:

  a_sha256, b_sha256   hashes of the fp16 bits of A and B as the reference drew them (the oracle's generator must
                       reproduce them bit for bit),
  c                    the fp16 bits of C written by the reference's Hopper kernel (the sm_100a path must agree with
                       it within the per-element tolerance),
  ref_idx, ref_val     the reference's fp64 result at 4096 fixed positions, ref_max its max |ref|, ref_sum its sum
                       (the oracle's fp64 GEMM must reproduce them to rounding).

Usage (needs the reference tree, so only in the build container):
    python tests/golden/make_golden.py
"""
import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
DUMP = os.path.join(ROOT, "oracle", "_ref", "emu_dump")

# (name, reference kernel label, M, N, K): one case per class of the reference's step-7 rule, plus the CPU config
# (256 x 256 x 512).
CASES = [
    ("cfg0_256x256x512", "step7 v0: 7c 6c, 3 blocks", 256, 256, 512),
    ("bands16_16x1024x1024", "step7 v0: bands 16 rows J=1 alone", 16, 1024, 1024),
    ("bands16w_16x2048x320", "step7 v0: 7b bands 16 rows J=2 in clusters of 8", 16, 2048, 320),
    ("bands64_80x512x192", "step7 v0: 7a bands 64 rows in pairs", 80, 512, 192),
    ("bands128_112x256x448", "step7 v0: 7d bands 128 rows", 112, 256, 448),
    ("tile128_208x512x192", "step7 v0: 128x128, 3 blocks", 208, 512, 192),
    ("tile7e_144x640x320", "step7 v0: 7e 128x320 alone, 3 blocks", 144, 640, 320),
    ("pairs_128x1024x448", "step7 v0: step 5's tile in pairs, 2 clusters", 128, 1024, 448),
]
N_SAMPLES = 4096


def main():
    if not os.path.exists(DUMP):
        subprocess.check_call(["make", "-f", os.path.join(ROOT, "oracle", "ref.mk"), "emu_dump"])
    with tempfile.TemporaryDirectory() as tmp:
        for name, label, m, n, k in CASES:
            prefix = os.path.join(tmp, name)
            subprocess.check_call([DUMP, label, str(m), str(n), str(k), prefix])
            a = np.fromfile(prefix + ".A.u16", dtype=np.uint16)
            b = np.fromfile(prefix + ".B.u16", dtype=np.uint16)
            c = np.fromfile(prefix + ".C.u16", dtype=np.uint16)
            ref = np.fromfile(prefix + ".ref.f64", dtype=np.float64)
            assert a.size == m * k and b.size == k * n and c.size == m * n and ref.size == m * n
            rng = np.random.default_rng(20261201)
            idx = np.sort(rng.choice(m * n, size=min(N_SAMPLES, m * n), replace=False)).astype(np.int64)
            out = os.path.join(HERE, name + ".npz")
            np.savez_compressed(
                out,
                label=np.array(label),
                shape=np.array([m, n, k], dtype=np.int64),
                seed=np.array(7, dtype=np.int64),
                a_sha256=np.array(hashlib.sha256(a.tobytes()).hexdigest()),
                b_sha256=np.array(hashlib.sha256(b.tobytes()).hexdigest()),
                c=c.reshape(m, n),
                ref_idx=idx,
                ref_val=ref[idx],
                ref_max=np.array(np.abs(ref).max()),
                ref_sum=np.array(ref.sum()),
            )
            print(f"{name}: {label} {m}x{n}x{k} -> {os.path.relpath(out, ROOT)}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
