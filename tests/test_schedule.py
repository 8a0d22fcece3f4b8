"""The rung's schedule and rule on the CPU: the same schedule.h the kernel runs, compiled with g++."""
import os
import subprocess

import pytest

from shapes import B200_EDGES, CONFIG1, DECODE_M, DECODE_WEIGHTS, JUDGE_B200, LADDER_4096, VERIF

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(ROOT, "gemm-ladder_b200", "csrc")


@pytest.fixture(scope="module", params=[(), ("BW_KSPLIT=1", "BW_SK_PART_WAVE=1", "BW_PAIR_WIDE=1", "BW_SWAP_PAIR=1")],
                ids=["library", "not_yet_measured"])
def checker(request, tmp_path_factory):
    """The checker over the library's rule, and over the rule with the options built but not yet measured (the K split
    on clusters of 2 to 8, stream-K over a part wave of pair tiles)."""
    exe = str(tmp_path_factory.mktemp("sched") / "schedule_check")
    subprocess.check_call(["g++", "-std=c++17", "-O2", "-Wall", *[f"-D{d}" for d in request.param], f"-I{CSRC}",
                           f"-I{os.path.join(ROOT, 'include')}", os.path.join(HERE, "schedule_check.cpp"), "-o", exe])
    return exe


def all_shapes():
    out = [(m, n, k) for _, m, n, k in JUDGE_B200] + [LADDER_4096[1:], CONFIG1[1:]] + list(VERIF) + list(B200_EDGES)
    out += [(m, n, k) for _, n, k in DECODE_WEIGHTS for m in DECODE_M]
    return out


@pytest.mark.parametrize("variant", range(8))
@pytest.mark.parametrize("sms", [148, 132, 7, 1])
def test_schedule_covers_every_kblock_once(checker, variant, sms):
    args = []
    for m, n, k in all_shapes():
        args += [str(m), str(n), str(k), str(sms), str(variant)]
    r = subprocess.run([checker, *args], capture_output=True, text=True)
    faults = [l for l in r.stdout.splitlines() if not l.startswith("OK")]
    assert r.returncode == 0 and not faults, "\n".join(faults[:5])


def test_schedule_exhaustive_small(checker):
    # every M (multiple of 16 up to 512), N (multiple of 64 up to 1024) at a few K and SM counts
    args = []
    for m in range(16, 513, 16):
        for n in range(64, 1025, 64):
            for k in (64, 192, 1024):
                for sms in (148, 5):
                    args += [str(m), str(n), str(k), str(sms), "0"]
    r = subprocess.run([checker, *args], capture_output=True, text=True)
    faults = [l for l in r.stdout.splitlines() if not l.startswith("OK")]
    assert r.returncode == 0 and not faults, "\n".join(faults[:5])
