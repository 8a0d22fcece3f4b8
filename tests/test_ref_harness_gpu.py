"""The reference's own harnesses, built where they lie (oracle/ref.mk) and linked with this rung's candidate
(gemm-ladder_b200/blackwell/candidate.cu), run on the B200:

  verif_bw   hopper/verif.cu: its 26 edge shapes, each variant against its fp64 CPU reference (max error / max |ref|
             <= 2e-3), 8 calls compared bit for bit, candidate_dirty() == 0 after each (hopper/verif.cu:186-229); its
             last line is "OK (tolerance 2e-3)" and its exit status 0.
  probe_bw   probe/probe.cu: the interleaved arms v0, twin and v1 on one shape, each checked against cublasGemmEx
             before and after its timing (probe/probe.cu:206-225; a line marked WRONG fails).

The binaries are built here by __graft_entry__.build() (make -f oracle/ref.mk) when the reference tree is present, and
travel prebuilt; without them the tests skip."""
import os
import subprocess

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

REF_BIN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")


def _binary(name):
    path = os.path.join(REF_BIN, name)
    if not os.path.exists(path):
        pytest.skip(f"{path} not built (make -f oracle/ref.mk needs the reference tree)")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return path


def test_reference_verif_accepts_the_rung():
    out = subprocess.run([_binary("verif_bw")], capture_output=True, text=True, timeout=600,
                         env=dict(os.environ, GEMM_LADDER_BUDGET="540"))
    lines = out.stdout.strip().splitlines()
    assert out.returncode == 0 and lines and lines[-1] == "OK (tolerance 2e-3)", out.stdout[-3000:] + out.stderr[-2000:]
    assert not any("FAILED" in line for line in lines), [line for line in lines if "FAILED" in line][:5]
    assert sum(line.startswith("shape ") for line in lines) >= 26


def test_reference_probe_runs_the_rung_arms():
    out = subprocess.run([_binary("probe_bw"), "512", "10240", "8192", "energy", "v0,twin,v1", "0.1", "2"],
                         capture_output=True, text=True, timeout=300)
    if out.returncode == 2 and "NVML energy unavailable" in out.stdout:
        pytest.skip("the probe needs NVML's energy counter")
    arms = [line for line in out.stdout.splitlines() if line.startswith("ARM ")]
    assert out.returncode == 0 and len(arms) == 3, out.stdout[-3000:] + out.stderr[-2000:]
    assert not any("WRONG" in line for line in arms), arms
