"""bench.py's pipelined end-to-end loop (e2e_pipelined) on the CPU: torch's streams and events replaced by fakes that log
what each stream is given, and the log checked as the GPU would order it.  Each stream runs its operations in order;
a wait on an event runs after the operation that recorded it.  Checked: a step's GEMM runs after its inputs' copies
and before the next copies into the same slot; a step's copy of C runs after its GEMM and before the next GEMM into
the same C; the timed region opens before the first copy and closes after the last one of every stream."""
import contextlib
import os
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import bench  # noqa: E402

torch = pytest.importorskip("torch")


class Stream:
    def __init__(self, name):
        self.name, self.log = name, []  # log: (kind, detail, dependency or None)

    def wait_event(self, ev):
        self.log.append(("wait", ev.name, ev.at))

    def wait_stream(self, other):
        self.log.append(("wait", other.name, (other, len(other.log) - 1) if other.log else None))


class Event:
    def __init__(self, enable_timing=False):
        self.name, self.at = f"ev{id(self)}", None

    def record(self, stream):
        stream.log.append(("record", self.name, None))
        self.at = (stream, len(stream.log) - 1)

    def synchronize(self):
        pass

    def elapsed_time(self, other):
        return 1.0


class Buf:
    shape, dtype = (4, 4), torch.float16

    def __init__(self, name):
        self.name = name

    def copy_(self, src, non_blocking=False):
        CURRENT[0].log.append(("copy", self.name, None))


CURRENT = [None]


def happens_before(a, b):
    """True if operation a = (stream, index) runs before operation b on the GPU: b's stream runs its operations in
    order, and a wait runs after the operation it waits for; a precedes b if it is reached going back from b."""
    seen, todo = set(), [b]
    while todo:
        s, i = todo.pop()
        if (id(s), i) in seen:
            continue
        seen.add((id(s), i))
        preds = [(s, i - 1)] if i > 0 else []
        kind, _, dep = s.log[i]
        if kind == "wait" and dep is not None:
            preds.append(dep)
        for q in preds:
            if q[0] is a[0] and q[1] == a[1]:
                return True
            todo.append(q)
    return False


def test_the_pipelined_loop_orders_every_reuse_of_a_slot(monkeypatch):
    st = Stream("compute")
    made = iter(["copy_in", "copy_out"])
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a: st)
    monkeypatch.setattr(torch.cuda, "Stream", lambda: Stream(next(made)))
    monkeypatch.setattr(torch.cuda, "Event", Event)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a: None)
    hc = iter(["hC0", "hC1"])
    monkeypatch.setattr(torch, "empty_like", lambda t: Buf("C1"))
    monkeypatch.setattr(torch, "empty", lambda *a, **k: Buf(next(hc)))

    @contextlib.contextmanager
    def on(stream):
        old, CURRENT[0] = CURRENT[0], stream
        try:
            yield
        finally:
            CURRENT[0] = old

    monkeypatch.setattr(torch.cuda, "stream", on)

    class Gemm:
        @staticmethod
        def gemm(A, B, C, stream=None):
            stream.log.append(("gemm", (A.name, B.name, C.name), None))

    steps = 5
    t = bench.e2e_pipelined(Gemm, Buf("hA"), Buf("hB"), [Buf("A0"), Buf("A1")], [Buf("B0"), Buf("B1")], Buf("C0"),
                            steps)
    assert t == pytest.approx(1e-3)
    streams = {"compute": st}
    for s in (st,):
        for kind, name, dep in s.log:
            if dep is not None:
                streams[dep[0].name] = dep[0]
    cs, ds = streams["copy_in"], streams["copy_out"]

    def ops(s, kind, name=None):
        return [(s, i) for i, (k, n, _) in enumerate(s.log) if k == kind and (name is None or n == name or
                                                                               (k == "gemm" and name in n))]

    gemms = ops(st, "gemm")
    assert len(gemms) == 2 + steps  # two warm-up steps, then the timed ones
    for slot in (0, 1):
        a_copies, c_copies = ops(cs, "copy", f"A{slot}"), ops(ds, "copy", f"hC{slot}")
        slot_gemms = [g for g in gemms if st.log[g[1]][1][0] == f"A{slot}"]
        assert len(a_copies) == len(slot_gemms) == len(c_copies)
        for n, g in enumerate(slot_gemms):
            assert happens_before(a_copies[n], g), "a GEMM may read its inputs before they arrive"
            assert happens_before(g, c_copies[n]), "C may be copied out before its GEMM"
            if n + 1 < len(slot_gemms):
                assert happens_before(g, a_copies[n + 1]), "a slot's inputs may be overwritten while read"
                assert happens_before(c_copies[n], slot_gemms[n + 1]), "C may be overwritten before it is copied out"
    # the timed region: its start is the compute stream's record before the timed steps; its end, the last record
    records = ops(st, "record")
    end = records[-1]
    assert happens_before((cs, len(cs.log) - 1), end) and happens_before((ds, len(ds.log) - 1), end)
    start = [r for r in records if r[1] < gemms[2][1]][-1]
    timed_first_copy = ops(cs, "copy", "A0")[1]
    assert happens_before(start, timed_first_copy)


def _bench(*argv, env=None):
    import subprocess
    e = dict(os.environ, **(env or {}))
    return subprocess.run([sys.executable, os.path.join(os.path.dirname(HERE), "bench.py"), *argv], env=e,
                          capture_output=True, text=True, timeout=600)


def test_the_reference_arm_prints_its_line_on_the_cpu():
    """bench.py --impl reference times the reference's CPU path (the oracle's restatement) on the host cores and
    prints one JSON line with the contract's keys; it needs no GPU."""
    import json
    r = _bench("--impl", "reference", "--shape", "64x256x128", "--steps", "2", "--warmup", "1",
               env={"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    out = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in out, key
    assert out["impl"] == "reference" and out["steps"] == 2 and out["warmup"] == 1 and out["value"] > 0
    assert out["cpu_baseline"]["value"] == out["value"] and out["cpu_baseline"]["kind"] in ("port", "reference")
    assert out["e2e"] == {"value": out["value"], "unit": out["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_the_reference_arm_runs_on_rank_0_only():
    r = _bench("--impl", "reference", "--shape", "64x256x128", "--steps", "1", "--warmup", "1",
               env={"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0 and r.stdout.strip() == "", (r.stdout, r.stderr[-2000:])
