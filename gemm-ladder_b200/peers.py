"""Host-side failure detection between the steps of a multi-rank run (one process per GPU), without touching a GPU.

Every rank calls `gate(step)` before it launches the step's kernels and collectives.  The gate is a counter in the
process group's key-value store: a rank adds 1 and waits until every rank has reached the same step.  While it waits
it looks for the `failed` key, which a rank posts (`fail(reason)`) when it leaves early -- an exception between
steps, a bad input, an operator's stop.  So:

- a rank that fails and says so: the others raise PeerFailed at their next gate, before launching anything that
  would wait for it;
- a rank that dies without a word (killed, crashed): the others raise PeerTimeout once the gate's limit passes;
- a rank that passed the gate and then never joins a collective: the process group's own timeout ends that
  collective with an error -- give the group a short one (`init_process_group(..., timeout=...)`).

A rank only ever leaves between steps, with none of its kernels or collectives in flight.  The ranks then tear their
process group down; nothing here aborts a GPU kernel.
"""
import time

FAILED_KEY = "bwgemm/peers/failed"
GATE_KEY = "bwgemm/peers/gate"


class PeerFailed(RuntimeError):
    """Another rank posted a failure."""


class PeerTimeout(RuntimeError):
    """Not every rank reached a gate within its limit (a rank died without posting)."""


class PeerWatch:
    def __init__(self, store, rank, world, gate_timeout_s=30.0, poll_s=0.0005):
        self.store, self.rank, self.world = store, rank, world
        self.gate_timeout_s, self.poll_s = gate_timeout_s, poll_s
        self.passed = 0  # gates this rank has passed

    @classmethod
    def from_default_group(cls, **kw):
        """The watch over the default process group's store."""
        import torch.distributed as dist
        from torch.distributed import distributed_c10d

        return cls(distributed_c10d._get_default_store(), dist.get_rank(), dist.get_world_size(), **kw)

    def failure(self):
        """The posted failure ('rank r: reason'), or None."""
        if self.store.check([FAILED_KEY]):
            return self.store.get(FAILED_KEY).decode()
        return None

    def fail(self, reason):
        """Posts this rank's failure for the others (the first post stays)."""
        self.store.compare_set(FAILED_KEY, "", f"rank {self.rank}: {reason}")

    def check(self):
        """Raises PeerFailed if any rank posted a failure."""
        f = self.failure()
        if f is not None:
            raise PeerFailed(f)

    def gate(self, step=None):
        """Waits until every rank has reached this gate (the ranks' `passed` counts agree), a rank posts a failure
        (PeerFailed) or gate_timeout_s passes (PeerTimeout)."""
        self.check()
        target = self.world * (self.passed + 1)
        n = self.store.add(GATE_KEY, 1)
        t0 = time.monotonic()
        while n < target:
            self.check()
            if time.monotonic() - t0 > self.gate_timeout_s:
                raise PeerTimeout(f"rank {self.rank}: {target - n} rank(s) did not reach gate "
                                  f"{self.passed if step is None else step} within {self.gate_timeout_s} s")
            time.sleep(self.poll_s)
            n = self.store.add(GATE_KEY, 0)
        self.passed += 1
