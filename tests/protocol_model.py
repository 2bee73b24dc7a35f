"""Shared machinery for the barrier-protocol models of the tensor-core kernels (CPU only).

A kernel's warp roles are restated as Python generators that yield the mbarrier waits of the
kernel (``Wait(bar, parity, m)``: the parity expression the kernel uses and the completion
index ``m`` it means) and arrive on barriers directly.  ``schedule`` runs the roles and an
in-order tensor pipe under a seeded random interleaving and checks mbarrier parity semantics:
a wait passes when the barrier's current phase parity differs from the waited parity, and it
must pass exactly on completion ``m + 1`` (never one phase early or after an overrun); an
arrival must belong to the barrier's current phase.  Buffer hazards are asserted by the
models themselves where the pipe, the copies and the warps touch shared buffers.
"""
import random


class Bar:
    """An mbarrier: ``count`` arrivals complete a phase; ``done`` counts completed phases."""

    def __init__(self, name, count):
        self.name, self.count, self.pending, self.done = name, count, count, 0

    def arrive(self, phase):
        assert phase == self.done, (self.name, "arrival for phase", phase, "current", self.done)
        self.pending -= 1
        if self.pending == 0:
            self.done += 1
            self.pending = self.count

    def passes(self, parity):
        return (self.done & 1) != parity

    def test(self, parity):  # mbarrier.test_wait: non-blocking
        return self.passes(parity)


class Wait:
    def __init__(self, bar, parity, m):
        assert parity == (m & 1), (bar.name, "parity", parity, "for completion", m)
        self.bar, self.parity, self.m = bar, parity, m


class Until:
    """A wait on something other than an mbarrier (e.g. a bulk-copy group count): passes when
    ``predicate()`` holds."""

    def __init__(self, predicate, name):
        self.predicate, self.name = predicate, name

    def passes(self):
        return self.predicate()


def _ready(w):
    return w is None or (w.passes() if isinstance(w, Until) else w.bar.passes(w.parity))


def schedule(roles, pipe, pipe_step, seed, max_steps=10_000_000):
    """Run generator ``roles`` (name -> generator) and the FIFO ``pipe`` (executed by
    ``pipe_step``) in a seeded random order until every role finishes and the pipe is empty."""
    rnd = random.Random(seed)
    waiting = {k: None for k in roles}
    finished = set()
    for _ in range(max_steps):
        runnable = [k for k in roles if k not in finished and _ready(waiting[k])]
        if pipe:
            runnable.append(None)
        if not runnable:
            if len(finished) == len(roles):
                return
            raise AssertionError("deadlock: " + ", ".join(
                (f"{k} waits {w.name}" if isinstance(w, Until) else f"{k} waits {w.bar.name} m={w.m} done={w.bar.done}")
                for k, w in waiting.items() if k not in finished))
        k = rnd.choice(runnable)
        if k is None:
            pipe_step(pipe.pop(0))
            continue
        w = waiting[k]
        if isinstance(w, Wait):
            assert w.bar.done == w.m + 1, (k, w.bar.name, "passes at", w.bar.done, "meant", w.m)
        waiting[k] = None
        try:
            nw = next(roles[k])
            if isinstance(nw, Wait):
                assert nw.bar.done <= nw.m + 1, (k, nw.bar.name, "phase overrun", nw.bar.done, nw.m)
            waiting[k] = nw
        except StopIteration:
            finished.add(k)
    raise AssertionError("step limit")
