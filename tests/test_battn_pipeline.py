"""Model check of k_battn's K/V pipeline protocol (csrc/q3_battn.cuh) on the CPU.

One producer thread streams chunk i into data stage i % kBaStages and arms
full barrier i % kBaFullBars; consumer warp w takes chunks w, w + 4, ... and
frees the stage on empty[i % kBaStages].  The model keeps the mbarrier rules
the kernel relies on -- a parity wait succeeds when the phase of that parity
is complete, which includes the phase before the pending one -- and lets TMA
copies land in any order.  Random schedules must never let a warp read a
stage before its chunk landed, refill a stage whose copy is in flight, or end
the CTA with a copy in flight.

The one-barrier-per-stage layout (full[i % kBaStages]) breaks under the same
model, so a failing schedule must be found for it; that is the check that the
model can see the aliasing at all.
"""
import pathlib
import random
import re

import pytest

HDR = pathlib.Path(__file__).resolve().parents[1] / "qwen3-iree_b200" / "csrc" / "q3_battn.cuh"


def _kernel_constants():
    src = HDR.read_text()
    stages = int(re.search(r"#define Q3_BA_STAGES (\d+)", src).group(1))
    warps = int(re.search(r"constexpr int kBaWarps = (\d+);", src).group(1))
    assert "kBaFullBars = ((kBaStages + kBaWarps - 1) / kBaWarps) * kBaWarps" in src
    return stages, warps, (stages + warps - 1) // warps * warps


class Barrier:
    def __init__(self, count=1):
        self.count, self.pending, self.tx, self.phase = count, count, 0, 0

    def done(self, parity):  # mbarrier.try_wait.parity
        return (self.phase & 1) != parity

    def _maybe_close(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self, tx=0):
        self.pending -= 1
        self.tx += tx
        assert self.pending >= 0, "more arrivals than the phase expects"
        self._maybe_close()

    def complete_tx(self, n):
        self.tx -= n
        self._maybe_close()


class Violation(AssertionError):
    pass


def run_cta(nch, stages, warps, nbars, rng, old_drain=False):
    full = [Barrier() for _ in range(nbars)]
    empty = [Barrier() for _ in range(stages)]
    content = [None] * stages      # chunk whose bytes a stage holds
    inflight = []                  # (stage, barrier, chunk)

    def producer():
        issued = 0
        for i in range(nch):
            st = i % stages
            if i >= stages:
                par = ((i // stages) - 1) & 1
                while not empty[st].done(par):
                    yield
            if any(c[0] == st for c in inflight):
                raise Violation(f"stage {st} refilled with chunk {i} while a copy is in flight")
            fb = full[i % nbars]
            fb.arrive(tx=2)
            inflight.append((st, fb, i))  # K tile
            inflight.append((st, fb, i))  # V tile
            issued = i + 1
            yield
        if old_drain:
            waits = [(st, ((issued - 1 - st) // stages) & 1) for st in range(min(stages, issued))]
        else:
            waits = [(i % nbars, (i // nbars) & 1) for i in range(max(0, issued - stages), issued)]
        for b, par in waits:
            while not full[b].done(par):
                yield

    def consumer(w):
        for i in range(w, nch, warps):
            st = i % stages
            par = (i // nbars) & 1
            while not full[i % nbars].done(par):
                yield
            if content[st] != i or any(c[0] == st for c in inflight):
                raise Violation(f"warp {w} read chunk {i} from stage {st} holding {content[st]}")
            yield  # the warp computes on the stage
            empty[st].arrive()

    actors = [producer()] + [consumer(w) for w in range(warps)]
    live = list(range(len(actors)))
    while live or inflight:
        # land a copy (any of them, not in issue order) or step a warp
        if inflight and (not live or rng.random() < 0.35):
            st, fb, i = inflight.pop(rng.randrange(len(inflight)))
            content[st] = i
            fb.complete_tx(1)
            continue
        if not live:
            break
        k = rng.choice(live)
        try:
            next(actors[k])
        except StopIteration:
            live.remove(k)
            if not live and inflight:
                raise Violation("the CTA exits with a copy in flight")


def _search(stages, warps, nbars, runs, old_drain=False):
    rng = random.Random(1234)
    for r in range(runs):
        nch = rng.randint(1, 32)
        try:
            run_cta(nch, stages, warps, nbars, rng, old_drain)
        except Violation as e:
            return f"run {r}, {nch} chunks: {e}"
    return None


def test_kernel_layout_has_no_failing_schedule():
    stages, warps, nbars = _kernel_constants()
    assert nbars % warps == 0 and nbars >= stages
    bad = _search(stages, warps, nbars, runs=3000)
    assert bad is None, bad


@pytest.mark.parametrize("stages", [4, 5, 6, 8])
def test_other_stage_counts_hold(stages):
    warps = 4
    nbars = (stages + warps - 1) // warps * warps
    assert _search(stages, warps, nbars, runs=600) is None


def test_one_barrier_per_stage_is_caught():
    stages, warps, _ = _kernel_constants()
    bad = _search(stages, warps, stages, runs=3000, old_drain=True)
    assert bad is not None, "the model found no aliasing in the one-barrier-per-stage layout"
