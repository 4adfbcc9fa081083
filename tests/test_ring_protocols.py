"""Model checks, on the CPU, of the other shared-memory rings' barrier
protocols (the attention ring has its own, tests/test_battn_pipeline.py).

* The Q8_0 GEMV / vocab ring (csrc/q3_gemv.cuh, k_gemv_q8 and
  k_vocab_argmax): one thread issues tile i's copy into stage i % ns after
  waiting on empty[s] with the parity of round i / ns - 1, and every
  consumer warp waits on full[s] for every tile, in order, then arrives on
  empty[s] (count = consumer warps).  The stage and the round parity are
  stepped, not divided out.  At the end the producer waits for the copies of
  the last ns tiles.
* The batched GEMM's weight-stage ring (csrc/q3_batch.cuh, k_bgemm_q8): the
  8 dequantising warps fill stage i % SUB and arrive on a_full (count 8);
  the MMA thread waits on a_full for every stage in order and releases it
  with a commit that arrives on a_empty later, when the MMAs reading it have
  finished (modelled as an asynchronous arrival).

Every consumer here sees every phase of the barriers it waits on, so a
parity wait cannot alias an older pending phase; random schedules must never
read a stage before it is filled, refill one still being read, or finish
with work in flight.
"""
import random

import pytest

from test_battn_pipeline import Barrier, Violation


def run_gemv_ring(ntiles, ns, consumers, rng):
    full = [Barrier(1) for _ in range(ns)]
    empty = [Barrier(consumers) for _ in range(ns)]
    content = [None] * ns
    readers = [set() for _ in range(ns)]
    inflight = []

    def producer():
        s, par, issued = 0, 0, 0
        for i in range(ntiles):
            if i >= ns:
                while not empty[s].done(par ^ 1):
                    yield
            if readers[s] or any(c[0] == s for c in inflight):
                raise Violation(f"stage {s} refilled with tile {i} while in use")
            full[s].arrive(tx=1)
            inflight.append((s, i))
            issued = i + 1
            s, par = (0, par ^ 1) if s + 1 == ns else (s + 1, par)
            yield
        for j in range(max(0, issued - ns), issued):
            while not full[j % ns].done((j // ns) & 1):
                yield

    def consumer(w):
        s, par = 0, 0
        for i in range(ntiles):
            while not full[s].done(par):
                yield
            if content[s] != i or any(c[0] == s for c in inflight):
                raise Violation(f"warp {w} read tile {i} from stage {s} holding {content[s]}")
            readers[s].add(w)
            yield
            readers[s].discard(w)
            empty[s].arrive()
            s, par = (0, par ^ 1) if s + 1 == ns else (s + 1, par)

    actors = [producer()] + [consumer(w) for w in range(consumers)]
    _schedule(actors, inflight, rng, land=lambda c: (content.__setitem__(c[0], c[1]),
                                                       full[c[0]].complete_tx(1)))


def run_mma_ring(nsub, sub, producers, rng):
    a_full = [Barrier(producers) for _ in range(sub)]
    a_empty = [Barrier(1) for _ in range(sub)]
    filled = [set() for _ in range(sub)]  # producers that wrote their part of stage s
    content = [None] * sub
    reading = [None] * sub                # sub-slice the MMAs of stage s are reading
    commits = []                          # (stage, sub-slice) releases still in flight

    def producer(w):
        for i in range(nsub):
            s = i % sub
            if i >= sub:
                while not a_empty[s].done(((i // sub) - 1) & 1):
                    yield
            if reading[s] is not None:
                raise Violation(f"warp {w} overwrote stage {s} while the MMAs read slice {reading[s]}")
            filled[s].add(w)
            if len(filled[s]) == producers:
                content[s] = i
                filled[s] = set()
            yield
            a_full[s].arrive()

    def mma():
        for i in range(nsub):
            s = i % sub
            while not a_full[s].done((i // sub) & 1):
                yield
            if content[s] != i:
                raise Violation(f"MMA read slice {i} from stage {s} holding {content[s]}")
            reading[s] = i
            commits.append((s, i))
            yield
        # the final commit (acc_full) completes after every earlier MMA; the
        # MMA thread waits for it before the CTA releases its TMEM and exits
        while commits:
            yield

    def land(c):
        s, i = c
        reading[s] = None
        a_empty[s].arrive()

    actors = [producer(w) for w in range(producers)] + [mma()]
    _schedule(actors, commits, rng, land=land)


def _schedule(actors, pending, rng, land):
    live = list(range(len(actors)))
    while live or pending:
        if pending and (not live or rng.random() < 0.35):
            land(pending.pop(rng.randrange(len(pending))))
            continue
        k = rng.choice(live)
        try:
            next(actors[k])
        except StopIteration:
            live.remove(k)
            if not live and pending:
                raise Violation("work still in flight at exit")


@pytest.mark.parametrize("ns", [1, 2, 3, 5, 8, 13])
def test_gemv_ring_schedules(ns):
    rng = random.Random(ns)
    for _ in range(300):
        run_gemv_ring(rng.randint(1, 40), ns, 8, rng)


@pytest.mark.parametrize("sub", [2, 3, 4])
def test_mma_ring_schedules(sub):
    rng = random.Random(100 + sub)
    for _ in range(300):
        run_mma_ring(rng.choice([4, 8]), sub, 8, rng)


def test_models_catch_a_missing_wait():
    """The same GEMV model with the producer's empty wait left out must fail
    (the check that the model can see a refill of a stage in use)."""
    rng = random.Random(7)

    def broken(ntiles, ns):
        full = [Barrier(1) for _ in range(ns)]
        inflight, content = [], [None] * ns

        def producer():
            for i in range(ntiles):
                s = i % ns
                if any(c[0] == s for c in inflight):
                    raise Violation("refill in flight")
                full[s].arrive(tx=1)
                inflight.append((s, i))
                yield

        def consumer():
            for i in range(ntiles):
                s = i % ns
                while not full[s].done((i // ns) & 1):
                    yield
                if content[s] != i:
                    raise Violation("stale read")
                yield

        _schedule([producer(), consumer()], inflight, rng,
                  land=lambda c: (content.__setitem__(c[0], c[1]), full[c[0]].complete_tx(1)))

    failures = 0
    for _ in range(200):
        try:
            broken(12, 2)
        except (Violation, AssertionError):
            failures += 1
    assert failures > 0
