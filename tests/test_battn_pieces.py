"""Model check of k_battn's per-piece protocol (csrc/q3_battn.cuh) on the CPU.

A CTA's share of the (b, h, chunk) list is cut into pieces, one per (b, h) it
touches.  The q warp stages piece p's q into slot p % kBaQSlots (after
qfree[slot] closed the phase of piece p - kBaQSlots) and arrives on
qready[slot]; each of the 4 consumer warps waits on qready[slot], works on
the piece, waits on wfree[p % 2] (the merge of piece p - 2) before writing its
state into state slot p % 2, and counts itself on pcnt[p % 2]; the warp that
counts last merges the four states, resets the count and arrives on wfree and
qfree.  Warps run in any interleaving and a warp may skip a piece's chunks
(pieces shorter than 4 chunks).  The model keeps the mbarrier parity rule
(a parity wait succeeds once the phase of that parity is complete, which
includes the phase before the pending one) and must never let a consumer read
another piece's q, overwrite a state another piece still needs, or merge
states of different pieces.  Dropping the wait on wfree must be caught.
"""
import pathlib
import random
import re

import pytest
from test_battn_pipeline import Barrier, Violation

HDR = pathlib.Path(__file__).resolve().parents[1] / "qwen3-iree_b200" / "csrc" / "q3_battn.cuh"


def _kernel_constants():
    src = HDR.read_text()
    qslots = int(re.search(r"constexpr int kBaQSlots = (\d+);", src).group(1))
    warps = int(re.search(r"constexpr int kBaWarps = (\d+);", src).group(1))
    assert "uint64_t qready[kBaQSlots], qfree[kBaQSlots], wfree[2];" in src
    assert "const int sl = p % kBaQSlots, ws = p & 1;" in src
    return qslots, warps, 2


def run_cta(npieces, qslots, warps, wslots, rng, wait_wfree=True):
    qready = [Barrier(1) for _ in range(qslots)]
    qfree = [Barrier(1) for _ in range(qslots)]
    wfree = [Barrier(1) for _ in range(wslots)]
    qslot = [None] * qslots            # piece whose q a slot holds
    readers = [set() for _ in range(qslots)]
    state = [[None] * warps for _ in range(wslots)]
    pcnt = [0] * wslots
    merged = []

    def qwarp():
        for p in range(npieces):
            sl = p % qslots
            if p >= qslots:
                par = ((p // qslots) - 1) & 1
                while not qfree[sl].done(par):
                    yield
            if readers[sl]:
                raise Violation(f"q slot {sl} refilled with piece {p} while {readers[sl]} read it")
            qslot[sl] = p
            yield
            qready[sl].arrive()

    def consumer(w):
        for p in range(npieces):
            sl, ws = p % qslots, p % wslots
            while not qready[sl].done((p // qslots) & 1):
                yield
            if qslot[sl] != p:
                raise Violation(f"warp {w} read piece {qslot[sl]}'s q for piece {p}")
            readers[sl].add((w, p))
            for _ in range(rng.randint(0, 2)):  # its chunks of the piece (maybe none)
                yield
            if p >= wslots and wait_wfree:
                par = ((p // wslots) - 1) & 1
                while not wfree[ws].done(par):
                    yield
            readers[sl].discard((w, p))
            if state[ws][w] is not None and state[ws][w] != p - wslots:
                raise Violation(f"warp {w} overwrote piece {state[ws][w]}'s state with piece {p}")
            state[ws][w] = p
            yield
            pcnt[ws] += 1
            if pcnt[ws] == warps:  # the last warp merges
                got = set(state[ws])
                if got != {p}:
                    raise Violation(f"merge of piece {p} saw states of pieces {got}")
                merged.append(p)
                pcnt[ws] = 0
                yield
                wfree[ws].arrive()
                qfree[sl].arrive()

    actors = [qwarp()] + [consumer(w) for w in range(warps)]
    live = list(range(len(actors)))
    while live:
        k = rng.choice(live)
        try:
            next(actors[k])
        except StopIteration:
            live.remove(k)
    if sorted(merged) != list(range(npieces)):
        raise Violation(f"pieces merged: {sorted(merged)} of {npieces}")


def _search(qslots, warps, wslots, runs, wait_wfree=True):
    rng = random.Random(99)
    for r in range(runs):
        n = rng.randint(1, 14)
        try:
            run_cta(n, qslots, warps, wslots, rng, wait_wfree)
        except Violation as e:
            return f"run {r}, {n} pieces: {e}"
    return None


def test_kernel_piece_protocol_has_no_failing_schedule():
    qslots, warps, wslots = _kernel_constants()
    bad = _search(qslots, warps, wslots, runs=3000)
    assert bad is None, bad


@pytest.mark.parametrize("qslots", [1, 2, 3, 4, 6])
def test_other_q_slot_counts_hold(qslots):
    assert _search(qslots, 4, 2, runs=500) is None


def test_missing_state_slot_wait_is_caught():
    qslots, warps, wslots = _kernel_constants()
    bad = _search(qslots, warps, wslots, runs=3000, wait_wfree=False)
    assert bad is not None, "the model found no hazard without the wfree wait"
