"""The buffer-reuse argument of the LL all-reduce (nanovllm-rs_b200/csrc/
allreduce.cu, allreduce_rms_norm_ll_kernel), checked on a model of it under
random interleavings, on the CPU.

Each rank runs its calls in order (a kernel starts after the previous one
ended); inside a call, CTA b of every rank handles rows u = b, b + C, ...;
every 8-byte word carries the call's epoch (the CTA's counter + 1) and lands
in the slot of the epoch's parity; a read spins until the word carries its
epoch.  Modelled as atomic steps of (rank, CTA) actors picked at random:

* one-shot (two ranks): push every row to every peer's receive slot, then
  read the peers' words and sum;
* column-owned two-shot (more ranks): push each row's slice o to owner o,
  owner sums its slice over the ranks and pushes the sum to every rank's
  gather slot, every rank reads all slices of its rows.

Asserted: every word read carries exactly the value of its own call (no word
of an earlier or later call with the same parity is ever seen, none is
overwritten before it was read), every call completes (no interleaving
deadlocks), and calls of different sizes -- CTAs with no rows in a call
included -- keep the per-CTA epochs of all ranks equal.  A mistake planted
in the model (the one-shot form with one slot instead of the parity pair)
must be caught.
"""
import random

import pytest


def _rows(b, C, T):
    return list(range(b, T, C))


def _run(W, C, sizes, seed, two_shot, parities=2):
    rng = random.Random(seed)
    recv = {}  # (dst, par, src, u, o) -> (epoch, value)
    gath = {}  # (dst, par, u, o) -> (epoch, value)
    epoch = {(r, b): 0 for r in range(W) for b in range(C)}
    done_calls = {r: 0 for r in range(W)}  # calls every CTA of rank r has finished
    data = lambda k, r, u, o: (k, r, u, o)  # noqa: E731
    reads = []

    def cta(r, b):
        for k, T in enumerate(sizes):
            while done_calls[r] < k:  # the previous kernel on this rank has not ended
                yield False
            e = epoch[(r, b)] + 1
            par = e % parities
            rows = _rows(b, C, T)
            if not two_shot:
                for u in rows:
                    for o in range(W):  # the whole row (its W slices) to every peer
                        for q in range(W):
                            if q != r:
                                recv[(q, par, r, u, o)] = (e, data(k, r, u, o))
                                yield True
                for u in rows:
                    for o in range(W):
                        for q in range(W):
                            if q == r:
                                continue
                            while recv.get((r, par, q, u, o), (None,))[0] != e:
                                yield False
                            got = recv[(r, par, q, u, o)][1]
                            reads.append((got, data(k, q, u, o)))
                            yield True
            else:
                for u in rows:  # phase 1: slice o of the row to its owner
                    for o in range(W):
                        if o != r:
                            recv[(o, par, r, u, o)] = (e, data(k, r, u, o))
                            yield True
                for u in rows:  # phase 2: own slice summed, pushed to every rank
                    total = [data(k, r, u, r)]
                    for q in range(W):
                        if q == r:
                            continue
                        while recv.get((r, par, q, u, r), (None,))[0] != e:
                            yield False
                        got = recv[(r, par, q, u, r)][1]
                        reads.append((got, data(k, q, u, r)))
                        total.append(got)
                        yield True
                    s = tuple(sorted(total))
                    for q in range(W):
                        gath[(q, par, u, r)] = (e, s)
                        yield True
                for u in rows:  # phase 3: every slice of the row
                    for o in range(W):
                        while gath.get((r, par, u, o), (None,))[0] != e:
                            yield False
                        got = gath[(r, par, u, o)][1]
                        want = tuple(sorted(data(k, q, u, o) for q in range(W)))
                        reads.append((got, want))
                        yield True
            epoch[(r, b)] = e
            yield "call-done"

    actors = {(r, b): cta(r, b) for r in range(W) for b in range(C)}
    finished_calls = {(r, b): 0 for r in range(W) for b in range(C)}
    live = set(actors)
    stalled = 0
    while live:
        key = rng.choice(sorted(live))
        try:
            res = next(actors[key])
        except StopIteration:
            live.discard(key)
            continue
        if res == "call-done":
            finished_calls[key] += 1
            r = key[0]
            done_calls[r] = min(finished_calls[(r, b)] for b in range(C))
            stalled = 0
        elif res:
            stalled = 0
        else:
            stalled += 1
            assert stalled < 20000, "no actor can progress: deadlock"
    for got, want in reads:
        assert got == want
    assert len(set(epoch.values())) == 1 and epoch[(0, 0)] == len(sizes)
    return len(reads)


@pytest.mark.parametrize("W,C,two_shot", [(2, 3, False), (3, 2, True), (4, 3, True),
                                          (2, 2, True)])
@pytest.mark.parametrize("seed", range(6))
def test_ll_slots_are_never_read_stale_or_overwritten(W, C, two_shot, seed):
    rng = random.Random(1000 + seed)
    sizes = [rng.randint(1, 2 * C + 1) for _ in range(7)]  # calls with idle CTAs among them
    assert _run(W, C, sizes, seed, two_shot) > 0


def test_model_catches_a_single_slot():
    """The model is sensitive: the one-shot form with one slot instead of
    the epoch-parity pair deadlocks under some interleaving (a rank finishes
    call e once its peer's pushes arrived, then overwrites the slot its peer
    has not read yet).  The column-owned two-shot needs no pair in this model
    -- its owners' sums order every overwrite after the read it could
    clobber -- and keeps it for the one-shot's sake (the same buffers)."""
    failures = 0
    for seed in range(40):
        rng = random.Random(seed)
        sizes = [rng.randint(1, 7) for _ in range(7)]
        try:
            _run(2, 3, sizes, seed, False, parities=1)
        except AssertionError:
            failures += 1
    assert failures > 0
