"""The exchange protocol of the peer-memory all-reduce (soc_b200/csrc/tp_allreduce.cu), checked
as a model on the CPU: ranks run the same sequence of all-reduces, each one
  1. storing its partial into slot [e & 1][rank] of every rank's buffer,
  2. raising flag [e & 1][rank] = e in every rank's buffer,
  3. waiting until every flag [e & 1][*] of its own buffer is >= e,
  4. summing the slots [e & 1][*] of its own buffer,
with every rank's steps interleaved at random (a step is one store, one flag or one read).
Two buffers must be enough: no read may see a slot written for another all-reduce, and every
rank must get the full sum."""
import random

import pytest


def _run(tp, rounds, seed):
    rng = random.Random(seed)
    slots = [[[None] * tp for _ in range(2)] for _ in range(tp)]  # [owner][buffer][writer] -> (epoch, value)
    flags = [[[0] * tp for _ in range(2)] for _ in range(tp)]      # [owner][buffer][writer] -> epoch
    results = [[] for _ in range(tp)]

    def rank_steps(r):
        for e in range(1, rounds + 1):
            b = e & 1
            value = (r + 1) * 1000 + e
            for p in rng.sample(range(tp), tp):          # 1. stores, in any order
                slots[p][b][r] = (e, value)
                yield
            for p in rng.sample(range(tp), tp):          # 2. flags
                flags[p][b][r] = e
                yield
            while min(flags[r][b]) < e:                  # 3. wait on the own buffer
                yield
            total = 0
            for w in rng.sample(range(tp), tp):          # 4. reads
                got_e, v = slots[r][b][w]
                assert got_e == e, f"rank {r} read writer {w}'s slot of all-reduce {got_e} during {e}"
                total += v
                yield
            results[r].append(total)

    live = {r: rank_steps(r) for r in range(tp)}
    while live:
        r = rng.choice(list(live))
        try:
            next(live[r])
        except StopIteration:
            del live[r]
    for r in range(tp):
        assert results[r] == [sum((w + 1) * 1000 + e for w in range(tp)) for e in range(1, rounds + 1)]


@pytest.mark.parametrize("tp", [2, 3, 4, 8])
def test_two_buffers_suffice_under_random_interleavings(tp):
    for seed in range(200 if tp <= 4 else 40):
        _run(tp, rounds=6, seed=seed)


def test_one_buffer_would_not():
    """The same protocol with a single buffer lets a fast rank overwrite a slot that a slow
    rank has not read yet: the model finds it, which is why the kernel alternates two."""
    found = False
    for seed in range(300):
        try:
            _run_single_buffer(3, 6, seed)
        except AssertionError:
            found = True
            break
    assert found


def _run_single_buffer(tp, rounds, seed):
    rng = random.Random(seed)
    slots = [[None] * tp for _ in range(tp)]
    flags = [[0] * tp for _ in range(tp)]

    def rank_steps(r):
        for e in range(1, rounds + 1):
            for p in rng.sample(range(tp), tp):
                slots[p][r] = (e, r)
                yield
            for p in rng.sample(range(tp), tp):
                flags[p][r] = e
                yield
            while min(flags[r]) < e:
                yield
            for w in rng.sample(range(tp), tp):
                got_e, _ = slots[r][w]
                assert got_e == e
                yield

    live = {r: rank_steps(r) for r in range(tp)}
    while live:
        r = rng.choice(list(live))
        try:
            next(live[r])
        except StopIteration:
            del live[r]


def _run_with_timeouts(tp, rounds, seed, poison):
    """The protocol with bounded waits: a rank whose wait gives up either carries on with the
    next all-reduce (poison=False, the behaviour before the exchange was poisoned on a
    timeout) or stops using the exchange for good (poison=True).  Returns the number of reads
    that followed a wait that succeeded yet saw a slot of another all-reduce."""
    rng = random.Random(seed)
    slots = [[[None] * tp for _ in range(2)] for _ in range(tp)]
    flags = [[[0] * tp for _ in range(2)] for _ in range(tp)]
    slow = rng.randrange(tp)  # one rank is delayed so that the others' waits run out
    bad = [0]

    def rank_steps(r):
        for e in range(1, rounds + 1):
            b = e & 1
            if r == slow and e == 2:
                for _ in range(rng.randint(0, 40)):
                    yield
            for p in rng.sample(range(tp), tp):
                slots[p][b][r] = (e, r)
                yield
            for p in rng.sample(range(tp), tp):
                flags[p][b][r] = e
                yield
            waited, limit, timed_out = 0, rng.randint(2, 12), False
            while min(flags[r][b]) < e:
                waited += 1
                if waited > limit:
                    timed_out = True
                    break
                yield
            if timed_out and poison:
                return  # the exchange is poisoned: no further all-reduce on this rank
            for w in rng.sample(range(tp), tp):
                got = slots[r][b][w]
                if not timed_out and (got is None or got[0] != e):
                    bad[0] += 1
                yield

    live = {r: rank_steps(r) for r in range(tp)}
    while live:
        r = rng.choice(list(live))
        try:
            next(live[r])
        except StopIteration:
            del live[r]
    return bad[0]


def test_carrying_on_after_a_timeout_breaks_the_two_buffer_guarantee():
    """After a rank gives up waiting and keeps using the exchange, a later all-reduce whose
    wait succeeds can read another all-reduce's slot: the model finds such a run."""
    assert any(_run_with_timeouts(3, 8, seed, poison=False) for seed in range(400))


@pytest.mark.parametrize("tp", [2, 3, 4, 8])
def test_poisoned_exchange_never_reads_a_wrong_slot(tp):
    """With the exchange poisoned on the first timeout, no completed wait is ever followed by
    a read of another all-reduce's slot."""
    for seed in range(300 if tp <= 4 else 60):
        assert _run_with_timeouts(tp, 8, seed, poison=True) == 0
