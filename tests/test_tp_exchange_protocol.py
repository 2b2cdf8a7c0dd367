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
