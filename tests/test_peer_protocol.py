"""CPU model of the peer gather's protocol (clove_b200/csrc/peer_gather.cu).

Every CTA of every rank is a sequence of atomic steps — store a chunk into a
peer's receive half, add 1 to the peer's per-source count, wait for a count,
copy a chunk out — and a seeded random scheduler interleaves them.  Within a
rank, call n+1's CTAs start only after all of call n's finished (stream
order); across ranks nothing is ordered except through the counts.  The model
checks that every call's output equals the all-gather of that call's slices,
for any interleaving, with the kernel's two alternating halves; with a single
half the scheduler finds an interleaving where a fast rank overwrites a slice
that a slow rank has not yet copied out.
"""
import random

import pytest


def _run(world, chunks, calls, halves, seed):
    rnd = random.Random(seed)
    # receive buffers: data[rank][half][src][chunk], count[rank][src]
    data = [[[[None] * chunks for _ in range(world)] for _ in range(halves)] for _ in range(world)]
    count = [[0] * world for _ in range(world)]
    out = [[None] * calls for _ in range(world)]

    def cta(rank, call, p, c, res):
        half = call % halves
        val = lambda r: (r, call, c)  # chunk c of rank r's slice in this call  # noqa: E731
        if p == rank:
            res[p][c] = val(rank)
            return
        data[p][half][rank][c] = val(rank)
        yield
        count[p][rank] += 1
        yield
        while count[rank][p] < (call + 1) * chunks:
            yield
        yield  # the copy is a separate step from the wait
        res[p][c] = data[rank][half][p][c]

    def rank_calls(rank):
        for call in range(calls):
            res = [[None] * chunks for _ in range(world)]
            ctas = [cta(rank, call, p, c, res) for p in range(world) for c in range(chunks)]
            while ctas:  # the CTAs of one launch interleave among themselves
                g = rnd.choice(ctas)
                try:
                    next(g)
                except StopIteration:
                    ctas.remove(g)
                yield
            out[rank][call] = res

    ranks = [rank_calls(r) for r in range(world)]
    live = list(range(world))
    steps = 0
    while live:
        r = rnd.choice(live) if rnd.random() < 0.5 else live[0]  # skewed: rank order favours a fast rank
        try:
            next(ranks[r])
        except StopIteration:
            live.remove(r)
        steps += 1
        assert steps < 10_000_000, "no progress"
    bad = 0
    for r in range(world):
        for call in range(calls):
            want = [[(p, call, c) for c in range(chunks)] for p in range(world)]
            bad += out[r][call] != want
    return bad


@pytest.mark.parametrize("world,chunks", [(2, 1), (2, 3), (4, 2), (8, 1)])
def test_two_halves_never_overwrite_unread_data(world, chunks):
    for seed in range(40):
        assert _run(world, chunks, calls=6, halves=2, seed=seed) == 0, seed


def test_one_half_is_not_enough():
    """The model is sharp enough to see the race the second half removes."""
    assert any(_run(2, 2, calls=6, halves=1, seed=s) for s in range(200))
