"""CPU model of the decode's equal-work partition (decode_common.cuh:
partition_prologue + the producer walk; decode_kernels.cu: the combine's
piece lists), checked for every invariant the kernels rely on: each
(sequence, KV head, block) is streamed by exactly one CTA, CTA loads (blocks
plus `alpha` per segment start) differ by at most one unit, every CTA keeps at
most two partial states (slots 0 and 1, never both for one piece), and the
combine merges exactly the split segments, each once, from the slots their
pieces wrote.

Stream: segment (b, h) is alpha + nblk(b) positions long (none when nblk(b)
is 0); its first alpha positions carry no blocks (they stand for the fixed
cost of a piece), the rest are its blocks in order."""
import numpy as np
import pytest


def range_begin(c, W, P):
    return c * W // P


def cta_of(x, W, P):
    return ((x + 1) * P + W - 1) // W - 1


def walk(nblk, H, P, alpha=0):
    """Pieces per CTA, as the producer walks them: (b, h, blk0, nblk, complete, slot)."""
    seg = np.where(nblk > 0, nblk + alpha, 0)
    W = H * int(seg.sum())
    pre = np.concatenate([[0], np.cumsum(seg)])
    out, loads = [], []
    for c in range(P):
        lo, hi = range_begin(c, W, P), range_begin(c + 1, W, P)
        loads.append(hi - lo)
        pieces = []
        if lo < hi:
            # segment of position lo (the prologue's pass 2)
            b = int(np.searchsorted(H * pre, lo, side="right") - 1)
            while seg[b] == 0:
                b += 1
            r = lo - H * pre[b]
            h, off = r // seg[b], r % seg[b]
            pos = lo
            while pos < hi:
                span = min(seg[b] - off, hi - pos)
                r0, r1 = max(off, alpha), off + span
                if r1 > r0:
                    pieces.append((b, h, r0 - alpha, r1 - r0, r0 == alpha and r1 == seg[b], 0 if not pieces else 1))
                pos += span
                off += span
                if off == seg[b] and pos < hi:
                    off = 0
                    h += 1
                    if h == H:
                        h = 0
                        b += 1
                        while seg[b] == 0:
                            b += 1
        out.append(pieces)
    return W, out, loads


def combine_lists(nblk, H, P, W, pieces, alpha=0):
    """The combine kernel's view: desc[c] = segment at the range start
    (offset counted from the segment's first position, virtual ones
    included); the iteration of the first boundary inside a segment's blocks
    merges it."""
    seg = np.where(nblk > 0, nblk + alpha, 0)
    pre = np.concatenate([[0], np.cumsum(seg)])
    desc = []
    for c in range(P):
        lo = range_begin(c, W, P)
        if lo >= range_begin(c + 1, W, P):
            desc.append((-1, 0, 0, 0))
            continue
        b = int(np.searchsorted(H * pre, lo, side="right") - 1)
        while seg[b] == 0:
            b += 1
        r = lo - H * pre[b]
        desc.append((b, r // seg[b], r % seg[b], int(seg[b])))
    merged = {}
    for c in range(1, P):
        b, h, off, ln = desc[c]
        if b < 0 or off <= alpha:
            continue
        S = range_begin(c, W, P) - off
        cf = cta_of(S + alpha, W, P)
        if cta_of(range_begin(c, W, P) - 1, W, P) != cf:
            continue
        cl = cta_of(S + ln - 1, W, P)
        lst = []
        for k in range(cf, cl + 1):
            if range_begin(k, W, P) == range_begin(k + 1, W, P):
                continue
            lst.append((k, 1 if (k == cf and range_begin(k, W, P) < S) else 0))
        assert (b, h) not in merged
        merged[(b, h)] = lst
    return merged


@pytest.mark.parametrize("alpha", [0, 1, 3])
@pytest.mark.parametrize("seed,B,H,P", [(0, 8, 8, 296), (1, 128, 8, 296), (2, 3, 1, 296), (3, 64, 32, 444),
                                        (4, 1, 8, 592), (5, 256, 8, 296), (6, 5, 2, 7), (7, 40, 4, 1),
                                        (8, 3, 2, 444), (9, 2, 1, 444), (10, 6, 8, 592)])
def test_partition_covers_every_block_once(seed, B, H, P, alpha):
    rng = np.random.default_rng(seed)
    nblk = rng.integers(0, 300 if seed < 8 else 4, B)  # seeds >= 8: less work than CTAs
    nblk[rng.random(B) < 0.2] = 0  # empty sequences
    if nblk.sum() == 0:
        nblk[0] = 1
    W, pieces, loads = walk(nblk, H, P, alpha)
    cover = {}
    for c, pl in enumerate(pieces):
        slots = [p[5] for p in pl if not p[4]]
        assert len(slots) == len(set(slots)) <= 2, (c, pl)  # at most one partial per slot
        for b, h, off, n, complete, slot in pl:
            assert n > 0
            for j in range(off, off + n):
                assert (b, h, j) not in cover
                cover[(b, h, j)] = (c, slot, complete)
    assert len(cover) == H * int(nblk.sum())
    assert max(loads) - min(loads) <= 1
    merged = combine_lists(nblk, H, P, W, pieces, alpha)
    # split segments are exactly the merged ones; their pieces come from the listed (cta, slot)
    for b in range(B):
        for h in range(H):
            if nblk[b] == 0:
                continue
            owners = {cover[(b, h, j)][:2] for j in range(nblk[b])}
            complete = {cover[(b, h, j)][2] for j in range(nblk[b])}
            if len(owners) == 1 and complete == {True}:
                assert (b, h) not in merged
            else:
                assert complete == {False}
                assert sorted(owners) == sorted(merged[(b, h)]), (b, h)


@pytest.mark.parametrize("alpha", [0, 3])
@pytest.mark.parametrize("seed,B,H,P", [(0, 8, 1, 296), (1, 128, 8, 296), (3, 64, 32, 444), (5, 256, 8, 296)])
def test_combine_helpers_cover_each_split_segment_once(seed, B, H, P, alpha):
    # work >= CTAs: the combine CTAs of all boundaries inside a split segment
    # share its outputs [k n / helpers, (k + 1) n / helpers)
    rng = np.random.default_rng(seed)
    nblk = rng.integers(1, 3000, B)
    W, pieces, _ = walk(nblk, H, P, alpha)
    assert W >= P
    seg = nblk + alpha
    pre = np.concatenate([[0], np.cumsum(seg)])
    n_out = 8 * 32
    done = {}
    for c in range(1, P):
        lo = range_begin(c, W, P)
        b = int(np.searchsorted(H * pre, lo, side="right") - 1)
        r = lo - H * pre[b]
        h, off = r // seg[b], r % seg[b]
        if off <= alpha:
            continue
        s0 = lo - off
        cf, cl = cta_of(s0 + alpha, W, P), cta_of(s0 + seg[b] - 1, W, P)
        k, n_h = c - cf - 1, cl - cf
        assert 0 <= k < n_h
        done.setdefault((b, h), []).append((k * n_out // n_h, (k + 1) * n_out // n_h, n_h))
    for key, parts in done.items():
        parts.sort()
        assert len(parts) == parts[0][2]  # every helper present
        assert parts[0][0] == 0 and parts[-1][1] == n_out
        assert all(parts[i][1] == parts[i + 1][0] for i in range(len(parts) - 1))
