"""CPU tests of the KV block manager (include/clove_blocks.h): allocation,
growth, fork with shared blocks, copy-on-write, free, exhaustion, export."""
import numpy as np
import pytest

from clove_b200 import _lib


@pytest.fixture()
def mgr():
    from clove_b200.blocks import BlockManager
    return BlockManager(num_blocks=16, block_size=4, max_seqs=8)


def test_add_grow_free(mgr):
    mgr.add(0, 5)  # 2 blocks
    assert mgr.num_free == 14 and mgr.seq_len(0) == 5
    assert mgr.reserve(0, 8) == []  # fits in the 2 blocks
    assert mgr.num_free == 14
    assert mgr.reserve(0, 9) == []  # third block
    assert mgr.num_free == 13
    t, l = mgr.export([0], 4)
    assert l.tolist() == [9] and (t[0, :3] >= 0).all() and t[0, 3] == -1
    assert len(set(t[0, :3].tolist())) == 3
    mgr.free(0)
    assert mgr.num_free == 16 and mgr.seq_len(0) == -1


def test_fork_shares_then_copy_on_write(mgr):
    mgr.add(0, 6)  # blocks: [a, b], b half full
    mgr.fork(0, 1)
    assert mgr.num_free == 14  # shared, nothing new
    t, _ = mgr.export([0, 1], 4)
    assert (t[0] == t[1]).all()
    # child appends token 6 -> lands in the shared block b: copy-on-write
    copies = mgr.reserve(1, 7)
    assert len(copies) == 1
    src, dst = copies[0]
    t2, l2 = mgr.export([0, 1], 4)
    assert src == t[0, 1] and dst == t2[1, 1] and dst != src
    assert t2[1, 0] == t[0, 0]  # the full prefix block stays shared
    assert l2.tolist() == [6, 7]
    # the parent now owns b alone: its append needs no copy
    assert mgr.reserve(0, 7) == []
    mgr.free(0)
    mgr.free(1)
    assert mgr.num_free == 16


def test_fork_at_block_boundary_needs_no_copy(mgr):
    mgr.add(0, 8)  # exactly 2 full blocks
    mgr.fork(0, 1)
    assert mgr.reserve(1, 9) == []  # new block, nothing shared is written
    t, _ = mgr.export([0, 1], 4)
    assert (t[0, :2] == t[1, :2]).all() and t[1, 2] not in t[0, :2]


def test_exhaustion_leaves_sequence_unchanged(mgr):
    mgr.add(0, 60)  # 15 blocks
    with pytest.raises(_lib.CloveError) as e:
        mgr.reserve(0, 70)  # needs 3 more, 1 free
    assert e.value.code == _lib.ERR_NO_BLOCKS
    assert mgr.seq_len(0) == 60 and mgr.num_free == 1
    with pytest.raises(_lib.CloveError) as e:
        mgr.add(1, 9)
    assert e.value.code == _lib.ERR_NO_BLOCKS


def test_bad_sequence_ids(mgr):
    with pytest.raises(_lib.CloveError):
        mgr.free(3)
    mgr.add(2, 1)
    with pytest.raises(_lib.CloveError):
        mgr.add(2, 1)  # in use
    with pytest.raises(_lib.CloveError):
        mgr.fork(5, 2)  # parent unknown, child in use
    with pytest.raises(_lib.CloveError):
        mgr.reserve(2, 0)  # shrinking
    with pytest.raises(_lib.CloveError):
        mgr.export([2], 0)


def test_random_workload_invariants():
    # Random add / grow / fork / free; block ownership stays consistent: every
    # block is free or referenced, and shared blocks are never written.
    from clove_b200.blocks import BlockManager
    rng = np.random.default_rng(3)
    nb, bs, ms = 64, 4, 12
    m = BlockManager(nb, bs, ms)
    live = {}
    for _ in range(400):
        op = rng.integers(0, 4)
        free_ids = [s for s in range(ms) if s not in live]
        if op == 0 and free_ids:
            s = int(rng.choice(free_ids))
            try:
                m.add(s, int(rng.integers(0, 20)))
                live[s] = m.seq_len(s)
            except _lib.CloveError:
                pass
        elif op == 1 and live:
            s = int(rng.choice(list(live)))
            try:
                m.reserve(s, live[s] + int(rng.integers(1, 6)))
                live[s] = m.seq_len(s)
            except _lib.CloveError:
                pass
        elif op == 2 and live and free_ids:
            p, c = int(rng.choice(list(live))), int(rng.choice(free_ids))
            m.fork(p, c)
            live[c] = live[p]
        elif op == 3 and live:
            s = int(rng.choice(list(live)))
            m.free(s)
            del live[s]
        seqs = sorted(live)
        if seqs:
            t, lens = m.export(seqs, 32)
            used = t[t >= 0]
            assert len(set(used.tolist())) + m.num_free <= nb
            assert len(set(used.tolist())) + m.num_free == nb
            assert (lens == [live[s] for s in seqs]).all()
        else:
            assert m.num_free == nb
