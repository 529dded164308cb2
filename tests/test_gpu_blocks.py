"""GPU: block copies are bit-exact, and a serving loop driven by the block
manager (prompts, decode steps, a fork that diverges through copy-on-write,
frees) decodes every step like the oracle run on each sequence's own
token history."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_copy_blocks_bit_exact():
    from clove_b200 import KVPool, _lib
    pool = KVPool(32, 16, 2, 128, torch.bfloat16, 0)
    pool.storage.normal_()
    before = pool.storage.clone()
    src = torch.tensor([3, 7, 0], dtype=torch.int32, device="cuda")
    dst = torch.tensor([10, 11, 31], dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().clove_cuda_copy_blocks(pool.handle, src.data_ptr(), dst.data_ptr(), 3, None))
    torch.cuda.synchronize()
    exp = before.clone()
    exp[:, [10, 11, 31]] = before[:, [3, 7, 0]]
    assert torch.equal(pool.storage.view(torch.int16), exp.view(torch.int16))
    bad = torch.tensor([99], dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().clove_cuda_copy_blocks(pool.handle, bad.data_ptr(), dst.data_ptr(), 1, None))
    assert pool.pool_status() & _lib.FLAG_BLOCK_OOB


def test_serving_loop_with_fork_and_copy_on_write():
    import oracle
    from clove_b200 import KVPool, _lib
    from clove_b200.blocks import BlockManager
    rng = np.random.default_rng(5)
    dev = torch.device("cuda", 0)
    nb, bs, hkv, hq, d = 128, 16, 2, 8, 64
    pool = KVPool(nb, bs, hkv, d, torch.float32, 0)
    pool.storage.zero_()
    mgr = BlockManager(nb, bs, max_seqs=8)
    hist = {}  # seq -> (list of K rows [hkv, d], list of V rows)
    L = _lib.lib()

    def write_tokens(seq, start, ks, vs):
        t, _ = mgr.export([seq], 64)
        slots = np.array([t[0, p // bs] * bs + p % bs for p in range(start, start + len(ks))], np.int32)
        pool.reshape_and_cache(torch.from_numpy(np.stack(ks)).to(dev), torch.from_numpy(np.stack(vs)).to(dev),
                               torch.from_numpy(slots).to(dev))

    def apply_copies(copies):
        if copies:
            s = torch.tensor([c[0] for c in copies], dtype=torch.int32, device=dev)
            t = torch.tensor([c[1] for c in copies], dtype=torch.int32, device=dev)
            _lib.check(L.clove_cuda_copy_blocks(pool.handle, s.data_ptr(), t.data_ptr(), len(copies), None))

    def rows(n):
        return [rng.standard_normal((hkv, d)).astype(np.float32) for _ in range(n)]

    # prompts
    for seq, plen in ((0, 37), (1, 16), (2, 5)):
        mgr.add(seq, plen)
        ks, vs = rows(plen), rows(plen)
        write_tokens(seq, 0, ks, vs)
        hist[seq] = (ks, vs)
    copies_seen = 0
    for step in range(40):
        if step == 7:  # fork sequence 0 mid-block: both branches then append
            mgr.fork(0, 3)
            hist[3] = (list(hist[0][0]), list(hist[0][1]))
        if step == 25:
            mgr.free(1)
            del hist[1]
        seqs = sorted(hist)
        old = {s: mgr.seq_len(s) for s in seqs}
        for s in seqs:
            copies = mgr.reserve(s, old[s] + 1)
            copies_seen += len(copies)
            apply_copies(copies)
        tables, _ = mgr.export(seqs, 16)
        ctx = np.array([old[s] for s in seqs], np.int32)
        kn, vn = rows(len(seqs)), rows(len(seqs))
        q = rng.standard_normal((len(seqs), hq, d)).astype(np.float32)
        out = pool.append_decode(torch.from_numpy(q).to(dev), torch.from_numpy(np.stack(kn)).to(dev),
                                 torch.from_numpy(np.stack(vn)).to(dev), torch.from_numpy(tables).to(dev),
                                 torch.from_numpy(ctx).to(dev), max_ctx=int(ctx.max()) + 1)
        assert pool.decode_status(len(seqs), hq, int(ctx.max()) + 1) == 0
        for i, s in enumerate(seqs):
            hist[s][0].append(kn[i])
            hist[s][1].append(vn[i])
        # oracle on each sequence's own history (dense, one block per token)
        for i, s in enumerate(seqs):
            K = np.stack(hist[s][0])[:, None]  # [T, 1, hkv, d] as a pool of 1-token blocks
            V = np.stack(hist[s][1])[:, None]
            T = K.shape[0]
            ref = oracle.decode_f64(0, q[i:i + 1], K, V, np.arange(T, dtype=np.int32)[None], np.array([T], np.int32),
                                    1.0 / np.sqrt(d))
            ok, worst = oracle.tolerance_ok(out[i:i + 1].cpu().numpy(), ref, 1e-5)
            assert ok, (step, s, worst)
    assert copies_seen >= 1  # the fork diverged through copy-on-write
