"""The append + decode entry point for callers that cannot allocate device
memory when they decode (their HBM is already handed to a KV pool, or their
only allocator may not be called on the serving path).  It takes no
workspace and uses the library's built-in scratch instead.

Checked through the C ABI against clove_cuda_paged_append_decode (which
takes a caller workspace) and against the fp64 oracle on the same inputs,
with the appended K/V rows compared bit for bit, on two calls in a row — the
second call finds the scratch holding the first call's leftovers.  A large
split-K call followed by a small one shows that leftovers of a bigger call
do not leak into a smaller one.  The device check flags of a call come back
through clove_cuda_noalloc_status.  This file is collected last so a run
that stops at the first failure has already run every other test.
"""
import numpy as np
import pytest
import torch

import oracle
from clove_b200 import _lib
from clove_b200.workload import dtype_code, to_numpy_bits
from workload_check import bits_equal, tol_check

pytestmark = pytest.mark.gpu

RT = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def _case(name, batch, ctx_scale):
    from clove_b200 import KVPool
    from clove_b200.workload import CONFIGS, fill_values, make_layout
    lay = make_layout(CONFIGS[name], batch=batch, ctx_scale=ctx_scale)
    s = lay.spec
    dev = torch.device("cuda", 0)
    pool = KVPool(lay.num_blocks, s.block_size, s.num_kv_heads, s.head_dim, s.dtype, 0)
    q, kn, vn, _ = fill_values(lay, dev, pool.storage)
    bt = torch.from_numpy(lay.block_tables).to(dev)
    cl = torch.from_numpy(lay.context_lens).to(dev)
    return lay, pool, q, kn, vn, bt, cl


def _noalloc(pool, q, kn, vn, bt, cl, lay, out):
    s = lay.spec
    return _lib.lib().clove_cuda_paged_append_decode_noalloc(
        pool.handle, q.data_ptr(), kn.data_ptr(), vn.data_ptr(), s.num_q_heads, bt.data_ptr(), bt.shape[1],
        cl.data_ptr(), lay.batch, float(1.0 / np.sqrt(s.head_dim)), lay.max_ctx, out.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


def _status(device=0):
    import ctypes as C
    flags = C.c_int(0)
    rc = _lib.lib().clove_cuda_noalloc_status(device, torch.cuda.current_stream().cuda_stream, C.byref(flags))
    assert rc in (_lib.OK, _lib.ERR_DEVICE_CHECK), _lib.last_error()
    return flags.value


def _oracle(lay, before, q, kn, vn):
    spec = lay.spec
    kc, vc = before[0].copy(), before[1].copy()
    slots = oracle.append_slots(lay.block_tables, lay.context_lens, spec.block_size)
    assert oracle.reshape_and_cache(kc, vc, to_numpy_bits(kn), to_numpy_bits(vn), slots) == 0
    ref = oracle.decode_f64(dtype_code(spec.dtype), to_numpy_bits(q), kc, vc, lay.block_tables,
                            lay.context_lens + 1, 1.0 / np.sqrt(spec.head_dim))
    return kc, vc, ref


def _check_calls(name, batch, ctx_scale, calls=2):
    lay, pool, q, kn, vn, bt, cl = _case(name, batch, ctx_scale)
    before = to_numpy_bits(pool.storage)
    kc, vc, ref64 = _oracle(lay, before, q, kn, vn)
    # The append writes the same token to the same slot each time, so the
    # cache is the same before every call below.
    ref = pool.append_decode(q, kn, vn, bt, cl, max_ctx=lay.max_ctx).cpu().numpy()
    for _ in range(calls):
        out = torch.full((lay.batch, lay.spec.num_q_heads, lay.spec.head_dim), float("nan"), device="cuda")
        _lib.check(_noalloc(pool, q, kn, vn, bt, cl, lay, out))
        torch.cuda.synchronize()
        assert _status() == 0
        got = out.cpu().numpy()
        tol_check(got, ref, RT[lay.spec.dtype])    # against the workspace entry point
        tol_check(got, ref64, RT[lay.spec.dtype])  # against the fp64 oracle
        after = to_numpy_bits(pool.storage)
        assert bits_equal(after[0], kc) and bits_equal(after[1], vc), "appended K/V rows not bit-exact"
    pool.close()


@pytest.mark.parametrize("name,batch,ctx_scale", [("c1", 8, 1.0), ("c3", 16, 0.5), ("c4", 2, 0.05)])
def test_noalloc_matches_workspace_entry_point(name, batch, ctx_scale):
    _check_calls(name, batch, ctx_scale)


def test_noalloc_large_then_small_call():
    # a split-K call with many chunks (long contexts), then a one-sequence
    # call: the second must not see the first call's item list, counters or
    # partials
    _check_calls("c4", 2, 0.2, calls=1)
    _check_calls("c1", 1, 1.0, calls=2)


def test_noalloc_reports_timeout_flag():
    # Failure detection without a GPU fault: the test hook leaves one stage
    # unfilled, the bounded wait runs out, the call completes, and the flag
    # comes back through clove_cuda_noalloc_status; the next call is right.
    import time
    L = _lib.lib()
    lay, pool, q, kn, vn, bt, cl = _case("c1", 4, 1.0)
    before = to_numpy_bits(pool.storage)
    _, _, ref64 = _oracle(lay, before, q, kn, vn)
    out = torch.empty((lay.batch, lay.spec.num_q_heads, lay.spec.head_dim), device="cuda")
    try:
        _lib.check(L.clove_cuda_debug_set(2000, 1))
        t0 = time.time()
        _lib.check(_noalloc(pool, q, kn, vn, bt, cl, lay, out))
        flags = _status()
        elapsed = time.time() - t0
    finally:
        L.clove_cuda_debug_set(0, 0)
    assert flags & _lib.FLAG_TIMEOUT, flags
    assert elapsed < 30
    _lib.check(_noalloc(pool, q, kn, vn, bt, cl, lay, out))
    torch.cuda.synchronize()
    assert _status() == 0
    tol_check(out.cpu().numpy(), ref64, RT[lay.spec.dtype])
    pool.close()


def test_noalloc_scratch_covers_every_decode_shape():
    # The decode splits its work evenly over a fixed number of CTAs, so its
    # scratch need depends only on the head shape; the built-in 16 MiB covers
    # the largest one built (head_dim 256, 8 query heads per KV head) at any
    # batch and context length.  (The size check in the entry point refuses
    # anything larger with CLOVE_ERR_WORKSPACE before launching.)
    from clove_b200 import KVPool
    for D in (64, 128, 256):
        pool = KVPool(16, 16, 8, D, torch.bfloat16, 0)
        for batch, max_ctx in ((1, 1), (1024, 131072), (65536, 1 << 20)):
            need = pool.workspace_bytes(batch, 64, max_ctx)
            assert 0 < need <= 16 << 20, (D, batch, max_ctx, need)
        pool.close()
