"""Error behaviour on the GPU: bad inputs give status codes or device check
flags, never a fault (out-of-range indices are clamped and flagged)."""
import numpy as np
import pytest
import torch

from clove_b200 import _lib

pytestmark = pytest.mark.gpu


def _setup(dtype=torch.float32):
    from clove_b200 import KVPool
    pool = KVPool(64, 16, 2, 128, dtype=dtype, device=0)
    pool.storage.normal_()
    dev = torch.device("cuda", 0)
    bt = torch.arange(8, dtype=torch.int32, device=dev).reshape(2, 4)
    cl = torch.tensor([20, 40], dtype=torch.int32, device=dev)
    q = torch.randn(2, 4, 128, device=dev).to(dtype)
    return pool, bt, cl, q


def test_bad_block_id_flagged():
    pool, bt, cl, q = _setup()
    bt[1, 1] = 10 ** 6
    pool.decode(q, bt, cl, max_ctx=64)
    assert pool.decode_status(2, 4, 64) & _lib.FLAG_BLOCK_OOB
    bt[1, 1] = -3
    pool.decode(q, bt, cl, max_ctx=64)
    assert pool.decode_status(2, 4, 64) & _lib.FLAG_BLOCK_OOB


def test_context_over_max_ctx_flagged_and_clamped():
    pool, bt, cl, q = _setup()
    out = pool.decode(q, bt, cl, max_ctx=30)
    assert pool.decode_status(2, 4, 30) & _lib.FLAG_CTX_RANGE
    assert torch.isfinite(out).all()
    cl[0] = -5
    out = pool.decode(q, bt, cl, max_ctx=64)
    assert pool.decode_status(2, 4, 64) & _lib.FLAG_CTX_RANGE
    assert (out[0] == 0).all()


def test_clean_call_clears_flags():
    pool, bt, cl, q = _setup()
    bt2 = bt.clone()
    bt2[0, 0] = 999
    pool.decode(q, bt2, cl, max_ctx=64)
    pool.decode(q, bt, cl, max_ctx=64)
    assert pool.decode_status(2, 4, 64) == 0


def test_slot_oob_flagged_by_append():
    pool, *_ = _setup()
    dev = torch.device("cuda", 0)
    k = torch.randn(3, 2, 128, device=dev)
    pool.reshape_and_cache(k, k, torch.tensor([0, 64 * 16, -1], dtype=torch.int32, device=dev))
    assert pool.pool_status() & _lib.FLAG_SLOT_OOB
    assert pool.pool_status() == 0  # read clears


def test_host_validation_codes():
    import ctypes as C
    pool, bt, cl, q = _setup()
    L = _lib.lib()
    out = torch.empty(2, 4, 128, device="cuda")
    ws = pool.workspace(2, 4, 64)
    # workspace too small
    rc = L.clove_cuda_paged_decode(pool.handle, q.data_ptr(), 4, bt.data_ptr(), 4, cl.data_ptr(), 2, 0.1, 64,
                                   out.data_ptr(), ws.data_ptr(), 8, None)
    assert rc == _lib.ERR_WORKSPACE
    # q heads not a multiple of kv heads
    rc = L.clove_cuda_paged_decode(pool.handle, q.data_ptr(), 3, bt.data_ptr(), 4, cl.data_ptr(), 2, 0.1, 64,
                                   out.data_ptr(), ws.data_ptr(), ws.numel(), None)
    assert rc == _lib.ERR_INVALID_ARG
    # max_ctx beyond the table capacity
    rc = L.clove_cuda_paged_decode(pool.handle, q.data_ptr(), 4, bt.data_ptr(), 4, cl.data_ptr(), 2, 0.1, 65,
                                   out.data_ptr(), ws.data_ptr(), ws.numel(), None)
    assert rc == _lib.ERR_INVALID_ARG
    # unsupported head_dim
    h = C.c_void_p()
    assert L.clove_cuda_pool_create(0, 4, 16, 1, 96, 0, C.byref(h)) == _lib.ERR_UNSUPPORTED
    # group > 8 not built
    q16 = torch.randn(2, 32, 128, device="cuda")
    with pytest.raises(_lib.CloveError):
        pool.decode(q16, bt, cl, max_ctx=64)


def test_empty_batch_and_zero_max_ctx():
    pool, bt, cl, q = _setup()
    out = torch.full((2, 4, 128), 7.0, device="cuda")
    cl0 = torch.zeros(2, dtype=torch.int32, device="cuda")
    pool.decode(q, bt, cl0, max_ctx=0, out=out)
    assert (out == 0).all()
    e = torch.empty(0, 4, 128, device="cuda")
    pool.decode(e, bt[:0], cl[:0], max_ctx=8)


def test_pool_create_owns_memory():
    import ctypes as C
    L = _lib.lib()
    h = C.c_void_p()
    _lib.check(L.clove_cuda_pool_create(0, 128, 16, 8, 64, 160, C.byref(h)))
    info = _lib.PoolInfo()
    _lib.check(L.clove_cuda_pool_info(h, C.byref(info)))
    assert info.owns_memory == 1 and info.plane_bytes == 128 * 16 * 8 * 64 * 2
    assert info.v_cache - info.k_cache == info.plane_bytes
    _lib.check(L.clove_cuda_pool_destroy(h))


@pytest.mark.parametrize("variant,group", [("mma", 4), ("mma", 2), ("simt", 3), ("simt", 1)])
def test_workspace_writes_stay_in_bounds(variant, group):
    # Multi-chunk sequences at the end of the batch write split-K partials at
    # the top of the workspace: a guard region right after the reported size
    # must come back untouched.
    from clove_b200 import set_decode_variant
    from clove_b200.workload import Spec, fill_values, make_layout
    from clove_b200 import KVPool
    spec = Spec("t", 64, 2 * group, 2, 128, 16, 0, torch.bfloat16, "uniform", 600, 3000, "permutation", seed=17)
    lay = make_layout(spec)
    dev = torch.device("cuda", 0)
    pool = KVPool(lay.num_blocks, 16, 2, 128, torch.bfloat16, 0)
    q, kn, vn, _ = fill_values(lay, dev, pool.storage)
    need = pool.workspace_bytes(lay.batch, spec.num_q_heads, lay.max_ctx)
    buf = torch.full((need + 65536,), 0xAB, dtype=torch.uint8, device=dev)
    out = torch.empty((lay.batch, spec.num_q_heads, 128), device=dev)
    bt = torch.from_numpy(lay.block_tables).to(dev)
    cl = torch.from_numpy(lay.context_lens).to(dev)
    set_decode_variant(variant)
    try:
        rc = _lib.lib().clove_cuda_paged_append_decode(
            pool.handle, q.data_ptr(), kn.data_ptr(), vn.data_ptr(), spec.num_q_heads, bt.data_ptr(),
            bt.shape[1], cl.data_ptr(), lay.batch, 0.0884, lay.max_ctx, out.data_ptr(), buf.data_ptr(), need,
            None)
        _lib.check(rc)
        torch.cuda.synchronize()
    finally:
        set_decode_variant("auto")
    assert (buf[need:] == 0xAB).all(), "decode wrote past the workspace size it reported"
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("variant,dtype,group", [("mma", torch.bfloat16, 4), ("simt", torch.float32, 1)])
def test_stuck_pipeline_wait_times_out_and_context_survives(variant, dtype, group):
    # Failure detection without a GPU fault: one stage is never filled (test
    # hook), so its consumer's bounded wait runs out; the call must finish,
    # report CLOVE_FLAG_TIMEOUT, and the next call must work normally.
    import time

    from clove_b200 import set_decode_variant
    from clove_b200.workload import Spec, make_layout
    from workload_check import run_layout_vs_oracle
    L = _lib.lib()
    spec = Spec("t", 8, 2 * group, 2, 128, 16, 0, dtype, "uniform", 200, 900, "permutation", seed=19)
    lay = make_layout(spec)
    from clove_b200 import KVPool
    from clove_b200.workload import fill_values
    dev = torch.device("cuda", 0)
    pool = KVPool(lay.num_blocks, 16, 2, 128, dtype, 0)
    q, kn, vn, _ = fill_values(lay, dev, pool.storage)
    bt = torch.from_numpy(lay.block_tables).to(dev)
    cl = torch.from_numpy(lay.context_lens).to(dev)
    set_decode_variant(variant)
    try:
        _lib.check(L.clove_cuda_debug_set(2000, 1))
        t0 = time.time()
        pool.append_decode(q, kn, vn, bt, cl, max_ctx=lay.max_ctx)
        flags = pool.decode_status(lay.batch, spec.num_q_heads, lay.max_ctx)
        elapsed = time.time() - t0
    finally:
        L.clove_cuda_debug_set(0, 0)
        set_decode_variant("auto")
    assert flags & _lib.FLAG_TIMEOUT, flags
    assert elapsed < 30
    # the context is intact: a normal call on a fresh workload is correct
    run_layout_vs_oracle(make_layout(spec, seed=23), 1e-5 if dtype == torch.float32 else 2e-2)
