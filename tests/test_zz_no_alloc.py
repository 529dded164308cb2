"""The append + decode entry point for callers that cannot allocate device
memory when they decode (their HBM is already handed to a KV pool, or their
only allocator may not be called on the serving path).  It takes no
workspace and uses the library's built-in scratch instead.

Checked through the C ABI against clove_cuda_paged_append_decode (which
takes a caller workspace) on the same inputs, on two calls in a row — the
second call finds the scratch holding the first call's leftovers.  This file
is collected last so a run that stops at the first failure has already run
every other test.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from clove_b200 import _lib

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


@pytest.mark.parametrize("name,batch,ctx_scale", [("c1", 8, 1.0), ("c3", 16, 0.5), ("c4", 2, 0.05)])
def test_noalloc_matches_workspace_entry_point(name, batch, ctx_scale):
    from workload_check import tol_check
    lay, pool, q, kn, vn, bt, cl = _case(name, batch, ctx_scale)
    # The append writes the same token to the same slot each time, so the
    # cache is the same before every call below.
    ref = pool.append_decode(q, kn, vn, bt, cl, max_ctx=lay.max_ctx).cpu().numpy()
    for _ in range(2):
        out = torch.full((lay.batch, lay.spec.num_q_heads, lay.spec.head_dim), float("nan"), device="cuda")
        _lib.check(_noalloc(pool, q, kn, vn, bt, cl, lay, out))
        torch.cuda.synchronize()
        tol_check(out.cpu().numpy(), ref, RT[lay.spec.dtype])


def test_noalloc_rejects_oversized_call():
    # 64 sequences of up to 60000 tokens with 64 query heads need far more
    # scratch than the built-in 32 MiB; the call is refused before any launch.
    from clove_b200 import KVPool
    big = KVPool(256, 16, 8, 128, torch.bfloat16, 0)
    need = big.workspace_bytes(64, 64, 60000)
    assert need > 32 << 20
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    out = torch.empty(16, device="cuda")
    rc = _lib.lib().clove_cuda_paged_append_decode_noalloc(
        big.handle, dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), 64, dummy.data_ptr(), 3750,
        dummy.data_ptr(), 64, 0.088, 60000, out.data_ptr(), None)
    assert rc == _lib.ERR_WORKSPACE
    assert "scratch" in _lib.last_error()
