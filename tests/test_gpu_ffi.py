"""The reference-facing tensor-handle FFI (include/clove_ffi.h) on the GPU:
clove_paged_attention on tensors made from host data matches the golden
fixtures; errors return NULL; freed buffers are reused."""
import ctypes as C

import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu


def _t(L, arr, dtype_code):
    arr = np.ascontiguousarray(arr)
    shape = (C.c_int64 * arr.ndim)(*arr.shape)
    h = L.clove_tensor_create_nd(arr.ctypes.data, shape, arr.ndim, dtype_code, 0)
    assert h, "tensor create failed"
    return h


@pytest.mark.parametrize("name", ["f32_mha_small", "f32_gqa_zero_ctx", "bf16_gqa_bs32"])
def test_ffi_paged_attention_matches_golden(name):
    import oracle
    from clove_b200 import _lib
    L = _lib.lib()
    g = load_golden(name)
    code = 160 if str(g["dtype"]) == "bf16" else 0
    B, hq, d = g["q"].shape
    kv = np.stack([g["k_cache"], g["v_cache"]])
    hs = [_t(L, g["q"].reshape(B, hq * d), code), _t(L, g["k_new"].reshape(B, -1), code),
          _t(L, g["v_new"].reshape(B, -1), code), _t(L, kv, code),
          _t(L, g["block_tables"], _lib.DTYPE_I32), _t(L, g["context_lens"], _lib.DTYPE_I32)]
    out = L.clove_paged_attention(*hs)
    assert out, _lib.last_error()
    shape = (C.c_int64 * 8)()
    assert L.clove_tensor_shape(out, shape) == 2 and (shape[0], shape[1]) == (B, hq * d)
    host = np.empty((B, hq * d), np.float32)
    L.clove_tensor_data(out, host.ctypes.data)
    ok, worst = oracle.tolerance_ok(host.reshape(B, hq, d), g["expected"], 2e-2 if code else 1e-5)
    assert ok, worst
    # the cache tensor now holds the appended token, bit for bit
    kv_after = np.empty_like(kv)
    L.clove_tensor_data(hs[3], kv_after.ctypes.data)
    assert np.array_equal(kv_after[0].view(np.uint8), g["k_cache_after"].view(np.uint8))
    for h in hs + [out]:
        L.clove_tensor_free(h)
    assert L.clove_tensor_cache_bytes(0) > 0  # freed buffers are kept for reuse


def test_ffi_errors_return_null():
    from clove_b200 import _lib
    L = _lib.lib()
    g = load_golden("f32_mha_small")
    B, hq, d = g["q"].shape
    kv = np.stack([g["k_cache"], g["v_cache"]])
    q = _t(L, g["q"].reshape(B, -1), 0)
    kv_h = _t(L, kv, 0)
    bt = _t(L, g["block_tables"], _lib.DTYPE_I32)
    cl = _t(L, g["context_lens"], _lib.DTYPE_I32)
    k_bad = _t(L, np.zeros((B, 3), np.float32), 0)
    assert not L.clove_paged_attention(q, k_bad, k_bad, kv_h, bt, cl)
    assert "k, v" in _lib.last_error()
    cl_f = _t(L, g["context_lens"].astype(np.float32), 0)
    assert not L.clove_paged_attention(q, k_bad, k_bad, kv_h, bt, cl_f)
    for h in (q, kv_h, bt, cl, k_bad, cl_f):
        L.clove_tensor_free(h)


def test_ffi_bad_block_id_returns_null_with_flags():
    """A block-table entry outside the pool is never followed: the call
    returns NULL and the error text names the flag, instead of a clamped
    answer."""
    from clove_b200 import _lib
    L = _lib.lib()
    g = load_golden("f32_mha_small")
    B, hq, d = g["q"].shape
    kv = np.stack([g["k_cache"], g["v_cache"]])
    bt_bad = g["block_tables"].copy()
    bt_bad[1, 0] = kv.shape[1] + 5  # past the pool's last block
    hs = [_t(L, g["q"].reshape(B, -1), 0), _t(L, g["k_new"].reshape(B, -1), 0), _t(L, g["v_new"].reshape(B, -1), 0),
          _t(L, kv, 0), _t(L, bt_bad, _lib.DTYPE_I32), _t(L, g["context_lens"], _lib.DTYPE_I32)]
    assert not L.clove_paged_attention(*hs)
    msg = _lib.last_error()
    assert "block id outside the pool" in msg, msg
    # the next good call on the same handles works
    good_bt = _t(L, g["block_tables"], _lib.DTYPE_I32)
    out = L.clove_paged_attention(hs[0], hs[1], hs[2], hs[3], good_bt, hs[5])
    assert out, _lib.last_error()
    for h in hs + [good_bt, out]:
        L.clove_tensor_free(h)


def test_ffi_device_context_lens_without_host_copy():
    """context_lens handed over as device memory: the call sizes its scratch
    from the block table (no device-to-host read) and gives the same result
    as the host-made tensor."""
    import torch

    import oracle
    from clove_b200 import _lib
    L = _lib.lib()
    g = load_golden("f32_mha_small")
    B, hq, d = g["q"].shape
    kv = np.stack([g["k_cache"], g["v_cache"]])
    cl_dev = torch.from_numpy(g["context_lens"].astype(np.int32)).cuda()
    shp = (C.c_int64 * 1)(B)
    cl_h = L.clove_tensor_from_device(cl_dev.data_ptr(), shp, 1, _lib.DTYPE_I32, 0)
    hs = [_t(L, g["q"].reshape(B, -1), 0), _t(L, g["k_new"].reshape(B, -1), 0), _t(L, g["v_new"].reshape(B, -1), 0),
          _t(L, kv, 0), _t(L, g["block_tables"], _lib.DTYPE_I32)]
    out = L.clove_paged_attention(*hs, cl_h)
    assert out, _lib.last_error()
    host = np.empty((B, hq * d), np.float32)
    L.clove_tensor_data(out, host.ctypes.data)
    ok, worst = oracle.tolerance_ok(host.reshape(B, hq, d), g["expected"], 1e-5)
    assert ok, worst
    for h in hs + [cl_h, out]:
        L.clove_tensor_free(h)
