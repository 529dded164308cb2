"""ctypes binding of libclove_cuda.so (the C ABI in include/clove_cuda.h).

The library is loaded from this package directory only; if it is missing the
import fails loudly — there is no CPU fallback behind these entry points.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libclove_cuda.so"

OK = 0
ERR_INVALID_ARG = -1
ERR_UNSUPPORTED = -2
ERR_CUDA = -3
ERR_OOM = -4
ERR_WORKSPACE = -5
ERR_DEVICE_CHECK = -6
ERR_NO_DEVICE = -7

FLAG_BLOCK_OOB = 1
FLAG_CTX_RANGE = 2
FLAG_SLOT_OOB = 4
FLAG_TIMEOUT = 8

IPC_HANDLE_BYTES = 64

DTYPE_F32 = 0
DTYPE_F16 = 16
DTYPE_BF16 = 160

# Every symbol include/clove_cuda.h declares, with (restype, argtypes).
_vp, _i, _f, _sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t
_ip = C.POINTER(C.c_int)


class PoolInfo(C.Structure):
    _fields_ = [("device", C.c_int), ("num_blocks", C.c_int), ("block_size", C.c_int),
                ("num_kv_heads", C.c_int), ("head_dim", C.c_int), ("dtype", C.c_int),
                ("owns_memory", C.c_int), ("k_cache", C.c_void_p), ("v_cache", C.c_void_p),
                ("plane_bytes", C.c_size_t)]


SIGNATURES = {
    "clove_cuda_init": (_i, [_ip]),
    "clove_cuda_get_last_error": (_i, [C.c_char_p, _sz]),
    "clove_cuda_pool_create": (_i, [_i, _i, _i, _i, _i, _i, C.POINTER(_vp)]),
    "clove_cuda_pool_wrap": (_i, [_i, _vp, _vp, _i, _i, _i, _i, _i, C.POINTER(_vp)]),
    "clove_cuda_pool_destroy": (_i, [_vp]),
    "clove_cuda_pool_status": (_i, [_vp, _vp, _ip]),
    "clove_cuda_pool_info": (_i, [_vp, C.POINTER(PoolInfo)]),
    "clove_cuda_reshape_and_cache": (_i, [_vp, _vp, _vp, _vp, _i, _vp]),
    "clove_cuda_gather_kv": (_i, [_vp, _vp, _i, _vp, _i, _i, _vp, _vp, _vp]),
    "clove_cuda_decode_workspace_size": (_sz, [_vp, _i, _i, _i]),
    "clove_cuda_paged_decode": (_i, [_vp, _vp, _i, _vp, _i, _vp, _i, _f, _i, _vp, _vp, _sz, _vp]),
    "clove_cuda_paged_append_decode": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _i, _vp, _i, _f, _i, _vp, _vp,
                                            _sz, _vp]),
    "clove_cuda_paged_append_decode_noalloc": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _i, _vp, _i, _f, _i, _vp, _vp]),
    "clove_cuda_noalloc_status": (_i, [_i, _vp, _ip]),
    "clove_cuda_peer_gather_buffer_bytes": (_sz, [_sz, _i]),
    "clove_cuda_peer_buffer_alloc": (_i, [_i, _sz, C.POINTER(_vp), _vp]),
    "clove_cuda_peer_buffer_open": (_i, [_i, _vp, C.POINTER(_vp)]),
    "clove_cuda_peer_buffer_close": (_i, [_vp]),
    "clove_cuda_peer_buffer_free": (_i, [_vp]),
    "clove_cuda_peer_gather": (_i, [_vp, _sz, _vp, _i, _i, _vp, _vp]),
    "clove_cuda_peer_gather_status": (_i, [_vp, _sz, _i, _vp, _ip]),
    "clove_cuda_prefill_workspace_size": (_sz, [_vp, _i, _i, _i, _i]),
    "clove_cuda_paged_prefill": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _f, _f, _i, _vp, _vp, _sz,
                                      _vp]),
    "clove_cuda_qkv_packed_bytes": (_sz, [_i, _i]),
    "clove_cuda_qkv_pack_weights": (_i, [_i, _vp, _i, _i, _vp, _vp]),
    "clove_cuda_qkv_workspace_size": (_sz, [_vp, _i, _i, _i]),
    "clove_cuda_qkv_append": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp, _i, _vp, _f, _vp, _vp, _vp, _sz, _vp]),
    "clove_cuda_decode_status": (_i, [_vp, _vp, _ip]),
    "clove_cuda_set_decode_variant": (_i, [_i]),
    "clove_cuda_launch_count": (C.c_uint64, []),
    "clove_cuda_debug_set": (_i, [C.c_uint32, _i]),
    "clove_cuda_debug_phase_timing": (_i, [_i]),
    "clove_cuda_debug_trace": (_i, [_vp]),
    "clove_cuda_debug_phase_ms": (_i, [C.POINTER(_f), C.POINTER(_f), C.POINTER(_f)]),
}


DTYPE_I32 = 32
_i64p = C.POINTER(C.c_int64)

# include/clove_ffi.h: the reference-facing tensor-handle FFI.
FFI_SIGNATURES = {
    "clove_tensor_create": (_vp, [C.POINTER(C.c_float), _sz, _sz]),
    "clove_tensor_create_nd": (_vp, [_vp, _i64p, _i, _i, _i]),
    "clove_tensor_from_device": (_vp, [_vp, _i64p, _i, _i, _i]),
    "clove_tensor_free": (None, [_vp]),
    "clove_tensor_data": (None, [_vp, _vp]),
    "clove_tensor_shape": (_i, [_vp, _i64p]),
    "clove_paged_attention": (_vp, [_vp, _vp, _vp, _vp, _vp, _vp]),
    "clove_tensor_cache_bytes": (_sz, [_i]),
}


ERR_NO_BLOCKS = -8
ERR_NO_SEQ = -9
_i32p = C.POINTER(C.c_int32)

# include/clove_blocks.h: the KV block manager.
BLOCKS_SIGNATURES = {
    "clove_blocks_create": (_i, [_i, _i, _i, C.POINTER(_vp)]),
    "clove_blocks_destroy": (_i, [_vp]),
    "clove_blocks_add": (_i, [_vp, _i, _i]),
    "clove_blocks_reserve": (_i, [_vp, _i, _i, _vp, _vp, _ip]),
    "clove_blocks_fork": (_i, [_vp, _i, _i]),
    "clove_blocks_free": (_i, [_vp, _i]),
    "clove_blocks_num_free": (_i, [_vp]),
    "clove_blocks_seq_len": (_i, [_vp, _i]),
    "clove_blocks_seq_blocks": (_i, [_vp, _i]),
    "clove_blocks_export": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "clove_cuda_copy_blocks": (_i, [_vp, _vp, _vp, _i, _vp]),
}


def load(path: Path | str = LIB_PATH) -> C.CDLL:
    path = Path(path)
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build it with `python -m clove_b200.build` "
            "(the CUDA extension is required; there is no fallback)")
    lib = C.CDLL(str(path))
    for name, (res, args) in {**SIGNATURES, **FFI_SIGNATURES, **BLOCKS_SIGNATURES}.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


class CloveError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"clove_cuda error {code}: {msg}")
        self.code = code


_LIB: C.CDLL | None = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = load()
    return _LIB


def last_error() -> str:
    buf = C.create_string_buffer(512)
    lib().clove_cuda_get_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(code: int) -> int:
    if code != OK:
        raise CloveError(code, last_error())
    return code
