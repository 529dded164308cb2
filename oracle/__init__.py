"""numpy front end of the CPU oracle (oracle/paged_oracle.cpp).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg use it as the checker or the timed CPU baseline; the product
path (clove_b200) never imports it.  PARITY UNPINNED: the reference holds no
PagedAttention vectors and cannot run here (see paged_oracle.cpp).

Arrays are numpy; 16-bit element types travel as uint16 bit patterns with a
dtype code (0 = f32, 16 = f16, 160 = bf16, the reference's FFI precision codes
at src/ffi.rs:305-313).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

F32, F16, BF16 = 0, 16, 160

_lib: C.CDLL | None = None


def build() -> Path:
    src = HERE / "paged_oracle.cpp"
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        vp, i, ll = C.c_void_p, C.c_int, C.c_longlong
        L.oracle_reshape_and_cache.argtypes = [vp, vp, vp, vp, vp, i, i, ll]
        L.oracle_reshape_and_cache.restype = i
        L.oracle_append_slots.argtypes = [vp, i, vp, i, i, vp]
        L.oracle_append_slots.restype = None
        L.oracle_gather_kv.argtypes = [vp, vp, vp, i, vp, i, i, i, i, i, vp, vp]
        L.oracle_gather_kv.restype = i
        L.oracle_decode_f64.argtypes = [i, vp, vp, vp, vp, i, vp, i, i, i, i, i, i, C.c_double, vp, i]
        L.oracle_decode_f64.restype = None
        L.oracle_decode_f32.argtypes = [i, vp, vp, vp, vp, i, vp, i, i, i, i, i, i, C.c_float, vp, i]
        L.oracle_decode_f32.restype = None
        L.oracle_mock_paged_attention.argtypes = [vp, vp, vp, C.c_uint, C.c_uint, C.c_uint, C.c_uint, vp]
        L.oracle_mock_paged_attention.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def default_threads() -> int:
    return os.cpu_count() or 1


def append_slots(block_tables, context_lens, block_size: int) -> np.ndarray:
    bt, cl = _i32(block_tables), _i32(context_lens)
    out = np.empty(cl.shape[0], np.int32)
    lib().oracle_append_slots(_p(bt), bt.shape[1], _p(cl), cl.shape[0], block_size, _p(out))
    return out


def reshape_and_cache(k_cache: np.ndarray, v_cache: np.ndarray, k: np.ndarray, v: np.ndarray,
                      slot_mapping) -> int:
    """In place on k_cache/v_cache ([NB, bs, Hkv, D]); returns # out-of-range slots."""
    sm = _i32(slot_mapping)
    nb, bs = k_cache.shape[0], k_cache.shape[1]
    row_bytes = k_cache[0, 0].nbytes
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    assert k.nbytes == sm.shape[0] * row_bytes
    return lib().oracle_reshape_and_cache(_p(k_cache), _p(v_cache), _p(k), _p(v), _p(sm), sm.shape[0],
                                          row_bytes, nb * bs)


def gather_kv(k_cache, v_cache, block_tables, context_lens, max_ctx: int):
    bt, cl = _i32(block_tables), _i32(context_lens)
    nb, bs = k_cache.shape[0], k_cache.shape[1]
    row_shape = k_cache.shape[2:]
    row_bytes = k_cache[0, 0].nbytes
    ko = np.empty((cl.shape[0], max_ctx) + row_shape, k_cache.dtype)
    vo = np.empty_like(ko)
    bad = lib().oracle_gather_kv(_p(k_cache), _p(v_cache), _p(bt), bt.shape[1], _p(cl), cl.shape[0], max_ctx, bs,
                                 nb, row_bytes, _p(ko), _p(vo))
    return ko, vo, bad


def _decode(fn: str, dtype_code: int, q, k_cache, v_cache, block_tables, context_lens, scale, out_dtype,
            nthreads):
    bt, cl = _i32(block_tables), _i32(context_lens)
    nb, bs, hkv, d = k_cache.shape
    batch = cl.shape[0]
    q = np.ascontiguousarray(q).reshape(batch, -1, d)
    hq = q.shape[1]
    out = np.empty((batch, hq, d), out_dtype)
    getattr(lib(), fn)(dtype_code, _p(q), _p(np.ascontiguousarray(k_cache)), _p(np.ascontiguousarray(v_cache)),
                       _p(bt), bt.shape[1], _p(cl), batch, hq, hkv, d, bs, nb, scale, _p(out),
                       nthreads or default_threads())
    return out


def decode_f64(dtype_code, q, k_cache, v_cache, block_tables, context_lens, scale, nthreads=0):
    """fp64 truth, out float64 [batch, hq, d]."""
    return _decode("oracle_decode_f64", dtype_code, q, k_cache, v_cache, block_tables, context_lens, scale,
                   np.float64, nthreads)


def decode_f32(dtype_code, q, k_cache, v_cache, block_tables, context_lens, scale, nthreads=0):
    """f32 restatement in the reference CPU idiom, out float32 [batch, hq, d]."""
    return _decode("oracle_decode_f32", dtype_code, q, k_cache, v_cache, block_tables, context_lens, scale,
                   np.float32, nthreads)


def mock_paged_attention(q: np.ndarray, kv_cache: np.ndarray, block_tables_1024: np.ndarray, seq_len: int,
                         head_dim: int, block_size: int) -> np.ndarray:
    """Literal restatement of the reference's placeholder kernel
    (src/lazy.rs:5255-5274); block_tables_1024 is uint32 with row stride 1024."""
    q = np.ascontiguousarray(q, np.float32)
    kv = np.ascontiguousarray(kv_cache, np.float32)
    bt = np.ascontiguousarray(block_tables_1024, np.uint32)
    out = np.empty_like(q)
    lib().oracle_mock_paged_attention(_p(q), _p(kv), _p(bt), q.size, seq_len, head_dim, block_size, _p(out))
    return out


# Every tolerance check made in this process: (test id, rtol, worst
# |x-r|/(|r|+rms), plain max |x-r|/|r|, fraction within plain rtol*|r|,
# elements).  The test session prints a summary of it.
PARITY_LOG: list[tuple] = []


def plain_relative_error(x: np.ndarray, ref: np.ndarray, rtol: float) -> tuple[float, float]:
    """(max |x - r| / |r| over the elements with r != 0, fraction of all
    elements with |x - r| <= rtol * |r|)."""
    x = np.asarray(x, np.float64)
    r = np.asarray(ref, np.float64)
    if not r.size:
        return 0.0, 1.0
    err = np.abs(x - r)
    nz = r != 0
    mx = float((err[nz] / np.abs(r[nz])).max()) if nz.any() else 0.0
    return mx, float((err <= rtol * np.abs(r)).mean())


def tolerance_ok(x: np.ndarray, ref: np.ndarray, rtol: float) -> tuple[bool, float]:
    """|x - r| <= rtol * (|r| + rms(r)) elementwise; returns (ok, worst ratio).
    The plain relative error (max |x - r| / |r|) is logged beside it in
    PARITY_LOG: near zeros of r it is large for any rounding, which is why
    the bar adds rms(r) to |r|."""
    x = np.asarray(x, np.float64)
    r = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(r * r))) if r.size else 0.0
    bound = rtol * (np.abs(r) + rms) + 1e-30
    ratio = np.abs(x - r) / bound
    worst = float(ratio.max()) * rtol if ratio.size else 0.0
    plain, within = plain_relative_error(x, r, rtol)
    PARITY_LOG.append((os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0], rtol, worst, plain, within,
                       int(r.size)))
    return bool((ratio <= 1.0).all()), worst


def rope(x: np.ndarray, positions, theta: float) -> np.ndarray:
    """float64 rotation of [..., tokens, heads, D] rows in adjacent pairs
    (2i, 2i+1) by pos * theta^(-2i/D) — apply_rope of the reference's
    FlashAttention shader (src/lazy.rs:4834-4842: angle = pos /
    10000^(i/head_dim) for the even index i).  positions: [tokens]."""
    x = np.asarray(x, np.float64)
    D = x.shape[-1]
    i = np.arange(D // 2)
    ang = np.asarray(positions, np.float64)[:, None] * theta ** (-2.0 * i / D)  # [T, D/2]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def linear(x: np.ndarray, w: np.ndarray, b: np.ndarray | None) -> np.ndarray:
    """float64 y = x W + b, the reference Linear (src/nn.rs:102-123:
    matmul(x, weights) then add(bias)); W is [in, out] as the reference
    stores it."""
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64)
    return y if b is None else y + np.asarray(b, np.float64)


def qkv_append(x, w_q, w_k, w_v, b_q, b_k, b_v, num_q_heads: int, num_kv_heads: int, positions,
               rope_theta: float = 0.0):
    """The projections of PagedAttention::forward (src/nn.rs:538-540) in
    float64, optionally rotated (RoPE) at each row's position: returns
    q [B, Hq, D], k [B, Hkv, D], v [B, Hkv, D] before rounding to the pool's
    element type.  The fused kernel writes k, v at slot positions[b]."""
    B = np.asarray(x).shape[0]
    q = linear(x, w_q, b_q).reshape(B, num_q_heads, -1)
    k = linear(x, w_k, b_k).reshape(B, num_kv_heads, -1)
    v = linear(x, w_v, b_v).reshape(B, num_kv_heads, -1)
    if rope_theta > 0:
        q = rope(q, positions, rope_theta)
        k = rope(k, positions, rope_theta)
    return q, k, v
