"""Torch-facing wrapper of the C ABI: a device KV block pool and the decode /
append / gather calls on it.

PyTorch only supplies device memory and the current CUDA stream; every
computation runs in libclove_cuda.so.  Shapes follow the reference's
PagedAttention documentation (src/nn.rs:534-536):

  K/V planes    [num_blocks, block_size, num_kv_heads, head_dim]
  block_tables  int32 [batch, max_blocks_per_seq]
  context_lens  int32 [batch]
  q             [batch, num_q_heads, head_dim]   (or [batch, num_q_heads*head_dim])
  out           float32 [batch, num_q_heads, head_dim]
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream: torch.cuda.Stream | None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def set_decode_variant(variant: str) -> None:
    """'auto', 'simt' (CUDA-core kernel) or 'mma' (tensor-core kernel)."""
    _lib.check(_lib.lib().clove_cuda_set_decode_variant({"auto": 0, "simt": 1, "mma": 2}[variant]))


def launch_count() -> int:
    return int(_lib.lib().clove_cuda_launch_count())


class KVPool:
    """A paged KV cache on one GPU: K and V planes in one torch allocation
    [2, num_blocks, block_size, num_kv_heads, head_dim], wrapped by a
    clove_pool_t handle (which encodes the tensor maps the decode kernel's
    bulk copies use)."""

    def __init__(self, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.float32, device: int | torch.device = 0,
                 storage: torch.Tensor | None = None):
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("KVPool lives on a CUDA device")
        if dtype not in _DTYPES:
            raise ValueError(f"dtype {dtype} not supported (float32, bfloat16, float16)")
        shape = (2, num_blocks, block_size, num_kv_heads, head_dim)
        if storage is None:
            storage = torch.empty(shape, dtype=dtype, device=self.device)
        if tuple(storage.shape) != shape or storage.dtype != dtype or not storage.is_contiguous():
            raise ValueError(f"storage must be a contiguous {dtype} tensor of shape {shape}")
        self.storage = storage
        self.num_blocks, self.block_size = num_blocks, block_size
        self.num_kv_heads, self.head_dim, self.dtype = num_kv_heads, head_dim, dtype
        self._lib = _lib.lib()
        h = C.c_void_p()
        _lib.check(self._lib.clove_cuda_pool_wrap(
            self.device.index, storage[0].data_ptr(), storage[1].data_ptr(), num_blocks, block_size,
            num_kv_heads, head_dim, _DTYPES[dtype], C.byref(h)))
        self.handle = h
        self._ws: torch.Tensor | None = None
        self._qkv_ws: torch.Tensor | None = None  # fused projection scratch (kept zeroed by the kernel)

    @property
    def k_cache(self) -> torch.Tensor:
        return self.storage[0]

    @property
    def v_cache(self) -> torch.Tensor:
        return self.storage[1]

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.clove_cuda_pool_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- scratch ---------------------------------------------------------
    def workspace_bytes(self, batch: int, num_q_heads: int, max_ctx: int) -> int:
        return int(self._lib.clove_cuda_decode_workspace_size(self.handle, batch, num_q_heads, max_ctx))

    def workspace(self, batch: int, num_q_heads: int, max_ctx: int) -> torch.Tensor:
        """The pool's decode scratch, grown (never shrunk) to fit this call.
        Calls on one stream may share it; the check-flag word lives at its
        start, so decode_status reads the most recent call's flags."""
        n = max(self.workspace_bytes(batch, num_q_heads, max_ctx), 256)
        if self._ws is None or self._ws.numel() < n:
            if self._ws is not None:
                torch.cuda.current_stream(self.device).synchronize()  # queued calls may still use the old one
            self._ws = torch.zeros(n, dtype=torch.uint8, device=self.device)
        return self._ws

    # ---- ops ---------------------------------------------------------------
    def _check_rows(self, t: torch.Tensor, rows: int, heads: int, name: str) -> torch.Tensor:
        t = t.reshape(rows, heads, self.head_dim)
        if t.dtype != self.dtype or t.device != self.device or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous {self.dtype} tensor on {self.device}")
        return t

    @staticmethod
    def _check_i32(t: torch.Tensor, name: str) -> None:
        if t.dtype != torch.int32 or not t.is_contiguous() or not t.is_cuda:
            raise ValueError(f"{name} must be a contiguous int32 CUDA tensor")

    def reshape_and_cache(self, k: torch.Tensor, v: torch.Tensor, slot_mapping: torch.Tensor,
                          stream: torch.cuda.Stream | None = None) -> None:
        n = slot_mapping.numel()
        k = self._check_rows(k, n, self.num_kv_heads, "k")
        v = self._check_rows(v, n, self.num_kv_heads, "v")
        self._check_i32(slot_mapping, "slot_mapping")
        _lib.check(self._lib.clove_cuda_reshape_and_cache(self.handle, _ptr(k), _ptr(v), _ptr(slot_mapping), n,
                                                          _stream(stream)))

    def gather_kv(self, block_tables: torch.Tensor, context_lens: torch.Tensor, max_ctx: int,
                  stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        self._check_i32(block_tables, "block_tables")
        self._check_i32(context_lens, "context_lens")
        b = context_lens.numel()
        shape = (b, max_ctx, self.num_kv_heads, self.head_dim)
        ko = torch.empty(shape, dtype=self.dtype, device=self.device)
        vo = torch.empty(shape, dtype=self.dtype, device=self.device)
        _lib.check(self._lib.clove_cuda_gather_kv(self.handle, _ptr(block_tables), block_tables.shape[1],
                                                  _ptr(context_lens), b, max_ctx, _ptr(ko), _ptr(vo),
                                                  _stream(stream)))
        return ko, vo

    def decode(self, q: torch.Tensor, block_tables: torch.Tensor, context_lens: torch.Tensor,
               scale: float | None = None, max_ctx: int | None = None, out: torch.Tensor | None = None,
               k_new: torch.Tensor | None = None, v_new: torch.Tensor | None = None,
               stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """Paged decode; with k_new/v_new, the fused append + decode
        (context_lens are then the pre-append lengths)."""
        batch = context_lens.numel()
        if q.dim() == 2:
            hq = q.shape[1] // self.head_dim
        else:
            hq = q.shape[1]
        q = self._check_rows(q, batch, hq, "q")
        self._check_i32(block_tables, "block_tables")
        self._check_i32(context_lens, "context_lens")
        if block_tables.shape[0] != batch:
            raise ValueError("block_tables rows != batch")
        append = k_new is not None
        if max_ctx is None:  # forces a device sync; pass it on hot paths
            max_ctx = int(context_lens.max().item()) + (1 if append else 0) if batch else 0
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        if out is None:
            out = torch.empty((batch, hq, self.head_dim), dtype=torch.float32, device=self.device)
        ws = self.workspace(batch, hq, max_ctx)
        if append:
            k_new = self._check_rows(k_new, batch, self.num_kv_heads, "k_new")
            v_new = self._check_rows(v_new, batch, self.num_kv_heads, "v_new")
            rc = self._lib.clove_cuda_paged_append_decode(
                self.handle, _ptr(q), _ptr(k_new), _ptr(v_new), hq, _ptr(block_tables), block_tables.shape[1],
                _ptr(context_lens), batch, float(scale), max_ctx, _ptr(out), _ptr(ws), ws.numel(),
                _stream(stream))
        else:
            rc = self._lib.clove_cuda_paged_decode(
                self.handle, _ptr(q), hq, _ptr(block_tables), block_tables.shape[1], _ptr(context_lens), batch,
                float(scale), max_ctx, _ptr(out), _ptr(ws), ws.numel(), _stream(stream))
        _lib.check(rc)
        return out

    def append_decode(self, q, k_new, v_new, block_tables, context_lens, **kw) -> torch.Tensor:
        return self.decode(q, block_tables, context_lens, k_new=k_new, v_new=v_new, **kw)

    def pack_qkv_weights(self, w_t: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """W^T [(Hq + 2 Hkv) D, hidden] (pool dtype; W_q|W_k|W_v transposed
        and stacked) -> the fused projection's streaming layout (uint8)."""
        if w_t.dim() != 2 or w_t.dtype != self.dtype or not w_t.is_contiguous() or w_t.device != self.device:
            raise ValueError("w_t must be a contiguous [n_out, hidden] tensor of the pool's dtype and device")
        n_out, hidden = w_t.shape
        packed = torch.empty(int(self._lib.clove_cuda_qkv_packed_bytes(n_out, hidden)), dtype=torch.uint8,
                             device=self.device)
        _lib.check(self._lib.clove_cuda_qkv_pack_weights(_DTYPES[self.dtype], _ptr(w_t), n_out, hidden,
                                                         _ptr(packed), _stream(stream)))
        return packed

    def qkv_append(self, x: torch.Tensor, w_packed: torch.Tensor, bias: torch.Tensor | None, num_q_heads: int,
                   block_tables: torch.Tensor, context_lens: torch.Tensor, rope_theta: float = 0.0,
                   q_out: torch.Tensor | None = None, lens_out: torch.Tensor | None = None,
                   stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Fused Q/K/V projection + append: x [B, hidden] (pool dtype),
        w_packed from pack_qkv_weights, bias f32 [(Hq + 2 Hkv) D] or None.
        Stores k, v at slot context_lens[b] and returns (q [B, Hq, D] pool
        dtype, context_lens + 1)."""
        B = x.shape[0]
        n_out = (num_q_heads + 2 * self.num_kv_heads) * self.head_dim
        if x.dim() != 2 or x.dtype != self.dtype or not x.is_contiguous() or x.device != self.device:
            raise ValueError("x must be a contiguous [batch, hidden] tensor of the pool's dtype and device")
        hidden = x.shape[1]
        if (w_packed.dtype != torch.uint8 or w_packed.device != self.device or not w_packed.is_contiguous()
                or w_packed.numel() != int(self._lib.clove_cuda_qkv_packed_bytes(n_out, hidden))):
            raise ValueError("w_packed must come from pack_qkv_weights for this shape")
        if bias is not None and (bias.shape != (n_out,) or bias.dtype != torch.float32 or not bias.is_contiguous()):
            raise ValueError(f"bias must be f32 [{n_out}]")
        self._check_i32(block_tables, "block_tables")
        self._check_i32(context_lens, "context_lens")
        if q_out is None:
            q_out = torch.empty((B, num_q_heads, self.head_dim), dtype=self.dtype, device=self.device)
        if lens_out is None:
            lens_out = torch.empty(B, dtype=torch.int32, device=self.device)
        n = int(self._lib.clove_cuda_qkv_workspace_size(self.handle, B, hidden, num_q_heads))
        if self._qkv_ws is None or self._qkv_ws.numel() < n:
            if self._qkv_ws is not None:
                torch.cuda.current_stream(self.device).synchronize()  # queued calls may still use the old one
            self._qkv_ws = torch.zeros(max(n, 256), dtype=torch.uint8, device=self.device)  # zero-filled: counters
        _lib.check(self._lib.clove_cuda_qkv_append(
            self.handle, _ptr(x), _ptr(w_packed), _ptr(bias), B, hidden, num_q_heads, _ptr(block_tables),
            block_tables.shape[1], _ptr(context_lens), float(rope_theta), _ptr(q_out), _ptr(lens_out),
            _ptr(self._qkv_ws), self._qkv_ws.numel(), _stream(stream)))
        return q_out, lens_out

    def prefill(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor,
                block_tables: torch.Tensor, context_lens: torch.Tensor, max_ctx: int, scale: float | None = None,
                rope_theta: float = 0.0, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """Prefill packed prompts: write their K/V (RoPE-rotated K when
        rope_theta > 0) into the cache and return each token's causal
        attention output, f32 [num_tokens, num_q_heads, head_dim]."""
        T = q.shape[0]
        hq = q.shape[1] if q.dim() == 3 else q.shape[1] // self.head_dim
        q = self._check_rows(q, T, hq, "q")
        k = self._check_rows(k, T, self.num_kv_heads, "k")
        v = self._check_rows(v, T, self.num_kv_heads, "v")
        for t, n in ((cu_seqlens, "cu_seqlens"), (block_tables, "block_tables"), (context_lens, "context_lens")):
            self._check_i32(t, n)
        batch = context_lens.numel()
        if scale is None:
            scale = 1.0 / math.sqrt(self.head_dim)
        out = torch.empty((T, hq, self.head_dim), dtype=torch.float32, device=self.device)
        n = int(self._lib.clove_cuda_prefill_workspace_size(self.handle, T, hq, block_tables.shape[1], max_ctx))
        ws = torch.empty(max(n, 256), dtype=torch.uint8, device=self.device)
        _lib.check(self._lib.clove_cuda_paged_prefill(
            self.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(cu_seqlens), _ptr(block_tables), block_tables.shape[1],
            _ptr(context_lens), batch, T, hq, float(scale), float(rope_theta), max_ctx, _ptr(out), _ptr(ws),
            ws.numel(), _stream(stream)))
        return out

    def decode_status(self, batch: int, num_q_heads: int, max_ctx: int,
                      stream: torch.cuda.Stream | None = None) -> int:
        """Device check flags of the most recent decode (the arguments are
        kept for the interface; every decode of the pool shares one workspace)."""
        if self._ws is None:
            return 0
        ws = self._ws
        flags = C.c_int(0)
        rc = self._lib.clove_cuda_decode_status(_ptr(ws), _stream(stream), C.byref(flags))
        if rc not in (_lib.OK, _lib.ERR_DEVICE_CHECK):
            _lib.check(rc)
        return flags.value

    def pool_status(self, stream: torch.cuda.Stream | None = None) -> int:
        flags = C.c_int(0)
        rc = self._lib.clove_cuda_pool_status(self.handle, _stream(stream), C.byref(flags))
        if rc not in (_lib.OK, _lib.ERR_DEVICE_CHECK):
            _lib.check(rc)
        return flags.value
