"""Python mirror of the reference's PagedAttention interface on the CUDA path.

  CudaBackend.paged_attention(q, k, v, kv_cache, block_tables, context_lens)
      <- Backend::paged_attention, src/backend.rs:249-256
  PagedAttention(dim, num_heads).forward(x, kv_cache, block_tables, context_lens)
      <- PagedAttention::forward, src/nn.rs:531-546

Tensors are torch CUDA tensors.  kv_cache is ONE tensor
[2, num_blocks, block_size, num_kv_heads, head_dim] (K plane, V plane): the
reference passes a single kv_cache and documents the per-plane layout at
src/nn.rs:534.  q: [B, Hq*D]; k, v: [B, Hkv*D] — the new token's projections;
context_lens: int32 [B] lengths before this token.  The call appends k, v
through the slot mapping and attends over ctx + 1 tokens; it returns f32
[B, Hq*D] (the reference output dtype, src/lazy.rs:5252).  context_lens is
not modified; the caller advances it.

Errors raise CloveError (the reference panics, src/backend.rs:2937-2948).
"""
from __future__ import annotations

import math
from collections import OrderedDict

import torch

from .ops import KVPool


class CudaBackend:
    """Stateless apart from a bounded cache of pool handles keyed by kv_cache
    storage.  A cached pool keeps its kv_cache alive, so the cache holds the
    most recently used MAX_POOLS caches only; an evicted one is wrapped again
    (tensor maps re-encoded) on its next use."""

    MAX_POOLS = 64
    _pools: OrderedDict[tuple[int, tuple, torch.dtype], KVPool] = OrderedDict()

    @classmethod
    def _pool(cls, kv_cache: torch.Tensor) -> KVPool:
        if kv_cache.dim() != 5 or kv_cache.shape[0] != 2:
            raise ValueError("kv_cache must be [2, num_blocks, block_size, num_kv_heads, head_dim]")
        key = (kv_cache.data_ptr(), tuple(kv_cache.shape), kv_cache.dtype)
        pool = cls._pools.get(key)
        if pool is None:
            _, nb, bs, hkv, d = kv_cache.shape
            pool = KVPool(nb, bs, hkv, d, dtype=kv_cache.dtype, device=kv_cache.device, storage=kv_cache)
            cls._pools[key] = pool
            while len(cls._pools) > cls.MAX_POOLS:
                cls._pools.popitem(last=False)  # the handle closes once nothing else holds the pool
        cls._pools.move_to_end(key)
        return pool

    @classmethod
    def paged_attention(cls, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_cache: torch.Tensor,
                        block_tables: torch.Tensor, context_lens: torch.Tensor,
                        max_ctx: int | None = None) -> torch.Tensor:
        pool = cls._pool(kv_cache)
        B = context_lens.numel()
        out = pool.append_decode(q.contiguous(), k.contiguous(), v.contiguous(), block_tables, context_lens,
                                 scale=1.0 / math.sqrt(pool.head_dim), max_ctx=max_ctx)
        return out.reshape(B, -1)


class Linear:
    """y = x W + b with W [in, out] (the reference Linear, src/nn.rs:102-123).
    A plain library GEMM: the projections are not part of the decode path."""

    def __init__(self, in_dim: int, out_dim: int, device, dtype=torch.float32, generator=None):
        bound = 1.0 / math.sqrt(in_dim)
        self.weight = (torch.rand((in_dim, out_dim), generator=generator, device=device) * 2 - 1).mul_(bound) \
            .to(dtype)
        self.bias = torch.zeros(out_dim, device=device, dtype=dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return torch.addmm(self.bias, x, self.weight)


class PagedAttention:
    """PagedAttention::new(dim, num_heads) (src/nn.rs:543-553) with the KV-head
    count added for GQA: w_k/w_v project to num_kv_heads*head_dim."""

    def __init__(self, dim: int, num_heads: int, num_kv_heads: int | None = None, device="cuda",
                 dtype=torch.float32, seed: int = 0):
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads or num_heads
        self.head_dim = dim // num_heads
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        kv_dim = self.num_kv_heads * self.head_dim
        self.w_q = Linear(dim, dim, device, dtype, g)
        self.w_k = Linear(dim, kv_dim, device, dtype, g)
        self.w_v = Linear(dim, kv_dim, device, dtype, g)
        self.w_o = Linear(dim, dim, device, torch.float32, g)
        self._fused: tuple[torch.Tensor, torch.Tensor] | None = None

    def forward(self, x: torch.Tensor, kv_cache: torch.Tensor, block_tables: torch.Tensor,
                context_lens: torch.Tensor, max_ctx: int | None = None) -> torch.Tensor:
        q = self.w_q.forward(x)
        k = self.w_k.forward(x)
        v = self.w_v.forward(x)
        attn = CudaBackend.paged_attention(q, k, v, kv_cache, block_tables, context_lens, max_ctx=max_ctx)
        return self.w_o.forward(attn)

    def fused_qkv(self, pool: KVPool) -> tuple[torch.Tensor, torch.Tensor]:
        """The projection weights in clove_cuda_qkv_append's streaming layout
        (W_q|W_k|W_v transposed, stacked and packed by the pool) and the f32
        bias b_q|b_k|b_v.  Built once per weight update."""
        if self._fused is None:
            w = torch.cat([self.w_q.weight, self.w_k.weight, self.w_v.weight], dim=1).t().contiguous()
            b = torch.cat([self.w_q.bias, self.w_k.bias, self.w_v.bias]).float().contiguous()
            self._fused = (pool.pack_qkv_weights(w.to(pool.dtype)), b)
        return self._fused

    def forward_fused(self, x: torch.Tensor, kv_cache: torch.Tensor, block_tables: torch.Tensor,
                      context_lens: torch.Tensor, max_ctx: int, rope_theta: float = 0.0) -> torch.Tensor:
        """forward() with the three projections and the append in one
        tensor-core kernel (16-bit caches): x [B, dim] in the cache dtype;
        max_ctx bounds context_lens + 1.  Same result as forward() up to the
        projections' rounding to the cache dtype."""
        pool = CudaBackend._pool(kv_cache)
        w, b = self.fused_qkv(pool)
        q, lens = pool.qkv_append(x.to(pool.dtype).contiguous(), w, b, self.num_heads, block_tables, context_lens,
                                  rope_theta=rope_theta)
        attn = pool.decode(q, block_tables, lens, max_ctx=max_ctx)
        return self.w_o.forward(attn.reshape(x.shape[0], -1))

    def prefill(self, x: torch.Tensor, kv_cache: torch.Tensor, block_tables: torch.Tensor,
                context_lens: torch.Tensor, cu_seqlens: torch.Tensor, max_ctx: int,
                rope_theta: float = 0.0) -> torch.Tensor:
        """Prompt pass: x [num_tokens, dim] packed by cu_seqlens; writes the
        prompt's K/V into the paged cache and returns [num_tokens, dim].  The
        attention is the reference's causal FlashAttention step
        (src/lazy.rs:4821-4923) on the paged cache (CudaBackend path)."""
        pool = CudaBackend._pool(kv_cache)
        T = x.shape[0]
        q = self.w_q.forward(x).reshape(T, self.num_heads, self.head_dim).contiguous()
        k = self.w_k.forward(x).reshape(T, self.num_kv_heads, self.head_dim).contiguous()
        v = self.w_v.forward(x).reshape(T, self.num_kv_heads, self.head_dim).contiguous()
        attn = pool.prefill(q, k, v, cu_seqlens, block_tables, context_lens, max_ctx=max_ctx, rope_theta=rope_theta)
        return self.w_o.forward(attn.reshape(T, -1))

    def parameters(self) -> list[torch.Tensor]:
        return [t for l in (self.w_q, self.w_k, self.w_v, self.w_o) for t in (l.weight, l.bias)]
