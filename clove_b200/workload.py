"""Seeded synthetic workloads for the five decode configurations.

No public dataset is involved: each configuration is generated from a fixed
seed with the shapes and value distributions of its specification.  Integer
metadata (context lengths, block tables) is drawn on the host with a numpy
Generator; K/V/Q values are drawn with a torch generator on the target device
(or on the CPU for small cases), so GPU and oracle consume the same numbers.

Conventions (one decode step = append one token per sequence, then attend
over ctx + 1 tokens):
  context_lens  int32 [B]   lengths BEFORE the append
  block_tables  int32 [B, MB], MB = max_b ceil((ctx_b + 1) / block_size);
                sequences own disjoint physical blocks.
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace

import numpy as np
import torch


@dataclass(frozen=True)
class Spec:
    name: str
    batch: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int  # 0: derived
    dtype: torch.dtype
    ctx: str                 # "uniform" | "fixed" | "lognormal"
    ctx_lo: int
    ctx_hi: int
    tables: str              # "permutation" | "contiguous_shuffled" | "fragmented"
    kv_scale: float = 1.0
    seed: int = 0
    description: str = ""


CONFIGS: dict[str, Spec] = {
    "c1": Spec("c1", 8, 8, 8, 64, 16, 512, torch.float32, "uniform", 64, 512, "permutation", seed=101,
               description="CPU-runnable f32 MHA 8x64, bs16, ctx U[64,512], 512-block pool"),
    "c2": Spec("c2", 64, 32, 32, 128, 16, 16384, torch.float32, "fixed", 2048, 2048, "contiguous_shuffled",
               seed=202, description="Llama-7B-shaped f32 MHA 32x128, bs16, ctx 2048, 16384-block pool"),
    "c3": Spec("c3", 128, 32, 8, 128, 16, 0, torch.bfloat16, "lognormal", 16, 8192, "permutation",
               kv_scale=0.5, seed=303,
               description="Llama-3-8B-shaped GQA 32q/8kv bf16, bs16, ctx lognormal(ln 1024, 0.8) in [16,8192]"),
    "c4": Spec("c4", 8, 64, 8, 128, 32, 40960, torch.bfloat16, "uniform", 32768, 131072, "permutation",
               seed=404, description="70B-shaped long context 64q/8kv bf16, bs32, ctx U[32768,131072]"),
    "c5": Spec("c5", 256, 32, 8, 128, 32, 65536, torch.bfloat16, "uniform", 1, 4096, "fragmented", seed=505,
               description="fragmented serving mix 32q/8kv bf16, bs32, ctx U[1,4096], 50% of 65536 blocks taken"),
}


@dataclass
class Layout:
    """Host-side metadata of one decode step."""
    spec: Spec
    context_lens: np.ndarray  # int32 [B] (pre-append)
    block_tables: np.ndarray  # int32 [B, MB]
    num_blocks: int
    seed: int
    extra: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return int(self.context_lens.shape[0])

    @property
    def max_ctx(self) -> int:
        """Tokens attended by the longest sequence (after the append)."""
        return int(self.context_lens.max()) + 1 if self.batch else 0

    def kv_bytes(self) -> int:
        """Algorithmic K+V bytes one decode step reads: sum (ctx+1)*2*Hkv*D*s."""
        s = torch.tensor([], dtype=self.spec.dtype).element_size()
        return int((self.context_lens.astype(np.int64) + 1).sum()) * 2 * self.spec.num_kv_heads * \
            self.spec.head_dim * s


def _context_lens(spec: Spec, rng: np.random.Generator, batch: int) -> np.ndarray:
    if spec.ctx == "fixed":
        c = np.full(batch, spec.ctx_lo)
    elif spec.ctx == "uniform":
        c = rng.integers(spec.ctx_lo, spec.ctx_hi + 1, size=batch)
    elif spec.ctx == "lognormal":
        c = np.clip(np.rint(np.exp(rng.normal(np.log(1024.0), 0.8, size=batch))), spec.ctx_lo, spec.ctx_hi)
    else:
        raise ValueError(spec.ctx)
    return c.astype(np.int32)


def make_layout(spec: Spec, seed: int | None = None, batch: int | None = None,
                ctx_scale: float = 1.0, context_lens: np.ndarray | None = None) -> Layout:
    """Context lengths and block tables for `spec` (optionally a smaller
    batch, or context lengths scaled down for CPU-sized parity cases).  With
    `context_lens`, those lengths are used as given and only the block
    tables are drawn."""
    seed = spec.seed if seed is None else seed
    rng = np.random.default_rng(seed)
    if context_lens is not None:
        ctx = np.asarray(context_lens, np.int32)
        batch = int(ctx.shape[0])
    else:
        batch = spec.batch if batch is None else batch
        ctx = _context_lens(spec, rng, batch)
    if ctx_scale != 1.0:
        ctx = np.maximum(1, np.rint(ctx * ctx_scale)).astype(np.int32)
    bs = spec.block_size
    need = (ctx.astype(np.int64) + 1 + bs - 1) // bs  # blocks incl. the appended token
    mb = int(need.max()) if batch else 1
    total = int(need.sum())
    nb = spec.num_blocks
    if spec.tables == "fragmented":
        nb = nb or 1 << max(1, int(np.ceil(np.log2(2 * total))))
        taken = np.zeros(nb, bool)
        taken[rng.permutation(nb)[: nb // 2]] = True  # 50% pre-allocated at random
        free = np.flatnonzero(~taken)
        free = free[rng.permutation(free.shape[0])]
        if total > free.shape[0]:
            raise ValueError("pool too small for this layout")
        ids = free[:total]
    elif spec.tables == "contiguous_shuffled":
        nb = nb or max(total, 1)
        perm = rng.permutation(nb)
        ids = perm[np.arange(total)]  # contiguous assignment, then a seeded relabelling
    else:  # permutation
        if not nb:
            nb = 1 << max(1, int(np.ceil(np.log2(2 * total))))  # next pow2 >= 2x need
        if total > nb:
            nb = total
        ids = rng.permutation(nb)[:total]
    bt = np.zeros((batch, mb), np.int32)
    off = 0
    for b in range(batch):
        n = int(need[b])
        bt[b, :n] = ids[off: off + n]
        off += n
    return Layout(spec, ctx, bt, nb, seed)


# How each configuration's batch shards over GPUs (sequences are
# independent; every rank owns its own block pool and tables).  c2 follows
# distribute_batch's contiguous split; the ragged configurations balance
# attended tokens.  c4 splits KV heads instead (see clove_b200.distributed).
SHARD_POLICY = {"c1": "contiguous", "c2": "contiguous", "c3": "tokens", "c5": "tokens"}


def shard_layout(spec: Spec, world: int, rank: int, policy: str | None = None,
                 batch: int | None = None) -> tuple[Layout, np.ndarray]:
    """Rank `rank`'s share of `spec`'s batch over `world` GPUs: the global
    context lengths are drawn from the configuration's seed (identical on
    every rank), the rank takes its sequences, and its own pool of
    num_blocks / world blocks (derived when the spec derives it) gets block
    tables drawn with the configuration's table rule and a rank-specific
    seed.  Returns (layout, global sequence indices of this rank)."""
    from .sharding import contiguous_shards, token_balanced_shards
    glob = make_layout(spec, batch=batch)
    if world <= 1:
        return glob, np.arange(glob.batch)
    policy = policy or SHARD_POLICY.get(spec.name, "contiguous")
    if policy == "contiguous":
        idx = contiguous_shards(glob.batch, world)[rank]
    elif policy == "tokens":
        idx = token_balanced_shards(glob.context_lens, world)[rank]
    else:
        raise ValueError(policy)
    local = spec if not spec.num_blocks else replace(spec, num_blocks=max(1, spec.num_blocks // world))
    lay = make_layout(local, seed=spec.seed + 7919 * (rank + 1), context_lens=glob.context_lens[idx])
    lay.extra["global_batch"] = glob.batch
    lay.extra["global_kv_bytes"] = glob.kv_bytes()
    return lay, idx


def fill_values(layout: Layout, device: torch.device | str, pool_storage: torch.Tensor | None = None,
                chunk_blocks: int = 4096):
    """Draw q, k_new, v_new and the pool contents.  Returns (q, k_new, v_new,
    storage) with storage [2, NB, bs, Hkv, D] in the spec dtype."""
    spec = layout.spec
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(layout.seed * 7919 + 17)
    B, hq, hkv, d, bs = layout.batch, spec.num_q_heads, spec.num_kv_heads, spec.head_dim, spec.block_size
    if pool_storage is None:
        pool_storage = torch.empty((2, layout.num_blocks, bs, hkv, d), dtype=spec.dtype, device=dev)
    flat = pool_storage.view(2, layout.num_blocks, -1)
    tmp = None
    for p in range(2):
        for b0 in range(0, layout.num_blocks, chunk_blocks):
            b1 = min(layout.num_blocks, b0 + chunk_blocks)
            shape = (b1 - b0, flat.shape[2])
            if tmp is None or tmp.shape != shape:
                tmp = torch.empty(shape, dtype=torch.float32, device=dev)
            tmp.normal_(generator=gen)
            if spec.kv_scale != 1.0:
                tmp.mul_(spec.kv_scale)
            flat[p, b0:b1].copy_(tmp)
    q = torch.randn((B, hq, d), generator=gen, device=dev).to(spec.dtype)
    k_new = (torch.randn((B, hkv, d), generator=gen, device=dev) * spec.kv_scale).to(spec.dtype)
    v_new = (torch.randn((B, hkv, d), generator=gen, device=dev) * spec.kv_scale).to(spec.dtype)
    return q, k_new, v_new, pool_storage


def to_numpy_bits(t: torch.Tensor) -> np.ndarray:
    """Host numpy view with 16-bit types as uint16 bit patterns."""
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def dtype_code(dtype: torch.dtype) -> int:
    return {torch.float32: 0, torch.float16: 16, torch.bfloat16: 160}[dtype]
