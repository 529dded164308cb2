"""Multi-GPU decode: one process per GPU over torch.distributed.

Two partitionings (the reference's orchestrator is MultiGPUOrchestrator,
src/distributed.rs:41-313, with distribute_batch at :184-200):

  sequence sharding   each rank owns a subset of sequences, its own KV block
                      pool and block tables; no collective on the data path.
  KV-head sharding    (long-context configuration) each rank owns a contiguous
                      range of KV heads of every sequence — its pool stores only
                      those heads — decodes the query heads that read them, and
                      one all-gather assembles [batch, num_q_heads, head_dim].

The compute is the single-GPU C-ABI path; torch.distributed (NCCL on GPUs,
gloo on CPU) carries only the output gather.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .sharding import head_shards


def init_from_env(backend: str | None = None) -> tuple[int, int, int]:
    """(world_size, rank, local_rank) from the torchrun environment; joins the
    process group when world_size > 1."""
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend)
    return ws, rank, local


def local_heads(num_kv_heads: int, group: int, world: int, rank: int) -> tuple[range, range]:
    """(KV heads, query heads) this rank owns under KV-head sharding."""
    return head_shards(num_kv_heads, group, world)[rank]


def gather_heads(out_local: torch.Tensor, world: int, group_pg=None) -> torch.Tensor:
    """All-gather per-rank outputs [B, hq_local, D] into [B, world*hq_local, D]
    (rank r's query heads land at r*hq_local .. (r+1)*hq_local - 1)."""
    if world == 1:
        return out_local
    B, hl, D = out_local.shape
    buf = torch.empty((world * B, hl, D), dtype=out_local.dtype, device=out_local.device)
    dist.all_gather_into_tensor(buf, out_local.contiguous(), group=group_pg)
    return buf.view(world, B, hl, D).permute(1, 0, 2, 3).reshape(B, world * hl, D)


def head_sharded_append_decode(pool_local, q_local: torch.Tensor, k_new_local: torch.Tensor,
                               v_new_local: torch.Tensor, block_tables: torch.Tensor,
                               context_lens: torch.Tensor, world: int, max_ctx: int,
                               scale: float | None = None, out_local: torch.Tensor | None = None,
                               gather_buf: torch.Tensor | None = None) -> torch.Tensor:
    """Append + decode under KV-head sharding.  Every argument is this rank's
    share: q_local [B, hq_local, D] holds the query heads of the KV heads in
    pool_local (rank r: query heads r*hq_local .. (r+1)*hq_local - 1, as
    local_heads gives them), k_new_local / v_new_local [B, hkv_local, D].
    Returns the full [B, world*hq_local, D] output on every rank.
    Preallocated out_local / gather_buf make the call free of allocations
    (e.g. for CUDA-graph capture)."""
    out_local = pool_local.append_decode(q_local, k_new_local, v_new_local, block_tables, context_lens,
                                         scale=scale, max_ctx=max_ctx, out=out_local)
    if world == 1:
        return out_local
    B, hl, D = out_local.shape
    if gather_buf is None:
        gather_buf = torch.empty((world * B, hl, D), dtype=out_local.dtype, device=out_local.device)
    dist.all_gather_into_tensor(gather_buf, out_local)
    return gather_buf.view(world, B, hl, D).permute(1, 0, 2, 3)  # [B, world, hl, D] view
