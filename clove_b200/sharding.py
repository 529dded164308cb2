"""Multi-GPU partitioning of a decode batch.

Sequences are independent, so the batch shards across ranks with no data-path
collective.  Only the long-context configuration splits KV heads across ranks
and all-gathers the per-rank outputs.
"""
from __future__ import annotations

import numpy as np


def distribute_batch(total_batch_size: int, num_shards: int) -> list[int]:
    """Contiguous split with the remainder going to the lowest ranks — the
    rule of MultiGPUOrchestrator::distribute_batch (src/distributed.rs:184-200);
    zero shards returns the whole batch as one shard."""
    if num_shards <= 0:
        return [total_batch_size]
    base, rem = divmod(total_batch_size, num_shards)
    return [base + 1 if i < rem else base for i in range(num_shards)]


def contiguous_shards(batch: int, num_shards: int) -> list[np.ndarray]:
    """Sequence indices per rank under distribute_batch."""
    sizes = distribute_batch(batch, num_shards)
    bounds = np.cumsum([0] + sizes)
    return [np.arange(bounds[i], bounds[i + 1]) for i in range(len(sizes))]


def token_balanced_shards(context_lens, num_shards: int) -> list[np.ndarray]:
    """Greedy longest-processing-time assignment of sequences to ranks by
    attended tokens (ragged batches); each rank's list is sorted.  Outputs do
    not depend on the assignment, only the step time does."""
    ctx = np.asarray(context_lens, np.int64)
    order = np.argsort(-ctx, kind="stable")
    load = np.zeros(max(num_shards, 1), np.int64)
    owner = np.empty(ctx.shape[0], np.int64)
    for i in order:
        r = int(np.argmin(load))
        owner[i] = r
        load[r] += ctx[i] + 1
    return [np.flatnonzero(owner == r) for r in range(max(num_shards, 1))]


def head_shards(num_kv_heads: int, group: int, num_shards: int) -> list[tuple[range, range]]:
    """KV-head split for the long-context configuration: rank r owns a
    contiguous range of KV heads and the query heads that read them."""
    if num_kv_heads % num_shards:
        raise ValueError(f"{num_kv_heads} KV heads do not split over {num_shards} ranks")
    per = num_kv_heads // num_shards
    return [(range(r * per, (r + 1) * per), range(r * per * group, (r + 1) * per * group))
            for r in range(num_shards)]
