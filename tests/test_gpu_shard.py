"""The multi-GPU decompositions, run on one GPU and checked against the fp64
oracle (so the driver's 1-GPU test run covers them):

  sequence sharding   a c3-shaped batch split into shards (distribute_batch's
                      contiguous split and the token-balanced split); each
                      shard decodes in its own pool with its own tables, as a
                      rank would, and every global sequence is produced
                      exactly once.
  KV-head sharding    a c4-shaped case whose pool is split into KV-head
                      slices; each slice decodes its query heads in its own
                      pool and the slices are assembled in the all-gather's
                      layout (rank-major [world, B, hq_local, D] viewed as
                      [B, world * hq_local, D]).
"""
import numpy as np
import pytest
import torch

import oracle
from clove_b200.workload import CONFIGS, dtype_code, fill_values, make_layout, shard_layout, to_numpy_bits
from workload_check import bits_equal, tol_check

pytestmark = pytest.mark.gpu

RT = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def _oracle_append_decode(lay, storage_bits, q, kn, vn):
    spec = lay.spec
    kc, vc = storage_bits[0].copy(), storage_bits[1].copy()
    slots = oracle.append_slots(lay.block_tables, lay.context_lens, spec.block_size)
    assert oracle.reshape_and_cache(kc, vc, to_numpy_bits(kn), to_numpy_bits(vn), slots) == 0
    ref = oracle.decode_f64(dtype_code(spec.dtype), to_numpy_bits(q), kc, vc, lay.block_tables,
                            lay.context_lens + 1, 1.0 / np.sqrt(spec.head_dim))
    return kc, vc, ref


@pytest.mark.parametrize("policy,world", [("contiguous", 2), ("contiguous", 3), ("tokens", 2), ("tokens", 4)])
def test_sequence_shards_match_oracle(policy, world):
    from dataclasses import replace

    from clove_b200 import KVPool
    spec = replace(CONFIGS["c3"], batch=24)
    dev = torch.device("cuda", 0)
    seen = np.zeros(spec.batch, int)
    glob = make_layout(spec)
    for rank in range(world):
        lay, idx = shard_layout(spec, world, rank, policy=policy)
        assert np.array_equal(lay.context_lens, glob.context_lens[idx])
        seen[idx] += 1
        pool = KVPool(lay.num_blocks, spec.block_size, spec.num_kv_heads, spec.head_dim, spec.dtype, 0)
        q, kn, vn, _ = fill_values(lay, dev, pool.storage)
        before = to_numpy_bits(pool.storage)
        out = pool.append_decode(q, kn, vn, torch.from_numpy(lay.block_tables).to(dev),
                                 torch.from_numpy(lay.context_lens).to(dev), max_ctx=lay.max_ctx)
        torch.cuda.synchronize()
        assert pool.decode_status(lay.batch, spec.num_q_heads, lay.max_ctx) == 0
        kc, vc, ref = _oracle_append_decode(lay, before, q, kn, vn)
        after = to_numpy_bits(pool.storage)
        assert bits_equal(after[0], kc) and bits_equal(after[1], vc), "append not bit-exact"
        tol_check(out.cpu().numpy(), ref, RT[spec.dtype])
    assert (seen == 1).all(), "every sequence is decoded by exactly one shard"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_kv_head_shards_match_oracle(world):
    """c4 shape (64 q / 8 kv heads, D 128, block 32, bf16) with contexts cut
    to a few thousand tokens so the oracle finishes in seconds; several
    chunks per sequence still exercise the split-K combine."""
    from dataclasses import replace

    from clove_b200 import KVPool
    from clove_b200.sharding import head_shards
    spec = replace(CONFIGS["c4"], batch=3, num_blocks=0)
    lay = make_layout(spec, ctx_scale=0.05)
    dev = torch.device("cuda", 0)
    full = torch.empty((2, lay.num_blocks, spec.block_size, spec.num_kv_heads, spec.head_dim), dtype=spec.dtype,
                       device=dev)
    q, kn, vn, _ = fill_values(lay, dev, full)
    before = to_numpy_bits(full)
    kc, vc, ref = _oracle_append_decode(lay, before, q, kn, vn)
    bt = torch.from_numpy(lay.block_tables).to(dev)
    cl = torch.from_numpy(lay.context_lens).to(dev)
    hl = spec.num_q_heads // world
    gbuf = torch.empty((world * lay.batch, hl, spec.head_dim), dtype=torch.float32, device=dev)
    for rank, (kvh, qh) in enumerate(head_shards(spec.num_kv_heads, spec.num_q_heads // spec.num_kv_heads, world)):
        local = KVPool(lay.num_blocks, spec.block_size, len(kvh), spec.head_dim, spec.dtype, 0,
                       storage=full[:, :, :, kvh.start:kvh.stop].contiguous())
        out = local.append_decode(q[:, qh.start:qh.stop].contiguous(), kn[:, kvh.start:kvh.stop].contiguous(),
                                  vn[:, kvh.start:kvh.stop].contiguous(), bt, cl, max_ctx=lay.max_ctx)
        gbuf[rank * lay.batch:(rank + 1) * lay.batch] = out  # what all_gather_into_tensor writes for rank r
        torch.cuda.synchronize()
        assert local.decode_status(lay.batch, hl, lay.max_ctx) == 0
        after = to_numpy_bits(local.storage)
        assert bits_equal(after[0], np.ascontiguousarray(kc[:, :, kvh.start:kvh.stop]))
        assert bits_equal(after[1], np.ascontiguousarray(vc[:, :, kvh.start:kvh.stop]))
    got = gbuf.view(world, lay.batch, hl, spec.head_dim).permute(1, 0, 2, 3).reshape(lay.batch, -1, spec.head_dim)
    tol_check(got.cpu().numpy(), ref, RT[spec.dtype])
