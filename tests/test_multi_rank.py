"""World-size-2 gloo tests (CPU) of the multi-rank host logic: sequence
sharding and KV-head sharding with one all-gather, each rank computing its
part with the CPU oracle in place of the GPU kernel, compared with the
unsharded oracle."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    from clove_b200.workload import Spec, fill_values, make_layout, to_numpy_bits
    spec = Spec("t", 6, 16, 4, 64, 16, 0, torch.float32, "uniform", 5, 300, "permutation", seed=31)
    lay = make_layout(spec)
    q, kn, vn, st = fill_values(lay, "cpu")
    return lay, to_numpy_bits(q), to_numpy_bits(st)


def _worker(rank, world, port, mode, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import oracle
    from clove_b200.distributed import gather_heads, init_from_env, local_heads
    from clove_b200.sharding import contiguous_shards, token_balanced_shards
    ws, r, _ = init_from_env("gloo")
    assert (ws, r) == (world, rank)
    lay, q, st = _case()
    scale = 1.0 / np.sqrt(lay.spec.head_dim)
    if mode == "heads":
        kvh, qh = local_heads(lay.spec.num_kv_heads, lay.spec.num_q_heads // lay.spec.num_kv_heads, world, rank)
        kc = np.ascontiguousarray(st[0][:, :, kvh.start:kvh.stop])
        vc = np.ascontiguousarray(st[1][:, :, kvh.start:kvh.stop])
        ql = np.ascontiguousarray(q[:, qh.start:qh.stop])
        out = oracle.decode_f64(0, ql, kc, vc, lay.block_tables, lay.context_lens, scale, nthreads=1)
        full = gather_heads(torch.from_numpy(out), world)
        result_q.put((rank, full.numpy()))
    else:
        shards = (contiguous_shards(lay.batch, world) if mode == "contiguous"
                  else token_balanced_shards(lay.context_lens, world))
        mine = shards[rank]
        out = oracle.decode_f64(0, np.ascontiguousarray(q[mine]), st[0], st[1],
                                np.ascontiguousarray(lay.block_tables[mine]), lay.context_lens[mine], scale,
                                nthreads=1)
        objs = [None] * world
        dist.all_gather_object(objs, (mine.tolist(), out))
        full = np.zeros((lay.batch,) + out.shape[1:])
        for idx, o in objs:
            full[idx] = o
        result_q.put((rank, full))
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["heads", "contiguous", "balanced"])
def test_two_rank_sharding_matches_unsharded(mode, oracle_lib):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    lay, qn, st = _case()
    ref = oracle_lib.decode_f64(0, qn, st[0], st[1], lay.block_tables, lay.context_lens,
                                1.0 / np.sqrt(lay.spec.head_dim))
    for r in range(2):
        np.testing.assert_array_equal(results[r], ref)


def _lonely_worker(port, q_out):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE="2", RANK="0", LOCAL_RANK="0")
    try:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=5))
        q_out.put("joined")
    except Exception as e:  # the peer never joins: a bounded error, not a hang
        q_out.put("error:" + type(e).__name__)


def test_rank_that_never_joins_gives_a_timeout_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_worker, args=(_free_port(), q))
    p.start()
    res = q.get(timeout=120)
    p.join(timeout=60)
    assert res.startswith("error:"), res
