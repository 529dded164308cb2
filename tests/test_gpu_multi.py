"""Two-GPU check of KV-head sharding (the long-context configuration): each
rank decodes its KV heads through the C ABI, one all-gather (NCCL, and the
library's P2P peer gather) assembles the output, and the gathered result on
every rank is compared with the fp64 oracle on the same inputs; the peer
gather is also checked bit for bit against NCCL's over repeated calls and
CUDA-graph replays.  Skipped with fewer than two GPUs (the same
decomposition runs on one GPU in test_gpu_shard.py)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from clove_b200 import KVPool
    from clove_b200.distributed import PeerGather, head_sharded_append_decode, init_from_env, local_heads
    from clove_b200.workload import Spec, fill_values, make_layout
    init_from_env("nccl")
    dev = torch.device("cuda", rank)
    spec = Spec("t", 4, 16, 4, 128, 32, 0, torch.bfloat16, "uniform", 500, 4000, "permutation", seed=41)
    lay = make_layout(spec)
    full = KVPool(lay.num_blocks, 32, 4, 128, torch.bfloat16, dev)
    q, kn, vn, _ = fill_values(lay, dev, full.storage)  # same seed: identical on every rank
    from clove_b200.workload import to_numpy_bits
    before = to_numpy_bits(full.storage) if rank == 0 else None
    kvh, qh = local_heads(4, 4, world, rank)
    local = KVPool(lay.num_blocks, 32, kvh.stop - kvh.start, 128, torch.bfloat16, dev,
                   storage=full.storage[:, :, :, kvh.start:kvh.stop].contiguous())
    bt = torch.from_numpy(lay.block_tables).to(dev)
    cl = torch.from_numpy(lay.context_lens).to(dev)
    got = head_sharded_append_decode(local, q[:, qh.start:qh.stop].contiguous(),
                                     kn[:, kvh.start:kvh.stop].contiguous(),
                                     vn[:, kvh.start:kvh.stop].contiguous(), bt, cl, world, lay.max_ctx)
    got = got.reshape(q.shape[0], q.shape[1], q.shape[2])
    # Same step again, outputs gathered by P2P stores (cache restored first).
    local.storage.copy_(full.storage[:, :, :, kvh.start:kvh.stop])
    hl = qh.stop - qh.start
    peer = PeerGather(q.shape[0] * hl * 128 * 4, dev)
    got_p = head_sharded_append_decode(local, q[:, qh.start:qh.stop].contiguous(),
                                       kn[:, kvh.start:kvh.stop].contiguous(),
                                       vn[:, kvh.start:kvh.stop].contiguous(), bt, cl, world, lay.max_ctx,
                                       peer=peer)
    got_p = got_p.reshape(q.shape[0], q.shape[1], q.shape[2])
    torch.cuda.synchronize()
    assert peer.status() == 0
    assert torch.equal(got, got_p), "peer gather differs from the NCCL all-gather"
    peer.close()
    extra = None
    if rank == 0:
        extra = (before, to_numpy_bits(q), to_numpy_bits(kn), to_numpy_bits(vn), lay.block_tables,
                 lay.context_lens)
    q_out.put((rank, got.cpu().numpy(), extra))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_head_split_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    import oracle
    from workload_check import tol_check
    before, qb, kb, vb, bt, cl = next(r[2] for r in res if r[2] is not None)
    kc, vc = before[0].copy(), before[1].copy()
    assert oracle.reshape_and_cache(kc, vc, kb, vb, oracle.append_slots(bt, cl, 32)) == 0
    ref = oracle.decode_f64(oracle.BF16, qb, kc, vc, bt, cl + 1, 1.0 / np.sqrt(128))
    for rank, got, _ in res:
        tol_check(got, ref, 2e-2)  # bf16 inputs, fp64 oracle


def _gather_worker(rank, world, port, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from clove_b200.distributed import PeerGather, init_from_env
    init_from_env("nccl")
    dev = torch.device("cuda", rank)
    errors = []
    for n in (4, 2048, 65536 + 4, 1 << 20):  # f32 words per rank: one chunk .. the 64-chunk cap
        peer = PeerGather(n * 4, dev)
        src = torch.empty(n, dtype=torch.float32, device=dev)
        out = torch.empty(world * n, dtype=torch.float32, device=dev)
        ref = torch.empty_like(out)
        g = torch.Generator(device=dev)
        for it in range(5):  # alternating receive halves
            g.manual_seed(1000 * rank + it)
            src.normal_(generator=g)
            peer(src, out)
            dist.all_gather_into_tensor(ref, src)
            torch.cuda.synchronize()
            if not torch.equal(out, ref):
                errors.append(f"n={n} call {it}")
        # Captured once, replayed with new inputs.
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            peer(src, out, stream=s)
        for it in range(3):
            g.manual_seed(7000 + 100 * rank + it)
            src.normal_(generator=g)
            torch.cuda.synchronize()
            graph.replay()
            dist.all_gather_into_tensor(ref, src)
            torch.cuda.synchronize()
            if not torch.equal(out, ref):
                errors.append(f"n={n} replay {it}")
        if peer.status() != 0:
            errors.append(f"n={n} flags")
        peer.close()
    q_out.put((rank, errors))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_peer_gather_matches_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, errors in res:
        assert not errors, (rank, errors)
