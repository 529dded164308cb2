"""Shared GPU-vs-oracle checking helpers for the -m gpu tests."""
from __future__ import annotations

import numpy as np
import torch

import oracle
from clove_b200.workload import Layout, dtype_code, fill_values, make_layout, to_numpy_bits


def bits_equal(t, ref: np.ndarray) -> bool:
    a = to_numpy_bits(t) if isinstance(t, torch.Tensor) else np.asarray(t)
    return np.array_equal(np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(ref).view(np.uint8))


def tol_check(x: np.ndarray, ref: np.ndarray, rtol: float) -> None:
    ok, worst = oracle.tolerance_ok(x, ref, rtol)
    assert ok, f"tolerance {rtol} exceeded: worst |x-r|/(|r|+rms) = {worst:.3e}"
    assert np.isfinite(x).all()


def run_layout_vs_oracle(lay: Layout, rtol: float, subset: int | None = None, append: bool = True) -> dict:
    """Append + decode `lay` on cuda:0 and compare with the oracle.  With
    `subset`, only that many sequences (spread over the batch) are checked,
    on a host copy of just their blocks — for full-size configurations."""
    from clove_b200 import KVPool
    spec = lay.spec
    dev = torch.device("cuda", 0)
    pool = KVPool(lay.num_blocks, spec.block_size, spec.num_kv_heads, spec.head_dim, dtype=spec.dtype, device=0)
    q, kn, vn, _ = fill_values(lay, dev, pool_storage=pool.storage)
    bt = torch.from_numpy(lay.block_tables).to(dev)
    cl = torch.from_numpy(lay.context_lens).to(dev)
    if subset is None:
        before = to_numpy_bits(pool.storage)
    if append:
        out = pool.append_decode(q, kn, vn, bt, cl, max_ctx=lay.max_ctx)
        ctx_after = lay.context_lens + 1
    else:
        out = pool.decode(q, bt, cl, max_ctx=int(lay.context_lens.max()))
        ctx_after = lay.context_lens
    torch.cuda.synchronize()
    flags = pool.decode_status(lay.batch, spec.num_q_heads, lay.max_ctx if append else int(lay.context_lens.max()))
    assert flags == 0, f"device check flags {flags}"
    out_np = out.cpu().numpy()
    code = dtype_code(spec.dtype)
    bs = spec.block_size
    if subset is None:
        kc, vc = before[0].copy(), before[1].copy()
        if append:
            slots = oracle.append_slots(lay.block_tables, lay.context_lens, bs)
            assert oracle.reshape_and_cache(kc, vc, to_numpy_bits(kn), to_numpy_bits(vn), slots) == 0
            after = to_numpy_bits(pool.storage)
            assert bits_equal(after[0], kc) and bits_equal(after[1], vc), "append not bit-exact"
        ref = oracle.decode_f64(code, to_numpy_bits(q), kc, vc, lay.block_tables, ctx_after,
                                1.0 / np.sqrt(spec.head_dim))
        tol_check(out_np, ref, rtol)
        return {"checked": lay.batch}
    seqs = np.unique(np.linspace(0, lay.batch - 1, subset).astype(int))
    need = (ctx_after.astype(np.int64) + bs - 1) // bs
    ids = [lay.block_tables[b, :need[b]] for b in seqs]
    allids = torch.from_numpy(np.concatenate(ids).astype(np.int64)).to(dev)
    mini = to_numpy_bits(pool.storage.index_select(1, allids))  # [2, n, bs, hkv, d]
    mbt = np.zeros((len(seqs), int(need[seqs].max())), np.int32)
    off = 0
    for i, b in enumerate(seqs):
        mbt[i, :need[b]] = np.arange(off, off + need[b])
        off += need[b]
    if append:  # the appended token's slot holds k_new / v_new bit for bit
        kn_np, vn_np = to_numpy_bits(kn), to_numpy_bits(vn)
        for i, b in enumerate(seqs):
            c = lay.context_lens[b]
            blk = mbt[i, c // bs]
            assert bits_equal(mini[0, blk, c % bs], kn_np[b]) and bits_equal(mini[1, blk, c % bs], vn_np[b])
    qs = to_numpy_bits(q)[seqs]
    ref = oracle.decode_f64(code, np.ascontiguousarray(qs), np.ascontiguousarray(mini[0]),
                            np.ascontiguousarray(mini[1]), mbt, ctx_after[seqs], 1.0 / np.sqrt(spec.head_dim))
    tol_check(out_np[seqs], ref, rtol)
    # the whole output is finite and rows are convex combinations of V rows
    assert np.isfinite(out_np).all()
    return {"checked": len(seqs)}


def small_layout(name: str, batch: int, ctx_scale: float, seed: int | None = None) -> Layout:
    from clove_b200.workload import CONFIGS
    return make_layout(CONFIGS[name], seed=seed, batch=batch, ctx_scale=ctx_scale)
