"""Generate the committed golden fixtures for the decode path.

PARITY UNPINNED: the reference (Rust + WGSL through wgpu) cannot run here and
its tests hold no PagedAttention vectors, so these fixtures are computed by an
independent numpy float64 implementation written below (vectorised gather +
softmax, sharing no code with oracle/paged_oracle.cpp).  They pin the C++
oracle and the CUDA kernels to the semantics the reference documents:
softmax(q K^T * scale) V (src/nn/attention.rs:52-69), scale 1/sqrt(head_dim)
(src/lazy.rs:5267), block-table gather (src/lazy.rs:5259-5270), append slot
block_tables[b][ctx/bs]*bs + ctx%bs, then attention over ctx+1 tokens.

The mock fixture records the literal output of the reference's placeholder
kernel (src/lazy.rs:5255-5274) restated in numpy.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    rounding = 0x7FFF + ((u >> 16) & 1)
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_to_f64(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def reference_decode(q, kc, vc, bt, ctx_after, scale):
    """float64 [B, Hq, D] over ctx_after[b] tokens (vectorised per sequence)."""
    B, hq, d = q.shape
    nb, bs, hkv, _ = kc.shape
    grp = hq // hkv
    out = np.zeros((B, hq, d))
    for b in range(B):
        L = int(ctx_after[b])
        if L == 0:
            continue
        t = np.arange(L)
        phys = bt[b, t // bs]
        K = kc[phys, t % bs]  # [L, hkv, d]
        V = vc[phys, t % bs]
        Kq = np.repeat(K, grp, axis=1)  # [L, hq, d]
        Vq = np.repeat(V, grp, axis=1)
        s = np.einsum("hd,lhd->hl", q[b] * scale, Kq)
        s = np.exp(s - s.max(axis=1, keepdims=True))
        p = s / s.sum(axis=1, keepdims=True)
        out[b] = np.einsum("hl,lhd->hd", p, Vq)
    return out


def make_case(name, rng, B, hq, hkv, d, bs, ctx_lo, ctx_hi, dtype, kv_scale=1.0, zero_ctx=False):
    ctx = rng.integers(ctx_lo, ctx_hi + 1, size=B).astype(np.int32)
    if zero_ctx:
        ctx[0] = 0
    need = (ctx + 1 + bs - 1) // bs
    nb = int(need.sum()) + 3
    ids = rng.permutation(nb)
    mb = int(need.max())
    bt = np.zeros((B, mb), np.int32)
    off = 0
    for b in range(B):
        bt[b, : need[b]] = ids[off: off + need[b]]
        off += need[b]
    kc = rng.standard_normal((nb, bs, hkv, d)).astype(np.float32) * kv_scale
    vc = rng.standard_normal((nb, bs, hkv, d)).astype(np.float32) * kv_scale
    q = rng.standard_normal((B, hq, d)).astype(np.float32)
    kn = rng.standard_normal((B, hkv, d)).astype(np.float32) * kv_scale
    vn = rng.standard_normal((B, hkv, d)).astype(np.float32) * kv_scale
    if dtype == "bf16":
        kc, vc, q, kn, vn = (bf16_round(a) for a in (kc, vc, q, kn, vn))
        widen = bf16_to_f64
    else:
        widen = lambda a: a.astype(np.float64)  # noqa: E731
    # append, then decode over ctx+1
    kc2, vc2 = kc.copy(), vc.copy()
    slots = bt[np.arange(B), ctx // bs] * bs + ctx % bs
    kc2.reshape(nb * bs, hkv, d)[slots] = kn
    vc2.reshape(nb * bs, hkv, d)[slots] = vn
    scale = 1.0 / np.sqrt(d)
    expected = reference_decode(widen(q), widen(kc2), widen(vc2), bt, ctx + 1, scale)
    # plain decode over the pre-append cache (no append)
    expected_noappend = reference_decode(widen(q), widen(kc), widen(vc), bt, ctx, scale)
    np.savez_compressed(HERE / f"{name}.npz", dtype=np.array(dtype), context_lens=ctx, block_tables=bt,
                        k_cache=kc, v_cache=vc, q=q, k_new=kn, v_new=vn, slots=slots.astype(np.int32),
                        k_cache_after=kc2, v_cache_after=vc2, scale=np.float64(scale), expected=expected,
                        expected_noappend=expected_noappend)


def make_mock(rng):
    # One sequence batch of 2, seq_len 40, head_dim 8, block_size 16.
    seq_len, hd, bs, B = 40, 8, 16, 2
    size = B * seq_len * hd
    nb = 8
    kv = rng.standard_normal(nb * bs * hd).astype(np.float32)
    bt = np.zeros(B * 1024, np.uint32)
    for b in range(B):
        bt[b * 1024: b * 1024 + 3] = rng.permutation(nb)[:3]
    q = rng.standard_normal(size).astype(np.float32)
    i = np.arange(size)
    token = i % seq_len
    phys = bt[(i // (seq_len * hd)) * 1024 + token // bs]
    kval = kv[phys * bs * hd + (token % bs) * hd + i % hd]
    out = q * kval * np.float32(1.0 / np.sqrt(np.float32(hd)))
    np.savez_compressed(HERE / "mock_lazy_kernel.npz", q=q, kv_cache=kv, block_tables=bt,
                        seq_len=np.int32(seq_len), head_dim=np.int32(hd), block_size=np.int32(bs),
                        expected=out.astype(np.float32))


def main():
    rng = np.random.default_rng(20261201)
    make_case("f32_mha_small", rng, B=4, hq=4, hkv=4, d=64, bs=16, ctx_lo=20, ctx_hi=80, dtype="f32")
    make_case("f32_gqa_zero_ctx", rng, B=5, hq=8, hkv=2, d=64, bs=16, ctx_lo=1, ctx_hi=40, dtype="f32",
              zero_ctx=True)
    make_case("bf16_gqa_bs32", rng, B=3, hq=8, hkv=2, d=128, bs=32, ctx_lo=1, ctx_hi=100, dtype="bf16",
              kv_scale=0.5)
    make_mock(rng)
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
