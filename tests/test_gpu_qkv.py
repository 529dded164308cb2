"""GPU: the fused Q/K/V projection + append (clove_cuda_qkv_append) against
the oracle's float64 Linear (src/nn.rs:102-123) and RoPE — q and the K/V
written into their cache slots within the rounding of the pool's element
type, every other slot untouched bit for bit, the advanced lengths exact —
and the fused module forward against the unfused one."""
import numpy as np
import pytest
import torch

from clove_b200.workload import to_numpy_bits

pytestmark = pytest.mark.gpu

# half an ulp of the element type, relative: bf16 keeps 8 significant bits, f16 11
_HALF_ULP = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}


def _within_rounding(got: np.ndarray, ref: np.ndarray, dtype) -> tuple[bool, float]:
    # |got - ref| <= half an ulp of ref (the final rounding) + a small absolute
    # term for the f32 accumulation order and the f32 RoPE angle
    bound = _HALF_ULP[dtype] * np.abs(ref) * 1.0001 + 2e-4 * np.sqrt(np.mean(ref ** 2))
    excess = np.abs(got - ref) - bound
    return bool((excess <= 0).all()), float(excess.max())


def _run(dtype, B, hidden, hq, hkv, D, bs, theta, with_bias=True, seed=0):
    import oracle
    from clove_b200 import KVPool
    rng = np.random.default_rng(seed)
    dev = torch.device("cuda", 0)
    n_out = (hq + 2 * hkv) * D
    ctx = rng.integers(0, 300, B).astype(np.int32)
    need = ctx // bs + 1
    nb = int(need.sum()) + 8
    ids = rng.permutation(nb).astype(np.int32)
    mb = int(need.max())
    bt = np.zeros((B, mb), np.int32)
    o = 0
    for b in range(B):
        bt[b, :need[b]] = ids[o:o + need[b]]
        o += need[b]
    pool = KVPool(nb, bs, hkv, D, dtype, 0)
    pool.storage.normal_()
    before = to_numpy_bits(pool.storage)
    x = torch.randn((B, hidden), device=dev).to(dtype)
    w = (torch.randn((n_out, hidden), device=dev) / np.sqrt(hidden)).to(dtype)
    bias = torch.randn(n_out, device=dev) * 0.1 if with_bias else None
    q, lens = pool.qkv_append(x, pool.pack_qkv_weights(w), bias, hq, torch.from_numpy(bt).to(dev), torch.from_numpy(ctx).to(dev),
                              rope_theta=theta)
    torch.cuda.synchronize()
    assert pool.pool_status() == 0
    assert np.array_equal(lens.cpu().numpy(), ctx + 1)
    # the per-tile arrival counters at the workspace's start are zero again
    tiles = -(-n_out // 256) if B <= 128 else 0  # stream-K: one counter per 256-feature tile
    assert int(pool._qkv_ws[:4 * tiles].view(torch.int32).abs().sum()) == 0
    # oracle: W [hidden, out] per projection as the reference stores it
    wf = w.double().cpu().numpy()
    bf = bias.double().cpu().numpy() if with_bias else np.zeros(n_out)
    xf = x.double().cpu().numpy()
    qd, kd = hq * D, hkv * D
    rq, rk, rv = oracle.qkv_append(xf, wf[:qd].T, wf[qd:qd + kd].T, wf[qd + kd:].T, bf[:qd], bf[qd:qd + kd],
                                   bf[qd + kd:], hq, hkv, ctx, theta)
    ok, worst = _within_rounding(q.double().cpu().numpy(), rq, dtype)
    assert ok, ("q", worst)
    slots = bt[np.arange(B), ctx // bs] * bs + ctx % bs
    kc = pool.storage[0].reshape(-1, hkv, D)
    vc = pool.storage[1].reshape(-1, hkv, D)
    st = torch.from_numpy(slots).to(dev).long()
    ok, worst = _within_rounding(kc[st].double().cpu().numpy(), rk, dtype)
    assert ok, ("k", worst)
    ok, worst = _within_rounding(vc[st].double().cpu().numpy(), rv, dtype)
    assert ok, ("v", worst)
    # nothing else in the pool changed
    after = to_numpy_bits(pool.storage)
    for plane in range(2):
        a = after[plane].reshape(-1, hkv * D).copy()
        e = before[plane].reshape(-1, hkv * D).copy()
        a[slots] = 0
        e[slots] = 0
        assert np.array_equal(a, e), plane


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,hidden,hq,hkv,D,bs,theta", [
    (128, 4096, 32, 8, 128, 16, 0.0),      # C3-shaped decode step
    (128, 4096, 32, 8, 128, 16, 10000.0),  # with RoPE
    (5, 512, 8, 2, 64, 16, 500.0),         # tiny ragged batch (x tile of 16 rows)
    (300, 1024, 16, 4, 128, 32, 0.0),      # three 128-row batch tiles
    (33, 520, 4, 4, 64, 8, 10000.0),       # hidden not a multiple of 64 (zero-filled tail)
    (64, 8192, 64, 8, 128, 16, 0.0),       # 70B-shaped projection
    (7, 384, 3, 1, 64, 16, 10000.0),       # 320 features: a partial last tile, q/k boundary mid-tile
    (140, 384, 3, 1, 64, 16, 10000.0),     # the same through the cluster schedule (two batch tiles)
    (1, 4096, 32, 8, 128, 16, 10000.0),    # batch 1: one live row of the 128-row tile
    (100, 2048, 16, 8, 128, 16, 0.0),      # ragged batch tile of 112 rows
    (16, 8192, 8, 2, 128, 16, 10000.0),    # stream-K: 6 tiles over 148 CTAs, ~25 pieces per tile
])
def test_qkv_append_matches_oracle(dtype, B, hidden, hq, hkv, D, bs, theta):
    _run(dtype, B, hidden, hq, hkv, D, bs, theta, seed=B + hidden)


def test_qkv_append_without_bias():
    _run(torch.bfloat16, 16, 256, 4, 2, 128, 16, 0.0, with_bias=False, seed=3)


@pytest.mark.parametrize("pad", [0, 38, 138])  # batch 2 (stream-K), 40 and 140 (cluster schedule, 1 and 2 batch tiles)
def test_qkv_append_flags_bad_slots_and_rejects_f32(pad):
    from clove_b200 import KVPool, _lib
    dev = torch.device("cuda", 0)
    pool = KVPool(8 + pad, 16, 2, 64, torch.bfloat16, 0)
    pool.storage.zero_()
    n_out = (4 + 4) * 64
    B = 2 + pad
    x = torch.randn((B, 128), device=dev).to(torch.bfloat16)
    w = torch.randn((n_out, 128), device=dev).to(torch.bfloat16)
    # seq 0: position past its table; seq 1: block id out of range; the rest valid
    bt = torch.tensor([[0, 1], [9999, 2]] + [[8 + i, 0] for i in range(pad)], dtype=torch.int32, device=dev)
    ctx = torch.tensor([40, 3] + [5] * pad, dtype=torch.int32, device=dev)
    pool.qkv_append(x, pool.pack_qkv_weights(w), None, 4, bt, ctx)
    torch.cuda.synchronize()
    st = pool.pool_status()
    assert st & _lib.FLAG_CTX_RANGE and st & _lib.FLAG_BLOCK_OOB
    written = pool.storage.view(torch.int16).reshape(2, -1, 16, 2 * 64).abs().sum(dim=(0, 3))  # [blocks, slots]
    assert int(written[:8].sum()) == 0  # the two bad rows wrote nothing
    if pad:
        assert bool((written[8:, 5] != 0).all())  # every valid row wrote its slot
    p32 = KVPool(8, 16, 2, 64, torch.float32, 0)
    with pytest.raises(_lib.CloveError):
        p32.pack_qkv_weights(w.float())


@pytest.mark.parametrize("theta", [0.0, 10000.0])
def test_fused_module_forward_matches_unfused(theta):
    import oracle
    from clove_b200.backend import PagedAttention
    rng = np.random.default_rng(11)
    dev = torch.device("cuda", 0)
    dim, hq, hkv, D, bs, B = 1024, 8, 2, 128, 16, 24
    m = PagedAttention(dim, hq, hkv, device=dev, dtype=torch.bfloat16, seed=4)
    ctx = rng.integers(1, 200, B).astype(np.int32)
    need = ctx // bs + 1
    nb = int(need.sum()) + 4
    ids = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((B, int(need.max())), np.int32)
    o = 0
    for b in range(B):
        bt[b, :need[b]] = ids[o:o + need[b]]
        o += need[b]
    kv = torch.randn((2, nb, bs, hkv, D), device=dev).to(torch.bfloat16)
    x = torch.randn((B, dim), device=dev).to(torch.bfloat16)
    btd, cld = torch.from_numpy(bt).to(dev), torch.from_numpy(ctx).to(dev)
    out = m.forward_fused(x, kv, btd, cld, max_ctx=int(ctx.max()) + 1, rope_theta=theta)
    # reference: the fp64 projections (rotated), appended by the bit-exact
    # scatter, then the fp64 decode over the cache the fused kernel wrote
    w = torch.cat([m.w_q.weight, m.w_k.weight, m.w_v.weight], 1).double().cpu().numpy()
    bb = torch.cat([m.w_q.bias, m.w_k.bias, m.w_v.bias]).double().cpu().numpy()
    qd, kd = hq * D, hkv * D
    rq, _, _ = oracle.qkv_append(x.double().cpu().numpy(), w[:, :qd], w[:, qd:qd + kd], w[:, qd + kd:],
                                 bb[:qd], bb[qd:qd + kd], bb[qd + kd:], hq, hkv, ctx, theta)
    kc = kv[0].float().cpu().numpy()
    vc = kv[1].float().cpu().numpy()
    attn = oracle.decode_f64(0, rq.astype(np.float32), kc, vc, bt, ctx + 1, 1.0 / np.sqrt(D))
    ref = oracle.linear(attn.reshape(B, -1), m.w_o.weight.double().cpu().numpy(), m.w_o.bias.double().cpu().numpy())
    ok, worst = oracle.tolerance_ok(out.double().cpu().numpy(), ref, 2e-2)
    assert ok, worst


@pytest.mark.parametrize("B", [5, 64, 160])  # stream-K, and the cluster schedule with 1 and 2 batch tiles
def test_stuck_wait_times_out_and_next_call_is_correct(B):
    # Failure detection without a GPU fault: the test hook leaves the first
    # stage of the first CTA unfilled, so the bounded waits run out; the call
    # must finish and report CLOVE_FLAG_TIMEOUT, the workspace counters must
    # be zero again, and the next call on the same pool and workspace must be
    # right.
    import time

    from clove_b200 import KVPool, _lib
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    hidden, hq, hkv, D, bs = 1024, 8, 2, 128, 16
    n_out = (hq + 2 * hkv) * D
    pool = KVPool(B + 4, bs, hkv, D, torch.bfloat16, 0)
    x = torch.randn((B, hidden), device=dev).to(torch.bfloat16)
    w = (torch.randn((n_out, hidden), device=dev) / 32).to(torch.bfloat16)
    wp = pool.pack_qkv_weights(w)
    bt = torch.arange(B, dtype=torch.int32, device=dev).reshape(B, 1)
    ctx = torch.full((B,), 3, dtype=torch.int32, device=dev)
    try:
        _lib.check(L.clove_cuda_debug_set(2000, 1))
        t0 = time.time()
        pool.qkv_append(x, wp, None, hq, bt, ctx)
        flags = pool.pool_status()
        elapsed = time.time() - t0
    finally:
        L.clove_cuda_debug_set(0, 0)
    assert flags & _lib.FLAG_TIMEOUT, flags
    assert elapsed < 30
    tiles = -(-n_out // 256) if B <= 128 else 0
    assert int(pool._qkv_ws[:4 * tiles].view(torch.int32).abs().sum()) == 0
    q, _ = pool.qkv_append(x, wp, None, hq, bt, ctx)
    torch.cuda.synchronize()
    assert pool.pool_status() == 0
    ref = (x.double() @ w.double().t())[:, :hq * D]
    got = q.double().reshape(B, -1)
    assert bool(((got - ref).abs() <= 2.0 ** -8 * ref.abs() * 1.0001 + 2e-4 * ref.pow(2).mean().sqrt()).all())
