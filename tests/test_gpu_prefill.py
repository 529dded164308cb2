"""GPU: prefill into the paged cache against the oracle — K/V slots written
bit for bit (no RoPE), causal outputs within tolerance, with and without
RoPE, fresh prompts and prompts continuing a cached context."""
import numpy as np
import pytest
import torch

from clove_b200.workload import to_numpy_bits

pytestmark = pytest.mark.gpu


def _bits_to_f64(a: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    if dtype == torch.float32:
        return a.astype(np.float64)
    return torch.from_numpy(a.view(np.int16)).view(dtype).double().numpy()


def _case(dtype, hq, hkv, d, bs, prior, prompt, seed):
    rng = np.random.default_rng(seed)
    B = len(prior)
    total = np.array(prior) + np.array(prompt)
    need = (total + bs - 1) // bs
    nb = int(need.sum()) + 4
    ids = rng.permutation(nb)
    mb = int(need.max())
    bt = np.zeros((B, mb), np.int32)
    o = 0
    for b in range(B):
        bt[b, :need[b]] = ids[o:o + need[b]]
        o += need[b]
    T = int(sum(prompt))
    cu = np.concatenate([[0], np.cumsum(prompt)]).astype(np.int32)
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    q = torch.randn((T, hq, d), device=dev, generator=gen).to(dtype)
    k = torch.randn((T, hkv, d), device=dev, generator=gen).to(dtype)
    v = torch.randn((T, hkv, d), device=dev, generator=gen).to(dtype)
    return dict(B=B, T=T, bt=bt, cu=cu, ctx=np.array(prior, np.int32), total=total, nb=nb, q=q, k=k, v=v)


@pytest.mark.parametrize("dtype,hq,hkv,d,bs,theta", [
    (torch.float32, 4, 4, 64, 16, 0.0),
    (torch.float32, 8, 2, 128, 16, 10000.0),
    (torch.bfloat16, 8, 2, 128, 32, 10000.0),
    (torch.float16, 16, 2, 64, 8, 500.0),
    (torch.bfloat16, 24, 8, 128, 16, 10000.0),
    (torch.bfloat16, 32, 2, 64, 16, 0.0),
    (torch.float16, 6, 2, 128, 64, 10000.0),
])
@pytest.mark.parametrize("variant", ["auto", "simt"])
def test_prefill_matches_oracle(dtype, hq, hkv, d, bs, theta, variant):
    import oracle
    from clove_b200 import KVPool, set_decode_variant
    if variant == "simt" and hq // hkv > 8:
        pytest.skip("the decode-reuse prefill covers groups <= 8 (the tensor-core path covers up to 16)")
    c = _case(dtype, hq, hkv, d, bs, prior=[0, 21, 0, 40], prompt=[17, 9, 1, 33], seed=hq + bs)
    pool = KVPool(c["nb"], bs, hkv, d, dtype, 0)
    pool.storage.normal_()
    before = to_numpy_bits(pool.storage)
    dev = torch.device("cuda", 0)
    set_decode_variant(variant)
    try:
        out = pool.prefill(c["q"], c["k"], c["v"], torch.from_numpy(c["cu"]).to(dev),
                           torch.from_numpy(c["bt"]).to(dev), torch.from_numpy(c["ctx"]).to(dev),
                           max_ctx=int(c["total"].max()), rope_theta=theta)
        torch.cuda.synchronize()
    finally:
        set_decode_variant("auto")
    assert pool.pool_status() == 0
    after = to_numpy_bits(pool.storage)
    # host reference: positions, (rotated) K written into the slots, V as is
    kn, vn, qn = (to_numpy_bits(t) for t in (c["k"], c["v"], c["q"]))
    pos = np.concatenate([c["ctx"][b] + np.arange(c["cu"][b + 1] - c["cu"][b]) for b in range(c["B"])])
    seq = np.concatenate([[b] * (c["cu"][b + 1] - c["cu"][b]) for b in range(c["B"])])
    slots = np.array([c["bt"][s, p // bs] * bs + p % bs for s, p in zip(seq, pos)])
    kc = _bits_to_f64(before[0], dtype).reshape(-1, hkv, d)
    vc = _bits_to_f64(before[1], dtype).reshape(-1, hkv, d)
    kf = _bits_to_f64(kn, dtype)
    qf = _bits_to_f64(qn, dtype)
    if theta > 0:
        kf = oracle.rope(kf, pos, theta)
        qf = oracle.rope(qf, pos, theta)
    else:
        # without rotation the slots hold the new rows bit for bit, nothing else changes
        exp_k = before[0].reshape(-1, hkv, d).copy()
        exp_k[slots] = kn
        assert np.array_equal(after[0].reshape(-1, hkv, d).view(np.uint8), exp_k.view(np.uint8))
    kc[slots] = kf
    vc[slots] = _bits_to_f64(vn, dtype)
    # every token: decode over its sequence's cache up to its own position
    ref = oracle.decode_f64(0, np.ascontiguousarray(qf.astype(np.float32)), kc.reshape(c["nb"], bs, hkv, d).astype(np.float32),
                            vc.reshape(c["nb"], bs, hkv, d).astype(np.float32), c["bt"][seq], pos + 1,
                            1.0 / np.sqrt(d))
    rtol = 1e-5 if dtype == torch.float32 and theta == 0 else 2e-2
    ok, worst = oracle.tolerance_ok(out.cpu().numpy(), ref, rtol)
    assert ok, worst


def test_prefill_long_prompt_multi_chunk():
    # one 3000-token prompt (the 2-CTA kernel): its late tokens attend over many 128-key steps
    import oracle
    from clove_b200 import KVPool
    c = _case(torch.bfloat16, 8, 1, 128, 32, prior=[0], prompt=[3000], seed=9)
    pool = KVPool(c["nb"], 32, 1, 128, torch.bfloat16, 0)
    dev = torch.device("cuda", 0)
    out = pool.prefill(c["q"], c["k"], c["v"], torch.from_numpy(c["cu"]).to(dev), torch.from_numpy(c["bt"]).to(dev),
                       torch.from_numpy(c["ctx"]).to(dev), max_ctx=3000)
    kc = _bits_to_f64(to_numpy_bits(pool.storage)[0], torch.bfloat16)
    vc = _bits_to_f64(to_numpy_bits(pool.storage)[1], torch.bfloat16)
    rows = np.array([0, 1, 15, 999, 2999])
    qf = _bits_to_f64(to_numpy_bits(c["q"])[rows], torch.bfloat16).astype(np.float32)
    ref = oracle.decode_f64(0, qf, kc.astype(np.float32), vc.astype(np.float32), np.repeat(c["bt"], len(rows), 0),
                            (rows + 1).astype(np.int32), 1.0 / np.sqrt(128))
    ok, worst = oracle.tolerance_ok(out.cpu().numpy()[rows], ref, 2e-2)
    assert ok, worst


def _prefill_vs_oracle(dtype, hq, hkv, d, bs, theta, prior, prompt, seed, variant="auto", tol=2e-2):
    import oracle
    from clove_b200 import KVPool, set_decode_variant
    c = _case(dtype, hq, hkv, d, bs, prior=prior, prompt=prompt, seed=seed)
    pool = KVPool(c["nb"], bs, hkv, d, dtype, 0)
    pool.storage.normal_()
    before = to_numpy_bits(pool.storage)
    dev = torch.device("cuda", 0)
    set_decode_variant(variant)
    try:
        out = pool.prefill(c["q"], c["k"], c["v"], torch.from_numpy(c["cu"]).to(dev),
                           torch.from_numpy(c["bt"]).to(dev), torch.from_numpy(c["ctx"]).to(dev),
                           max_ctx=int(c["total"].max()), rope_theta=theta)
        torch.cuda.synchronize()
    finally:
        set_decode_variant("auto")
    assert pool.pool_status() == 0
    kn, vn, qn = (to_numpy_bits(t) for t in (c["k"], c["v"], c["q"]))
    pos = np.concatenate([c["ctx"][b] + np.arange(c["cu"][b + 1] - c["cu"][b]) for b in range(c["B"])])
    seq = np.concatenate([[b] * (c["cu"][b + 1] - c["cu"][b]) for b in range(c["B"])])
    slots = np.array([c["bt"][s, p // bs] * bs + p % bs for s, p in zip(seq, pos)])
    # the kernels store the rotated rows in the pool dtype: attend over the
    # cache as written (its prompt rows checked against the rotation below)
    # with q rotated and rounded the same way
    after = to_numpy_bits(pool.storage)
    kc = _bits_to_f64(after[0], dtype).reshape(-1, hkv, d)
    vc = _bits_to_f64(after[1], dtype).reshape(-1, hkv, d)
    kf, qf = _bits_to_f64(kn, dtype), _bits_to_f64(qn, dtype)
    if theta > 0:
        kf, qf = oracle.rope(kf, pos, theta), oracle.rope(qf, pos, theta)
    qf = torch.from_numpy(qf).to(dtype).double().numpy()
    assert np.abs(kc[slots] - kf).max() <= 2.0 ** -7 * np.abs(kf).max()  # one 16-bit rounding of the rotation
    assert np.array_equal(vc[slots], _bits_to_f64(vn, dtype))
    unchanged = np.ones(kc.shape[0], bool)
    unchanged[slots] = False
    assert np.array_equal(after[0].reshape(-1, hkv, d)[unchanged].view(np.uint8),
                          before[0].reshape(-1, hkv, d)[unchanged].view(np.uint8))
    ref = oracle.decode_f64(0, np.ascontiguousarray(qf.astype(np.float32)),
                            kc.reshape(c["nb"], bs, hkv, d).astype(np.float32),
                            vc.reshape(c["nb"], bs, hkv, d).astype(np.float32), c["bt"][seq], pos + 1, 1.0 / np.sqrt(d))
    from workload_check import tol_check
    tol_check(out.cpu().numpy(), ref, tol)
    return out


@pytest.mark.parametrize("ctas", ["1", "2"])  # the one-CTA kernel and the 2-CTA (SM pair) kernel
@pytest.mark.parametrize("dtype,hq,hkv,bs,theta", [
    (torch.bfloat16, 8, 2, 32, 10000.0),   # group 4
    (torch.bfloat16, 16, 2, 16, 0.0),      # group 8
    (torch.float16, 32, 2, 64, 500.0),     # group 16
    (torch.bfloat16, 4, 4, 8, 10000.0),    # group 1
    (torch.float16, 4, 2, 128, 0.0),       # group 2, one block per key step
])
def test_prefill_tensor_core_multi_step(dtype, hq, hkv, bs, theta, ctas, monkeypatch):
    # contexts and prompts spanning several 128-key steps, prompt tails
    # shorter than a query tile, and a prompt continuing a cached context
    monkeypatch.setenv("CLOVE_PREFILL_CTAS", ctas)
    _prefill_vs_oracle(dtype, hq, hkv, 128, bs, theta, prior=[300, 0, 129, 7], prompt=[200, 257, 1, 95], seed=hq + bs)


def test_prefill_long_prompts_default_kernel_choice(monkeypatch):
    # prompts averaging over 1024 tokens (the 2-CTA kernel by default): many
    # 128-key steps, a continued prompt, quads of tiles cut by both prompt ends
    # P is rounded to bf16 before P.V (in every 16-bit prefill kernel here,
    # the warp-MMA one included); over rows of 1000+ keys its worst element
    # reaches ~2.15e-2 of |r| + rms on this seed in all three kernels alike,
    # hence 3e-2 here (2e-2 in the shorter cases above)
    monkeypatch.delenv("CLOVE_PREFILL_CTAS", raising=False)
    _prefill_vs_oracle(torch.bfloat16, 8, 2, 128, 32, 10000.0, prior=[0, 300], prompt=[1500, 700], seed=21, tol=3e-2)


@pytest.mark.parametrize("ctas", ["1", "2"])
def test_prefill_tensor_core_matches_warp_mma(ctas, monkeypatch):
    # the tcgen05 kernels and the warp-MMA kernel agree (both against the oracle)
    monkeypatch.setenv("CLOVE_PREFILL_CTAS", ctas)
    a = _prefill_vs_oracle(torch.bfloat16, 16, 4, 128, 32, 10000.0, prior=[50, 0], prompt=[400, 130], seed=3)
    b = _prefill_vs_oracle(torch.bfloat16, 16, 4, 128, 32, 10000.0, prior=[50, 0], prompt=[400, 130], seed=3,
                           variant="mma")
    assert torch.isfinite(a).all() and torch.isfinite(b).all()


@pytest.mark.parametrize("ctas", ["1", "2"])
def test_prefill_tensor_core_stuck_wait_times_out(ctas, monkeypatch):
    # failure detection without a GPU fault: one K/V step is never filled, the
    # bounded waits run out, the call completes with CLOVE_FLAG_TIMEOUT in the
    # pool's status word, and the next call on the same context is correct
    import time

    from clove_b200 import KVPool, _lib
    monkeypatch.setenv("CLOVE_PREFILL_CTAS", ctas)
    L = _lib.lib()
    c = _case(torch.bfloat16, 8, 2, 128, 32, prior=[0, 100], prompt=[300, 60], seed=5)
    pool = KVPool(c["nb"], 32, 2, 128, torch.bfloat16, 0)
    dev = torch.device("cuda", 0)
    try:
        _lib.check(L.clove_cuda_debug_set(2000, 1))
        t0 = time.time()
        pool.prefill(c["q"], c["k"], c["v"], torch.from_numpy(c["cu"]).to(dev), torch.from_numpy(c["bt"]).to(dev),
                     torch.from_numpy(c["ctx"]).to(dev), max_ctx=int(c["total"].max()))
        flags = pool.pool_status()
        elapsed = time.time() - t0
    finally:
        L.clove_cuda_debug_set(0, 0)
    assert flags & _lib.FLAG_TIMEOUT, flags
    assert elapsed < 30
    _prefill_vs_oracle(torch.bfloat16, 8, 2, 128, 32, 0.0, prior=[0, 100], prompt=[300, 60], seed=5)
