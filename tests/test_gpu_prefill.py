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
    q = torch.randn((T, hq, d), device=dev).to(dtype)
    k = torch.randn((T, hkv, d), device=dev).to(dtype)
    v = torch.randn((T, hkv, d), device=dev).to(dtype)
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
    # one 3000-token prompt: its late tokens attend over many chunks (split-K path)
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
