"""CPU tests of the oracle against the committed golden fixtures, an
independent torch implementation, and the append / gather / mock rules."""
import numpy as np
import pytest
import torch

from conftest import load_golden

CASES = ["f32_mha_small", "f32_gqa_zero_ctx", "bf16_gqa_bs32"]


def _code(g):
    return 160 if str(g["dtype"]) == "bf16" else 0


@pytest.mark.parametrize("name", CASES)
def test_append_matches_golden(oracle_lib, name):
    g = load_golden(name)
    kc, vc = g["k_cache"].copy(), g["v_cache"].copy()
    slots = oracle_lib.append_slots(g["block_tables"], g["context_lens"], kc.shape[1])
    assert np.array_equal(slots, g["slots"])
    bad = oracle_lib.reshape_and_cache(kc, vc, g["k_new"], g["v_new"], slots)
    assert bad == 0
    assert np.array_equal(kc.view(np.uint8), g["k_cache_after"].view(np.uint8))
    assert np.array_equal(vc.view(np.uint8), g["v_cache_after"].view(np.uint8))


@pytest.mark.parametrize("name", CASES)
def test_decode_f64_matches_golden(oracle_lib, name):
    g = load_golden(name)
    out = oracle_lib.decode_f64(_code(g), g["q"], g["k_cache_after"], g["v_cache_after"], g["block_tables"],
                                g["context_lens"] + 1, float(g["scale"]))
    np.testing.assert_allclose(out, g["expected"], rtol=1e-12, atol=1e-13)
    out0 = oracle_lib.decode_f64(_code(g), g["q"], g["k_cache"], g["v_cache"], g["block_tables"],
                                 g["context_lens"], float(g["scale"]))
    np.testing.assert_allclose(out0, g["expected_noappend"], rtol=1e-12, atol=1e-13)


@pytest.mark.parametrize("name", CASES)
def test_decode_f32_within_tolerance(oracle_lib, name):
    # f32 restatement vs fp64 truth: |x - r| <= 1e-5 (|r| + rms(r)).
    g = load_golden(name)
    out = oracle_lib.decode_f32(_code(g), g["q"], g["k_cache_after"], g["v_cache_after"], g["block_tables"],
                                g["context_lens"] + 1, float(g["scale"]))
    ok, worst = oracle_lib.tolerance_ok(out, g["expected"], 1e-5)
    assert ok, worst


def test_decode_matches_torch_independent(oracle_lib):
    # Secondary cross-check: torch CPU softmax(q K^T scale) V on gathered K/V.
    rng = np.random.default_rng(7)
    B, hq, hkv, d, bs = 3, 6, 3, 64, 8
    ctx = np.array([5, 17, 33], np.int32)
    need = (ctx + bs - 1) // bs
    nb = int(need.sum()) + 2
    ids = rng.permutation(nb)
    bt = np.zeros((B, need.max()), np.int32)
    o = 0
    for b in range(B):
        bt[b, :need[b]] = ids[o:o + need[b]]
        o += need[b]
    kc = rng.standard_normal((nb, bs, hkv, d)).astype(np.float32)
    vc = rng.standard_normal((nb, bs, hkv, d)).astype(np.float32)
    q = rng.standard_normal((B, hq, d)).astype(np.float32)
    scale = 1 / np.sqrt(d)
    got = oracle_lib.decode_f64(0, q, kc, vc, bt, ctx, scale)
    for b in range(B):
        t = np.arange(ctx[b])
        K = torch.from_numpy(kc[bt[b, t // bs], t % bs]).double().repeat_interleave(hq // hkv, dim=1)
        V = torch.from_numpy(vc[bt[b, t // bs], t % bs]).double().repeat_interleave(hq // hkv, dim=1)
        Q = torch.from_numpy(q[b]).double() * scale
        P = torch.softmax(torch.einsum("hd,lhd->hl", Q, K), dim=1)
        ref = torch.einsum("hl,lhd->hd", P, V).numpy()
        np.testing.assert_allclose(got[b], ref, rtol=1e-12, atol=1e-13)


def test_gather_follows_block_tables(oracle_lib):
    g = load_golden("f32_mha_small")
    ctx = g["context_lens"]
    max_ctx = int(ctx.max())
    ko, vo, bad = oracle_lib.gather_kv(g["k_cache"], g["v_cache"], g["block_tables"], ctx, max_ctx)
    assert bad == 0
    bs = g["k_cache"].shape[1]
    for b in range(ctx.shape[0]):
        for t in range(max_ctx):
            if t < ctx[b]:
                phys = g["block_tables"][b, t // bs]
                assert np.array_equal(ko[b, t], g["k_cache"][phys, t % bs])
                assert np.array_equal(vo[b, t], g["v_cache"][phys, t % bs])
            else:
                assert not ko[b, t].any() and not vo[b, t].any()


def test_gather_counts_bad_blocks(oracle_lib):
    g = load_golden("f32_mha_small")
    bt = g["block_tables"].copy()
    bt[0, 0] = 10 ** 6
    _, _, bad = oracle_lib.gather_kv(g["k_cache"], g["v_cache"], bt, g["context_lens"],
                                     int(g["context_lens"].max()))
    assert bad == g["k_cache"].shape[1]  # every token of the bad block


def test_reshape_and_cache_skips_padding_and_counts_oob(oracle_lib):
    kc = np.zeros((4, 2, 1, 4), np.float32)
    vc = np.zeros_like(kc)
    k = np.arange(12, dtype=np.float32).reshape(3, 1, 4)
    v = -k
    bad = oracle_lib.reshape_and_cache(kc, vc, k, v, np.array([-1, 5, 8], np.int32))
    assert bad == 1
    assert np.array_equal(kc.reshape(8, 4)[5], k[1, 0]) and np.array_equal(vc.reshape(8, 4)[5], v[1, 0])
    assert np.count_nonzero(kc.reshape(8, 4)[[0, 1, 2, 3, 4, 6, 7]]) == 0


def test_mock_kernel_characterisation(oracle_lib):
    # The reference's placeholder kernel (src/lazy.rs:5255-5274): not the op's
    # semantics, recorded so its behaviour is characterised.
    g = load_golden("mock_lazy_kernel")
    out = oracle_lib.mock_paged_attention(g["q"], g["kv_cache"], g["block_tables"], int(g["seq_len"]),
                                          int(g["head_dim"]), int(g["block_size"]))
    np.testing.assert_array_equal(out, g["expected"])


def test_bf16_widening_is_exact(oracle_lib):
    g = load_golden("bf16_gqa_bs32")
    bits = g["q"]
    t = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).float().numpy()
    mine = (bits.astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(t, mine)
