"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle and the
golden fixtures.

Bars: append and gather bit-exact; f32 decode |x - r| <= 1e-5 (|r| + rms(r))
against the fp64 oracle; bf16/f16 decode the same form with 2e-2 against the
fp64 oracle on the same 16-bit inputs.
"""
import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu

RTOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}
GOLDEN = ["f32_mha_small", "f32_gqa_zero_ctx", "bf16_gqa_bs32"]


def _dev():
    return torch.device("cuda", 0)


def _from_bits(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    if dtype == torch.float32:
        return torch.from_numpy(np.ascontiguousarray(a)).to(_dev())
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(dtype).to(_dev())


def _golden_pool(g):
    from clove_b200 import KVPool
    dtype = torch.bfloat16 if str(g["dtype"]) == "bf16" else torch.float32
    nb, bs, hkv, d = g["k_cache"].shape
    pool = KVPool(nb, bs, hkv, d, dtype=dtype, device=0)
    pool.k_cache.copy_(_from_bits(g["k_cache"], dtype))
    pool.v_cache.copy_(_from_bits(g["v_cache"], dtype))
    return pool, dtype


def _i32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(_dev())


@pytest.mark.parametrize("name,variant", [(n, v) for n in GOLDEN for v in ("auto", "simt")] +
                         [("bf16_gqa_bs32", "mma")])
def test_golden_append_decode(name, variant):
    from clove_b200 import set_decode_variant
    from workload_check import bits_equal, tol_check
    g = load_golden(name)
    pool, dtype = _golden_pool(g)
    set_decode_variant(variant)
    try:
        bt, cl = _i32(g["block_tables"]), _i32(g["context_lens"])
        out = pool.append_decode(_from_bits(g["q"], dtype), _from_bits(g["k_new"], dtype),
                                 _from_bits(g["v_new"], dtype), bt, cl, scale=float(g["scale"]))
        torch.cuda.synchronize()
    finally:
        set_decode_variant("auto")
    assert pool.decode_status(cl.numel(), g["q"].shape[1], int(g["context_lens"].max()) + 1) == 0
    assert bits_equal(pool.k_cache, g["k_cache_after"]) and bits_equal(pool.v_cache, g["v_cache_after"])
    tol_check(out.cpu().numpy(), g["expected"], RTOL[dtype])


@pytest.mark.parametrize("name", GOLDEN)
def test_golden_decode_no_append(name):
    from workload_check import tol_check
    g = load_golden(name)
    pool, dtype = _golden_pool(g)
    out = pool.decode(_from_bits(g["q"], dtype), _i32(g["block_tables"]), _i32(g["context_lens"]),
                      scale=float(g["scale"]))
    tol_check(out.cpu().numpy(), g["expected_noappend"], RTOL[dtype])


@pytest.mark.parametrize("name", GOLDEN)
def test_golden_reshape_and_cache_and_gather(name):
    from workload_check import bits_equal
    g = load_golden(name)
    pool, dtype = _golden_pool(g)
    pool.reshape_and_cache(_from_bits(g["k_new"], dtype), _from_bits(g["v_new"], dtype), _i32(g["slots"]))
    torch.cuda.synchronize()
    assert bits_equal(pool.k_cache, g["k_cache_after"]) and bits_equal(pool.v_cache, g["v_cache_after"])
    import oracle
    ctx = g["context_lens"] + 1
    max_ctx = int(ctx.max()) + 3
    ko, vo = pool.gather_kv(_i32(g["block_tables"]), _i32(ctx), max_ctx)
    rk, rv, bad = oracle.gather_kv(g["k_cache_after"], g["v_cache_after"], g["block_tables"], ctx, max_ctx)
    assert bad == 0
    assert bits_equal(ko, rk) and bits_equal(vo, rv)
    assert pool.pool_status() == 0
