"""GPU parity on the five configurations: full oracle checks at CPU-sized
batches, and subset checks at the full sizes."""
import numpy as np
import pytest
import torch

from workload_check import run_layout_vs_oracle, small_layout

pytestmark = pytest.mark.gpu

RT = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def _rt(name):
    from clove_b200.workload import CONFIGS
    return RT[CONFIGS[name].dtype]


def test_c1_full_vs_oracle():
    run_layout_vs_oracle(small_layout("c1", batch=8, ctx_scale=1.0), _rt("c1"))


@pytest.mark.parametrize("name,batch,scale", [("c2", 4, 1.0), ("c3", 16, 0.25), ("c4", 2, 0.02),
                                              ("c5", 24, 0.25)])
@pytest.mark.parametrize("variant", ["auto", "simt"])
def test_configs_reduced_vs_oracle(name, batch, scale, variant):
    from clove_b200 import set_decode_variant
    set_decode_variant(variant)
    try:
        run_layout_vs_oracle(small_layout(name, batch=batch, ctx_scale=scale), _rt(name))
    finally:
        set_decode_variant("auto")


@pytest.mark.parametrize("name", ["c2", "c3", "c4", "c5"])
def test_configs_full_size_subset(name):
    from clove_b200.workload import CONFIGS, make_layout
    lay = make_layout(CONFIGS[name])
    run_layout_vs_oracle(lay, _rt(name), subset=4)
    torch.cuda.empty_cache()


def test_plain_decode_without_append():
    run_layout_vs_oracle(small_layout("c3", batch=8, ctx_scale=0.1), _rt("c3"), append=False)


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("group", [1, 2, 3, 4, 8])
def test_shapes_dtypes_groups(d, dtype, group):
    from clove_b200.workload import Layout, Spec, make_layout
    hkv = 2
    spec = Spec("t", 3, hkv * group, hkv, d, 16, 0, dtype, "uniform", 1, 300, "permutation", seed=11)
    run_layout_vs_oracle(make_layout(spec), RT[dtype])


@pytest.mark.parametrize("bs", [8, 16, 32, 64])
def test_block_sizes(bs):
    from clove_b200.workload import Spec, make_layout
    spec = Spec("t", 4, 4, 4, 128, bs, 0, torch.float32, "uniform", 1, 700, "permutation", seed=12)
    run_layout_vs_oracle(make_layout(spec), 1e-5)


def test_block_boundaries_and_tiny_contexts():
    # ctx such that the appended token starts a new block, ends one, and ctx=0.
    from clove_b200.workload import Layout, Spec
    spec = Spec("t", 6, 8, 2, 128, 16, 0, torch.bfloat16, "fixed", 1, 1, "permutation", seed=13)
    ctx = np.array([0, 15, 16, 31, 1, 47], np.int32)
    need = (ctx + 1 + 15) // 16
    rng = np.random.default_rng(5)
    nb = int(need.sum()) + 5
    ids = rng.permutation(nb)
    bt = np.zeros((6, need.max()), np.int32)
    o = 0
    for b in range(6):
        bt[b, :need[b]] = ids[o:o + need[b]]
        o += need[b]
    run_layout_vs_oracle(Layout(spec, ctx, bt, nb, 13), 2e-2)


def test_long_context_split_chunks():
    # one very long sequence forces many chunks and the last-CTA combine
    from clove_b200.workload import Spec, make_layout
    spec = Spec("t", 2, 16, 2, 128, 32, 0, torch.bfloat16, "uniform", 60000, 70000, "permutation", seed=14)
    run_layout_vs_oracle(make_layout(spec), 2e-2)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("group", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("bs", [8, 16, 32])
def test_tensor_core_variant_forced(d, dtype, group, bs):
    from clove_b200 import set_decode_variant
    from clove_b200.workload import Spec, make_layout
    spec = Spec("t", 3, 2 * group, 2, d, bs, 0, dtype, "uniform", 1, 500, "permutation", seed=15)
    set_decode_variant("mma")
    try:
        run_layout_vs_oracle(make_layout(spec), RT[dtype])
    finally:
        set_decode_variant("auto")


def test_tensor_core_nan_rows_past_context():
    # Pool memory past the context holds NaN bit patterns; the output must
    # not see them (P is zero there and the tensor-core kernel clears V rows).
    from clove_b200 import KVPool
    from clove_b200.workload import Spec, fill_values, make_layout
    spec = Spec("t", 4, 16, 2, 128, 32, 0, torch.bfloat16, "uniform", 1, 90, "permutation", seed=16)
    lay = make_layout(spec)
    dev = torch.device("cuda", 0)
    pool = KVPool(lay.num_blocks, 32, 2, 128, torch.bfloat16, 0)
    q, kn, vn, _ = fill_values(lay, dev, pool.storage)
    # poison every slot past each sequence's (post-append) length
    for b in range(lay.batch):
        L = int(lay.context_lens[b]) + 1
        blk = int(lay.block_tables[b, (L - 1) // 32])
        pool.storage[:, blk, (L - 1) % 32 + 1:] = float("nan")
    out = pool.append_decode(q, kn, vn, torch.from_numpy(lay.block_tables).to(dev),
                             torch.from_numpy(lay.context_lens).to(dev), max_ctx=lay.max_ctx)
    assert torch.isfinite(out).all()
