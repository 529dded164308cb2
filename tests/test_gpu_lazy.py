"""GPU: a traced-and-compiled PagedAttention::forward graph (projections +
paged attention + output projection) dispatches PagedAttention to the CUDA
path; its result is checked against the fp64 oracle of the whole module
(Linear, append, decode, Linear) and equals the eager module's bit for bit;
a symbolic batch binds at execution."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,bs", [(torch.float32, 16), (torch.bfloat16, 32)])
def test_compiled_forward_matches_eager(dtype, bs):
    from clove_b200.backend import PagedAttention
    from clove_b200.lazy import LazyBackend, compile, execute
    dev = torch.device("cuda", 0)
    dim, hq, hkv, D, B = 512, 8, 2, 64, 6
    m = PagedAttention(dim, hq, hkv, device=dev, dtype=dtype, seed=1)
    rng = np.random.default_rng(2)
    ctx = rng.integers(0, 90, B).astype(np.int32)
    need = ctx // bs + 1
    nb = int(need.sum()) + 2
    ids = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((B, int(need.max())), np.int32)
    o = 0
    for b in range(B):
        bt[b, :need[b]] = ids[o:o + need[b]]
        o += need[b]
    kv0 = torch.randn((2, nb, bs, hkv, D), device=dev).to(dtype)
    x = torch.randn((B, dim), device=dev).to(dtype)
    btd, cld = torch.from_numpy(bt).to(dev), torch.from_numpy(ctx).to(dev)
    max_ctx = int(ctx.max()) + 1

    kv_e = kv0.clone()
    eager = m.forward(x, kv_e, btd, cld, max_ctx=max_ctx)

    lb = LazyBackend()
    t = {n: lb.input(n, s) for n, s in (("x", ("B", dim)), ("wq", (dim, dim)), ("bq", (dim,)),
                                         ("wk", (dim, hkv * D)), ("bk", (hkv * D,)), ("wv", (dim, hkv * D)),
                                         ("bv", (hkv * D,)), ("wo", (dim, dim)), ("bo", (dim,)),
                                         ("kv_cache", tuple(kv0.shape)), ("block_tables", ("B", bt.shape[1])),
                                         ("context_lens", ("B",)))}
    q = lb.add(lb.matmul(t["x"], t["wq"]), t["bq"])
    k = lb.add(lb.matmul(t["x"], t["wk"]), t["bk"])
    v = lb.add(lb.matmul(t["x"], t["wv"]), t["bv"])
    a = lb.paged_attention(q, k, v, t["kv_cache"], t["block_tables"], t["context_lens"])
    out = lb.add(lb.matmul(a, t["wo"]), t["bo"])
    steps = compile(lb.graph, [out])
    kv_l = kv0.clone()
    feeds = {"x": x, "wq": m.w_q.weight, "bq": m.w_q.bias, "wk": m.w_k.weight, "bk": m.w_k.bias,
             "wv": m.w_v.weight, "bv": m.w_v.bias, "wo": m.w_o.weight, "bo": m.w_o.bias, "kv_cache": kv_l,
             "block_tables": btd, "context_lens": cld}
    lazy = execute(lb.graph, steps, feeds, max_ctx=max_ctx)[out.id]
    torch.cuda.synchronize()

    # fp64 oracle of the module: the three projections (src/nn.rs:538-540,
    # rounded to the cache dtype as the library GEMMs store them), the
    # slot-mapping append, the decode (src/nn/attention.rs:52-69) and the
    # output projection (src/nn.rs:545)
    import oracle
    from workload_check import tol_check

    def lin(a, w, b):
        return oracle.linear(a, w.double().cpu().numpy(), b.double().cpu().numpy())

    def rnd(a):  # round to the module dtype, back to f32 (exact)
        return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).float().numpy()

    x64 = x.double().cpu().numpy()
    qr = rnd(lin(x64, m.w_q.weight, m.w_q.bias)).reshape(B, hq, D)
    kr = rnd(lin(x64, m.w_k.weight, m.w_k.bias)).reshape(B, hkv, D)
    vr = rnd(lin(x64, m.w_v.weight, m.w_v.bias)).reshape(B, hkv, D)
    kc, vc = kv0[0].float().cpu().numpy(), kv0[1].float().cpu().numpy()
    assert oracle.reshape_and_cache(kc, vc, kr, vr, oracle.append_slots(bt, ctx, bs)) == 0
    attn = oracle.decode_f64(oracle.F32, qr, kc, vc, bt, ctx + 1, 1.0 / np.sqrt(D))
    ref = lin(attn.reshape(B, -1), m.w_o.weight, m.w_o.bias)
    # bf16: the 16-bit bar; f32: three f32 library GEMMs around the decode
    tol_check(lazy.double().cpu().numpy(), ref, 2e-2 if dtype == torch.bfloat16 else 1e-4)
    assert torch.equal(lazy, eager)
    assert torch.equal(kv_l.view(torch.uint8), kv_e.view(torch.uint8))  # same appended slots
