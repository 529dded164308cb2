"""CPU: the lazy planner turns a traced PagedAttention node into a step sized
from the kv_cache shape (head_dim, block_size, KV heads), where the
reference's planner reads head_dim from q's last dimension and fixes the
block size at 16 (src/lazy.rs:2369-2372, :2384)."""
import pytest

from clove_b200.lazy import LazyBackend, Opcode, PagedAttentionStep, compile


def _trace(q_shape, kv_shape, with_projection=False):
    lb = LazyBackend()
    B = q_shape[0]
    if with_projection:
        x = lb.input("x", (B, 4096))
        wq, bq = lb.input("wq", (4096, 4096)), lb.input("bq", (4096,))
        q = lb.add(lb.matmul(x, wq), bq)
    else:
        q = lb.input("q", q_shape)
    k = lb.input("k", (B, kv_shape[-2] * kv_shape[-1]))
    v = lb.input("v", (B, kv_shape[-2] * kv_shape[-1]))
    kv = lb.input("kv_cache", kv_shape)
    bt = lb.input("block_tables", (B, 64))
    cl = lb.input("context_lens", (B,))
    out = lb.paged_attention(q, k, v, kv, bt, cl)
    return lb, out


def test_node_shape_is_q_shape_and_step_sizes_come_from_the_cache():
    lb, out = _trace(("B", 64 * 128), (2, 40960, 32, 8, 128))
    assert out.shape == ("B", 64 * 128)
    (st,) = compile(lb.graph, [out])
    assert isinstance(st, PagedAttentionStep)
    # the reference's planner would say head_dim 8192 (q's last dim) and block 16
    assert (st.head_dim, st.block_size, st.num_kv_heads, st.num_q_heads) == (128, 32, 8, 64)
    assert st.deps == [n.id for n in lb.graph.nodes[:6]]


def test_three_dim_q_and_projection_chain_order():
    lb, out = _trace((16, 32, 128), (2, 1024, 16, 8, 128), with_projection=True)
    steps = compile(lb.graph, [out])
    # the projection's MatMul + bias Add plan as one Linear step
    assert [s.op for s in steps] == [Opcode.LINEAR, Opcode.PAGED_ATTENTION]
    assert steps[-1].num_q_heads == 32


@pytest.mark.parametrize("q_shape,kv_shape,msg", [
    ((4, 100), (2, 64, 16, 2, 64), "multiple of head_dim"),
    ((4, 3 * 64), (2, 64, 16, 2, 64), "multiple of num_kv_heads"),
    ((4, 128), (64, 16, 2, 64), "kv_cache must be"),
    ((4, 128), (2, 64, "bs", 2, 64), "block_size must be a constant"),
])
def test_planner_rejects_inconsistent_shapes(q_shape, kv_shape, msg):
    lb, out = _trace(q_shape, kv_shape)
    with pytest.raises(ValueError, match=msg):
        compile(lb.graph, [out])


def test_unused_nodes_are_not_planned():
    lb, out = _trace((4, 128), (2, 64, 16, 2, 64))
    lb.matmul(lb.input("a", (4, 4)), lb.input("b", (4, 4)))  # dead branch
    assert [s.op for s in compile(lb.graph, [out])] == [Opcode.PAGED_ATTENTION]


def test_execute_binds_symbols_and_runs_linear_steps_on_any_device():
    # host logic of execute(): symbolic dims bind from the feeds, a mismatch
    # raises, and a Linear step is one addmm (bit-equal to torch.addmm)
    import torch

    from clove_b200.lazy import execute
    lb = LazyBackend()
    x = lb.input("x", ("B", 8))
    w, b = lb.input("w", (8, 4)), lb.input("b", (4,))
    y = lb.add(lb.matmul(x, w), b)
    steps = compile(lb.graph, [y])
    assert [s.op for s in steps] == [Opcode.LINEAR]
    g = torch.Generator().manual_seed(0)
    feeds = {"x": torch.randn(3, 8, generator=g), "w": torch.randn(8, 4, generator=g), "b": torch.randn(4, generator=g)}
    out = execute(lb.graph, steps, feeds)[y.id]
    assert torch.equal(out, torch.addmm(feeds["b"], feeds["x"], feeds["w"]))
    with pytest.raises(ValueError, match="dimension"):
        execute(lb.graph, steps, {**feeds, "w": torch.randn(9, 4)})
    lb2 = LazyBackend()
    a1, a2 = lb2.input("a1", ("B", 4)), lb2.input("a2", ("B", 4))
    s2 = lb2.add(a1, a2)
    with pytest.raises(ValueError, match="symbol B"):
        execute(lb2.graph, compile(lb2.graph, [s2]), {"a1": torch.zeros(2, 4), "a2": torch.zeros(3, 4)})


def test_requested_matmul_is_not_fused_away():
    # a MatMul that is also a requested output keeps its own step, so its
    # value exists after execute(); the Add then runs as a plain step
    lb = LazyBackend()
    x, w, b = lb.input("x", (4, 64)), lb.input("w", (64, 32)), lb.input("b", (32,))
    mm = lb.matmul(x, w)
    y = lb.add(mm, b)
    ops = [s.op for s in compile(lb.graph, [y, mm])]
    assert Opcode.LINEAR not in ops
    assert ops.count(Opcode.MATMUL) == 1 and ops.count(Opcode.ADD) == 1
    assert [s.op for s in compile(lb.graph, [y])] == [Opcode.LINEAR]
