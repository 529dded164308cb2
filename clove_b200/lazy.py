"""Lazy-graph dispatch of PagedAttention to the CUDA path.

A mirror of the reference's lazy JIT for the one op on the path:

  LazyBackend.paged_attention   <- LazyBackend::paged_attention, src/lazy.rs:860-899
      records a PagedAttention node whose shape is q's shape (:875, :886)
  compile()                     <- the planner, src/lazy.rs:2353-2387
      turns the node into Step.PagedAttention (src/lazy.rs:1354-1366)
  execute()                     <- the dispatch, src/lazy.rs:4133-4256
      runs the step through CudaBackend.paged_attention (clove_cuda_paged_append_decode)

The planner takes head_dim, block_size and the KV-head count from the
kv_cache node's shape [2, num_blocks, block_size, num_kv_heads, head_dim].
The reference reads head_dim from q's last dimension, which is Hq * D for the
2-D q that PagedAttention::forward produces, with a fallback of 64
(src/lazy.rs:2369-2372), and hard-codes block_size 16 (:2384).  Shapes may
hold symbols (the reference's SymInt): a str dimension is bound at execute()
from the fed tensors.

MatMul / Add (the projections of PagedAttention::forward, src/nn.rs:538-545)
run as torch ops: they are off the path and not part of its kernels.  The
planner fuses a MatMul whose only consumer adds a bias row into one Linear
step (one GEMM with the bias in its epilogue, as the eager Linear runs it),
so a compiled graph reproduces the eager module bit for bit.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from enum import Enum

import torch

from .backend import CudaBackend

SymInt = int | str


class Opcode(Enum):
    INPUT = "input"
    MATMUL = "matmul"
    ADD = "add"
    LINEAR = "linear"  # planner only: MatMul whose single consumer adds a bias row
    PAGED_ATTENTION = "paged_attention"


@dataclass
class Node:
    id: int
    op: Opcode
    shape: tuple[SymInt, ...]
    deps: list[int] = field(default_factory=list)
    name: str = ""


class LazyGraph:
    """The traced graph (the reference's thread-local GLOBAL_GRAPH)."""

    def __init__(self):
        self.nodes: list[Node] = []

    def push(self, op: Opcode, shape, deps=(), name: str = "") -> int:
        self.nodes.append(Node(len(self.nodes), op, tuple(shape), list(deps), name))
        return len(self.nodes) - 1


@dataclass(frozen=True)
class LazyTensor:
    graph: LazyGraph
    id: int

    @property
    def shape(self) -> tuple[SymInt, ...]:
        return self.graph.nodes[self.id].shape


class LazyBackend:
    """Records ops instead of running them."""

    def __init__(self, graph: LazyGraph | None = None):
        self.graph = graph or LazyGraph()

    def input(self, name: str, shape) -> LazyTensor:
        return LazyTensor(self.graph, self.graph.push(Opcode.INPUT, shape, name=name))

    def matmul(self, a: LazyTensor, b: LazyTensor) -> LazyTensor:
        sa, sb = a.shape, b.shape
        return LazyTensor(self.graph, self.graph.push(Opcode.MATMUL, (sa[0], sb[-1]), [a.id, b.id]))

    def add(self, a: LazyTensor, b: LazyTensor) -> LazyTensor:
        return LazyTensor(self.graph, self.graph.push(Opcode.ADD, a.shape, [a.id, b.id]))

    def paged_attention(self, q: LazyTensor, k: LazyTensor, v: LazyTensor, kv_cache: LazyTensor,
                        block_tables: LazyTensor, context_lens: LazyTensor) -> LazyTensor:
        # output shape = q's shape (src/lazy.rs:875, :886); no backward (:897)
        deps = [q.id, k.id, v.id, kv_cache.id, block_tables.id, context_lens.id]
        return LazyTensor(self.graph, self.graph.push(Opcode.PAGED_ATTENTION, q.shape, deps))


@dataclass
class Step:
    op: Opcode
    out_id: int
    deps: list[int]


@dataclass
class PagedAttentionStep(Step):
    """Step::PagedAttention (src/lazy.rs:1354-1366) with the sizes the CUDA
    path needs, all from the kv_cache shape."""
    size: tuple[SymInt, ...] = ()  # factors of the element count (resolved at execute)
    head_dim: int = 0
    block_size: int = 0
    num_kv_heads: int = 0
    num_q_heads: SymInt = 0


def _const(d: SymInt, what: str) -> int:
    if not isinstance(d, int):
        raise ValueError(f"{what} must be a constant dimension, got symbol {d!r}")
    return d


def compile(graph: LazyGraph, outputs: list[LazyTensor]) -> list[Step]:
    """Planner: the steps that compute `outputs`, in dependency order."""
    need: set[int] = set()
    stack = [t.id for t in outputs]
    while stack:
        i = stack.pop()
        if i not in need:
            need.add(i)
            stack.extend(graph.nodes[i].deps)
    users: dict[int, int] = {}
    for node in graph.nodes:
        if node.id in need:
            for d in node.deps:
                users[d] = users.get(d, 0) + 1
    # MatMul + bias Add -> one Linear step (the reference Linear, src/nn.rs:114-117),
    # run as one GEMM with the bias in its epilogue.  A MatMul that is itself
    # a requested output keeps its own step (its value must exist).
    requested = {t.id for t in outputs}
    fused_mm: set[int] = set()
    linear_of: dict[int, list[int]] = {}
    for node in graph.nodes:
        if node.id in need and node.op is Opcode.ADD:
            mm = graph.nodes[node.deps[0]]
            if (mm.op is Opcode.MATMUL and users.get(mm.id) == 1 and mm.id not in requested
                    and len(graph.nodes[node.deps[1]].shape) == 1):
                fused_mm.add(mm.id)
                linear_of[node.id] = [mm.deps[0], mm.deps[1], node.deps[1]]
    steps: list[Step] = []
    for node in graph.nodes:  # push order is a topological order
        if node.id not in need or node.op is Opcode.INPUT or node.id in fused_mm:
            continue
        if node.id in linear_of:
            steps.append(Step(Opcode.LINEAR, node.id, linear_of[node.id]))
        elif node.op is Opcode.PAGED_ATTENTION:
            q, _, _, kv, bt, cl = (graph.nodes[d] for d in node.deps)
            if len(kv.shape) != 5 or kv.shape[0] != 2:
                raise ValueError("kv_cache must be [2, num_blocks, block_size, num_kv_heads, head_dim]")
            block_size = _const(kv.shape[2], "block_size")
            hkv = _const(kv.shape[3], "num_kv_heads")
            head_dim = _const(kv.shape[4], "head_dim")
            if len(q.shape) == 2:
                width = _const(q.shape[1], "q width")
                if width % head_dim:
                    raise ValueError(f"q width {width} is not a multiple of head_dim {head_dim}")
                hq = width // head_dim
            elif len(q.shape) == 3:
                hq = _const(q.shape[1], "num_q_heads")
                if _const(q.shape[2], "q head_dim") != head_dim:
                    raise ValueError("q head_dim differs from the cache's")
            else:
                raise ValueError("q must be [batch, Hq*D] or [batch, Hq, D]")
            if hq % hkv:
                raise ValueError(f"num_q_heads {hq} is not a multiple of num_kv_heads {hkv}")
            steps.append(PagedAttentionStep(Opcode.PAGED_ATTENTION, node.id, list(node.deps), size=node.shape,
                                            head_dim=head_dim, block_size=block_size, num_kv_heads=hkv,
                                            num_q_heads=hq))
        else:
            steps.append(Step(node.op, node.id, list(node.deps)))
    return steps


def _bind(shape, t: torch.Tensor, env: dict[str, int], name: str) -> None:
    if len(shape) != t.dim():
        raise ValueError(f"{name}: rank {t.dim()} fed for shape {shape}")
    for s, n in zip(shape, t.shape):
        if isinstance(s, str):
            if env.setdefault(s, n) != n:
                raise ValueError(f"{name}: symbol {s} bound to {env[s]} and {n}")
        elif s != n:
            raise ValueError(f"{name}: dimension {n} fed for {s}")


def execute(graph: LazyGraph, steps: list[Step], feeds: dict[str, torch.Tensor],
            max_ctx: int | None = None) -> dict[int, torch.Tensor]:
    """Run compiled steps; feeds maps input names to tensors.  Returns every
    computed value by node id."""
    env: dict[str, int] = {}
    vals: dict[int, torch.Tensor] = {}
    for node in graph.nodes:
        if node.op is Opcode.INPUT and node.name in feeds:
            _bind(node.shape, feeds[node.name], env, node.name)
            vals[node.id] = feeds[node.name]
    for st in steps:
        args = [vals[d] for d in st.deps]
        if st.op is Opcode.LINEAR:
            out = torch.addmm(args[2], args[0], args[1])
        elif st.op is Opcode.MATMUL:
            out = args[0] @ args[1]
        elif st.op is Opcode.ADD:
            out = args[0] + args[1]
        elif isinstance(st, PagedAttentionStep):
            q, k, v, kv, bt, cl = args
            elems = math.prod(env[s] if isinstance(s, str) else s for s in st.size)
            if q.numel() != elems:
                raise ValueError(f"PagedAttention: q has {q.numel()} elements, the plan {elems}")
            out = CudaBackend.paged_attention(q.reshape(q.shape[0], -1), k, v, kv, bt, cl, max_ctx=max_ctx)
        else:
            raise ValueError(f"no dispatch for {st.op}")
        vals[st.out_id] = out
    return vals
