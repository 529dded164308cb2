"""Multi-GPU decode: one process per GPU over torch.distributed.

Two partitionings (the reference's orchestrator is MultiGPUOrchestrator,
src/distributed.rs:41-313, with distribute_batch at :184-200):

  sequence sharding   each rank owns a subset of sequences, its own KV block
                      pool and block tables; no collective on the data path.
  KV-head sharding    (long-context configuration) each rank owns a contiguous
                      range of KV heads of every sequence — its pool stores only
                      those heads — decodes the query heads that read them, and
                      one all-gather assembles [batch, num_q_heads, head_dim].

The compute is the single-GPU C-ABI path.  The output gather runs either
through torch.distributed (NCCL on GPUs, gloo on CPU) or, on GPUs, through
PeerGather: one kernel of the library that stores each rank's slice straight
into its peers' memory over NVLink (CUDA IPC mappings, no multicast).
"""
from __future__ import annotations

import ctypes as C
import os

import torch
import torch.distributed as dist

from . import _lib
from .sharding import head_shards


def init_from_env(backend: str | None = None) -> tuple[int, int, int]:
    """(world_size, rank, local_rank) from the torchrun environment; joins the
    process group when world_size > 1."""
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend)
    return ws, rank, local


def local_heads(num_kv_heads: int, group: int, world: int, rank: int) -> tuple[range, range]:
    """(KV heads, query heads) this rank owns under KV-head sharding."""
    return head_shards(num_kv_heads, group, world)[rank]


def gather_heads(out_local: torch.Tensor, world: int, group_pg=None) -> torch.Tensor:
    """All-gather per-rank outputs [B, hq_local, D] into [B, world*hq_local, D]
    (rank r's query heads land at r*hq_local .. (r+1)*hq_local - 1)."""
    if world == 1:
        return out_local
    B, hl, D = out_local.shape
    buf = torch.empty((world * B, hl, D), dtype=out_local.dtype, device=out_local.device)
    dist.all_gather_into_tensor(buf, out_local.contiguous(), group=group_pg)
    return buf.view(world, B, hl, D).permute(1, 0, 2, 3).reshape(B, world * hl, D)


def head_sharded_append_decode(pool_local, q_local: torch.Tensor, k_new_local: torch.Tensor,
                               v_new_local: torch.Tensor, block_tables: torch.Tensor,
                               context_lens: torch.Tensor, world: int, max_ctx: int,
                               scale: float | None = None, out_local: torch.Tensor | None = None,
                               gather_buf: torch.Tensor | None = None,
                               peer: "PeerGather | None" = None) -> torch.Tensor:
    """Append + decode under KV-head sharding.  Every argument is this rank's
    share: q_local [B, hq_local, D] holds the query heads of the KV heads in
    pool_local (rank r: query heads r*hq_local .. (r+1)*hq_local - 1, as
    local_heads gives them), k_new_local / v_new_local [B, hkv_local, D].
    Returns the full [B, world*hq_local, D] output on every rank.
    Preallocated out_local / gather_buf make the call free of allocations
    (e.g. for CUDA-graph capture).  With `peer` (a PeerGather over slices of
    out_local's size) the outputs travel by P2P stores instead of NCCL."""
    out_local = pool_local.append_decode(q_local, k_new_local, v_new_local, block_tables, context_lens,
                                         scale=scale, max_ctx=max_ctx, out=out_local)
    if world == 1:
        return out_local
    B, hl, D = out_local.shape
    if gather_buf is None:
        gather_buf = torch.empty((world * B, hl, D), dtype=out_local.dtype, device=out_local.device)
    if peer is not None:
        peer(out_local, gather_buf)
    else:
        dist.all_gather_into_tensor(gather_buf, out_local)
    return gather_buf.view(world, B, hl, D).permute(1, 0, 2, 3)  # [B, world, hl, D] view


class PeerGather:
    """All-gather of a fixed-size slice over NVLink peer memory
    (clove_cuda_peer_gather): every rank allocates a receive buffer, the IPC
    handles travel once through torch.distributed, and each call is one kernel
    that stores this rank's slice into every peer's buffer and collects the
    peers' slices into `out` — no NCCL on the data path, capturable in a CUDA
    graph.  Output layout as all_gather_into_tensor: out[r] = rank r's slice.

    The reference assembles per-shard results through host staging buffers
    (MultiGPUOrchestrator::synchronize_gradients, src/distributed.rs:204-300).
    """

    def __init__(self, slice_bytes: int, device: torch.device, group_pg=None):
        self.world = dist.get_world_size(group_pg) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group_pg) if dist.is_initialized() else 0
        self.slice_bytes = int(slice_bytes)
        self.device = torch.device(device)
        self._pg = group_pg
        self._lib = _lib.lib()
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self._dev = dev
        nbytes = int(self._lib.clove_cuda_peer_gather_buffer_bytes(self.slice_bytes, self.world))
        own = C.c_void_p()
        handle = C.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        _lib.check(self._lib.clove_cuda_peer_buffer_alloc(dev, nbytes, C.byref(own), handle))
        self._own = own
        self._opened: list[C.c_void_p] = []
        handles = [handle.raw]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group_pg)
        ptrs = []
        for r in range(self.world):
            if r == self.rank:
                ptrs.append(own.value)
                continue
            p = C.c_void_p()
            _lib.check(self._lib.clove_cuda_peer_buffer_open(dev, C.c_char_p(handles[r]), C.byref(p)))
            self._opened.append(p)
            ptrs.append(p.value)
        self.ptrs = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        if self.world > 1:  # every peer mapped before anyone stores into it
            dist.barrier(group=group_pg)

    def __call__(self, src: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
        if src.device != self.device or not src.is_contiguous() or \
                src.numel() * src.element_size() != self.slice_bytes:
            raise ValueError("src must be a contiguous tensor of slice_bytes on this rank's device")
        if out.device != self.device or not out.is_contiguous() or \
                out.numel() * out.element_size() != self.slice_bytes * self.world:
            raise ValueError("out must be a contiguous tensor of world * slice_bytes")
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.check(self._lib.clove_cuda_peer_gather(src.data_ptr(), self.slice_bytes, self.ptrs.data_ptr(),
                                                    self.rank, self.world, out.data_ptr(), s.cuda_stream))
        return out

    def status(self, stream=None) -> int:
        """Flags (CLOVE_FLAG_*) raised by calls since the last status read.
        After CLOVE_FLAG_TIMEOUT the ranks' counts are out of step: close this
        gather on every rank and make a new one."""
        flags = C.c_int(0)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        rc = self._lib.clove_cuda_peer_gather_status(self._own, self.slice_bytes, self.world, s.cuda_stream,
                                                     C.byref(flags))
        if rc not in (_lib.OK, _lib.ERR_DEVICE_CHECK):
            _lib.check(rc)
        return flags.value

    def close(self) -> None:
        """Unmap the peers' buffers and, once every rank has, free this one."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self._lib.clove_cuda_peer_buffer_close(p)
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self._pg)
        self._lib.clove_cuda_peer_buffer_free(self._own)
        self._own = None
