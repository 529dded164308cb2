"""One-GPU checks of the peer gather kernel (clove_cuda_peer_gather).  Two
ranks' calls would wait on each other, so they never run as two launches on
one GPU: the peer's side is played by the host instead — it writes the peer's
slice and delivery count into rank 0's receive buffer before the launch, and
the test checks what rank 0 stored into the peer's buffer.  A second call
with nothing delivered checks the bounded wait (CLOVE_FLAG_TIMEOUT, no
hang).  The two-process exchange runs in test_gpu_multi.py."""
import ctypes as C

import pytest
import torch

from clove_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _layout(slice_bytes, world):
    """Receive-buffer layout the kernel uses: two halves of world slots of
    slice_bytes rounded up to 256, then one u32 delivery count per source and
    the local state words; 8 KB chunks per CTA, at most 64."""
    slot = (slice_bytes + 255) // 256 * 256
    count_off = 2 * world * slot
    chunks = max(1, min(64, -(-slice_bytes // 8192)))
    return slot, count_off, chunks


def _gather(src, bufs, rank, out):
    ptrs = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=DEV)
    s = torch.cuda.current_stream(DEV)
    _lib.check(_lib.lib().clove_cuda_peer_gather(src.data_ptr(), src.numel() * 4, ptrs.data_ptr(), rank, len(bufs),
                                                 out.data_ptr(), s.cuda_stream))
    torch.cuda.synchronize()


def _status(buf, slice_bytes, world):
    flags = C.c_int(0)
    _lib.lib().clove_cuda_peer_gather_status(buf.data_ptr(), slice_bytes, world,
                                             torch.cuda.current_stream(DEV).cuda_stream, C.byref(flags))
    return flags.value


@pytest.mark.parametrize("n", [4, 3000, 200000])
def test_peer_gather_emulated_peer(n):
    lib = _lib.lib()
    sb = n * 4
    nbytes = int(lib.clove_cuda_peer_gather_buffer_bytes(sb, 2))
    slot, count_off, chunks = _layout(sb, 2)
    assert nbytes >= count_off + 20
    buf0 = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    buf1 = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    g = torch.Generator(device=DEV)
    for call in (1, 2, 3):  # halves alternate with the call number
        g.manual_seed(call)
        src = torch.randn(n, generator=g, device=DEV)
        peer = torch.randn(n, generator=g, device=DEV)
        half = (call & 1) * 2 * slot
        buf0[half + slot: half + slot + sb].copy_(peer.view(torch.uint8))
        buf0[count_off + 4: count_off + 8].view(torch.int32).fill_(call * chunks)  # peer 1 delivered
        out = torch.full((2 * n,), float("nan"), device=DEV)
        _gather(src, [buf0, buf1], 0, out)
        assert torch.equal(out[:n], src) and torch.equal(out[n:], peer)
        assert torch.equal(buf1[half: half + sb].view(torch.float32), src)  # stored at rank 0's slot
        assert int(buf1[count_off: count_off + 4].view(torch.int32).item()) == call * chunks
        assert _status(buf0, sb, 2) == 0


def test_peer_gather_single_rank_copies():
    n = 1000
    buf = torch.zeros(int(_lib.lib().clove_cuda_peer_gather_buffer_bytes(n * 4, 1)), dtype=torch.uint8, device=DEV)
    src = torch.randn(n, device=DEV)
    out = torch.empty(n, device=DEV)
    _gather(src, [buf], 0, out)
    assert torch.equal(out, src)


def test_peer_gather_missing_peer_times_out():
    """Nothing delivers: the bounded wait runs out, the call completes and
    the flag reports it; the context stays usable."""
    lib = _lib.lib()
    n = 512
    nbytes = int(lib.clove_cuda_peer_gather_buffer_bytes(n * 4, 2))
    buf0 = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    buf1 = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    src = torch.randn(n, device=DEV)
    out = torch.zeros(2 * n, device=DEV)
    _lib.check(lib.clove_cuda_debug_set(20000, 0))
    try:
        _gather(src, [buf0, buf1], 0, out)
    finally:
        _lib.check(lib.clove_cuda_debug_set(0, 0))
    assert _status(buf0, n * 4, 2) == _lib.FLAG_TIMEOUT
    assert _status(buf0, n * 4, 2) == 0  # cleared by the read
    assert torch.equal(out[:n], src)
    assert float((src * 2).sum()) == pytest.approx(float(src.sum()) * 2, rel=1e-5)  # context alive


def test_peer_buffer_alloc_and_handle():
    lib = _lib.lib()
    p = C.c_void_p()
    h = C.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    _lib.check(lib.clove_cuda_peer_buffer_alloc(0, 4096, C.byref(p), h))
    assert p.value and any(h.raw)
    _lib.check(lib.clove_cuda_peer_buffer_free(p))
