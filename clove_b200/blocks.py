"""Python face of the KV block manager (include/clove_blocks.h)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib


class BlockManager:
    """Sequence -> physical block mapping of one KV pool, with reference-
    counted sharing (fork) and copy-on-write on append."""

    def __init__(self, num_blocks: int, block_size: int, max_seqs: int):
        self._lib = _lib.lib()
        h = C.c_void_p()
        _lib.check(self._lib.clove_blocks_create(num_blocks, block_size, max_seqs, C.byref(h)))
        self.handle = h
        self.block_size = block_size

    def __del__(self):
        try:
            if self.handle:
                self._lib.clove_blocks_destroy(self.handle)
        except Exception:
            pass

    def add(self, seq: int, length: int) -> None:
        _lib.check(self._lib.clove_blocks_add(self.handle, seq, length))

    def reserve(self, seq: int, length: int, max_copies: int = 64) -> list[tuple[int, int]]:
        """Grow `seq` to `length` tokens; returns the (src, dst) block copies
        the caller must perform before writing (copy-on-write)."""
        src = np.zeros(max_copies, np.int32)
        dst = np.zeros(max_copies, np.int32)
        n = C.c_int(max_copies)
        _lib.check(self._lib.clove_blocks_reserve(self.handle, seq, length, src.ctypes.data, dst.ctypes.data,
                                                  C.byref(n)))
        return [(int(src[i]), int(dst[i])) for i in range(n.value)]

    def fork(self, parent: int, child: int) -> None:
        _lib.check(self._lib.clove_blocks_fork(self.handle, parent, child))

    def free(self, seq: int) -> None:
        _lib.check(self._lib.clove_blocks_free(self.handle, seq))

    @property
    def num_free(self) -> int:
        return int(self._lib.clove_blocks_num_free(self.handle))

    def seq_len(self, seq: int) -> int:
        return int(self._lib.clove_blocks_seq_len(self.handle, seq))

    def export(self, seqs, stride: int) -> tuple[np.ndarray, np.ndarray]:
        s = np.ascontiguousarray(seqs, np.int32)
        tables = np.empty((s.shape[0], stride), np.int32)
        lens = np.empty(s.shape[0], np.int32)
        _lib.check(self._lib.clove_blocks_export(self.handle, s.ctypes.data, s.shape[0], stride,
                                                 tables.ctypes.data, lens.ctypes.data))
        return tables, lens
