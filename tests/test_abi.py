"""CPU tests of the C-ABI library: it loads, exports every symbol the header
declares, and its no-compute entry points behave without a GPU."""
import ctypes as C
import re
from pathlib import Path

import pytest

from conftest import ROOT, cuda_ok


def _declared(header: Path) -> set[str]:
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(clove_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    from clove_b200 import _lib
    if not _lib.LIB_PATH.exists():
        from clove_b200 import build
        build.build()
    return _lib.load()


def test_exports_every_declared_symbol(lib):
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= _declared(h)
    assert names, "no declarations found"
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_header():
    from clove_b200 import _lib
    declared = _declared(ROOT / "include" / "clove_cuda.h")
    assert declared == set(_lib.SIGNATURES), declared ^ set(_lib.SIGNATURES)


def test_ffi_bindings_cover_header():
    from clove_b200 import _lib
    declared = _declared(ROOT / "include" / "clove_ffi.h")
    assert declared == set(_lib.FFI_SIGNATURES), declared ^ set(_lib.FFI_SIGNATURES)


def test_blocks_bindings_cover_header():
    from clove_b200 import _lib
    declared = _declared(ROOT / "include" / "clove_blocks.h")
    assert declared == set(_lib.BLOCKS_SIGNATURES), declared ^ set(_lib.BLOCKS_SIGNATURES)


def test_ffi_null_handles(lib):
    assert lib.clove_tensor_create(None, 2, 2) is None
    assert lib.clove_paged_attention(None, None, None, None, None, None) is None
    lib.clove_tensor_free(None)
    lib.clove_tensor_data(None, None)
    assert lib.clove_tensor_shape(None, None) == -1


def test_last_error_and_variant(lib):
    assert lib.clove_cuda_set_decode_variant(7) == -1
    buf = C.create_string_buffer(256)
    assert lib.clove_cuda_get_last_error(buf, 256) == 0
    assert b"set_decode_variant" in buf.value
    assert lib.clove_cuda_set_decode_variant(0) == 0
    assert lib.clove_cuda_get_last_error(None, 0) == -1


def test_null_arguments_rejected(lib):
    assert lib.clove_cuda_pool_destroy(None) == 0
    assert lib.clove_cuda_pool_info(None, None) == -1
    assert lib.clove_cuda_decode_workspace_size(None, 1, 1, 1) == 0
    assert lib.clove_cuda_paged_decode(None, None, 1, None, 1, None, 1, 1.0, 1, None, None, 0, None) == -1
    assert lib.clove_cuda_reshape_and_cache(None, None, None, None, 1, None) == -1
    assert lib.clove_cuda_decode_status(None, None, None) == -1


@pytest.mark.skipif(cuda_ok(), reason="checks the no-device path")
def test_no_device_reported(lib):
    n = C.c_int(-1)
    assert lib.clove_cuda_init(C.byref(n)) == -7
    assert n.value == 0
    h = C.c_void_p()
    assert lib.clove_cuda_pool_create(0, 16, 16, 1, 64, 0, C.byref(h)) == -7


def test_package_fails_loudly_without_library(tmp_path):
    from clove_b200 import _lib
    with pytest.raises(ImportError):
        _lib.load(tmp_path / "missing.so")


def test_sharding_rules():
    from clove_b200 import distribute_batch, head_shards, token_balanced_shards
    assert distribute_batch(10, 4) == [3, 3, 2, 2]
    assert distribute_batch(5, 0) == [5]
    assert sum(distribute_batch(64, 8)) == 64
    sh = token_balanced_shards([100, 1, 50, 50, 3], 2)
    assert sorted(int(i) for s in sh for i in s) == [0, 1, 2, 3, 4]
    loads = [sum([100, 1, 50, 50, 3][i] + 1 for i in s) for s in sh]
    assert max(loads) - min(loads) <= 52
    hs = head_shards(8, 8, 4)
    assert [list(k) for k, _ in hs] == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert list(hs[1][1]) == list(range(16, 32))
    with pytest.raises(ValueError):
        head_shards(8, 1, 3)


def test_workload_layouts_disjoint():
    import numpy as np

    from clove_b200.workload import CONFIGS, make_layout
    for name, spec in CONFIGS.items():
        lay = make_layout(spec)
        bs = spec.block_size
        need = (lay.context_lens.astype(np.int64) + 1 + bs - 1) // bs
        ids = np.concatenate([lay.block_tables[b, :need[b]] for b in range(lay.batch)])
        assert len(np.unique(ids)) == ids.size, name
        assert ids.min() >= 0 and ids.max() < lay.num_blocks, name
        assert lay.block_tables.shape[1] == need.max()
        assert lay.context_lens.min() >= spec.ctx_lo and lay.context_lens.max() <= spec.ctx_hi, name
    c2 = make_layout(CONFIGS["c2"])
    assert c2.block_tables.shape == (64, 129) and (c2.context_lens == 2048).all()
    assert c2.kv_bytes() == 64 * 2049 * 2 * 32 * 128 * 4


def test_rust_binding_declares_every_entry_point():
    # rust/src/cuda_ffi.rs (the crate's extern "C" block) names exactly the
    # functions include/clove_cuda.h declares
    from clove_b200 import _lib
    text = (ROOT / "rust" / "src" / "cuda_ffi.rs").read_text()
    assert set(re.findall(r"pub fn (clove_\w+)", text)) == set(_lib.SIGNATURES)
