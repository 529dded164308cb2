"""B200-native PagedAttention decode (+ slot-mapping KV append) behind the
reference's Backend::paged_attention / PagedAttention / clove_paged_attention
interface.  The compute lives in libclove_cuda.so (CUDA, sm_100a); importing
the ops without it raises — there is no CPU fallback."""
from .sharding import distribute_batch, head_shards, token_balanced_shards  # noqa: F401

__all__ = ["distribute_batch", "head_shards", "token_balanced_shards"]


def __getattr__(name):
    # Lazy: the torch/ctypes layer loads the CUDA library on first use.
    if name in ("KVPool", "set_decode_variant", "launch_count"):
        from . import ops
        return getattr(ops, name)
    if name in ("CudaBackend", "PagedAttention"):
        from . import backend
        return getattr(backend, name)
    raise AttributeError(name)
