"""metagross_b200 -- B200-native paged quantized KV-cache and decode attention.

Drop-in for the reference's Python surface:
  metagross_b200.allocator.BlockAllocator        (metagross/allocator.py)
  metagross_b200.cache.LayerKVCache/PagedKVCache (metagross/cache.py)
  metagross_b200.attention.paged_attention       (metagross/attention.py)
  metagross_b200._C                              (metagross._C, csrc/bindings.cpp)
plus the batched device-resident path (``BatchedPagedKVCache``,
``paged_decode_attention``).  All device work runs in libmgb200.so (sm_100a);
there is no CPU or pure-PyTorch fallback: if the native library is missing the
import of ``metagross_b200._C`` fails.
"""

__version__ = "0.1.0"


def sanity_add(a, b):
    """Elementwise add through the native library (the reference's build check, metagross/__init__.py:4-8)."""
    from . import _C

    return _C.add(a, b)


def __getattr__(name):
    # lazy re-exports, so importing the package never needs a GPU
    if name in ("BatchedPagedKVCache", "DecodeGraph", "paged_decode_attention"):
        from . import batched

        return getattr(batched, name)
    raise AttributeError(name)
