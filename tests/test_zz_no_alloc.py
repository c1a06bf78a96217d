"""mg_paged_decode_attention_noalloc (metagross_b200/csrc/mg_noalloc.cu): the
batched decode attention with its workspace in the library's static device
scratch.  Compared bit for bit with mg_paged_decode_attention (caller
workspace) on the same cache, two no-alloc calls in a row; and an oversized
request is refused before any launch.  Named to be collected last, after every
other test has used the library."""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "metagross_b200", "libmgb200.so")
MG_F32, MG_F16 = 0, 1


class Layout(ctypes.Structure):
    _fields_ = [("kv_dtype", ctypes.c_int32), ("staging_dtype", ctypes.c_int32), ("page_size", ctypes.c_int32),
                ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("max_blocks", ctypes.c_int32),
                ("num_pages", ctypes.c_int64), ("scale_layout", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class LayerPtrs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("k_pool", "v_pool", "k_scales", "v_scales", "staging_k", "staging_v")]


def _lib():
    import metagross_b200._C  # noqa: F401  (loads libmgb200.so; ctypes gets the same handle)

    lib = ctypes.CDLL(LIB)
    lib.mg_last_error.restype = ctypes.c_char_p
    lib.mg_paged_decode_workspace_bytes.restype = ctypes.c_int64
    return lib


def _filled_cache(kv, B, hkv, hq, seed):
    from metagross_b200.batched import BatchedPagedKVCache

    g = torch.Generator().manual_seed(seed)
    cache = BatchedPagedKVCache(1, B, hkv, 64, page_size=16, num_pages=B * 24, max_blocks=24, kv_dtype=kv,
                                device="cuda")
    lens = torch.randint(1, 300, (B,), generator=g, dtype=torch.int32)
    cache.begin_step(lens)
    T = int(lens.max())
    k = torch.randn(B, T, hkv, 64, generator=g).half().cuda()
    v = torch.randn(B, T, hkv, 64, generator=g).half().cuda()
    cache.append(0, k, v)
    q = torch.randn(B, hq, 64, generator=g).half().cuda()
    torch.cuda.synchronize()
    cache.check()
    return cache, q


def _args(cache):
    L = Layout(0 if cache.kv_dtype == "int8" else 1, MG_F16, cache.page_size, cache.num_kv_heads, cache.head_dim,
               cache.max_blocks, cache.num_pages)
    ptrs = LayerPtrs(cache.k_pool[0].data_ptr(), cache.v_pool[0].data_ptr(), cache.k_scales[0].data_ptr(),
                     cache.v_scales[0].data_ptr(), cache.staging_k[0].data_ptr(), cache.staging_v[0].data_ptr())
    return L, ptrs


@pytest.mark.parametrize("kv,B,hkv,hq", [("int8", 6, 12, 12), ("int4", 9, 4, 32), ("int4", 5, 2, 32)])
def test_noalloc_matches_workspace_entry_point(kv, B, hkv, hq):
    lib = _lib()
    cache, q = _filled_cache(kv, B, hkv, hq, seed=11 + B)
    L, ptrs = _args(cache)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    maxctx = cache.max_blocks * cache.page_size
    nbytes = lib.mg_paged_decode_workspace_bytes(ctypes.byref(L), B, hq, maxctx)
    assert nbytes > 0, lib.mg_last_error()
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")

    def with_workspace():
        out = torch.empty_like(q)
        rc = lib.mg_paged_decode_attention(
            ctypes.byref(L), ctypes.byref(ptrs), ctypes.c_void_p(cache.block_tables.data_ptr()),
            ctypes.c_void_p(cache.seq_lens.data_ptr()), B, ctypes.c_void_p(q.data_ptr()), MG_F16, hq,
            ctypes.c_float(1.0 / 8), ctypes.c_void_p(out.data_ptr()), MG_F16, maxctx,
            ctypes.c_void_p(ws.data_ptr()), ctypes.c_int64(nbytes), ctypes.c_void_p(status.data_ptr()), stream)
        assert rc == 0, lib.mg_last_error()
        return out

    def no_alloc():
        out = torch.empty_like(q)
        rc = lib.mg_paged_decode_attention_noalloc(
            ctypes.byref(L), ctypes.byref(ptrs), ctypes.c_void_p(cache.block_tables.data_ptr()),
            ctypes.c_void_p(cache.seq_lens.data_ptr()), B, ctypes.c_void_p(q.data_ptr()), MG_F16, hq,
            ctypes.c_float(1.0 / 8), ctypes.c_void_p(out.data_ptr()), MG_F16, maxctx,
            ctypes.c_void_p(status.data_ptr()), stream)
        assert rc == 0, lib.mg_last_error()
        return out

    ref = with_workspace()
    a = no_alloc()
    b = no_alloc()  # the second call in a row reuses the scratch the first one left
    ref2 = with_workspace()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.isfinite(ref.float()).all()
    assert torch.equal(a, ref)
    assert torch.equal(b, ref)
    assert torch.equal(ref2, ref)


def test_noalloc_refuses_a_workspace_larger_than_its_scratch():
    lib = _lib()
    # 8192 sequences x 64 q heads x head_dim 128: the split partials alone need ~10 MB > 4 MiB
    L = Layout(0, MG_F16, 16, 8, 128, 64, 8192 * 64)
    ptrs = LayerPtrs(1 << 20, 1 << 20, 1 << 20, 1 << 20, None, None)  # never dereferenced: refused first
    rc = lib.mg_paged_decode_attention_noalloc(
        ctypes.byref(L), ctypes.byref(ptrs), ctypes.c_void_p(1 << 20), ctypes.c_void_p(1 << 20), 8192,
        ctypes.c_void_p(1 << 20), MG_F32, 64, ctypes.c_float(0.1), ctypes.c_void_p(1 << 20), MG_F32, 1024, None,
        None)
    assert rc == 1
    assert b"static scratch" in lib.mg_last_error()
