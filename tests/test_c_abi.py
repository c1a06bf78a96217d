"""CPU checks of the drop-in boundary: the C-ABI library loads, exports every
entry point include/metagross_b200.h declares, rejects bad arguments before
touching the device, and the ``_C`` module exposes the reference's op names
(csrc/bindings.cpp:4-18) plus the batched ops.  No kernel runs here."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "metagross_b200.h")
LIB = os.path.join(ROOT, "metagross_b200", "libmgb200.so")

REFERENCE_OPS = ["add", "quantize_new_scale", "quantize_fixed_scale", "dequantize_page", "paged_attention_committed",
                 "quantize_int4_new_scale", "dequantize_int4_page"]
BATCHED_OPS = ["alloc_init", "plan_append", "free_sequences", "truncate_sequences", "kv_append", "decode_workspace_bytes",
               "paged_decode_attention", "gather_dequant"]


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^MG_API\s+[\w\s\*]+?\b(mg_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ["mg_quantize_int8_new_scale", "mg_quantize_int8_fixed_scale", "mg_dequantize_int8_page",
              "mg_quantize_int4_new_scale", "mg_dequantize_int4_page", "mg_paged_attention_committed",
              "mg_add_f32", "mg_plan_append", "mg_kv_append", "mg_paged_decode_attention", "mg_gather_dequant",
              "mg_alloc_init", "mg_free_sequences", "mg_truncate_sequences"]:
        assert s in syms, s


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_version_and_error_text():
    lib = ctypes.CDLL(LIB)
    lib.mg_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.mg_version()
    lib.mg_last_error.restype = ctypes.c_char_p
    f = lib.mg_quantize_int8_fixed_scale
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                  ctypes.c_double, ctypes.c_void_p]
    f.restype = ctypes.c_int
    # invalid scale, negative offset, overflow: rejected before any CUDA call
    assert f(None, 4, 8, None, 16, 0, -1.0, None) == 1
    assert b"scale" in lib.mg_last_error()
    assert f(None, 4, 8, None, 16, -1, 0.5, None) == 1
    assert b"token_offset" in lib.mg_last_error()
    assert f(None, 20, 8, None, 16, 0, 0.5, None) == 1
    assert b"overflow" in lib.mg_last_error()


def test_int4_rejects_odd_head_dim_before_launch():
    lib = ctypes.CDLL(LIB)
    f = lib.mg_quantize_int4_new_scale
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    assert f(None, 4, 2, 5, None, 16, 0, None, None) == 1
    assert f(None, 4, 2, 0, None, 16, 0, None, None) == 1


def test_extension_module_surface():
    from metagross_b200 import _C

    for name in REFERENCE_OPS + BATCHED_OPS:
        assert callable(getattr(_C, name)), name
    assert "sm_100a" in _C.version()


def test_extension_links_the_c_abi_library():
    import metagross_b200._C as C

    maps = open("/proc/self/maps").read()
    assert "libmgb200.so" in maps, "the _C extension must load the in-tree C-ABI library"
    assert C.__file__.startswith(os.path.join(ROOT, "metagross_b200"))


@pytest.mark.parametrize("op", ["quantize_new_scale", "dequantize_page"])
def test_extension_rejects_cpu_tensors(op):
    import torch
    from metagross_b200 import _C

    x = torch.zeros(4, 2, 8)
    page = torch.zeros(16, 2, 8, dtype=torch.int8)
    with pytest.raises(RuntimeError):
        if op == "quantize_new_scale":
            _C.quantize_new_scale(x, page, 0)
        else:
            _C.dequantize_page(page, 0, 4, 0.1)


class _Layout(ctypes.Structure):
    _fields_ = [("kv_dtype", ctypes.c_int32), ("staging_dtype", ctypes.c_int32), ("page_size", ctypes.c_int32),
                ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("max_blocks", ctypes.c_int32),
                ("num_pages", ctypes.c_int64), ("scale_layout", ctypes.c_int32), ("reserved", ctypes.c_int32)]


@pytest.mark.parametrize("hq,hkv", [(32, 2), (16, 1), (8, 1), (12, 12)])
def test_workspace_size_covers_every_supported_group(hq, hkv):
    """Groups of 9-16 q heads per kv head run with fp16 queries only; the
    workspace size (independent of the query dtype) must still be given."""
    lib = ctypes.CDLL(LIB)
    lib.mg_paged_decode_workspace_bytes.restype = ctypes.c_int64
    lib.mg_last_error.restype = ctypes.c_char_p
    L = _Layout(1, 1, 16, hkv, 64, 64, 4096)
    n = lib.mg_paged_decode_workspace_bytes(ctypes.byref(L), 8, hq, 1024)
    assert n > 0, lib.mg_last_error()


def test_workspace_size_rejects_an_unsupported_group():
    lib = ctypes.CDLL(LIB)
    lib.mg_paged_decode_workspace_bytes.restype = ctypes.c_int64
    lib.mg_last_error.restype = ctypes.c_char_p
    L = _Layout(0, 1, 16, 1, 64, 64, 4096)
    assert lib.mg_paged_decode_workspace_bytes(ctypes.byref(L), 8, 17, 1024) == 0
    assert b"GQA group 17" in lib.mg_last_error()


def test_append_rejects_more_pages_than_one_launch_covers():
    lib = ctypes.CDLL(LIB)
    lib.mg_last_error.restype = ctypes.c_char_p

    class _Ptrs(ctypes.Structure):
        _fields_ = [(n, ctypes.c_void_p) for n in ("k_pool", "v_pool", "k_scales", "v_scales", "staging_k",
                                                    "staging_v")]

    L = _Layout(0, 1, 16, 4, 64, 70000, 1 << 20)
    ptrs = _Ptrs(*([1 << 20] * 6))  # never dereferenced: refused before launch
    f = lib.mg_kv_append
    f.restype = ctypes.c_int
    rc = f(ctypes.byref(L), ctypes.byref(ptrs), ctypes.c_void_p(1 << 20), ctypes.c_void_p(1 << 20),
           ctypes.c_void_p(1 << 20), 1, ctypes.c_void_p(1 << 20), ctypes.c_void_p(1 << 20), 1, 16 * 65535,
           None, None)
    assert rc == 1
    assert b"65534 pages" in lib.mg_last_error()


def test_planned_attention_rejects_unknown_flags_before_launch():
    lib = ctypes.CDLL(LIB)
    lib.mg_last_error.restype = ctypes.c_char_p
    f = lib.mg_paged_decode_attention_planned_flags
    f.restype = ctypes.c_int
    L = _Layout(0, 1, 16, 4, 64, 64, 1024)
    p = ctypes.c_void_p(1 << 20)  # never dereferenced: refused before launch
    rc = f(ctypes.byref(L), p, p, p, ctypes.c_int64(1 << 20), 1, p, 1, 32, ctypes.c_float(0.125), p, 1, p,
           ctypes.c_int64(1 << 20), ctypes.c_uint32(0x2), None, None)
    assert rc == 1
    assert b"unknown attention flags" in lib.mg_last_error()


def test_append_rejects_unknown_flags_before_launch():
    lib = ctypes.CDLL(LIB)
    lib.mg_last_error.restype = ctypes.c_char_p
    f = lib.mg_kv_append_flags
    f.restype = ctypes.c_int
    L = _Layout(0, 1, 16, 4, 64, 64, 1024)
    p = ctypes.c_void_p(1 << 20)  # never dereferenced: refused before launch
    rc = f(ctypes.byref(L), p, p, p, p, 1, p, p, 1, 1, ctypes.c_uint32(0x4), None, None)
    assert rc == 1
    assert b"unknown append flags" in lib.mg_last_error()
