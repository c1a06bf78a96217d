"""CPU oracle for the paged quantized KV-cache + decode-attention path.

TEST INFRASTRUCTURE ONLY -- this module is the checker, never the thing
measured or shipped.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import it.  The product package
(``metagross_b200``) never imports anything under ``oracle/``.

Layers:
  * byte/integer arithmetic (quantize, dequantize, INT4 packing, allocator
    replay) lives in plain C (``mg_oracle.c``) and is loaded with ctypes; those
    functions are bit-exact restatements of the reference's CUDA ops
    (csrc/quantize.cu, csrc/quantize_int4.cu, csrc/dequantize*.cu) and of
    metagross/allocator.py;
  * attention is float64 numpy "dequantize, then attend", the reference's own
    oracle path (tests/test_attention.py:14-20 ``_reference_full_attention``
    over ``LayerKVCache.read_fp32``, metagross/cache.py:74-85), with GQA head
    expansion as metagross/attention.py:53-59 (kv head h serves q heads
    h*G .. h*G+G-1);
  * ``PagedCacheModel`` replays the cache semantics of metagross/cache.py:45-72
    (stage tokens, commit a page with one fresh absmax scale when it fills,
    allocate ids LIFO) for a batch of sequences sharing one page pool: the
    batch is processed in sequence order, so page ids equal the ones a single
    reference BlockAllocator hands out for the same sequence of commits.

Pinned by tests/test_oracle_golden.py against fixtures generated from the
reference's own Python (tests/golden/make_golden.py) and against the
reference's known-answer tests.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmgoracle.so")
_SRC = os.path.join(HERE, "mg_oracle.c")

_lib = None


def build_oracle_lib(force: bool = False) -> str:
    """Compile mg_oracle.c with gcc (IEEE division, no FMA contraction)."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(_SRC):
        subprocess.check_call([
            "gcc", "-O2", "-fno-fast-math", "-ffp-contract=off", "-fPIC", "-shared",
            "-o", LIB_PATH, _SRC, "-lm",
        ])
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) and os.path.exists(_SRC):
            build_oracle_lib()
        L = ctypes.CDLL(LIB_PATH)
        f32p = ctypes.POINTER(ctypes.c_float)
        i64 = ctypes.c_int64
        L.mgo_absmax.argtypes = [f32p, i64]
        L.mgo_absmax.restype = ctypes.c_float
        L.mgo_scale_from_absmax.argtypes = [ctypes.c_float, ctypes.c_double]
        L.mgo_scale_from_absmax.restype = ctypes.c_double
        L.mgo_quantize_int8.argtypes = [f32p, i64, i64, ctypes.c_void_p, i64, ctypes.c_int, ctypes.c_double]
        L.mgo_quantize_int8.restype = ctypes.c_double
        L.mgo_dequantize_int8.argtypes = [ctypes.c_void_p, i64, i64, i64, ctypes.c_double, f32p]
        L.mgo_dequantize_int8.restype = None
        L.mgo_quantize_int4.argtypes = [f32p, i64, i64, i64, ctypes.c_void_p, i64, ctypes.c_int, ctypes.c_double]
        L.mgo_quantize_int4.restype = ctypes.c_double
        L.mgo_dequantize_int4.argtypes = [ctypes.c_void_p, i64, i64, i64, ctypes.c_double, f32p]
        L.mgo_dequantize_int4.restype = None
        L.mgo_allocator_replay.argtypes = [ctypes.c_void_p, i64, i64, ctypes.c_void_p, i64, ctypes.c_void_p]
        L.mgo_allocator_replay.restype = i64
        _lib = L
    return _lib


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _fp(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


# --------------------------------------------------------------------------
# byte / integer arithmetic (C)
# --------------------------------------------------------------------------

def absmax(x) -> float:
    x = _f32(x)
    return float(lib().mgo_absmax(_fp(x), x.size))


def scale_from_absmax(a: float, qmax: float) -> float:
    return float(lib().mgo_scale_from_absmax(ctypes.c_float(a), qmax))


def quantize_int8(x, page: np.ndarray | None = None, offset: int = 0, scale: float | None = None):
    """Quantize fp32 ``x[T,H,D]`` into ``page[P,H,D]`` (int8) at ``offset``.

    ``scale=None`` picks a fresh absmax scale (csrc/quantize.cu:65-120);
    otherwise the fixed scale is used (csrc/quantize.cu:122-167).
    Returns ``(page, scale_as_double)``.
    """
    x = _f32(x)
    if x.ndim != 3:
        raise ValueError("x must be [T,H,D]")
    T, H, D = x.shape
    if page is None:
        page = np.zeros((offset + T, H, D), dtype=np.int8)
    assert page.dtype == np.int8 and page.flags.c_contiguous
    assert offset + T <= page.shape[0]
    s = lib().mgo_quantize_int8(_fp(x), T, H * D, page.ctypes.data, offset,
                                1 if scale is None else 0, 0.0 if scale is None else float(scale))
    return page, float(s)


def dequantize_int8(page: np.ndarray, offset: int, num_tokens: int, scale: float) -> np.ndarray:
    page = np.ascontiguousarray(page, dtype=np.int8)
    P, H, D = page.shape
    out = np.empty((num_tokens, H, D), dtype=np.float32)
    lib().mgo_dequantize_int8(page.ctypes.data, offset, num_tokens, H * D, float(scale), _fp(out))
    return out


def quantize_int4(x, packed: np.ndarray | None = None, offset: int = 0, scale: float | None = None):
    """Packed INT4 quantize (csrc/quantize_int4.cu:33-125) into ``packed[P,H,D/2]``."""
    x = _f32(x)
    T, H, D = x.shape
    assert D % 2 == 0 and D > 0
    if packed is None:
        packed = np.zeros((offset + T, H, D // 2), dtype=np.uint8)
    assert packed.dtype == np.uint8 and packed.flags.c_contiguous
    s = lib().mgo_quantize_int4(_fp(x), T, H, D, packed.ctypes.data, offset,
                                1 if scale is None else 0, 0.0 if scale is None else float(scale))
    return packed, float(s)


def dequantize_int4(packed: np.ndarray, offset: int, num_tokens: int, scale: float) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    P, H, Dh = packed.shape
    out = np.empty((num_tokens, H, 2 * Dh), dtype=np.float32)
    lib().mgo_dequantize_int4(packed.ctypes.data, offset, num_tokens, H * Dh, float(scale), _fp(out))
    return out


def quantize_token_head(x, kv_dtype: str = "int8"):
    """One fresh absmax scale per (token, head) D-vector: the reference's
    ``quantize_new_scale`` / ``quantize_int4_new_scale`` (csrc/quantize.cu:65-120,
    csrc/quantize_int4.cu:67-125) applied to each ``[1, 1, D]`` slice of
    ``x[T, H, D]``.  The reference cache has only per-page scales
    (metagross/cache.py:39,69-70); this is the per-token-per-head layout of its
    CPU reference config, with the kernels' rounding.
    Returns ``(codes [T, H, D] int8 or [T, H, D/2] uint8, scales float64 [T, H])``."""
    x = _f32(x)
    T, H, D = x.shape
    int8 = kv_dtype == "int8"
    codes = np.zeros((T, H, D if int8 else D // 2), np.int8 if int8 else np.uint8)
    scales = np.zeros((T, H), np.float64)
    for t in range(T):
        for h in range(H):
            sl = x[t:t + 1, h:h + 1]
            c, sc = quantize_int8(sl) if int8 else quantize_int4(sl)
            codes[t, h] = c[0, 0]
            scales[t, h] = sc
    return codes, scales


def dequantize_token_head(codes: np.ndarray, scales: np.ndarray, kv_dtype: str = "int8") -> np.ndarray:
    """Inverse of ``quantize_token_head``: each [D] vector dequantized with its
    own scale as csrc/dequantize.cu:9-26 / csrc/dequantize_int4.cu:9-37 do."""
    T, H = codes.shape[:2]
    D = codes.shape[2] if kv_dtype == "int8" else 2 * codes.shape[2]
    out = np.empty((T, H, D), np.float32)
    for t in range(T):
        for h in range(H):
            sl = codes[t:t + 1, h:h + 1]
            out[t, h] = (dequantize_int8(sl, 0, 1, scales[t, h]) if kv_dtype == "int8"
                         else dequantize_int4(sl, 0, 1, scales[t, h]))[0, 0]
    return out


def allocator_replay(num_pages: int, ops, free_list: np.ndarray | None = None):
    """Replay allocate (-1) / free (id) ops; returns (results, free_list, n_free)."""
    if free_list is None:
        free_list = np.arange(num_pages, dtype=np.int32)
        n_free = num_pages
    else:
        n_free = len(free_list)
        free_list = np.concatenate([free_list.astype(np.int32), np.zeros(num_pages, np.int32)])[:num_pages].copy()
    ops = np.ascontiguousarray(np.asarray(ops, dtype=np.int32))
    out = np.zeros(len(ops), dtype=np.int32)
    n = lib().mgo_allocator_replay(free_list.ctypes.data, n_free, num_pages, ops.ctypes.data, len(ops),
                                   out.ctypes.data)
    return out, free_list[:n].copy(), int(n)


# --------------------------------------------------------------------------
# attention (float64 numpy): dequantize-then-attend
# --------------------------------------------------------------------------

def repeat_kv_heads(x: np.ndarray, n_rep: int) -> np.ndarray:
    """[C, Hkv, D] -> [C, Hkv*n_rep, D]; kv head h serves q heads h*n_rep.. (attention.py:53-59)."""
    if n_rep == 1:
        return x
    return np.repeat(x, n_rep, axis=1)


def attention_unnormalized(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float):
    """(wv[Hq,D], l[Hq], m[Hq]) with s = scale*q.k, m = max s, l = sum e^(s-m).

    Matches the outputs of csrc/paged_attention.cu:63-134; (0, 0, -inf) when
    there are no tokens.
    """
    q = np.asarray(q, dtype=np.float64)
    Hq, D = q.shape
    if k.shape[0] == 0:
        return np.zeros((Hq, D)), np.zeros(Hq), np.full(Hq, -np.inf)
    G = Hq // k.shape[1]
    kk = repeat_kv_heads(np.asarray(k, dtype=np.float64), G)
    vv = repeat_kv_heads(np.asarray(v, dtype=np.float64), G)
    s = np.einsum("thd,hd->ht", kk, q) * scale
    m = s.max(axis=1)
    p = np.exp(s - m[:, None])
    return np.einsum("ht,thd->hd", p, vv), p.sum(axis=1), m


def attention(q, k, v, scale: float) -> np.ndarray:
    wv, l, _ = attention_unnormalized(q, k, v, scale)
    return wv / l[:, None]


def merge_unnormalized(m1, l1, wv1, m2, l2, wv2):
    """LSE merge of two partial softmax states (attention.py:15-26)."""
    m = np.maximum(m1, m2)
    with np.errstate(invalid="ignore"):
        a = np.where(np.isneginf(m1), 0.0, np.exp(m1 - m))
        b = np.where(np.isneginf(m2), 0.0, np.exp(m2 - m))
    return wv1 * a[:, None] + wv2 * b[:, None], l1 * a + l2 * b, m


# --------------------------------------------------------------------------
# batched paged cache model (metagross/cache.py semantics, shared pool)
# --------------------------------------------------------------------------

class PagedCacheModel:
    """Replay of the reference cache semantics for B sequences on one pool.

    kv_dtype "int8": pools int8 [N, P, Hkv, D]; "int4": uint8 [N, P, Hkv, D/2].
    scale_granularity "page": one fp32 scale per physical page for K and one
    for V (metagross/cache.py:39,69-70); "token_head": one per (page, token,
    kv head), scales [N, P, Hkv] (``quantize_token_head``).  Staged tokens are
    kept exactly (metagross/cache.py:57-61) in ``staging_dtype``.
    """

    def __init__(self, batch, num_pages, page_size, num_kv_heads, head_dim,
                 kv_dtype="int8", staging_dtype=np.float32, max_blocks=None, scale_granularity="page"):
        self.B, self.N, self.P, self.H, self.D = batch, num_pages, page_size, num_kv_heads, head_dim
        self.kv_dtype = kv_dtype
        self.scale_granularity = scale_granularity
        row = head_dim if kv_dtype == "int8" else head_dim // 2
        dt = np.int8 if kv_dtype == "int8" else np.uint8
        self.k_pool = np.zeros((num_pages, page_size, num_kv_heads, row), dt)
        self.v_pool = np.zeros_like(self.k_pool)
        sshape = (num_pages,) + ((page_size, num_kv_heads) if scale_granularity == "token_head" else ())
        self.k_scales = np.zeros(sshape, np.float32)
        self.v_scales = np.zeros(sshape, np.float32)
        self.k_scales64 = np.zeros(sshape, np.float64)
        self.v_scales64 = np.zeros(sshape, np.float64)
        self.max_blocks = max_blocks if max_blocks is not None else num_pages
        self.block_tables = np.zeros((batch, self.max_blocks), np.int32)
        self.num_blocks = np.zeros(batch, np.int32)
        self.seq_lens = np.zeros(batch, np.int32)
        self.staging_dtype = staging_dtype
        self.staging_k = [[] for _ in range(batch)]
        self.staging_v = [[] for _ in range(batch)]
        self.free_list = list(range(num_pages))

    def _allocate(self) -> int:
        if not self.free_list:
            raise RuntimeError("out of pages")
        return self.free_list.pop()

    def free_sequence(self, b: int):
        """Return seq b's pages to the pool in block-table order and reset it."""
        for j in range(int(self.num_blocks[b])):
            self.free_list.append(int(self.block_tables[b, j]))
        self.num_blocks[b] = 0
        self.seq_lens[b] = 0
        self.staging_k[b] = []
        self.staging_v[b] = []

    def truncate(self, b: int, new_len: int):
        """Drop seq b's tokens beyond new_len (a page boundary, or inside the
        staged tail); freed pages return to the pool in block-table order."""
        old = int(self.seq_lens[b])
        committed = (old // self.P) * self.P
        assert 0 <= new_len <= old and (new_len % self.P == 0 or new_len >= committed)
        keep = new_len // self.P
        for j in range(keep, int(self.num_blocks[b])):
            self.free_list.append(int(self.block_tables[b, j]))
        if new_len < committed:
            self.staging_k[b] = []
            self.staging_v[b] = []
        else:
            r = new_len - committed
            self.staging_k[b] = self.staging_k[b][:r]
            self.staging_v[b] = self.staging_v[b][:r]
        self.num_blocks[b] = keep
        self.seq_lens[b] = new_len

    def _commit(self, b: int):
        m = self._allocate()
        j = int(self.num_blocks[b])
        self.block_tables[b, j] = m
        self.num_blocks[b] = j + 1
        kp = np.stack(self.staging_k[b]).astype(np.float32)
        vp = np.stack(self.staging_v[b]).astype(np.float32)
        if self.scale_granularity == "token_head":
            self.k_pool[m], sk = quantize_token_head(kp, self.kv_dtype)
            self.v_pool[m], sv = quantize_token_head(vp, self.kv_dtype)
        elif self.kv_dtype == "int8":
            self.k_pool[m], sk = quantize_int8(kp, np.zeros_like(self.k_pool[m]))
            self.v_pool[m], sv = quantize_int8(vp, np.zeros_like(self.v_pool[m]))
        else:
            self.k_pool[m], sk = quantize_int4(kp, np.zeros_like(self.k_pool[m]))
            self.v_pool[m], sv = quantize_int4(vp, np.zeros_like(self.v_pool[m]))
        self.k_scales64[m], self.v_scales64[m] = sk, sv
        self.k_scales[m], self.v_scales[m] = np.float32(sk), np.float32(sv)
        self.staging_k[b] = []
        self.staging_v[b] = []

    def append(self, k_new, v_new, n_new=None):
        """k_new/v_new: [B, T, Hkv, D]; n_new[b] <= T tokens of seq b are appended.

        Sequences are processed in index order; within a sequence tokens go
        one by one as metagross/cache.py:57-61 does.
        """
        k_new = np.asarray(k_new)
        v_new = np.asarray(v_new)
        B, T = k_new.shape[:2]
        if n_new is None:
            n_new = [T] * B
        for b in range(B):
            n = int(n_new[b])
            i = 0
            while i < n:
                r = len(self.staging_k[b])
                if r == 0 and n - i >= self.P:
                    # a whole page with nothing staged: the same commit as pushing
                    # its P tokens one by one (metagross/cache.py:57-61), in one go
                    self.staging_k[b] = list(k_new[b, i:i + self.P].astype(self.staging_dtype))
                    self.staging_v[b] = list(v_new[b, i:i + self.P].astype(self.staging_dtype))
                    self.seq_lens[b] += self.P
                    i += self.P
                    self._commit(b)
                    continue
                self.staging_k[b].append(k_new[b, i].astype(self.staging_dtype))
                self.staging_v[b].append(v_new[b, i].astype(self.staging_dtype))
                self.seq_lens[b] += 1
                i += 1
                if len(self.staging_k[b]) == self.P:
                    self._commit(b)

    def dequantized_sequence(self, b: int, which: str = "k") -> np.ndarray:
        """``read_fp32`` (metagross/cache.py:74-85): committed pages in block-table order + exact tail."""
        pool = self.k_pool if which == "k" else self.v_pool
        scales = self.k_scales64 if which == "k" else self.v_scales64
        parts = []
        for j in range(int(self.num_blocks[b])):
            m = int(self.block_tables[b, j])
            if self.scale_granularity == "token_head":
                parts.append(dequantize_token_head(pool[m], scales[m], self.kv_dtype))
            elif self.kv_dtype == "int8":
                parts.append(dequantize_int8(pool[m], 0, self.P, scales[m]))
            else:
                parts.append(dequantize_int4(pool[m], 0, self.P, scales[m]))
        st = self.staging_k[b] if which == "k" else self.staging_v[b]
        if st:
            parts.append(np.stack(st).astype(np.float32))
        if not parts:
            return np.zeros((0, self.H, self.D), np.float32)
        return np.concatenate(parts, axis=0)

    def attend(self, q, scale: float) -> np.ndarray:
        """Decode attention for every sequence: q [B, Hq, D] -> [B, Hq, D] (float64)."""
        q = np.asarray(q, dtype=np.float64)
        out = np.zeros(q.shape, np.float64)
        for b in range(self.B):
            k = self.dequantized_sequence(b, "k")
            v = self.dequantized_sequence(b, "v")
            if k.shape[0]:
                out[b] = attention(q[b], k, v, scale)
        return out
