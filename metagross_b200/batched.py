"""Batched, device-resident paged KV cache and decode attention.

This is the fast path behind the reference's per-sequence API: the same page
layout, scale layout, commit rule and allocator order as metagross/cache.py
and metagross/allocator.py, but for a batch of sequences and all layers, with
every piece of state in device memory and no host synchronisation per step.

State (per cache):
  k_pool, v_pool   [L, N, P, Hkv, D] int8  or [L, N, P, Hkv, D/2] uint8 (INT4)
  k_scales, v_scales [L, N] fp32, one scale per physical page (the
                   reference's layout), or with scale_granularity="token_head"
                   [L, N, P, Hkv]: one absmax scale per token and kv head
  staging_k/v      [L, B, P, Hkv, D] (fp16 or fp32): the page being filled,
                   exact, never quantized
  block_tables     [B, max_blocks] int32, shared by all layers (every layer
                   commits at the same token counts, so one table serves all)
  seq_lens         [B] int32 tokens cached per sequence
  allocator        DeviceBlockAllocator (LIFO, reference order)
  status           [1] int32 error bits set by kernels (see MG_DEV_* in
                   include/metagross_b200.h); ``check()`` reads it

A decode/prefill step is:
  cache.begin_step(n_new)              # allocate committing pages (once)
  for layer: cache.append(layer, k, v) # quantize filled pages, stage the rest
             out = cache.attend(layer, q)

The first ``attend`` after the lengths or block tables change (begin_step,
truncate, free, reset) builds the step's decode plan -- the split of the
batch's pages over the SMs, with a copy of each CTA's first page ids -- and
the other layers reuse it.  Code that writes ``seq_lens`` or
``block_tables`` directly must call ``invalidate_plan()``.
"""
from __future__ import annotations

import math

import torch

from .allocator import DeviceBlockAllocator

MG_DEV_BITS = {
    0x1: "out of pages",
    0x2: "block-table id out of range",
    0x4: "double free",
    0x8: "bulk-copy wait timed out",
    0x10: "block-table row full",
    0x20: "work skipped after an earlier error",
    0x40: "sequence longer than max_context",
    0x80: "inconsistent per-sequence argument",
    0x100: "negative length or token count",
}


def _get_C():
    from . import _C

    return _C


class BatchedPagedKVCache:
    def __init__(self, num_layers, batch, num_kv_heads, head_dim, page_size=16, num_pages=None, max_blocks=None,
                 kv_dtype="int8", staging_dtype=torch.float16, device="cuda", scale_granularity="page"):
        if kv_dtype not in ("int8", "int4"):
            raise ValueError(f"kv_dtype must be 'int8' or 'int4', got {kv_dtype!r}")
        if scale_granularity not in ("page", "token_head"):
            raise ValueError(f"scale_granularity must be 'page' or 'token_head', got {scale_granularity!r}")
        if scale_granularity == "token_head" and (head_dim > 256 or head_dim & (head_dim - 1)):
            raise ValueError("token_head scales need head_dim a power of two <= 256")
        for name, v in (("num_layers", num_layers), ("batch", batch), ("num_kv_heads", num_kv_heads),
                        ("head_dim", head_dim), ("page_size", page_size)):
            if v <= 0:
                raise ValueError(f"{name} must be positive, got {v}")
        if kv_dtype == "int4" and head_dim % 32:
            raise ValueError("INT4 pools need head_dim % 32 == 0")
        if staging_dtype not in (torch.float16, torch.float32):
            raise ValueError("staging_dtype must be torch.float16 or torch.float32")
        self.num_layers, self.batch = num_layers, batch
        self.num_kv_heads, self.head_dim, self.page_size = num_kv_heads, head_dim, page_size
        self.kv_dtype = kv_dtype
        self.scale_granularity = scale_granularity
        self.staging_dtype = staging_dtype
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.max_blocks = int(max_blocks) if max_blocks else 64
        self.num_pages = int(num_pages) if num_pages else batch * self.max_blocks
        row = head_dim if kv_dtype == "int8" else head_dim // 2
        dt = torch.int8 if kv_dtype == "int8" else torch.uint8
        shape = (num_layers, self.num_pages, page_size, num_kv_heads, row)
        self.k_pool = torch.zeros(shape, dtype=dt, device=self.device)
        self.v_pool = torch.zeros(shape, dtype=dt, device=self.device)
        sshape = (num_layers, self.num_pages) + ((page_size, num_kv_heads) if scale_granularity == "token_head" else ())
        self.k_scales = torch.zeros(sshape, dtype=torch.float32, device=self.device)
        self.v_scales = torch.zeros_like(self.k_scales)
        st = (num_layers, batch, page_size, num_kv_heads, head_dim)
        self.staging_k = torch.zeros(st, dtype=staging_dtype, device=self.device)
        self.staging_v = torch.zeros(st, dtype=staging_dtype, device=self.device)
        self.block_tables = torch.zeros(batch, self.max_blocks, dtype=torch.int32, device=self.device)
        self.seq_lens = torch.zeros(batch, dtype=torch.int32, device=self.device)
        self.n_new = torch.zeros(batch, dtype=torch.int32, device=self.device)
        self._n_new_val = 0  # the one value every entry of n_new holds, or None
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.allocator = DeviceBlockAllocator(self.num_pages, self.device)
        self._max_len = 0  # host-side upper bound on seq_lens
        self._ws = torch.zeros(0, dtype=torch.uint8, device=self.device)
        self._ws_key = None
        self._plan = None
        self._plan_ok = False
        self._plan_last = False  # the plan kernel is the cache's latest launch (nothing after it yet)

    # ------------------------------------------------------------------ steps
    def begin_step(self, n_new, plan: bool = False) -> None:
        """Grow every sequence by n_new tokens (int or int32 tensor [B]); allocate the pages that fill.
        plan=True also builds the step's decode plan, in the same launch (mg_plan_step): call it so
        before the step's first append, and every attention launch of the step reads its plan early."""
        C = _get_C()
        if isinstance(n_new, int):
            if n_new < 0:
                raise ValueError("n_new must be >= 0")
            self._ensure_n_new(n_new)
            self._max_len += n_new
        else:
            t = torch.as_tensor(n_new, dtype=torch.int32)
            if t.device.type == "cpu":
                self._max_len += int(t.max()) if t.numel() else 0
            else:
                self._max_len = self.max_blocks * self.page_size + self.page_size - 1
            self.n_new.copy_(t.to(self.device), non_blocking=True)
            self._n_new_val = None
        self._max_len = min(self._max_len, self.max_blocks * self.page_size + self.page_size - 1)
        if plan:
            if self._plan is None:
                self._plan = torch.zeros(C.decode_plan_bytes(self.batch), dtype=torch.uint8, device=self.device)
            C.plan_step(self.allocator.free_stack, self.allocator.n_free, self.allocator.in_use, self.k_pool[0],
                        self.block_tables, self.seq_lens, self.n_new, True, self._plan, self.status)
            self._plan_ok = True
            self._plan_last = True
            return
        self._plan_ok = False
        C.plan_append(self.allocator.free_stack, self.allocator.n_free, self.allocator.in_use, self.block_tables,
                      self.seq_lens, self.n_new, self.page_size, self.status)
        self._plan_last = False

    def _ensure_n_new(self, n: int) -> None:
        """Every entry of the device n_new equal to n; no launch when it already is (a
        decode graph then replays without the fill)."""
        if self._n_new_val != n:
            self.n_new.fill_(n)
            self._n_new_val = n

    def append(self, layer: int, k_new: torch.Tensor, v_new: torch.Tensor, early_launch: bool = False) -> None:
        """Write this step's tokens of one layer: k_new/v_new [B, T, Hkv, D] (fp16/fp32), n_new[b] <= T used.
        early_launch: a programmatic dependent launch (MG_APPEND_EARLY_LAUNCH) -- for an append that follows
        this library's own kernels (the previous layer's attention, the step plan), not a GEMM."""
        if k_new.dim() == 3:
            k_new, v_new = k_new.unsqueeze(1), v_new.unsqueeze(1)
        _get_C().kv_append(self.k_pool[layer], self.v_pool[layer], self.k_scales[layer], self.v_scales[layer],
                           self.staging_k[layer], self.staging_v[layer], self.block_tables, self.seq_lens,
                           self.n_new, k_new, v_new, self.status, early_launch=early_launch)
        self._plan_last = False

    def append_rope(self, layer: int, qkv: torch.Tensor, num_q_heads: int, cos: torch.Tensor, sin: torch.Tensor,
                    q_out: torch.Tensor) -> None:
        """``append`` for a step whose tokens come straight from a fused q|k|v
        projection, qkv fp16 [B, T, (num_q_heads + 2 Hkv) * D]: K is rotated
        (rotate-half, at each token's position = cached length before it) as it
        is written, V as it is, and the rotated q goes to q_out (B * T *
        num_q_heads * D fp16 elements) -- one launch (mg_kv_append_rope).
        cos / sin: fp32 [positions, D / 2]."""
        if qkv.dim() == 2:
            qkv = qkv.unsqueeze(1)
        _get_C().kv_append_rope(self.k_pool[layer], self.v_pool[layer], self.k_scales[layer], self.v_scales[layer],
                                self.staging_k[layer], self.staging_v[layer], self.block_tables, self.seq_lens,
                                self.n_new, qkv, num_q_heads, cos, sin, q_out, self.status)
        self._plan_last = False

    def invalidate_plan(self) -> None:
        """Mark the decode plan stale (after writing seq_lens or block_tables directly)."""
        self._plan_ok = False

    def prepare_plan(self) -> None:
        """Build the step's decode plan now if the lengths changed since the last
        one (right after ``begin_step``, before the step's first append): the
        attention launches that follow a launch other than the plan's then read
        it, and warm L2 with their first pages, before they wait for that launch
        (MG_ATTN_PLAN_SETTLED)."""
        self._decode_plan()

    def _decode_plan(self) -> torch.Tensor:
        """The step's decode plan, rebuilt on the device when the lengths changed."""
        C = _get_C()
        if self._plan is None:
            self._plan = torch.zeros(C.decode_plan_bytes(self.batch), dtype=torch.uint8, device=self.device)
        if not self._plan_ok:
            C.decode_plan(self.k_pool[0], self.block_tables, self.seq_lens, True, self._plan, self.status)
            self._plan_ok = True
            self._plan_last = True
        return self._plan

    def _workspace(self, num_q_heads: int, max_context: int) -> torch.Tensor:
        key = (num_q_heads, max_context)
        if key != self._ws_key:
            nbytes = _get_C().decode_workspace_bytes(self.k_pool[0], self.block_tables, num_q_heads, max_context)
            if nbytes > self._ws.numel():
                self._ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._ws_key = key
        return self._ws

    def attend(self, layer: int, q: torch.Tensor, scale: float | None = None, out: torch.Tensor | None = None,
               max_context: int | None = None) -> torch.Tensor:
        """softmax(scale q K^T) V over committed pages + staged tail; q [B, Hq, D] fp16/fp32."""
        if q.dim() != 3 or q.shape[0] != self.batch or q.shape[2] != self.head_dim:
            raise ValueError(f"q must be [{self.batch}, num_q_heads, {self.head_dim}], got {tuple(q.shape)}")
        hq = q.shape[1]
        if hq % self.num_kv_heads:
            raise ValueError(f"num_q_heads={hq} must be divisible by num_kv_heads={self.num_kv_heads}")
        sc = 1.0 / math.sqrt(self.head_dim) if scale is None else float(scale)
        if not (sc > 0 and math.isfinite(sc)):
            raise ValueError(f"scale must be a positive finite number, got {scale}")
        mc = int(max_context) if max_context else max(self._max_len, 1)
        ws = self._workspace(hq, mc)
        if out is None:
            out = torch.empty_like(q)
        plan = self._decode_plan()
        # settled: the plan kernel is not the launch right before this one (an
        # append or another attention of the cache came in between)
        _get_C().paged_decode_attention_planned(q.contiguous(), self.k_pool[layer], self.v_pool[layer],
                                                self.k_scales[layer], self.v_scales[layer], self.staging_k[layer],
                                                self.staging_v[layer], self.block_tables, plan, sc, ws, out,
                                                self.status, settled=not self._plan_last)
        self._plan_last = False
        return out

    def gather(self, layer: int, dtype=torch.float32, include_staging: bool = True):
        """Dequantized K, V of every sequence, packed: ([total, Hkv, D], [total, Hkv, D], cu_seqlens [B+1])."""
        lens = self.seq_lens.to("cpu")
        if not include_staging:
            lens = (lens // self.page_size) * self.page_size
        cu = torch.zeros(self.batch + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(lens, 0)
        total = int(cu[-1])
        ok = torch.empty(total, self.num_kv_heads, self.head_dim, dtype=dtype, device=self.device)
        ov = torch.empty_like(ok)
        mc = max(int(lens.max()) if lens.numel() else 0, 1)
        _get_C().gather_dequant(self.k_pool[layer], self.v_pool[layer], self.k_scales[layer], self.v_scales[layer],
                                self.staging_k[layer] if include_staging else None,
                                self.staging_v[layer] if include_staging else None, self.block_tables,
                                self.seq_lens, cu.to(self.device), mc, ok, ov, self.status)
        return ok, ov, cu

    def free(self, seq_ids) -> None:
        """Return every page of the given sequences to the pool and reset them to length 0."""
        ids = torch.as_tensor(seq_ids, dtype=torch.int32).to(self.device)
        self._plan_ok = False
        _get_C().free_sequences(self.allocator.free_stack, self.allocator.n_free, self.allocator.in_use,
                                self.block_tables, self.seq_lens, ids, self.page_size, self.status)

    def truncate(self, new_lens, seq_ids=None) -> None:
        """Shrink sequences to new_lens (int or per-sequence), freeing whole trailing pages.

        A new length may not cut a committed page (multiple of page_size, or within
        the staged tail); pages go back to the allocator in block-table order."""
        if seq_ids is None:
            seq_ids = torch.arange(self.batch, dtype=torch.int32)
        ids = torch.as_tensor(seq_ids, dtype=torch.int32)
        if isinstance(new_lens, int):
            nl = torch.full((ids.numel(),), new_lens, dtype=torch.int32)
        else:
            nl = torch.as_tensor(new_lens, dtype=torch.int32)
        self._plan_ok = False
        _get_C().truncate_sequences(self.allocator.free_stack, self.allocator.n_free, self.allocator.in_use,
                                    self.block_tables, self.seq_lens, ids.to(self.device), nl.to(self.device),
                                    self.page_size, self.status)

    def reset(self) -> None:
        self.allocator.reset()
        self.seq_lens.zero_()
        self.block_tables.zero_()
        self.status.zero_()
        self._max_len = 0
        self._plan_ok = False

    # ------------------------------------------------------------- inspection
    def check(self) -> None:
        """Raise RuntimeError if a kernel reported an error (synchronises)."""
        s = int(self.status.item())
        if s:
            names = [v for k, v in MG_DEV_BITS.items() if s & k]
            raise RuntimeError(f"paged KV cache device error 0x{s:x}: {', '.join(names)}")

    def memory_bytes(self) -> int:
        """Bytes of the quantized pools (codes only, as the reference's LayerKVCache.memory_bytes)."""
        return self.k_pool.numel() + self.v_pool.numel()


class DecodeGraph:
    """One decode step over every layer of ``cache`` captured as a CUDA graph:
    begin_step(n_new, plan=True) (page allocation and the step's decode plan in
    one launch, before the first append, so that every attention launch reads
    its plan early), then per layer
    append(k_new[l], v_new[l]) and attend(q[l]) -> out[l], all on the fixed
    device buffers given here.  ``replay()`` runs a step with one launch from
    the host, so the step is bound by the GPU, not by per-kernel launch cost.
    Refill q / k_new / v_new in place between replays; truncate / free stay
    eager calls on the cache (they take a different set of sequences each time).

    q [L, B, Hq, D], k_new / v_new [L, B, T, Hkv, D] (or [L, B, Hkv, D] for
    T = 1), out [L, B, Hq, D]."""

    def __init__(self, cache: BatchedPagedKVCache, q, k_new, v_new, out, n_new=1, scale=None):
        if not isinstance(n_new, int) or n_new < 0:
            raise ValueError("n_new must be a non-negative int")
        L = cache.num_layers
        for name, t in (("q", q), ("k_new", k_new), ("v_new", v_new), ("out", out)):
            if t.device != cache.device or t.shape[0] != L:
                raise ValueError(f"{name} must be a [{L}, ...] tensor on {cache.device}")
        self.cache, self.q, self.k_new, self.v_new, self.out = cache, q, k_new, v_new, out
        self.n_new, self.scale = n_new, scale
        # buffers the step reuses must exist before capture; n_new is filled
        # outside the graph (replay() refills it if an eager step changed it)
        cache._workspace(q.shape[2], cache.max_blocks * cache.page_size)
        cache._decode_plan()
        cache._ensure_n_new(n_new)
        stream = torch.cuda.Stream(cache.device)
        stream.wait_stream(torch.cuda.current_stream(cache.device))
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(self.graph, stream=stream):
                self._step()
        torch.cuda.current_stream(cache.device).wait_stream(stream)
        cache._plan_ok = False  # the capture ran nothing; the plan buffer holds the eager plan

    def _step(self):
        c = self.cache
        c.begin_step(self.n_new, plan=True)
        for layer in range(c.num_layers):
            # every append follows one of the library's kernels (the plan step, the previous attention)
            c.append(layer, self.k_new[layer], self.v_new[layer], early_launch=True)
            c.attend(layer, self.q[layer], scale=self.scale, out=self.out[layer],
                     max_context=c.max_blocks * c.page_size)

    def replay(self) -> None:
        self.cache._ensure_n_new(self.n_new)
        self.graph.replay()
        self.cache._max_len = min(self.cache._max_len + self.n_new,
                                  self.cache.max_blocks * self.cache.page_size + self.cache.page_size - 1)
        self.cache._plan_ok = False  # lengths moved on the device


def paged_decode_attention(cache: BatchedPagedKVCache, layer: int, q: torch.Tensor, scale=None, out=None):
    """Functional form of ``BatchedPagedKVCache.attend``."""
    return cache.attend(layer, q, scale=scale, out=out)
