"""Batched greedy decode of a Llama-architecture model on the paged cache.

The reference decodes TinyLlama one sequence at a time through Hugging Face's
model with its cache in Python (metagross/generate_llama.py:41-126, the
per-token append at :103-107 after the rotary embedding at :20-37).  Here a
batch decodes together.  The dense parts -- embedding, RMSNorm, the q/k/v/o
projections, the rotary embedding, the SwiGLU MLP and the lm_head -- are plain
torch fp16 ops (cuBLAS GEMMs); the cache side is this package's: every layer
appends its new K/V (quantized full pages, exact staged tail) and runs the
fused paged decode attention.  A decode step is captured in one CUDA graph.

Weights are random (seeded) unless given: the benchmarked quantity is the
decode throughput of the architecture, not its text.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .batched import BatchedPagedKVCache, _get_C


@dataclass(frozen=True)
class LlamaShape:
    vocab: int = 32000
    hidden: int = 2048
    layers: int = 22
    heads: int = 32
    kv_heads: int = 4
    ffn: int = 5632
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


TINYLLAMA_1_1B = LlamaShape()


class LlamaDecoder:
    """Greedy decoder for ``batch`` sequences of up to ``max_len`` tokens.

    ``prefill(prompt)`` runs the prompts ([B, T] token ids, one length T) with
    exact causal attention and appends their K/V to the cache; ``decode(n)``
    generates n tokens per sequence, one captured decode step per token, and
    returns them [B, n].
    """

    def __init__(self, shape: LlamaShape, batch: int, max_len: int, kv_dtype: str = "int8", page_size: int = 16,
                 device="cuda", seed: int = 0, weights: dict | None = None, keep_logits: bool = False,
                 fused_rope: bool = True):
        self.s = shape
        self.batch, self.max_len = batch, max_len
        self.device = torch.device(device)
        dt = torch.float16
        H, D, Hq, Hkv, Fd = shape.hidden, shape.head_dim, shape.heads, shape.kv_heads, shape.ffn
        if weights is None:
            g = torch.Generator(device=self.device).manual_seed(seed)

            def rnd(*sh, std=0.02):
                return (torch.randn(*sh, generator=g, device=self.device) * std).to(dt)

            weights = {"embed": rnd(shape.vocab, H), "norm": torch.ones(H, device=self.device, dtype=dt),
                       "lm_head": rnd(H, shape.vocab)}
            for i in range(shape.layers):
                weights[f"{i}.wqkv"] = rnd(H, (Hq + 2 * Hkv) * D)
                weights[f"{i}.wo"] = rnd(Hq * D, H)
                weights[f"{i}.wgu"] = rnd(H, 2 * Fd)
                weights[f"{i}.wdown"] = rnd(Fd, H)
                weights[f"{i}.n1"] = torch.ones(H, device=self.device, dtype=dt)
                weights[f"{i}.n2"] = torch.ones(H, device=self.device, dtype=dt)
        self.w = weights
        inv = 1.0 / (shape.rope_theta ** (torch.arange(0, D, 2, device=self.device, dtype=torch.float32) / D))
        ang = torch.outer(torch.arange(max_len, device=self.device, dtype=torch.float32), inv)
        self.cos, self.sin = ang.cos(), ang.sin()  # [max_len, D/2]
        mb = (max_len + page_size - 1) // page_size + 1
        self.cache = BatchedPagedKVCache(shape.layers, batch, Hkv, D, page_size=page_size, num_pages=batch * mb,
                                         max_blocks=mb, kv_dtype=kv_dtype, staging_dtype=dt, device=self.device)
        self.pos = torch.zeros(batch, dtype=torch.int64, device=self.device)
        self.ids = torch.zeros(batch, dtype=torch.int64, device=self.device)
        self.attn_out = torch.empty(batch, Hq, D, dtype=dt, device=self.device)
        self.qb = torch.empty(batch, Hq, D, dtype=dt, device=self.device)  # rotated q / k and v of a step
        self.kb = torch.empty(batch, Hkv, D, dtype=dt, device=self.device)
        self.vb = torch.empty(batch, Hkv, D, dtype=dt, device=self.device)
        # the last step's logits, kept only on request (tests)
        self.logits = torch.empty(batch, shape.vocab, dtype=dt, device=self.device) if keep_logits else None
        self.graph = None
        # rotary embedding inside the KV append (one launch per layer) or as its
        # own launch before a plain append (the same results)
        self.fused_rope = fused_rope

    # ------------------------------------------------- torch restatement of the pieces
    # (the decode step below runs the fused kernels; these are the plain torch
    # form of the same math, kept as the reference the tests compare against)
    def _rms(self, x, w):
        x32 = x.float()
        return (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + self.s.rms_eps)).to(x.dtype) * w

    def _rope(self, x, pos):
        """Rotary embedding (rotate-half convention) of x [..., heads, D] at positions pos [...]."""
        d2 = x.shape[-1] // 2
        c = self.cos[pos].unsqueeze(-2)
        s = self.sin[pos].unsqueeze(-2)
        x1, x2 = x[..., :d2].float(), x[..., d2:].float()
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)

    def _qkv(self, i, h):
        s = self.s
        D = s.head_dim
        qkv = h @ self.w[f"{i}.wqkv"]
        q, k, v = qkv.split([s.heads * D, s.kv_heads * D, s.kv_heads * D], dim=-1)
        return (q.unflatten(-1, (s.heads, D)), k.unflatten(-1, (s.kv_heads, D)), v.unflatten(-1, (s.kv_heads, D)))

    def _mlp(self, i, x):
        h = self._rms(x, self.w[f"{i}.n2"])
        gate, up = (h @ self.w[f"{i}.wgu"]).chunk(2, dim=-1)
        return x + (F.silu(gate) * up) @ self.w[f"{i}.wdown"]

    def _logits(self, x):
        return self._rms(x, self.w["norm"]) @ self.w["lm_head"]

    # ---------------------------------------------------------------- fused pieces
    def _norm(self, x, w):
        return _get_C().rmsnorm(x, w, self.s.rms_eps)

    def _ffn(self, i, x):
        """x [rows, hidden] += SwiGLU-MLP(RMSNorm(x)), in place."""
        C = _get_C()
        gu = C.rmsnorm(x, self.w[f"{i}.n2"], self.s.rms_eps) @ self.w[f"{i}.wgu"]
        x.addmm_(C.silu_mul(gu), self.w[f"{i}.wdown"])
        return x

    # ---------------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Prompts [B, T] -> first generated token per sequence [B]."""
        B, T = prompt.shape
        if B != self.batch or T + 1 > self.max_len:
            raise ValueError("prompt must be [batch, T] with T < max_len")
        s, c, C = self.s, self.cache, _get_C()
        D = s.head_dim
        x = self.w["embed"][prompt.to(self.device)].reshape(B * T, s.hidden)
        pos = torch.arange(T, device=self.device).repeat(B)
        q = torch.empty(B * T, s.heads, D, dtype=x.dtype, device=self.device)
        k = torch.empty(B * T, s.kv_heads, D, dtype=x.dtype, device=self.device)
        v = torch.empty_like(k)
        c.begin_step(T)
        for i in range(s.layers):
            qkv = self._norm(x, self.w[f"{i}.n1"]) @ self.w[f"{i}.wqkv"]
            C.rope_qkv(qkv, pos, self.cos, self.sin, q, k, v)  # k and v also feed the prompt's own attention
            c.append(i, k.view(B, T, s.kv_heads, D), v.view(B, T, s.kv_heads, D))
            o = F.scaled_dot_product_attention(q.view(B, T, s.heads, D).transpose(1, 2),
                                               k.view(B, T, s.kv_heads, D).transpose(1, 2),
                                               v.view(B, T, s.kv_heads, D).transpose(1, 2), is_causal=True,
                                               enable_gqa=True)
            x.addmm_(o.transpose(1, 2).reshape(B * T, s.heads * D), self.w[f"{i}.wo"])
            self._ffn(i, x)
        self.pos.fill_(T)
        last = x.view(B, T, s.hidden)[:, -1].contiguous()
        nxt = (self._norm(last, self.w["norm"]) @ self.w["lm_head"]).argmax(-1)
        self.ids.copy_(nxt)
        return nxt

    # ---------------------------------------------------------------- decode
    def _step(self):
        """One token for every sequence: self.ids at positions self.pos -> self.ids.
        Per layer: RMSNorm, the qkv GEMM, the KV append with the rotary
        embedding fused in (it also writes the rotated q), paged attention, the
        o-projection GEMM accumulated into x, then the MLP."""
        c, C = self.cache, _get_C()
        x = self.w["embed"][self.ids]
        c.begin_step(1, plan=True)
        for i in range(self.s.layers):
            qkv = self._norm(x, self.w[f"{i}.n1"]) @ self.w[f"{i}.wqkv"]
            if self.fused_rope:
                c.append_rope(i, qkv, self.s.heads, self.cos, self.sin, self.qb)
            else:
                C.rope_qkv(qkv, self.pos, self.cos, self.sin, self.qb, self.kb, self.vb)
                c.append(i, self.kb, self.vb)
            o = c.attend(i, self.qb, out=self.attn_out, max_context=c.max_blocks * c.page_size)
            x.addmm_(o.view(self.batch, -1), self.w[f"{i}.wo"])
            self._ffn(i, x)
        logits = self._norm(x, self.w["norm"]) @ self.w["lm_head"]
        if self.logits is not None:
            self.logits.copy_(logits)
        self.ids.copy_(logits.argmax(-1))
        self.pos += 1

    def capture(self) -> None:
        """Capture the decode step in a CUDA graph (after prefill)."""
        c = self.cache
        c._workspace(self.s.heads, c.max_blocks * c.page_size)
        c._decode_plan()
        c._ensure_n_new(1)  # filled outside the graph
        st = torch.cuda.Stream(self.device)
        st.wait_stream(torch.cuda.current_stream(self.device))
        self.graph = torch.cuda.CUDAGraph()
        saved = (self.ids.clone(), self.pos.clone())
        with torch.cuda.stream(st), torch.no_grad():
            with torch.cuda.graph(self.graph, stream=st):
                self._step()
        torch.cuda.current_stream(self.device).wait_stream(st)
        self.ids.copy_(saved[0])
        self.pos.copy_(saved[1])
        c._plan_ok = False

    @torch.no_grad()
    def decode(self, n: int) -> torch.Tensor:
        """n greedy tokens per sequence [B, n] (the first is the prefill's)."""
        c = self.cache
        out = torch.empty(self.batch, n, dtype=torch.int64, device=self.device)
        for t in range(n):
            out[:, t] = self.ids
            if t + 1 == n:
                break
            if self.graph is not None:
                c._ensure_n_new(1)
                self.graph.replay()
                c._max_len = min(c._max_len + 1, c.max_blocks * c.page_size + c.page_size - 1)
                c._plan_ok = False
            else:
                self._step()
        return out
