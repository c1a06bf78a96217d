"""Decode attention over a ``PagedKVCache`` with the reference's interface.

``paged_attention(cache, layer_idx, query, scale=None)`` keeps the signature,
validation and ValueError behaviour of metagross/attention.py:62-134.  Where
the reference runs its committed-page kernel, then the staging tail in torch,
then a log-sum-exp merge, this module makes ONE call to the fused native
kernel (``_C.paged_decode_attention``): committed INT8 pages through the block
table and the exact fp32 staged tail in the same online softmax, normalised in
the kernel.

The three helpers below are kept with the reference's semantics because
callers and tests use them directly:
  _merge_unnormalized    metagross/attention.py:15-26
  _staging_contribution  metagross/attention.py:29-50
  _repeat_kv_heads       metagross/attention.py:53-59 (kv head h -> q heads h*n..h*n+n-1)
"""
from __future__ import annotations

import math

import torch

from .cache import PagedKVCache

_KERNEL_HEAD_DIMS = (64, 128)


def _get_C():
    from . import _C

    return _C


def _merge_unnormalized(max1, sum1, wv1: torch.Tensor, max2, sum2, wv2: torch.Tensor):
    m = torch.maximum(max1, max2)
    a = torch.exp(max1 - m)
    b = torch.exp(max2 - m)
    return wv1 * a.unsqueeze(-1) + wv2 * b.unsqueeze(-1), sum1 * a + sum2 * b


def _staging_contribution(query, staging_k, staging_v, inv_sqrt_head_dim):
    hq, d = query.shape
    dev = query.device
    if staging_k.shape[0] == 0:
        return (
            torch.full((hq,), float("-inf"), device=dev),
            torch.zeros(hq, device=dev),
            torch.zeros(hq, d, device=dev),
        )
    s = torch.einsum("thd,hd->ht", staging_k, query) * inv_sqrt_head_dim
    m = s.max(dim=-1).values
    e = torch.exp(s - m.unsqueeze(-1))
    return m, e.sum(dim=-1), torch.einsum("ht,thd->hd", e, staging_v)


def _repeat_kv_heads(x: torch.Tensor, n_rep) -> torch.Tensor:
    if n_rep == 1:
        return x
    seq, h, d = x.shape
    return x[:, :, None, :].expand(seq, h, n_rep, d).reshape(seq, h * n_rep, d)


class _Scratch:
    """Per-device reusable workspace for the single-sequence path."""

    def __init__(self):
        self.ws = {}

    def get(self, device, nbytes):
        t = self.ws.get(device)
        if t is None or t.numel() < nbytes:
            t = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            self.ws[device] = t
        return t


_scratch = _Scratch()


def _scales_tensor(scales, device):
    return torch.tensor([s if s is not None else 0.0 for s in scales], dtype=torch.float32, device=device)


def paged_attention(cache: PagedKVCache, layer_idx, query, scale=None) -> torch.Tensor:
    if query.dim() != 2:
        raise ValueError(f"query must be 2-D [num_q_heads, head_dim], got {query.dim()}-D")
    hq, d = query.shape
    if scale is not None:
        if isinstance(scale, torch.Tensor):
            scale = scale.item()
        if math.isnan(scale) or math.isinf(scale) or scale <= 0:
            raise ValueError(f"scale must be a positive finite number, got {scale}")
    sc = scale if scale is not None else 1.0 / (d ** 0.5)

    kc = cache.k_layers[layer_idx]
    vc = cache.v_layers[layer_idx]
    dev = query.device
    hkv = kc.num_heads
    if hkv <= 0:
        raise ValueError("num_kv_heads must be positive")
    if hq % hkv != 0:
        raise ValueError(f"num_q_heads={hq} must be divisible by num_kv_heads={hkv}")
    if not kc.block_table and not kc._staging:
        raise ValueError(
            "paged_attention requires at least one cached token (both committed pages and staging are empty "
            "for this layer) -- call cache.append(...) before paged_attention(...)"
        )
    C = _get_C()
    if d not in _KERNEL_HEAD_DIMS or kc.head_dim != d:
        # Shapes outside the fused kernel: same composition (and errors) as the
        # reference -- committed pages through the op, which rejects them with
        # RuntimeError, the staged tail with the torch helpers on the device.
        n_rep = hq // hkv
        if kc.block_table:
            bt = torch.tensor(kc.block_table, dtype=torch.int32, device=dev)
            wv1, s1, m1 = C.paged_attention_committed(
                query.float(), kc.storage, vc.storage, _scales_tensor(kc.page_scales, dev),
                _scales_tensor(vc.page_scales, dev), bt, sc)
        else:
            m1 = torch.full((hq,), float("-inf"), device=dev)
            s1 = torch.zeros(hq, device=dev)
            wv1 = torch.zeros(hq, d, device=dev)
        sk = torch.stack(kc._staging).float() if kc._staging else torch.empty(0, hkv, d, device=dev)
        sv = torch.stack(vc._staging).float() if vc._staging else torch.empty(0, hkv, d, device=dev)
        m2, s2, wv2 = _staging_contribution(query.float(), _repeat_kv_heads(sk, n_rep), _repeat_kv_heads(sv, n_rep), sc)
        wv, l = _merge_unnormalized(m1, s1, wv1, m2, s2, wv2)
        return wv / l.unsqueeze(-1)

    P = kc.page_size
    nb = len(kc.block_table)
    r = len(kc._staging)
    q = query.float().contiguous().unsqueeze(0)
    bt = torch.tensor([kc.block_table or [0]], dtype=torch.int32, device=dev)
    seq_lens = torch.tensor([nb * P + r], dtype=torch.int32, device=dev)
    staging_k = torch.zeros(1, P, hkv, d, dtype=torch.float32, device=dev)
    staging_v = torch.zeros(1, P, hkv, d, dtype=torch.float32, device=dev)
    if r:
        staging_k[0, :r] = torch.stack(kc._staging)
        staging_v[0, :r] = torch.stack(vc._staging)
    max_ctx = nb * P + r
    ws_bytes = C.decode_workspace_bytes(kc.storage, bt, hq, max_ctx)
    ws = _scratch.get(dev, ws_bytes)
    out = torch.empty(1, hq, d, dtype=torch.float32, device=dev)
    C.paged_decode_attention(q, kc.storage, vc.storage, _scales_tensor(kc.page_scales, dev),
                             _scales_tensor(vc.page_scales, dev), staging_k, staging_v, bt, seq_lens, sc, max_ctx,
                             ws, out)
    return out[0]
