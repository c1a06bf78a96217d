"""CPU baseline: the reference's CPU path for decode attention, timed.

TEST / CPU-baseline infrastructure only (used by bench.py's CPU-baseline leg and
its ``--impl reference`` arm).  It restates the reference's CPU implementation
of the path -- tests/reference.py's dequantize (``codes.astype(float32) *
float32(scale)`` per page; the INT4 nibble unpack of
``dequantize_symmetric_int4_packed``, vectorised here) followed by the fp32
dequantize-then-attend of ``_reference_full_attention``
(tests/test_attention.py:14-20) with GQA head expansion -- in numpy float32,
plus the per-token append with a page commit (oracle C quantizer) every
``page_size`` tokens.  numpy's BLAS runs the products on all host threads.
"""
from __future__ import annotations

import os
import time

import numpy as np

import oracle as O


def _blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return 1


def _dequant_pages(pool, scales, ids, kv):
    codes = pool[ids]  # [n, P, H, row]
    if kv == "int8":
        x = codes.astype(np.float32)
    else:
        lo = (codes & 0x0F).astype(np.int8)
        hi = (codes >> 4).astype(np.int8)
        lo = np.where(lo >= 8, lo - 16, lo)
        hi = np.where(hi >= 8, hi - 16, hi)
        x = np.stack([lo, hi], axis=-1).reshape(*codes.shape[:-1], codes.shape[-1] * 2).astype(np.float32)
    x *= scales[ids].astype(np.float32)[:, None, None, None]
    return x.reshape(-1, x.shape[2], x.shape[3])


def _attend_fp32(q, k, v, scale):
    hq, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    kk = np.repeat(k, g, axis=1).transpose(1, 0, 2)  # [Hq, T, D]
    vv = np.repeat(v, g, axis=1).transpose(1, 0, 2)
    s = np.matmul(kk, q[:, :, None])[:, :, 0] * np.float32(scale)  # [Hq, T]
    s -= s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=1, keepdims=True)
    return np.matmul(p[:, None, :], vv)[:, 0, :]


def time_decode_sample(w, seconds=10.0, seed=0, max_seqs=8):
    """Run decode steps (append one token + attend, one layer) over a sample of
    the workload's sequences until ``seconds`` of CPU time pass.  Returns
    (GB/s over the same algorithmic bytes as the GPU metric, threads, text)."""
    rng = np.random.default_rng(seed)
    P, hkv, d, hq, kv = w["page"], w["hkv"], w["d"], w["hq"], w["kv"]
    if w["ctx"] == "uniform128_2048":
        ctx = rng.integers(128, 2049, size=max_seqs)
    elif w["ctx"] == "lognormal2048":
        ctx = np.exp(rng.normal(np.log(2048.0), 1.0, size=max_seqs)).round().clip(2, 32768).astype(np.int64) - 1
    else:
        ctx = np.full(max_seqs, int(w["ctx"]) - 1)
    nseq = max_seqs
    row = d if kv == "int8" else d // 2
    seqs = []
    for c in ctx:
        n = int(c) // P
        k = rng.standard_normal((n * P, hkv, d)).astype(np.float32)
        v = rng.standard_normal((n * P, hkv, d)).astype(np.float32)
        pool_k = np.zeros((n + 8, P, hkv, row), np.int8 if kv == "int8" else np.uint8)
        pool_v = np.zeros_like(pool_k)
        sk = np.zeros(n + 8, np.float64)
        sv = np.zeros(n + 8, np.float64)
        quant = O.quantize_int8 if kv == "int8" else O.quantize_int4
        for j in range(n):
            pool_k[j], sk[j] = quant(k[j * P:(j + 1) * P], np.zeros_like(pool_k[j]))
            pool_v[j], sv[j] = quant(v[j * P:(j + 1) * P], np.zeros_like(pool_v[j]))
        rest = int(c) - n * P
        seqs.append(dict(pool_k=pool_k, pool_v=pool_v, sk=sk, sv=sv, n=n,
                         stk=[rng.standard_normal((hkv, d)).astype(np.float32) for _ in range(rest)],
                         stv=[rng.standard_normal((hkv, d)).astype(np.float32) for _ in range(rest)]))
    q = rng.standard_normal((hq, d)).astype(np.float32)
    scale = 1.0 / np.sqrt(d)

    def bytes_for(c_after):
        bq = 1.0 if kv == "int8" else 0.5
        n, r = c_after // P, c_after % P
        att = 2 * n * P * hkv * d * bq + 12 * n + 4 * r * hkv * d + 4 * hq * d
        app = 4 * hkv * d + (4 * (P - 1) * hkv * d + 2 * P * hkv * d * bq + 8 if r == 0 else 4 * hkv * d)
        return att + app

    total_bytes = 0.0
    steps = 0
    t0 = time.perf_counter()
    while True:
        for s in seqs:
            # append one token (stage; commit a full page with one fresh scale)
            s["stk"].append(rng.standard_normal((hkv, d)).astype(np.float32))
            s["stv"].append(rng.standard_normal((hkv, d)).astype(np.float32))
            if len(s["stk"]) == P:
                j = s["n"]
                if j >= s["pool_k"].shape[0]:
                    s["pool_k"] = np.concatenate([s["pool_k"], np.zeros_like(s["pool_k"])])
                    s["pool_v"] = np.concatenate([s["pool_v"], np.zeros_like(s["pool_v"])])
                    s["sk"] = np.concatenate([s["sk"], np.zeros_like(s["sk"])])
                    s["sv"] = np.concatenate([s["sv"], np.zeros_like(s["sv"])])
                quant = O.quantize_int8 if kv == "int8" else O.quantize_int4
                s["pool_k"][j], s["sk"][j] = quant(np.stack(s["stk"]), np.zeros_like(s["pool_k"][j]))
                s["pool_v"][j], s["sv"][j] = quant(np.stack(s["stv"]), np.zeros_like(s["pool_v"][j]))
                s["n"] += 1
                s["stk"], s["stv"] = [], []
            ids = np.arange(s["n"])
            kd = _dequant_pages(s["pool_k"], s["sk"], ids, kv)
            vd = _dequant_pages(s["pool_v"], s["sv"], ids, kv)
            if s["stk"]:
                kd = np.concatenate([kd, np.stack(s["stk"])])
                vd = np.concatenate([vd, np.stack(s["stv"])])
            _attend_fp32(q, kd, vd, scale)
            total_bytes += bytes_for(s["n"] * P + len(s["stk"]))
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = total_bytes / el / 1e9
    threads = _blas_threads()
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    sample = (f"{nseq} sequences x 1 layer (contexts {int(ctx.min())}-{int(ctx.max())}), {steps} decode steps "
              f"(append + dequantize-then-attend fp32 numpy) in {el:.1f} s; {threads} BLAS threads on {cores} "
              f"host cores")
    return gbs, threads, sample


# --------------------------------------------------------------------------
# The CPU reference configuration itself: batch 4, 12 heads, head_dim 64,
# page 16, contexts U[1, 512], fp32 N(0, 1), INT8 with one absmax scale per
# (token, head) vector, shuffled physical pages, one decode step.
# --------------------------------------------------------------------------

def _quantize_rows_int8(x):
    """tests/reference.py:4-11 ``quantize_symmetric_int8`` applied to every
    last-axis vector of ``x`` at once: scale = absmax / 127 (1e-8 when the
    absmax is <= 1e-12), codes = clip(round-half-even(x / scale), -127, 127)."""
    a = np.abs(x).max(axis=-1, keepdims=True)
    s = np.where(a > 1e-12, a / 127.0, 1e-8)
    q = np.clip(np.round(x / s), -127, 127).astype(np.int8)
    return q, s[..., 0]


def _dequantize_rows_int8(q, s):
    """tests/reference.py:14-15 ``dequantize_symmetric_int8``: codes as float32
    times float32(scale), per vector."""
    return q.astype(np.float32) * s.astype(np.float32)[..., None]


def time_cpu_reference_config(seconds=10.0, seed=0):
    """One decode step of the CPU reference configuration, repeated until
    ``seconds`` pass: per sequence, quantize the new token's K and V vectors
    (per token and head), dequantize the cached codes through the shuffled
    block table, and run fp32 attention in torch on the CPU (scores by einsum,
    max-subtracted softmax, einsum with V: the steps of
    tests/test_attention.py:14-20).  Returns (GB/s over the bytes the step
    reads and writes -- codes and per-(token, head) scales of the cache, the new
    token, q and out -- threads, description)."""
    import torch

    rng = np.random.default_rng(seed)
    B, H, D, P = 4, 12, 64, 16
    ctx = rng.integers(1, 513, size=B)
    nblocks = [int(c + 1 + P - 1) // P for c in ctx]
    num_pages = sum(nblocks) + 8
    perm = rng.permutation(num_pages)
    codes_k = np.zeros((num_pages, P, H, D), np.int8)
    codes_v = np.zeros_like(codes_k)
    sc_k = np.zeros((num_pages, P, H), np.float64)
    sc_v = np.zeros_like(sc_k)
    tables, nxt = [], 0
    for b in range(B):
        tables.append(perm[nxt:nxt + nblocks[b]])
        nxt += nblocks[b]
    lens = [int(c) for c in ctx]
    for b in range(B):
        x = rng.standard_normal((lens[b], H, D)).astype(np.float32)
        y = rng.standard_normal((lens[b], H, D)).astype(np.float32)
        qk, sk = _quantize_rows_int8(x)
        qv, sv = _quantize_rows_int8(y)
        for t in range(lens[b]):
            pg, off = tables[b][t // P], t % P
            codes_k[pg, off], sc_k[pg, off] = qk[t], sk[t]
            codes_v[pg, off], sc_v[pg, off] = qv[t], sv[t]
    q = [torch.from_numpy(rng.standard_normal((H, D)).astype(np.float32)) for _ in range(B)]
    new_k = rng.standard_normal((B, H, D)).astype(np.float32)
    new_v = rng.standard_normal((B, H, D)).astype(np.float32)
    inv = 1.0 / np.sqrt(D)
    steps = 0
    t0 = time.perf_counter()
    total = 0.0
    while True:
        for b in range(B):
            c = lens[b]  # the step appends token c, then attends over c + 1 tokens
            pg, off = tables[b][c // P], c % P
            codes_k[pg, off], sc_k[pg, off] = _quantize_rows_int8(new_k[b])
            codes_v[pg, off], sc_v[pg, off] = _quantize_rows_int8(new_v[b])
            n = c + 1
            tb = tables[b][: (n + P - 1) // P]
            k = _dequantize_rows_int8(codes_k[tb], sc_k[tb]).reshape(-1, H, D)[:n]
            v = _dequantize_rows_int8(codes_v[tb], sc_v[tb]).reshape(-1, H, D)[:n]
            kt, vt = torch.from_numpy(k), torch.from_numpy(v)
            s = torch.einsum("thd,hd->ht", kt, q[b]) * inv
            s = s - s.max(dim=-1, keepdim=True).values
            pr = torch.softmax(s, dim=-1)
            torch.einsum("ht,thd->hd", pr, vt)
            total += 2 * n * H * (D + 4) + 2 * H * (D * 4 + D + 4) + 2 * H * D * 4
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = total / el / 1e9
    threads = max(_blas_threads(), torch.get_num_threads())
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    desc = (f"CPU reference configuration: batch 4, 12 heads, head_dim 64, page 16, contexts "
            f"{int(ctx.min())}..{int(ctx.max())} (U[1, 512]), fp32, INT8 per-(token, head) scales, shuffled pages; "
            f"{steps} decode steps (quantize the new token, dequantize, fp32 torch attention) in {el:.1f} s, "
            f"ms/step {1e3 * el / steps:.3f}; {threads} threads on {cores} host cores")
    return gbs, threads, desc, 1e3 * el / steps
