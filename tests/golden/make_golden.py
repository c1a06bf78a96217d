"""Generate the golden fixtures in tests/golden/ from the reference's own Python.

Run in a container where the reference is mounted (it is NOT needed at test
time; the .npz files are committed):

    python tests/golden/make_golden.py /root/reference [all|page|token_head]

Every fixture is produced by calling the reference's code, never by this
repository's code:
  * tests/reference.py         quantize_symmetric_int8 / int4_packed and their
                               dequantizers (the reference's CPU path)
  * metagross/allocator.py     BlockAllocator driven by a seeded op script
  * metagross/attention.py     _staging_contribution, _merge_unnormalized,
                               _repeat_kv_heads (torch CPU, fp32)
Inputs are seeded with torch.Generator(seed) on the CPU, like the reference's
stress tests (tests/test_cuda_stress.py:13-28, BASE_SEED = 20260822).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

OUT = os.path.dirname(os.path.abspath(__file__))
BASE_SEED = 20260822


def _gen(offset):
    return torch.Generator().manual_seed(BASE_SEED + offset)


def main(ref_root: str):
    sys.path.insert(0, ref_root)
    from tests import reference as R  # reference's numpy CPU path
    from metagross.allocator import BlockAllocator
    from metagross import attention as A

    # ---- INT8: reference tests' shapes + randomized shapes -----------------
    cases = {}
    shapes = [(16, 4, 8, 3.0), (8, 4, 8, 3.0), (16, 12, 64, 1.0), (16, 4, 64, 1.0)]
    g = _gen(0)
    for i in range(25):
        t = int(torch.randint(1, 17, (1,), generator=g))
        h = int(torch.randint(1, 9, (1,), generator=g))
        d = int(torch.randint(1, 33, (1,), generator=g))
        sc = float(torch.rand((1,), generator=g)) * 10 + 0.01
        shapes.append((t, h, d, sc))
    for i, (t, h, d, sc) in enumerate(shapes):
        x = (torch.randn(t, h, d, generator=_gen(100 + i)) * sc).numpy().astype(np.float32)
        q, s = R.quantize_symmetric_int8(x)
        deq = R.dequantize_symmetric_int8(q, s)
        cases[f"x{i}"] = x
        cases[f"q{i}"] = q
        cases[f"s{i}"] = np.array([s], np.float64)
        cases[f"deq{i}"] = deq
    cases["n"] = np.array([len(shapes)])
    np.savez_compressed(os.path.join(OUT, "int8_quant.npz"), **cases)

    # ---- INT4 packed ----------------------------------------------------------
    cases = {}
    shapes4 = [(16, 4, 8, 3.0), (8, 2, 8, 3.0), (16, 4, 64, 1.0)]
    g = _gen(1000)
    for i in range(25):
        t = int(torch.randint(1, 17, (1,), generator=g))
        h = int(torch.randint(1, 9, (1,), generator=g))
        d = int(torch.randint(1, 17, (1,), generator=g)) * 2
        sc = float(torch.rand((1,), generator=g)) * 10 + 0.01
        shapes4.append((t, h, d, sc))
    for i, (t, h, d, sc) in enumerate(shapes4):
        x = (torch.randn(t, h, d, generator=_gen(200 + i)) * sc).numpy().astype(np.float32)
        packed, s = R.quantize_symmetric_int4_packed(x.reshape(-1))
        deq = R.dequantize_symmetric_int4_packed(packed, s)
        cases[f"x{i}"] = x
        cases[f"p{i}"] = packed
        cases[f"s{i}"] = np.array([s], np.float64)
        cases[f"deq{i}"] = deq.reshape(x.shape)
    cases["n"] = np.array([len(shapes4)])
    np.savez_compressed(os.path.join(OUT, "int4_quant.npz"), **cases)

    # ---- known-answer: integer inputs, absmax 127 -> scale exactly 1.0 --------
    g = _gen(7100)
    kat = {}
    for i in range(5):
        x = torch.randint(-127, 128, (16, 4, 64), generator=g).float()
        x[0, 0, 0] = 127.0
        q, s = R.quantize_symmetric_int8(x.numpy())
        kat[f"x{i}"] = x.numpy()
        kat[f"q{i}"] = q
        kat[f"s{i}"] = np.array([s])
    np.savez_compressed(os.path.join(OUT, "int8_kat_scale1.npz"), **kat)

    # ---- allocator: seeded script of allocate / free, errors included ---------
    g = _gen(9000)
    scripts = {}
    for case in range(6):
        n = int(torch.randint(1, 40, (1,), generator=g))
        alloc = BlockAllocator(n)
        held = []
        ops, res = [], []
        for _ in range(200):
            r = float(torch.rand((1,), generator=g))
            if r < 0.55:
                ops.append(-1)
                try:
                    p = alloc.allocate()
                    held.append(p)
                    res.append(p)
                except RuntimeError:
                    res.append(-1)
            elif r < 0.9 and held:
                idx = int(torch.randint(0, len(held), (1,), generator=g))
                p = held.pop(idx)
                ops.append(p)
                alloc.free(p)
                res.append(p)
            elif r < 0.95:
                # double free of a page that is free right now (if any)
                free_now = [p for p in range(n) if p not in held]
                if not free_now:
                    continue
                p = free_now[int(torch.randint(0, len(free_now), (1,), generator=g))]
                ops.append(p)
                try:
                    alloc.free(p)
                    res.append(p)
                except RuntimeError:
                    res.append(-2)
            else:
                p = n + int(torch.randint(0, 5, (1,), generator=g))
                ops.append(p)
                try:
                    alloc.free(p)
                    res.append(p)
                except ValueError:
                    res.append(-3)
        scripts[f"n{case}"] = np.array([n])
        scripts[f"ops{case}"] = np.array(ops, np.int32)
        scripts[f"res{case}"] = np.array(res, np.int32)
        scripts[f"free{case}"] = np.array(alloc._free, np.int32)
    scripts["n"] = np.array([6])
    np.savez_compressed(os.path.join(OUT, "allocator_script.npz"), **scripts)

    # ---- attention helpers (torch CPU fp32) ------------------------------------
    att = {}
    cfgs = [(4, 4, 64, 7, 10), (32, 4, 64, 16, 5), (12, 12, 64, 33, 0), (8, 2, 64, 1, 20), (6, 3, 64, 5, 9)]
    for i, (hq, hkv, d, n1, n2) in enumerate(cfgs):
        gg = _gen(300 + i)
        q = torch.randn(hq, d, generator=gg)
        k1 = torch.randn(n1, hkv, d, generator=gg) * 2
        v1 = torch.randn(n1, hkv, d, generator=gg) * 2
        k2 = torch.randn(n2, hkv, d, generator=gg) * 2
        v2 = torch.randn(n2, hkv, d, generator=gg) * 2
        sc = 1.0 / d ** 0.5
        rep = hq // hkv
        m1, s1, wv1 = A._staging_contribution(q, A._repeat_kv_heads(k1, rep), A._repeat_kv_heads(v1, rep), sc)
        m2, s2, wv2 = A._staging_contribution(q, A._repeat_kv_heads(k2, rep), A._repeat_kv_heads(v2, rep), sc)
        wv, l = A._merge_unnormalized(m1, s1, wv1, m2, s2, wv2)
        for name, val in dict(q=q, k1=k1, v1=v1, k2=k2, v2=v2, m1=m1, s1=s1, wv1=wv1, m2=m2, s2=s2,
                              wv2=wv2, wv=wv, l=l, out=wv / l.unsqueeze(-1)).items():
            att[f"{name}{i}"] = val.numpy()
        att[f"scale{i}"] = np.array([sc])
    att["n"] = np.array([len(cfgs)])
    np.savez_compressed(os.path.join(OUT, "attention_helpers.npz"), **att)

    print("wrote fixtures to", OUT)


def make_token_head(ref_root: str):
    """Per-token-per-head INT8 scales on a GPT-2-small decode step: batch 4, 12
    heads, head_dim 64, contexts U[1, 512], fp32 N(0, 1) K/V/q.  As in the
    reference cache, the full 16-token pages of a context are quantized and the
    partial last page stays exact; each (token, head) D-vector of a full page is
    quantized by the reference's CPU path on its own.  The output is the
    reference's exact attention math (_staging_contribution) over the
    dequantized pages followed by the exact tail.  The test regenerates the
    inputs from the seed (th_inputs is the recipe), so only digests of the
    committed codes / scales, the first page of each sequence in full, the
    rounding ties (t, h, d, CPU-path code, kernel code) and the outputs are
    stored."""
    import hashlib

    sys.path.insert(0, ref_root)
    from tests import reference as R
    from metagross import attention as A

    lens, ks, vs, q = th_inputs()
    th = {"lens": lens.numpy(), "q": q.numpy()}
    for b in range(len(lens)):
        deqs = {}
        n = int(lens[b]) // 16 * 16  # committed rows
        for name, x in (("k", ks[b]), ("v", vs[b])):
            xn = x.numpy()[:n]
            codes = np.zeros(xn.shape, np.int8)
            scales = np.zeros(xn.shape[:2], np.float32)
            deq = np.zeros(xn.shape, np.float32)
            ties = []
            for t in range(xn.shape[0]):
                for h in range(xn.shape[1]):
                    c, sc = R.quantize_symmetric_int8(xn[t, h])
                    # x / s landing exactly on k + 0.5: the CPU path rounds half to
                    # even (np.round), the reference's CUDA kernels half away from
                    # zero (roundf); the fixture keeps the kernels' code and lists
                    # the position with both codes
                    r = xn[t, h] / sc
                    for d in np.nonzero(np.abs(r - np.trunc(r)) == 0.5)[0]:
                        away = int(np.clip(np.trunc(r[d]) + np.sign(r[d]), -127, 127))
                        ties.append((t, h, d, int(c[d]), away))
                        c[d] = away
                    codes[t, h], scales[t, h] = c, np.float32(sc)
                    deq[t, h] = R.dequantize_symmetric_int8(c, sc)
            th[f"{name}_ties{b}"] = np.array(ties, np.int32).reshape(-1, 5)
            th[f"{name}_codes_sha{b}"] = np.frombuffer(hashlib.sha256(codes.tobytes()).digest(), np.uint8)
            th[f"{name}_scales_sha{b}"] = np.frombuffer(hashlib.sha256(scales.tobytes()).digest(), np.uint8)
            th[f"{name}_codes_page0_{b}"] = codes[:16]
            th[f"{name}_scales_page0_{b}"] = scales[:16]
            deqs[name] = torch.cat([torch.from_numpy(deq), x[n:]])
        m, ssum, wv = A._staging_contribution(q[b], deqs["k"], deqs["v"], 1.0 / 8)
        th[f"out{b}"] = (wv / ssum.unsqueeze(-1)).numpy()
    np.savez_compressed(os.path.join(OUT, "token_head_int8.npz"), **th)
    print("wrote token_head_int8.npz to", OUT)


def th_inputs():
    """Seeded inputs of the per-token-per-head fixture: (lens [4], K list, V list, q [4, 12, 64])."""
    g = _gen(7300)
    lens = torch.randint(1, 513, (4,), generator=g, dtype=torch.int32)
    ks = [torch.randn(int(n), 12, 64, generator=g) for n in lens]
    vs = [torch.randn(int(n), 12, 64, generator=g) for n in lens]
    q = torch.randn(4, 12, 64, generator=g)
    return lens, ks, vs, q


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    which = sys.argv[2] if len(sys.argv) > 2 else "all"
    if which in ("all", "page"):
        main(root)
    if which in ("all", "token_head"):
        make_token_head(root)
