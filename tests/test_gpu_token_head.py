"""Per-(token, kv head) scales (scale_granularity="token_head") on the GPU.

The reference cache has one scale per page; its CPU-reference workload (batch 4,
12 heads, head_dim 64, contexts U[1, 512], fp32 N(0, 1)) quantizes with one
absmax scale per token and head.  Checked here:
  * append: codes / packed nibbles and the fp32 scales [N, P, Hkv] bit-exact
    with the oracle's PagedCacheModel(scale_granularity="token_head") after
    every step, INT8 and INT4, page sizes 16 and 8;
  * gather/dequantize: bit-exact with the oracle's per-vector dequantization;
  * attention: within 2e-3 (fp16 out) / 1e-3 (fp32 out) of float64
    dequantize-then-attend, 16-token pages (per-row scales of one page) and
    8-token pages (tiles spanning pages);
  * the golden fixture of the CPU-reference workload (tests/golden/
    token_head_int8.npz, made by the reference's own Python): codes and scales
    hash to the fixture's, outputs within 1e-3 of the reference's torch math.
"""
import hashlib
import os
import sys

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _cache(*args, **kw):
    from metagross_b200.batched import BatchedPagedKVCache

    return BatchedPagedKVCache(*args, scale_granularity="token_head", **kw)


def _assert_pages_equal(cache, model, layer=0):
    nb = model.num_blocks
    bt = cache.block_tables.cpu().numpy()
    kp, vp = cache.k_pool[layer].cpu().numpy(), cache.v_pool[layer].cpu().numpy()
    ks, vs = cache.k_scales[layer].cpu().numpy(), cache.v_scales[layer].cpu().numpy()
    for b in range(model.B):
        np.testing.assert_array_equal(bt[b, :nb[b]], model.block_tables[b, :nb[b]])
        for j in range(nb[b]):
            p = int(model.block_tables[b, j])
            np.testing.assert_array_equal(kp[p], model.k_pool[p], err_msg=f"k page {p}")
            np.testing.assert_array_equal(vp[p], model.v_pool[p], err_msg=f"v page {p}")
            np.testing.assert_array_equal(ks[p], model.k_scales[p], err_msg=f"k scales of page {p}")
            np.testing.assert_array_equal(vs[p], model.v_scales[p], err_msg=f"v scales of page {p}")


@pytest.mark.parametrize("kv", ["int8", "int4"])
@pytest.mark.parametrize("P", [16, 8])
def test_append_token_head_bit_exact(kv, P):
    g = torch.Generator().manual_seed(21 + P)
    B, H, D = 5, 3, 64
    cache = _cache(1, B, H, D, page_size=P, num_pages=200, max_blocks=60, kv_dtype=kv, staging_dtype=torch.float16)
    model = O.PagedCacheModel(B, 200, P, H, D, kv_dtype=kv, staging_dtype=np.float16, max_blocks=60,
                              scale_granularity="token_head")
    for step, T in enumerate([3, 1, 17, 1, 40, 2]):
        n_new = torch.randint(0, T + 1, (B,), generator=g, dtype=torch.int32)
        k = (torch.randn(B, T, H, D, generator=g) * 2).half()
        v = (torch.randn(B, T, H, D, generator=g) * 2).half()
        k[torch.rand(k.shape, generator=g) < 0.01] *= 8
        if step == 2:  # an all-zero vector takes the 1e-8 scale
            k[:, 0, 0] = 0
        cache.begin_step(n_new)
        cache.append(0, k.cuda(), v.cuda())
        model.append(k.numpy(), v.numpy(), n_new.numpy())
        cache.check()
        _assert_pages_equal(cache, model)


@pytest.mark.parametrize("kv", ["int8", "int4"])
def test_gather_token_head_bit_exact(kv):
    g = torch.Generator().manual_seed(31)
    B, H, D, P = 4, 4, 64, 16
    cache = _cache(1, B, H, D, page_size=P, num_pages=64, max_blocks=16, kv_dtype=kv, staging_dtype=torch.float16)
    model = O.PagedCacheModel(B, 64, P, H, D, kv_dtype=kv, staging_dtype=np.float16, max_blocks=16,
                              scale_granularity="token_head")
    lens = torch.tensor([0, 5, 16, 77], dtype=torch.int32)
    k = torch.randn(B, 77, H, D, generator=g).half()
    v = torch.randn(B, 77, H, D, generator=g).half()
    cache.begin_step(lens)
    cache.append(0, k.cuda(), v.cuda())
    model.append(k.numpy(), v.numpy(), lens.numpy())
    ok, ov, cu = cache.gather(0, dtype=torch.float32)
    cache.check()
    for b in range(B):
        sl = slice(int(cu[b]), int(cu[b + 1]))
        np.testing.assert_array_equal(ok[sl].cpu().numpy(), model.dequantized_sequence(b, "k"))
        np.testing.assert_array_equal(ov[sl].cpu().numpy(), model.dequantized_sequence(b, "v"))


@pytest.mark.parametrize("kv", ["int8", "int4"])
@pytest.mark.parametrize("hq,hkv", [(12, 12), (32, 4), (8, 2)])
@pytest.mark.parametrize("P,qdt", [(16, torch.float16), (8, torch.float16), (16, torch.float32)])
def test_attention_token_head(kv, hq, hkv, P, qdt):
    g = torch.Generator().manual_seed(hq * 5 + hkv + P)
    B, D = 4, 64
    cache = _cache(1, B, hkv, D, page_size=P, num_pages=B * 80, max_blocks=80, kv_dtype=kv,
                   staging_dtype=torch.float32 if qdt == torch.float32 else torch.float16)
    model = O.PagedCacheModel(B, B * 80, P, hkv, D, kv_dtype=kv, max_blocks=80, scale_granularity="token_head")
    lens = torch.randint(100, 600, (B,), generator=g, dtype=torch.int32)
    k = torch.randn(B, 600, hkv, D, generator=g).to(qdt)
    v = torch.randn(B, 600, hkv, D, generator=g).to(qdt)
    k[torch.rand(k.shape, generator=g) < 0.01] *= 8
    cache.begin_step(lens)
    cache.append(0, k.cuda(), v.cuda())
    model.append(k.float().numpy(), v.float().numpy(), lens.numpy())
    for step in range(2):
        q = torch.randn(B, hq, D, generator=g).to(qdt)
        out = cache.attend(0, q.cuda())
        cache.check()
        ref = model.attend(q.float().numpy(), 1.0 / 8)
        err = np.abs(out.float().cpu().numpy() - ref).max()
        assert err < (2e-3 if qdt == torch.float16 else 1e-3), err
        kn = torch.randn(B, 1, hkv, D, generator=g).to(qdt)
        vn = torch.randn(B, 1, hkv, D, generator=g).to(qdt)
        cache.begin_step(1)
        cache.append(0, kn.cuda(), vn.cuda())
        model.append(kn.float().numpy(), vn.float().numpy())


def test_cpu_reference_workload_fixture():
    """The fixture's GPT-2-small decode step through the batched cache: fp32
    K/V appended in one prefill; the committed codes and scales, read in
    block-table order, hash to the reference CPU path's, and the fp32
    attention output is within 1e-3 of the reference's torch math."""
    if GOLD not in sys.path:
        sys.path.insert(0, GOLD)
    import make_golden

    z = np.load(os.path.join(GOLD, "token_head_int8.npz"))
    lens, ks, vs, q = make_golden.th_inputs()
    B, H, D, P = 4, 12, 64, 16
    T = int(lens.max())
    mb = (T + P - 1) // P
    cache = _cache(1, B, H, D, page_size=P, num_pages=B * mb, max_blocks=mb, staging_dtype=torch.float32)
    k = torch.zeros(B, T, H, D)
    v = torch.zeros(B, T, H, D)
    for b in range(B):
        k[b, :int(lens[b])] = ks[b]
        v[b, :int(lens[b])] = vs[b]
    cache.begin_step(lens)
    cache.append(0, k.cuda(), v.cuda())
    out = cache.attend(0, q.cuda(), scale=1.0 / 8)
    cache.check()
    bt = cache.block_tables.cpu().numpy()
    for b in range(B):
        n = int(lens[b]) // P
        pages = bt[b, :n]
        for name, pool, scales in (("k", cache.k_pool[0], cache.k_scales[0]),
                                   ("v", cache.v_pool[0], cache.v_scales[0])):
            codes = pool.cpu().numpy()[pages].reshape(n * P, H, D)
            s32 = scales.cpu().numpy()[pages].reshape(n * P, H)
            if n:
                np.testing.assert_array_equal(codes[:16], z[f"{name}_codes_page0_{b}"])
                np.testing.assert_array_equal(s32[:16], z[f"{name}_scales_page0_{b}"])
            assert hashlib.sha256(codes.tobytes()).digest() == z[f"{name}_codes_sha{b}"].tobytes()
            assert hashlib.sha256(s32.tobytes()).digest() == z[f"{name}_scales_sha{b}"].tobytes()
    ref = np.stack([z[f"out{b}"] for b in range(B)])
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err < 1e-3, err
