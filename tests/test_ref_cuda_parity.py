"""Side-by-side parity with the reference's own CUDA ops on the same inputs.

The reference's ``_C`` (csrc/*.cu, compiled from its sources by
oracle/build_ref.py into oracle/_ref/, test infrastructure only) runs next to
this package's ops and the CPU oracle:
  * INT8 / INT4 quantize (new and fixed scale) and dequantize: codes, packed
    nibbles, scales and dequantized floats bit-exact, three ways;
  * paged_attention_committed (one sequence, shuffled block table): the
    unnormalised (wv, sum, max) agree within fp32 rounding of the different
    summation orders.
Skipped when the reference build is absent (it is built where the reference
sources are mounted and travels with the working tree)."""
import glob
import importlib.util
import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def _ref():
    hits = sorted(glob.glob(os.path.join(ROOT, "oracle", "_ref", "metagross_ref_C*.so")))
    if not hits:
        pytest.skip("reference _C not built (oracle/_ref)")
    spec = importlib.util.spec_from_file_location("metagross_ref_C", hits[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _ours():
    from metagross_b200 import _C

    return _C


def _inputs(seed, T, H, D, special=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, D, generator=g) * (1 + 3 * torch.rand(T, H, D, generator=g))
    if special:
        x.view(-1)[::97] = float("nan")
        x.view(-1)[5] = 0.0
    return x


@pytest.mark.parametrize("seed,T,off,special", [(1, 16, 0, False), (2, 7, 3, False), (3, 1, 15, True),
                                                 (4, 16, 0, True)])
def test_int8_ops_match_reference(seed, T, off, special):
    import oracle as O

    ref, ours = _ref(), _ours()
    H, D, P = 4, 64, 16
    x = _inputs(seed, T, H, D, special).cuda()
    pr = torch.zeros(P, H, D, dtype=torch.int8, device="cuda")
    po = torch.zeros_like(pr)
    sr = ref.quantize_new_scale(x, pr, off)
    so = ours.quantize_new_scale(x, po, off)
    assert sr == so
    assert torch.equal(pr, po)
    codes, s_orc = O.quantize_int8(x.cpu().numpy())
    assert s_orc == sr
    np.testing.assert_array_equal(pr[off:off + T].cpu().numpy(), codes)
    # fixed scale and dequantize
    pr2, po2 = torch.zeros_like(pr), torch.zeros_like(pr)
    ref.quantize_fixed_scale(x, pr2, off, 0.0375)
    ours.quantize_fixed_scale(x, po2, off, 0.0375)
    assert torch.equal(pr2, po2)
    dr = ref.dequantize_page(pr, off, T, sr)
    do = ours.dequantize_page(po, off, T, so)
    assert torch.equal(dr, do)


@pytest.mark.parametrize("seed,T,off", [(5, 16, 0), (6, 9, 4), (7, 1, 0)])
def test_int4_ops_match_reference(seed, T, off):
    import oracle as O

    ref, ours = _ref(), _ours()
    H, D, P = 4, 64, 16
    x = _inputs(seed, T, H, D).cuda()
    pr = torch.zeros(P, H, D // 2, dtype=torch.uint8, device="cuda")
    po = torch.zeros_like(pr)
    sr = ref.quantize_int4_new_scale(x, pr, off)
    so = ours.quantize_int4_new_scale(x, po, off)
    assert sr == so
    assert torch.equal(pr, po)
    packed, s_orc = O.quantize_int4(x.cpu().numpy())
    assert s_orc == sr
    np.testing.assert_array_equal(pr[off:off + T].cpu().numpy(), packed)
    assert torch.equal(ref.dequantize_int4_page(pr, off, T, sr), ours.dequantize_int4_page(po, off, T, so))


@pytest.mark.parametrize("hq,hkv,pages,P", [(12, 12, 9, 16), (8, 2, 5, 16), (4, 4, 3, 8), (16, 4, 33, 32)])
def test_paged_attention_committed_matches_reference(hq, hkv, pages, P):
    ref, ours = _ref(), _ours()
    D = 64
    g = torch.Generator().manual_seed(100 + pages)
    n_phys = pages + 7
    k_store = torch.randint(-127, 128, (n_phys, P, hkv, D), generator=g, dtype=torch.int8).cuda()
    v_store = torch.randint(-127, 128, (n_phys, P, hkv, D), generator=g, dtype=torch.int8).cuda()
    sk = (torch.rand(n_phys, generator=g) * 0.05 + 0.005).cuda()
    sv = (torch.rand(n_phys, generator=g) * 0.05 + 0.005).cuda()
    bt = torch.randperm(n_phys, generator=g)[:pages].to(torch.int32).cuda()
    q = torch.randn(hq, D, generator=g).cuda()
    scale = 1.0 / D ** 0.5
    wr, lr, mr = ref.paged_attention_committed(q, k_store, v_store, sk, sv, bt, scale)
    wo, lo, mo = ours.paged_attention_committed(q, k_store, v_store, sk, sv, bt, scale)
    torch.cuda.synchronize()
    np.testing.assert_allclose(mo.cpu().numpy(), mr.cpu().numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lo.cpu().numpy(), lr.cpu().numpy(), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(wo.cpu().numpy(), wr.cpu().numpy(), rtol=1e-4, atol=1e-4)
    # the normalised outputs, which are what a caller uses
    np.testing.assert_allclose((wo / lo[:, None]).cpu().numpy(), (wr / lr[:, None]).cpu().numpy(), atol=2e-5)


@pytest.mark.parametrize("kv", ["int8", "int4"])
def test_token_head_commit_matches_reference_per_vector(kv):
    """Pages committed with one scale per (token, head): every D-vector's codes /
    nibbles and fp32 scale equal the reference's own quantize op run on that
    [1, 1, D] slice (NaN, zero and outlier elements included)."""
    from metagross_b200.batched import BatchedPagedKVCache

    ref = _ref()
    H, D, P = 4, 64, 16
    x = _inputs(41, 2 * P, H, D, special=True)
    x[3, 1] = 0.0  # an all-zero vector: scale 1e-8
    y = _inputs(42, 2 * P, H, D) * 0.5
    cache = BatchedPagedKVCache(1, 1, H, D, page_size=P, num_pages=4, max_blocks=4, kv_dtype=kv,
                                staging_dtype=torch.float32, scale_granularity="token_head")
    cache.begin_step(torch.tensor([2 * P], dtype=torch.int32))
    cache.append(0, x[None].cuda(), y[None].cuda())
    cache.check()
    bt = cache.block_tables[0, :2].cpu().tolist()
    for src, pool, scales in ((x, cache.k_pool[0], cache.k_scales[0]), (y, cache.v_pool[0], cache.v_scales[0])):
        for j, page in enumerate(bt):
            for t in range(P):
                for h in range(H):
                    sl = src[j * P + t:j * P + t + 1, h:h + 1].contiguous().cuda()
                    if kv == "int8":
                        buf = torch.zeros(1, 1, D, dtype=torch.int8, device="cuda")
                        s = ref.quantize_new_scale(sl, buf, 0)
                    else:
                        buf = torch.zeros(1, 1, D // 2, dtype=torch.uint8, device="cuda")
                        s = ref.quantize_int4_new_scale(sl, buf, 0)
                    assert np.float32(s) == scales[page, t, h].item(), (page, t, h)
                    assert torch.equal(buf[0, 0], pool[page, t, h]), (page, t, h)
