"""Reference-API attention (``paged_attention`` and ``_C.paged_attention_committed``)
against the oracle's dequantize-then-attend (float64), ported from the
reference's tests/test_attention.py, tests/test_cuda_stress.py and
tests/test_edge_cases.py.

Inputs here are fp32 (the reference API), so the kernel runs in its split
(hi+lo fp16) mode; tolerances are the reference's own: 1e-3 for N(0,1) data,
5e-3 for the x3 stress data, 1e-4 for the exact staging-only path.
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

BASE_SEED = 20260822
N_TRIALS = 25


def _rng(off):
    return torch.Generator().manual_seed(BASE_SEED + off)


def _randn(g, *shape, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).cuda()


def _modules():
    from metagross_b200 import _C
    from metagross_b200.attention import paged_attention
    from metagross_b200.cache import LayerKVCache, PagedKVCache

    return _C, paged_attention, LayerKVCache, PagedKVCache


def _oracle_attention(cache, layer, q, scale):
    """Dequantize-then-attend in float64 from the cache's own state (codes via the oracle)."""
    kc, vc = cache.k_layers[layer], cache.v_layers[layer]

    def seq(lc):
        parts = [O.dequantize_int8(lc.storage[p].cpu().numpy(), 0, lc.page_size, lc.page_scales[p])
                 for p in lc.block_table]
        if lc._staging:
            parts.append(torch.stack(lc._staging).float().cpu().numpy())
        return np.concatenate(parts)

    return O.attention(q.double().cpu().numpy(), seq(kc), seq(vc), scale)


def _check_cache_codes_against_oracle(lc, inputs):
    """Every committed page's codes and scale equal the oracle quantizing the same tokens."""
    P = lc.page_size
    for j, p in enumerate(lc.block_table):
        ref, s = O.quantize_int8(inputs[j * P:(j + 1) * P].cpu().numpy())
        assert lc.page_scales[p] == s
        np.testing.assert_array_equal(lc.storage[p].cpu().numpy(), ref)


def test_committed_kernel_matches_oracle():
    C, _, _, PagedKVCache = _modules()
    torch.manual_seed(0)
    h, d, P, npages = 4, 64, 16, 3
    k, v = torch.randn(npages * P, h, d, device="cuda"), torch.randn(npages * P, h, d, device="cuda")
    cache = PagedKVCache(num_layers=1, num_heads=h, head_dim=d, page_size=P, max_pages=npages, device="cuda")
    cache.append(0, k, v)
    kc, vc = cache.k_layers[0], cache.v_layers[0]
    assert kc.block_table == [2, 1, 0] and not kc._staging
    _check_cache_codes_against_oracle(kc, k)
    _check_cache_codes_against_oracle(vc, v)
    q = torch.randn(h, d, device="cuda")
    sc = 1.0 / d ** 0.5
    bt = torch.tensor(kc.block_table, dtype=torch.int32, device="cuda")
    sk = torch.tensor([s if s is not None else 0.0 for s in kc.page_scales], device="cuda")
    sv = torch.tensor([s if s is not None else 0.0 for s in vc.page_scales], device="cuda")
    wv, l, m = C.paged_attention_committed(q, kc.storage, vc.storage, sk, sv, bt, sc)
    ref_k = np.concatenate([O.dequantize_int8(kc.storage[p].cpu().numpy(), 0, P, kc.page_scales[p])
                            for p in kc.block_table])
    ref_v = np.concatenate([O.dequantize_int8(vc.storage[p].cpu().numpy(), 0, P, vc.page_scales[p])
                            for p in kc.block_table])
    rwv, rl, rm = O.attention_unnormalized(q.double().cpu().numpy(), ref_k, ref_v, sc)
    np.testing.assert_allclose(m.cpu().numpy(), rm, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(l.cpu().numpy(), rl, rtol=1e-4)
    np.testing.assert_allclose((wv / l.unsqueeze(-1)).cpu().numpy(), rwv / rl[:, None], atol=1e-3, rtol=1e-3)


def test_committed_kernel_no_pages_is_identity():
    C, _, _, _ = _modules()
    st = torch.zeros(2, 16, 4, 64, dtype=torch.int8, device="cuda")
    sc = torch.ones(2, device="cuda")
    wv, l, m = C.paged_attention_committed(torch.randn(4, 64, device="cuda"), st, st, sc, sc,
                                           torch.empty(0, dtype=torch.int32, device="cuda"), 0.125)
    assert (wv == 0).all() and (l == 0).all() and torch.isinf(m).all() and (m < 0).all()


@pytest.mark.parametrize("committed,staged", [(16, 5), (0, 5), (32, 0), (48, 15)])
def test_paged_attention_mixed(committed, staged):
    _, paged_attention, _, PagedKVCache = _modules()
    torch.manual_seed(4 + committed + staged)
    h, d, P = 4, 64, 16
    k = torch.randn(committed + staged, h, d, device="cuda")
    v = torch.randn(committed + staged, h, d, device="cuda")
    cache = PagedKVCache(num_layers=1, num_heads=h, head_dim=d, page_size=P, max_pages=4, device="cuda")
    cache.append(0, k, v)
    q = torch.randn(h, d, device="cuda")
    got = paged_attention(cache, 0, q)
    ref = _oracle_attention(cache, 0, q, 1.0 / d ** 0.5)
    tol = 1e-4 if committed == 0 else 1e-3
    np.testing.assert_allclose(got.cpu().numpy(), ref, atol=tol, rtol=tol)


@pytest.mark.parametrize("hq,hkv", [(8, 8), (8, 4), (16, 4), (32, 4), (32, 8), (6, 3), (7, 1)])
def test_gqa_ratios(hq, hkv):
    _, paged_attention, _, PagedKVCache = _modules()
    g = _rng(hq * 100 + hkv)
    d, P = 64, 16
    k, v = _randn(g, 2 * P + 5, hkv, d), _randn(g, 2 * P + 5, hkv, d)
    cache = PagedKVCache(num_layers=1, num_heads=hkv, head_dim=d, page_size=P, max_pages=4, device="cuda")
    cache.append(0, k, v)
    q = _randn(g, hq, d)
    got = paged_attention(cache, 0, q)
    assert got.shape == (hq, d)
    np.testing.assert_allclose(got.cpu().numpy(), _oracle_attention(cache, 0, q, 1.0 / 8), atol=1e-3, rtol=1e-3)


def test_invalid_gqa_ratio_rejected():
    C, paged_attention, _, PagedKVCache = _modules()
    cache = PagedKVCache(num_layers=1, num_heads=4, head_dim=64, page_size=16, max_pages=2, device="cuda")
    cache.append(0, torch.randn(16, 4, 64, device="cuda"), torch.randn(16, 4, 64, device="cuda"))
    with pytest.raises(ValueError):
        paged_attention(cache, 0, torch.randn(7, 64, device="cuda"))
    kc, vc = cache.k_layers[0], cache.v_layers[0]
    bt = torch.tensor(kc.block_table, dtype=torch.int32, device="cuda")
    s = torch.ones(2, device="cuda")
    with pytest.raises(RuntimeError):
        C.paged_attention_committed(torch.randn(7, 64, device="cuda"), kc.storage, vc.storage, s, s, bt, 0.125)


@pytest.mark.parametrize("trial", range(N_TRIALS))
def test_random_shapes(trial):
    _, paged_attention, _, PagedKVCache = _modules()
    g = _rng(3000 + trial)
    d = 64
    hkv = int(torch.randint(1, 5, (1,), generator=g))
    P = int(torch.randint(1, 17, (1,), generator=g))
    npg = int(torch.randint(0, 4, (1,), generator=g))
    st = int(torch.randint(0, P, (1,), generator=g))
    n = npg * P + st
    if n == 0:
        pytest.skip("empty draw")
    cache = PagedKVCache(num_layers=1, num_heads=hkv, head_dim=d, page_size=P, max_pages=npg + 2, device="cuda")
    cache.append(0, _randn(g, n, hkv, d, scale=3.0), _randn(g, n, hkv, d, scale=3.0))
    q = _randn(g, hkv, d)
    got = paged_attention(cache, 0, q)
    assert torch.isfinite(got).all()
    np.testing.assert_allclose(got.cpu().numpy(), _oracle_attention(cache, 0, q, 1.0 / 8), atol=5e-3, rtol=5e-3)


@pytest.mark.parametrize("trial", range(N_TRIALS))
def test_random_gqa(trial):
    _, paged_attention, _, PagedKVCache = _modules()
    g = _rng(4000 + trial)
    hkv = [1, 2, 4, 8][int(torch.randint(0, 4, (1,), generator=g))]
    rep = int(torch.randint(1, 9, (1,), generator=g))
    n = int(torch.randint(1, 3, (1,), generator=g)) * 16
    cache = PagedKVCache(num_layers=1, num_heads=hkv, head_dim=64, page_size=16, max_pages=n // 16 + 1, device="cuda")
    cache.append(0, _randn(g, n, hkv, 64, scale=3.0), _randn(g, n, hkv, 64, scale=3.0))
    q = _randn(g, hkv * rep, 64)
    got = paged_attention(cache, 0, q)
    np.testing.assert_allclose(got.cpu().numpy(), _oracle_attention(cache, 0, q, 1.0 / 8), atol=5e-3, rtol=5e-3)


@pytest.mark.parametrize("trial", range(N_TRIALS))
def test_staging_only(trial):
    _, paged_attention, _, PagedKVCache = _modules()
    g = _rng(6000 + trial)
    n = int(torch.randint(1, 16, (1,), generator=g))
    cache = PagedKVCache(num_layers=1, num_heads=4, head_dim=64, page_size=16, max_pages=2, device="cuda")
    k, v = _randn(g, n, 4, 64, scale=3.0), _randn(g, n, 4, 64, scale=3.0)
    cache.append(0, k, v)
    q = _randn(g, 4, 64)
    got = paged_attention(cache, 0, q)
    ref = O.attention(q.double().cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), 1.0 / 8)
    np.testing.assert_allclose(got.cpu().numpy(), ref, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("trial", range(N_TRIALS))
def test_shuffled_block_table(trial):
    C, _, _, PagedKVCache = _modules()
    g = _rng(7000 + trial)
    d, h, P, npg = 64, 4, 16, 4
    cache = PagedKVCache(num_layers=1, num_heads=h, head_dim=d, page_size=P, max_pages=npg, device="cuda")
    for _ in range(npg):
        cache.append(0, _randn(g, P, h, d, scale=3.0), _randn(g, P, h, d, scale=3.0))
    kc, vc = cache.k_layers[0], cache.v_layers[0]
    perm = torch.randperm(npg, generator=g).tolist()
    shuffled = [kc.block_table[i] for i in perm]
    q = _randn(g, h, d)
    sk = torch.tensor([s for s in kc.page_scales], device="cuda")
    sv = torch.tensor([s for s in vc.page_scales], device="cuda")
    wv, l, _ = C.paged_attention_committed(q, kc.storage, vc.storage, sk, sv,
                                           torch.tensor(shuffled, dtype=torch.int32, device="cuda"), 1.0 / 8)
    rk = np.concatenate([O.dequantize_int8(kc.storage[p].cpu().numpy(), 0, P, kc.page_scales[p]) for p in shuffled])
    rv = np.concatenate([O.dequantize_int8(vc.storage[p].cpu().numpy(), 0, P, vc.page_scales[p]) for p in shuffled])
    ref = O.attention(q.double().cpu().numpy(), rk, rv, 1.0 / 8)
    np.testing.assert_allclose((wv / l.unsqueeze(-1)).cpu().numpy(), ref, atol=5e-3, rtol=5e-3)


def test_exact_quantization_kat_attention():
    C, _, _, PagedKVCache = _modules()
    for trial in range(5):
        g = _rng(7100 + trial)
        d, h, P, npg = 64, 4, 16, 4
        cache = PagedKVCache(num_layers=1, num_heads=h, head_dim=d, page_size=P, max_pages=npg, device="cuda")
        ks, vs = [], []
        for _ in range(npg):
            k = torch.randint(-127, 128, (P, h, d), generator=g).float()
            v = torch.randint(-127, 128, (P, h, d), generator=g).float()
            k[0, 0, 0] = 127.0
            v[0, 0, 0] = 127.0
            cache.append(0, k.cuda(), v.cuda())
            ks.append(k)
            vs.append(v)
        kc, vc = cache.k_layers[0], cache.v_layers[0]
        assert all(kc.page_scales[p] == 1.0 for p in kc.block_table)
        perm = torch.randperm(npg, generator=g).tolist()
        bt = torch.tensor([kc.block_table[i] for i in perm], dtype=torch.int32, device="cuda")
        q = _randn(g, h, d)
        one = torch.ones(npg, device="cuda")
        wv, l, _ = C.paged_attention_committed(q, kc.storage, vc.storage, one, one, bt, 1.0 / 8)
        ref = O.attention(q.double().cpu().numpy(), torch.cat([ks[i] for i in perm]).numpy(),
                          torch.cat([vs[i] for i in perm]).numpy(), 1.0 / 8)
        np.testing.assert_allclose((wv / l.unsqueeze(-1)).cpu().numpy(), ref, atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("P", [4, 16])
@pytest.mark.parametrize("n", [1, 2, 15, 16, 17, 31, 32, 33, 47, 48, 49, 63, 64, 65])
def test_page_boundaries(P, n):
    _, paged_attention, LayerKVCache, PagedKVCache = _modules()
    g = _rng(n * 10 + P)
    lc = LayerKVCache(num_heads=2, head_dim=8, page_size=P, max_pages=n // P + 2, device="cuda")
    x = _randn(g, n, 2, 8)
    lc.append(x)
    assert lc.seq_len == n and len(lc.block_table) == n // P and len(lc._staging) == n % P
    _check_cache_codes_against_oracle(lc, x)
    out = lc.read_fp32()
    assert out.shape[0] == n
    torch.testing.assert_close(out[(n // P) * P:], x[(n // P) * P:], atol=0, rtol=0)
    # attention at head_dim 64 across the same boundary
    cache = PagedKVCache(num_layers=1, num_heads=2, head_dim=64, page_size=P, max_pages=n // P + 2, device="cuda")
    cache.append(0, _randn(g, n, 2, 64), _randn(g, n, 2, 64))
    q = _randn(g, 4, 64)
    np.testing.assert_allclose(paged_attention(cache, 0, q).cpu().numpy(), _oracle_attention(cache, 0, q, 0.125),
                               atol=1e-3, rtol=1e-3)


def test_incremental_equals_one_shot_and_exhaustion():
    _, _, LayerKVCache, _ = _modules()
    x = torch.randn(20, 4, 8, device="cuda")
    a = LayerKVCache(num_heads=4, head_dim=8, page_size=16, max_pages=4, device="cuda")
    a.append(x)
    b = LayerKVCache(num_heads=4, head_dim=8, page_size=16, max_pages=4, device="cuda")
    for i in range(20):
        b.append(x[i:i + 1])
    assert a.block_table == b.block_table == [3]
    assert a.page_scales[3] == b.page_scales[3]
    assert torch.equal(a.storage, b.storage)
    c = LayerKVCache(num_heads=4, head_dim=8, page_size=16, max_pages=1, device="cuda")
    with pytest.raises(RuntimeError):
        c.append(torch.randn(32, 4, 8, device="cuda"))


def test_kernel_shape_validation():
    C, _, _, PagedKVCache = _modules()

    def args(h=4, d=64, P=16, mp=2):
        cache = PagedKVCache(num_layers=1, num_heads=h, head_dim=d, page_size=P, max_pages=mp, device="cuda")
        cache.append(0, torch.randn(P, h, d, device="cuda"), torch.randn(P, h, d, device="cuda"))
        kc, vc = cache.k_layers[0], cache.v_layers[0]
        return (torch.randn(h, d, device="cuda"), kc.storage, vc.storage,
                torch.tensor([s or 0.0 for s in kc.page_scales], device="cuda"),
                torch.tensor([s or 0.0 for s in vc.page_scales], device="cuda"),
                torch.tensor(kc.block_table, dtype=torch.int32, device="cuda"), 0.125)

    a = args()
    assert torch.isfinite(C.paged_attention_committed(*a)[0]).all()
    bad = [
        (a[0].reshape(-1),) + a[1:],
        (torch.randn(4, 32, device="cuda"),) + a[1:],
        a[:2] + (a[2][:1],) + a[3:],
        a[:2] + (torch.zeros(2, 16, 8, 64, dtype=torch.int8, device="cuda"),) + a[3:],
        a[:2] + (torch.zeros(2, 4, 4, 64, dtype=torch.int8, device="cuda"),) + a[3:],
        a[:5] + (torch.tensor([-1], dtype=torch.int32, device="cuda"), 0.125),
        a[:5] + (torch.tensor([2], dtype=torch.int32, device="cuda"), 0.125),
        a[:5] + (torch.tensor([999], dtype=torch.int32, device="cuda"), 0.125),
    ] + [a[:6] + (s,) for s in [0.0, -1.0, float("nan"), float("inf"), float("-inf")]]
    for b in bad:
        with pytest.raises(RuntimeError):
            C.paged_attention_committed(*b)
    # page_size 128 rejected, 4 and 16 accepted (reference limits)
    with pytest.raises(RuntimeError):
        C.paged_attention_committed(*args(P=128, mp=1))
    for P in (4, 16):
        wv, l, _ = C.paged_attention_committed(*args(P=P))
        assert torch.isfinite(wv).all() and (l > 0).all()
    # non-contiguous storage rejected, non-contiguous query accepted
    ks = a[1]
    wide = torch.zeros(*ks.shape[:-1], 65, dtype=torch.int8, device="cuda")
    wide[..., :64] = ks
    with pytest.raises(RuntimeError):
        C.paged_attention_committed(a[0], wide[..., :64], a[2], a[3], a[4], a[5], 0.125)
    qt = torch.randn(64, 4, device="cuda").t()
    assert torch.isfinite(C.paged_attention_committed(qt, *a[1:])[0]).all()


@pytest.mark.parametrize("good", [1.0, 0.125, 1e-6, 1e6])
def test_paged_attention_accepts_valid_scale(good):
    _, paged_attention, _, PagedKVCache = _modules()
    cache = PagedKVCache(num_layers=1, num_heads=4, head_dim=64, page_size=16, max_pages=2, device="cuda")
    cache.append(0, torch.randn(16, 4, 64, device="cuda"), torch.randn(16, 4, 64, device="cuda"))
    assert torch.isfinite(paged_attention(cache, 0, torch.randn(4, 64, device="cuda"), scale=good)).all()


def test_long_context_beyond_reference_cap():
    """The reference kernel stops at 4096 tokens; the split kernel does not."""
    _, paged_attention, _, PagedKVCache = _modules()
    g = _rng(99)
    n = 5000
    cache = PagedKVCache(num_layers=1, num_heads=2, head_dim=64, page_size=16, max_pages=n // 16 + 1, device="cuda")
    cache.append(0, _randn(g, n, 2, 64), _randn(g, n, 2, 64))
    q = _randn(g, 8, 64)
    np.testing.assert_allclose(paged_attention(cache, 0, q).cpu().numpy(), _oracle_attention(cache, 0, q, 0.125),
                               atol=1e-3, rtol=1e-3)
