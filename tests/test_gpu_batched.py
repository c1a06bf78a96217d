"""Batched device-resident cache against the oracle's PagedCacheModel.

Bit-exact after every step: pools (INT8 codes / packed INT4 nibbles), page
scales, block tables (LIFO allocator order), sequence lengths, staged rows.
Attention: max-abs within 2e-3 of float64 dequantize-then-attend for fp16
outputs (the parity bar), 1e-3 for fp32.  The gather/dequantize kernel is
bit-exact against the oracle's dequantization.
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def _cache_cls():
    from metagross_b200.batched import BatchedPagedKVCache

    return BatchedPagedKVCache


def _assert_state_equal(cache, model, layer=0):
    np.testing.assert_array_equal(cache.seq_lens.cpu().numpy(), model.seq_lens)
    nb = model.num_blocks
    bt = cache.block_tables.cpu().numpy()
    for b in range(model.B):
        np.testing.assert_array_equal(bt[b, :nb[b]], model.block_tables[b, :nb[b]], err_msg=f"block table {b}")
    used = sorted({int(model.block_tables[b, j]) for b in range(model.B) for j in range(nb[b])})
    kp = cache.k_pool[layer].cpu().numpy()
    vp = cache.v_pool[layer].cpu().numpy()
    ks = cache.k_scales[layer].cpu().numpy()
    vs = cache.v_scales[layer].cpu().numpy()
    for p in used:
        np.testing.assert_array_equal(kp[p], model.k_pool[p], err_msg=f"k page {p}")
        np.testing.assert_array_equal(vp[p], model.v_pool[p], err_msg=f"v page {p}")
        assert ks[p] == model.k_scales[p] and vs[p] == model.v_scales[p]
    stk = cache.staging_k[layer].float().cpu().numpy()
    for b in range(model.B):
        r = len(model.staging_k[b])
        if r:
            np.testing.assert_array_equal(stk[b, :r], np.stack(model.staging_k[b]).astype(np.float32))
    assert cache.allocator.free_list() == model.free_list


@pytest.mark.parametrize("kv", ["int8", "int4"])
@pytest.mark.parametrize("P", [16, 4, 7])
def test_append_steps_bit_exact(kv, P):
    g = torch.Generator().manual_seed(11)
    B, H, D = 5, 3, 64
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=200, max_blocks=40, kv_dtype=kv,
                         staging_dtype=torch.float16)
    model = O.PagedCacheModel(B, 200, P, H, D, kv_dtype=kv, staging_dtype=np.float16, max_blocks=40)
    for step, T in enumerate([3, 1, 1, 17, 1, 40, 2, 1]):
        n_new = torch.randint(0, T + 1, (B,), generator=g, dtype=torch.int32)
        k = (torch.randn(B, T, H, D, generator=g) * 2).half()
        v = (torch.randn(B, T, H, D, generator=g) * 2).half()
        if step == 5:  # 1% outliers x8 as in the INT4 config
            k[torch.rand(k.shape, generator=g) < 0.01] *= 8
        cache.begin_step(n_new)
        cache.append(0, k.cuda(), v.cuda())
        model.append(k.numpy(), v.numpy(), n_new.numpy())
        cache.check()
        _assert_state_equal(cache, model)


def test_decode_attention_matches_oracle_fp16_int8_mha():
    g = torch.Generator().manual_seed(5)
    B, H, D, P = 6, 12, 64, 16
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=B * 20, max_blocks=20, staging_dtype=torch.float16)
    model = O.PagedCacheModel(B, B * 20, P, H, D, staging_dtype=np.float16, max_blocks=20)
    lens = torch.tensor([1, 16, 17, 100, 255, 300], dtype=torch.int32)
    k = torch.randn(B, 300, H, D, generator=g).half()
    v = torch.randn(B, 300, H, D, generator=g).half()
    cache.begin_step(lens)
    cache.append(0, k.cuda(), v.cuda())
    model.append(k.numpy(), v.numpy(), lens.numpy())
    _assert_state_equal(cache, model)
    for step in range(3):
        q = torch.randn(B, H, D, generator=g).half()
        out = cache.attend(0, q.cuda())
        cache.check()
        ref = model.attend(q.float().numpy(), 1.0 / 8)
        err = np.abs(out.float().cpu().numpy() - ref).max()
        assert err < 2e-3, err
        kn = torch.randn(B, 1, H, D, generator=g).half()
        vn = torch.randn(B, 1, H, D, generator=g).half()
        cache.begin_step(1)
        cache.append(0, kn.cuda(), vn.cuda())
        model.append(kn.numpy(), vn.numpy())


@pytest.mark.parametrize("kv", ["int8", "int4"])
@pytest.mark.parametrize("hq,hkv", [(32, 4), (8, 8), (12, 4), (16, 2), (32, 2)])
@pytest.mark.parametrize("qdt", [torch.float16, torch.float32])
def test_decode_attention_gqa(kv, hq, hkv, qdt):
    if qdt == torch.float32 and hq // hkv > 8:
        pytest.skip("fp32 q supports groups <= 8")
    g = torch.Generator().manual_seed(hq * 7 + hkv)
    B, D, P = 4, 64, 16
    cache = _cache_cls()(1, B, hkv, D, page_size=P, num_pages=B * 40, max_blocks=40, kv_dtype=kv,
                         staging_dtype=torch.float32 if qdt == torch.float32 else torch.float16)
    model = O.PagedCacheModel(B, B * 40, P, hkv, D, kv_dtype=kv, max_blocks=40)
    lens = torch.randint(128, 600, (B,), generator=g, dtype=torch.int32)
    k = torch.randn(B, 600, hkv, D, generator=g).to(qdt)
    v = torch.randn(B, 600, hkv, D, generator=g).to(qdt)
    out_mask = torch.rand(k.shape, generator=g) < 0.01
    k[out_mask] *= 8
    cache.begin_step(lens)
    cache.append(0, k.cuda(), v.cuda())
    model.append(k.float().numpy(), v.float().numpy(), lens.numpy())
    q = torch.randn(B, hq, D, generator=g).to(qdt)
    out = cache.attend(0, q.cuda())
    cache.check()
    ref = model.attend(q.float().numpy(), 1.0 / 8)
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err < (2e-3 if qdt == torch.float16 else 1e-3), err


@pytest.mark.parametrize("kv", ["int8", "int4"])
def test_gather_dequant_bit_exact(kv):
    g = torch.Generator().manual_seed(3)
    B, H, D, P = 4, 4, 64, 16
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=64, max_blocks=16, kv_dtype=kv,
                         staging_dtype=torch.float16)
    model = O.PagedCacheModel(B, 64, P, H, D, kv_dtype=kv, staging_dtype=np.float16, max_blocks=16)
    lens = torch.tensor([0, 5, 16, 77], dtype=torch.int32)
    k = torch.randn(B, 77, H, D, generator=g).half()
    v = torch.randn(B, 77, H, D, generator=g).half()
    cache.begin_step(lens)
    cache.append(0, k.cuda(), v.cuda())
    model.append(k.numpy(), v.numpy(), lens.numpy())
    ok, ov, cu = cache.gather(0, dtype=torch.float32)
    for b in range(B):
        sl = slice(int(cu[b]), int(cu[b + 1]))
        np.testing.assert_array_equal(ok[sl].cpu().numpy(), model.dequantized_sequence(b, "k"))
        np.testing.assert_array_equal(ov[sl].cpu().numpy(), model.dequantized_sequence(b, "v"))


def test_free_and_reuse_is_lifo():
    B, H, D, P = 3, 2, 64, 16
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=12, max_blocks=8)
    model = O.PagedCacheModel(B, 12, P, H, D, staging_dtype=np.float16, max_blocks=8)
    g = torch.Generator().manual_seed(1)
    lens = torch.tensor([33, 50, 20], dtype=torch.int32)
    k = torch.randn(B, 50, H, D, generator=g).half()
    cache.begin_step(lens)
    cache.append(0, k.cuda(), k.cuda())
    model.append(k.numpy(), k.numpy(), lens.numpy())
    cache.free([1, 0])
    model.free_sequence(1)
    model.free_sequence(0)
    assert cache.allocator.free_list() == model.free_list
    lens2 = torch.tensor([40, 17, 0], dtype=torch.int32)
    cache.begin_step(lens2)
    cache.append(0, k.cuda(), k.cuda())
    model.append(k.numpy(), k.numpy(), lens2.numpy())
    cache.check()
    _assert_state_equal(cache, model)


@pytest.mark.parametrize("order", [[2, 0, 1], [1, 2, 1], [0, 5, 2]])
def test_free_many_sequences_lifo_order(order):
    """Several sequences freed in one call, in list order then block-table order,
    as the reference allocator would receive them: distinct ids (the parallel
    walk), a repeated id (the sequential walk; the second entry frees nothing)
    and an id out of range (flagged and skipped)."""
    B, H, D, P = 3, 2, 64, 16
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=24, max_blocks=8)
    model = O.PagedCacheModel(B, 24, P, H, D, staging_dtype=np.float16, max_blocks=8)
    g = torch.Generator().manual_seed(2)
    lens = torch.tensor([70, 33, 100], dtype=torch.int32)
    k = torch.randn(B, 100, H, D, generator=g).half()
    cache.begin_step(lens)
    cache.append(0, k.cuda(), k.cuda())
    model.append(k.numpy(), k.numpy(), lens.numpy())
    cache.free(order)
    for b in order:
        if b < B:
            model.free_sequence(b)
    assert cache.allocator.free_list() == model.free_list
    assert cache.seq_lens.tolist() == [int(x) for x in model.seq_lens]
    if max(order) >= B:
        with pytest.raises(RuntimeError, match="inconsistent per-sequence argument"):
            cache.check()
    else:
        cache.check()


def test_truncate_many_sequences_matches_oracle():
    B, H, D, P = 6, 2, 64, 16
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=64, max_blocks=10)
    model = O.PagedCacheModel(B, 64, P, H, D, staging_dtype=np.float16, max_blocks=10)
    g = torch.Generator().manual_seed(4)
    lens = torch.tensor([150, 16, 77, 130, 5, 64], dtype=torch.int32)
    k = torch.randn(B, 150, H, D, generator=g).half()
    cache.begin_step(lens)
    cache.append(0, k.cuda(), k.cuda())
    model.append(k.numpy(), k.numpy(), lens.numpy())
    ids, new = [5, 0, 3, 2], [32, 80, 128, 64]
    cache.truncate(torch.tensor(new, dtype=torch.int32), ids)
    for b, n in zip(ids, new):
        model.truncate(b, n)
    cache.check()
    assert cache.allocator.free_list() == model.free_list
    assert cache.seq_lens.tolist() == [int(x) for x in model.seq_lens]


def test_out_of_pages_is_all_or_nothing():
    B, H, D, P = 2, 2, 64, 16
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=3, max_blocks=8)
    k = torch.randn(B, 64, H, D).half().cuda()
    cache.begin_step(torch.tensor([32, 32], dtype=torch.int32))  # needs 4 pages, has 3
    cache.append(0, k, k)
    assert cache.seq_lens.tolist() == [0, 0]
    assert cache.allocator.num_free == 3
    with pytest.raises(RuntimeError, match="out of pages"):
        cache.check()


def test_negative_count_is_rejected_and_changes_nothing():
    B, H, D, P = 3, 2, 64, 16
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=8, max_blocks=4)
    k = torch.randn(B, 20, H, D).half().cuda()
    cache.begin_step(torch.tensor([20, -1, 5], dtype=torch.int32))
    cache.append(0, k, k)
    q = torch.randn(B, H, D).half().cuda()
    cache.attend(0, q)
    assert cache.seq_lens.tolist() == [0, 0, 0]
    assert cache.allocator.num_free == 8
    s = int(cache.status.item())
    assert s & 0x100 and not s & 0x10, hex(s)  # the cause is named, not reported as a full block-table row
    with pytest.raises(RuntimeError, match="negative length"):
        cache.check()


def test_double_free_flagged():
    cache = _cache_cls()(1, 2, 2, 64, page_size=16, num_pages=8, max_blocks=4)
    k = torch.randn(2, 16, 2, 64).half().cuda()
    cache.begin_step(16)
    cache.append(0, k, k)
    bt = cache.block_tables.clone()
    sl = cache.seq_lens.clone()
    cache.free([0])
    cache.seq_lens.copy_(sl)  # resurrect the length so the same page is freed again
    cache.block_tables.copy_(bt)
    cache.free([0])
    with pytest.raises(RuntimeError, match="double free"):
        cache.check()


def test_full_size_config2_properties():
    """Config-2 sizes (B=32, H=12, D=64, 1024 tokens, shuffled pool): the
    output of a constant-V cache is that constant, and attention is invariant
    to relabelling physical pages (permuting pool rows + block-table ids)."""
    B, H, D, P, C = 32, 12, 64, 16, 1024
    g = torch.Generator().manual_seed(2)
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=B * C // P + 64, max_blocks=C // P + 4)
    k = torch.randn(B, C, H, D, generator=g).half()
    v = torch.full((B, C, H, D), 0.75).half()
    cache.begin_step(C)
    cache.append(0, k.cuda(), v.cuda())
    q = torch.randn(B, H, D, generator=g).half().cuda()
    out = cache.attend(0, q)
    cache.check()
    assert torch.allclose(out.float(), torch.full_like(out.float(), 0.75), atol=1e-3)
    # relabel pages: new_pool[perm[p]] = pool[p], block ids mapped through perm
    v2 = torch.randn(B, C, H, D, generator=g).half()
    cache.reset()
    cache.begin_step(C)
    cache.append(0, k.cuda(), v2.cuda())
    out1 = cache.attend(0, q).float()
    perm = torch.randperm(cache.num_pages, generator=g).cuda()
    kp, vp = cache.k_pool[0].clone(), cache.v_pool[0].clone()
    ks, vs = cache.k_scales[0].clone(), cache.v_scales[0].clone()
    cache.k_pool[0][perm] = kp
    cache.v_pool[0][perm] = vp
    cache.k_scales[0][perm] = ks
    cache.v_scales[0][perm] = vs
    cache.block_tables.copy_(perm[cache.block_tables.long()].int())
    cache.invalidate_plan()  # the decode plan keeps a copy of the first block-table entries
    out2 = cache.attend(0, q).float()
    assert torch.equal(out1, out2)


def test_truncate_then_regrow_matches_oracle():
    """Truncation frees trailing pages in block-table order (LIFO reuse), keeps a
    staged-tail prefix, and later commits reuse the freed ids as the reference
    allocator would."""
    B, H, D, P = 3, 2, 64, 16
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=24, max_blocks=8)
    model = O.PagedCacheModel(B, 24, P, H, D, staging_dtype=np.float16, max_blocks=8)
    g = torch.Generator().manual_seed(4)
    k = torch.randn(B, 70, H, D, generator=g).half()
    v = torch.randn(B, 70, H, D, generator=g).half()
    lens = torch.tensor([70, 37, 48], dtype=torch.int32)
    cache.begin_step(lens)
    cache.append(0, k.cuda(), v.cuda())
    model.append(k.numpy(), v.numpy(), lens.numpy())
    new = [32, 36, 0]  # page boundary, inside the staged tail, everything
    cache.truncate(new)
    for b, n in enumerate(new):
        model.truncate(b, n)
    cache.check()
    _assert_state_equal(cache, model)
    k2 = torch.randn(B, 40, H, D, generator=g).half()
    grow = torch.tensor([40, 30, 17], dtype=torch.int32)
    cache.begin_step(grow)
    cache.append(0, k2.cuda(), k2.cuda())
    model.append(k2.numpy(), k2.numpy(), grow.numpy())
    cache.check()
    _assert_state_equal(cache, model)
    q = torch.randn(B, 4, D, generator=g).half()
    err = np.abs(cache.attend(0, q.cuda()).float().cpu().numpy() - model.attend(q.float().numpy(), 0.125)).max()
    assert err < 2e-3


def test_truncate_rejects_cutting_a_committed_page():
    cache = _cache_cls()(1, 1, 2, 64, page_size=16, num_pages=8, max_blocks=4)
    k = torch.randn(1, 40, 2, 64).half().cuda()
    cache.begin_step(40)
    cache.append(0, k, k)
    cache.truncate([20])  # inside committed page 1
    assert cache.seq_lens.tolist() == [40]
    with pytest.raises(RuntimeError, match="inconsistent"):
        cache.check()


@pytest.mark.parametrize("kv", ["int8", "int4"])
def test_append_rounds_half_integer_quotients_like_the_reference(kv):
    """Codes of values whose quotient x / s is exactly a half-integer (ties go
    away from zero, csrc/quantize.cu:51-57) or 2^-4 (INT8) / 2^-7 (INT4) beside
    one: each page has absmax = qmax, so s = 1 and x / s = x.  The append forms
    x / s as x * (1 / s) and must take the IEEE quotient at the ties."""
    qmax = 127 if kv == "int8" else 7
    B, H, D, P = 2, 2, 64, 16
    step = 2.0 ** -4 if kv == "int8" else 2.0 ** -7  # fp16 spacing near the largest halves used
    base = np.arange(-qmax, qmax) + 0.5  # every half-integer in range
    vals = np.concatenate([base, base + step, base - step])
    rng = np.random.default_rng(11)
    k = rng.choice(vals, size=(B, P, H, D)).astype(np.float16)
    v = rng.choice(vals, size=(B, P, H, D)).astype(np.float16)
    k[:, 0, 0, 0] = qmax  # absmax of every page = qmax -> scale exactly 1
    v[:, 0, 0, 0] = -qmax
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=8, max_blocks=4, kv_dtype=kv)
    model = O.PagedCacheModel(B, 8, P, H, D, kv_dtype=kv, staging_dtype=np.float16, max_blocks=4)
    cache.begin_step(P)
    cache.append(0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    model.append(k, v)
    torch.cuda.synchronize()
    cache.check()
    _assert_state_equal(cache, model)
    assert all(model.k_scales[int(model.block_tables[b, 0])] == 1.0 for b in range(B))


def _record_words(B, G):
    """Indices of the segment records' last word (r1.w) in a plan of batch B on G CTAs (plan_layout)."""
    off_offs = 16 + G
    off_recs = (off_offs + G + 7) // 8 * 8
    off_pids = off_recs + G * 4 * 8
    off_flat = off_pids + G * 128
    off_empty = off_flat + (B + G) * 8
    return list(range(off_recs + 7, off_pids, 8)) + list(range(off_flat + 7, off_empty, 8))


@pytest.mark.parametrize("case", ["grow", "out_of_pages", "prefill"])
def test_plan_step_equals_plan_append_then_plan(case):
    """mg_plan_step (allocation + decode plan in one launch) leaves the same
    lengths, block tables, free stack, status and plan words as mg_plan_append
    followed by mg_paged_decode_plan -- except each segment record's count of
    pages that predate the step (r1.w), which only the step plan knows:
    clamp((new length - n_new) // P - lo, 0, npg)."""
    B, H, D, P = 40, 4, 64, 16
    g = np.random.default_rng(3)
    caches = [_cache_cls()(1, B, H, D, page_size=P, num_pages=B * 70 if case != "out_of_pages" else 300,
                           max_blocks=70, kv_dtype="int4") for _ in range(2)]
    lens = torch.tensor(g.integers(0, 600, B), dtype=torch.int32)
    if case == "out_of_pages":
        lens = torch.tensor(g.integers(0, 120, B), dtype=torch.int32)
    for c in caches:
        c.begin_step(lens)
    steps = [torch.tensor(g.integers(0, 40, B), dtype=torch.int32)] if case != "grow" else [1] * 20
    if case == "out_of_pages":
        steps = [torch.full((B,), 200, dtype=torch.int32)]
    G = torch.cuda.get_device_properties(0).multi_processor_count
    wi = _record_words(B, G)
    for n in steps:
        a, b = caches
        a.begin_step(n)
        a._decode_plan()
        b.begin_step(n, plan=True)
        torch.cuda.synchronize()
        assert torch.equal(a.seq_lens, b.seq_lens)
        assert torch.equal(a.block_tables, b.block_tables)
        assert torch.equal(a.status, b.status)
        assert a.allocator.free_list() == b.allocator.free_list()
        wa = a._plan.view(torch.int32).cpu().numpy().copy()
        wb = b._plan.view(torch.int32).cpu().numpy().copy()
        assert np.all(wa[wi] == 0)
        nn = np.full(B, n) if isinstance(n, int) else n.numpy()
        lens_now = b.seq_lens.cpu().numpy()
        for w in wi:
            rec = wb[w - 7:w + 1]
            bb, lo, npg = int(rec[0]), int(rec[1]), int(rec[2])
            if npg == 0 and rec[3] == 0 and wb[w] == 0:
                continue  # unused or tail-only record
            # (after a refused step the lengths did not grow, and the count only comes out lower: still safe)
            add = int(nn[bb])
            old = lens_now[bb] - add if 0 <= add <= lens_now[bb] else -1
            expect = min(max(old // P - lo, 0), npg) if old >= 0 else 0
            assert wb[w] == expect, (w, rec)
        wb[wi] = 0
        assert np.array_equal(wa, wb)
    if case == "out_of_pages":
        assert int(caches[1].status.item()) & 0x1  # MG_DEV_OUT_OF_PAGES, nothing grew
        assert torch.equal(caches[1].seq_lens, lens.cuda())
