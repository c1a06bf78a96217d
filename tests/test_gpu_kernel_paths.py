"""Both decode-attention kernels on the layouts either can serve.

16-token pages with page scales and fp16 staged tails run the bulk-copy
kernel: with its producer's bulk copies for INT8 pools, in its self-copying
mode (consumer warps copy their own tiles) for INT4 pools
(metagross_b200/csrc/mg_attention.cu, tma_mode).  The environment variable
METAGROSS_B200_ATTENTION forces a path: ``registers`` (the
register-streaming kernel), ``bulk`` (bulk copies for INT4 pools too);
``self`` is the default behaviour.  Each case here runs under each and is compared
with the oracle's float64 dequantize-then-attend path (|out - ref| <= 2e-3 +
2^-11 |ref|), and the kernels' outputs with each other.
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def _cache_cls():
    from metagross_b200.batched import BatchedPagedKVCache

    return BatchedPagedKVCache


CASES = {
    # name: (kv, B, hq, hkv, lens)
    "int8_mha_tails": ("int8", 6, 12, 12, [1, 16, 17, 100, 255, 1023]),
    "int8_gqa8": ("int8", 5, 32, 4, [128, 600, 16, 33, 1500]),
    "int4_gqa8": ("int4", 5, 32, 4, [128, 600, 16, 33, 1500]),
    "int4_mha": ("int4", 4, 8, 8, [5, 64, 300, 901]),
    "int8_group16": ("int8", 3, 32, 2, [40, 700, 1200]),
}


def _build(kv, B, hq, hkv, lens, seed):
    P, D = 16, 64
    g = torch.Generator().manual_seed(seed)
    mb = max(lens) // P + 2
    cache = _cache_cls()(1, B, hkv, D, page_size=P, num_pages=B * mb, max_blocks=mb, kv_dtype=kv)
    model = O.PagedCacheModel(B, B * mb, P, hkv, D, kv_dtype=kv, staging_dtype=np.float16, max_blocks=mb)
    T = max(lens)
    k = torch.randn(B, T, hkv, D, generator=g)
    v = torch.randn(B, T, hkv, D, generator=g)
    k[torch.rand(k.shape, generator=g) < 0.01] *= 8
    k, v = k.half(), v.half()
    n = torch.tensor(lens, dtype=torch.int32)
    cache.begin_step(n)
    cache.append(0, k.cuda(), v.cuda())
    model.append(k.numpy(), v.numpy(), n.numpy())
    q = torch.randn(B, hq, D, generator=g).half()
    return cache, model, q


@pytest.mark.parametrize("case", sorted(CASES))
def test_both_kernels_match_the_oracle_and_each_other(case, monkeypatch):
    kv, B, hq, hkv, lens = CASES[case]
    cache, model, q = _build(kv, B, hq, hkv, lens, seed=sum(map(ord, case)))
    ref = model.attend(q.float().numpy(), 1.0 / 8)
    outs = {}
    for path in ("registers", "bulk", "self"):
        monkeypatch.setenv("METAGROSS_B200_ATTENTION", path)
        cache.invalidate_plan()
        out = cache.attend(0, q.cuda())
        torch.cuda.synchronize()
        cache.check()
        o = out.float().cpu().numpy()
        err = float((np.abs(o - ref) - np.abs(ref) * 2.0 ** -11).max())
        assert err < 2e-3, (path, err)
        outs[path] = o
    assert np.abs(outs["registers"] - outs["bulk"]).max() < 4e-3
    assert np.abs(outs["registers"] - outs["self"]).max() < 4e-3


def test_bulk_kernel_stream_k_int8():
    """More non-empty sequences than SMs on the bulk-copy kernel (INT8): CTAs
    hold several segments, and cut sequences merge through the tickets."""
    rng = np.random.default_rng(7)
    B = 200
    lens = np.maximum(1, np.exp(rng.normal(np.log(300), 1.0, B)).round().astype(int)).clip(max=3000).tolist()
    lens[3] = 0
    cache, model, q = _build("int8", B, 12, 12, lens, seed=9)
    out = cache.attend(0, q.cuda())
    torch.cuda.synchronize()
    cache.check()
    assert int(cache._plan.view(torch.int32)[5].item()) == 2  # stream-K
    ref = model.attend(q.float().numpy(), 1.0 / 8)
    o = out.float().cpu().numpy()
    assert np.all(o[3] == 0.0)
    err = float((np.abs(o - ref) - np.abs(ref) * 2.0 ** -11).max())
    assert err < 2e-3, err


@pytest.mark.parametrize("case", ["int8_gqa8", "int4_gqa8", "int8_mha_tails"])
@pytest.mark.parametrize("path", ["registers", "bulk", "self"])
def test_settled_plan_launch_matches_the_plain_launch(case, path, monkeypatch):
    """MG_ATTN_PLAN_SETTLED moves the plan reads, and the copies of the pages
    that predate the step (or an L2 warm-up), before the wait on the previous
    launch; the outputs are the plain launch's bit for bit, with an append
    (which commits pages) right before."""
    from metagross_b200 import _C

    monkeypatch.setenv("METAGROSS_B200_ATTENTION", path)
    kv, B, hq, hkv, lens = CASES[case]
    cache, model, q = _build(kv, B, hq, hkv, lens, seed=5)
    g = torch.Generator().manual_seed(6)
    outs = []
    for settled in (False, True, False, True):
        # the step plan: it records each segment's pages that predate the step, which a settled
        # bulk-copy launch copies before its wait
        cache.begin_step(1, plan=True)
        kn = torch.randn(B, hkv, 64, generator=g).half()
        vn = torch.randn(B, hkv, 64, generator=g).half()
        cache.append(0, kn.cuda(), vn.cuda())
        model.append(kn.numpy()[:, None], vn.numpy()[:, None])
        qq = q.cuda()
        out = torch.empty_like(qq)
        _C.paged_decode_attention_planned(qq, cache.k_pool[0], cache.v_pool[0], cache.k_scales[0],
                                          cache.v_scales[0], cache.staging_k[0], cache.staging_v[0],
                                          cache.block_tables, cache._decode_plan(), 0.125,
                                          cache._workspace(hq, cache.max_blocks * cache.page_size), out,
                                          cache.status, settled=settled)
        torch.cuda.synchronize()
        cache.check()
        ref = model.attend(q.float().numpy(), 1.0 / 8)
        o = out.float().cpu().numpy()
        err = float((np.abs(o - ref) - np.abs(ref) * 2.0 ** -11).max())
        assert err < 2e-3, (settled, err)
        outs.append(out)
    # same inputs give the same outputs: re-run the last step's attention unsettled
    out2 = torch.empty_like(outs[-1])
    _C.paged_decode_attention_planned(q.cuda(), cache.k_pool[0], cache.v_pool[0], cache.k_scales[0],
                                      cache.v_scales[0], cache.staging_k[0], cache.staging_v[0], cache.block_tables,
                                      cache._decode_plan(), 0.125,
                                      cache._workspace(hq, cache.max_blocks * cache.page_size), out2, cache.status,
                                      settled=False)
    torch.cuda.synchronize()
    assert torch.equal(out2, outs[-1])


def test_self_copy_stream_k_int4(monkeypatch):
    """The self-copying mode in stream-K (CTAs over several segments, page-id
    windows refilled from the block table past the plan's first page ids),
    INT4 32 q / 4 kv heads, with an empty and tail-only sequences."""
    monkeypatch.setenv("METAGROSS_B200_ATTENTION", "self")
    rng = np.random.default_rng(11)
    B = 220
    lens = np.maximum(1, np.exp(rng.normal(np.log(400), 1.0, B)).round().astype(int)).clip(max=4200).tolist()
    lens[2] = 0
    lens[9] = 7
    lens[10] = 16 * 150 + 3
    cache, model, q = _build("int4", B, 32, 4, lens, seed=12)
    out = cache.attend(0, q.cuda())
    torch.cuda.synchronize()
    cache.check()
    assert int(cache._plan.view(torch.int32)[5].item()) == 2  # stream-K
    ref = model.attend(q.float().numpy(), 1.0 / 8)
    o = out.float().cpu().numpy()
    assert np.all(o[2] == 0.0)
    err = float((np.abs(o - ref) - np.abs(ref) * 2.0 ** -11).max())
    assert err < 2e-3, err
