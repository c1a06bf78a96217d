"""Decode attention against the oracle at the sizes the benchmarks run.

The small cases elsewhere never leave the plan's chunk mode (every non-empty
sequence on its own SMs).  These cases cover what the benchmarks exercise:

* stream-K mode: more non-empty sequences than SMs, log-normal contexts with
  one beyond 4096 tokens (the reference kernel's per-call cap,
  csrc/paged_attention.cu:212-216), empty and tail-only sequences, so CTAs
  straddle sequences and cut sequences merge through the per-(sequence, kv
  head) tickets;
* the TinyLlama-shape INT4 GQA batch at full size (B=64, contexts
  U[128, 2048], 1 % outliers x8);
* the GPT-2-shape INT8 batch at full size (B=32, 12 heads, 1024 tokens,
  physical pages shuffled through the allocator's free stack);
* the CUDA-graph decode step (DecodeGraph) replayed across page commits and
  an eager truncation, against the same steps run eagerly and the oracle.

Parity bar: |out - ref| <= 2e-3 + 2^-11 |ref| elementwise against the
float64 dequantize-then-attend oracle (tests/test_attention.py:14-20 of the
reference over read_fp32, with the log-sum-exp merge of
metagross/attention.py:15-26 for the staged tail).  2^-11 |ref| is the
rounding of an fp16 output itself: with 1 % of the K/V elements scaled by 8,
some outputs reach |16|, where fp16 values are 2^-6 apart, so no fp16 output
can be within a flat 2e-3 of them.  Cache state (codes, scales, block tables,
free list) bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _excess(out, ref):
    """max over elements of |out - ref| - 2^-11 |ref| (the fp16 rounding of ref)."""
    out = out.float().cpu().numpy() if isinstance(out, torch.Tensor) else out
    return float((np.abs(out - ref) - np.abs(ref) * 2.0 ** -11).max())


def _cache_cls():
    from metagross_b200.batched import BatchedPagedKVCache

    return BatchedPagedKVCache


def _plan_mode(cache):
    """Header word 5 of the step's decode plan: 1 chunk mode, 2 stream-K."""
    return int(cache._plan.view(torch.int32)[5].item())


def _fill_in_chunks(cache, model, lens, g, hkv, D, chunk=1024, outliers=0.0):
    """Append each sequence's lens[b] tokens in steps of at most `chunk` tokens
    per sequence (several begin_step/append calls, as a chunked prefill)."""
    lens = np.asarray(lens, dtype=np.int64)
    done = np.zeros_like(lens)
    while (done < lens).any():
        n = np.minimum(chunk, lens - done).astype(np.int32)
        T = int(n.max())
        k = torch.zeros(len(lens), T, hkv, D, dtype=torch.float16)
        v = torch.zeros_like(k)
        for b in np.flatnonzero(n):
            for t in (k, v):
                x = torch.randn(int(n[b]), hkv, D, generator=g)
                if outliers:
                    x[torch.rand(x.shape, generator=g) < outliers] *= 8
                t[b, :n[b]] = x.half()
        cache.begin_step(torch.from_numpy(n))
        cache.append(0, k.cuda(), v.cuda())
        model.append(k.numpy(), v.numpy(), n)
        done += n
    torch.cuda.synchronize()
    cache.check()


def _check_state(cache, model):
    np.testing.assert_array_equal(cache.seq_lens.cpu().numpy(), model.seq_lens)
    bt = cache.block_tables.cpu().numpy()
    kp, vp = cache.k_pool[0].cpu().numpy(), cache.v_pool[0].cpu().numpy()
    ks, vs = cache.k_scales[0].cpu().numpy(), cache.v_scales[0].cpu().numpy()
    for b in range(model.B):
        nb = int(model.num_blocks[b])
        np.testing.assert_array_equal(bt[b, :nb], model.block_tables[b, :nb])
    used = np.array(sorted({int(model.block_tables[b, j]) for b in range(model.B)
                            for j in range(int(model.num_blocks[b]))}), dtype=np.int64)
    if used.size:
        np.testing.assert_array_equal(kp[used], model.k_pool[used])
        np.testing.assert_array_equal(vp[used], model.v_pool[used])
        np.testing.assert_array_equal(ks[used], model.k_scales[used])
        np.testing.assert_array_equal(vs[used], model.v_scales[used])
    assert cache.allocator.free_list() == model.free_list


def test_stream_k_lognormal_int4_gqa_matches_oracle():
    """320 sequences (> 148 SMs): stream-K.  Log-normal contexts (median 1024,
    sigma 1) plus one of 9000 tokens, 12 empty, 10 tail-only (1..15 tokens) and
    some exact page multiples; INT4, 32 q / 4 kv heads."""
    B, hq, hkv, D, P = 320, 32, 4, 64, 16
    rng = np.random.default_rng(20260822)
    lens = np.minimum(np.exp(rng.normal(np.log(1024), 1.0, B)).round(), 8192).astype(np.int64)
    lens = np.maximum(lens, 1)
    lens[rng.choice(B, 12, replace=False)] = 0
    tail_only = rng.choice(np.flatnonzero(lens > 0), 10, replace=False)
    lens[tail_only] = rng.integers(1, 16, 10)
    lens[7] = 9000
    lens[11] = 4096
    lens[13] = 16 * 300
    pages = int(((lens + P - 1) // P).sum()) + 64
    mb = int(lens.max()) // P + 2
    cache = _cache_cls()(1, B, hkv, D, page_size=P, num_pages=pages, max_blocks=mb, kv_dtype="int4")
    model = O.PagedCacheModel(B, pages, P, hkv, D, kv_dtype="int4", staging_dtype=np.float16, max_blocks=mb)
    g = torch.Generator().manual_seed(20260822)
    _fill_in_chunks(cache, model, lens, g, hkv, D, chunk=2048)
    _check_state(cache, model)
    q = torch.randn(B, hq, D, generator=g).half()
    out = cache.attend(0, q.cuda())
    torch.cuda.synchronize()
    cache.check()
    assert _plan_mode(cache) == 2, "expected the stream-K partition"
    ref = model.attend(q.float().numpy(), 1.0 / 8)
    o = out.float().cpu().numpy()
    empty = lens == 0
    assert np.all(o[empty] == 0.0)
    err = (np.abs(o - ref) - np.abs(ref) * 2.0 ** -11).max(axis=(1, 2))
    assert err.max() < TOL, (int(err.argmax()), float(err.max()), int(lens[err.argmax()]))
    # a second call on the same plan: the merge tickets were left at zero
    out2 = cache.attend(0, q.cuda())
    torch.cuda.synchronize()
    assert torch.equal(out2, out)


def test_tinyllama_shape_int4_full_size_matches_oracle():
    """B=64, 32 q / 4 kv heads, contexts U[128, 2048], 1 % outliers x8, INT4."""
    B, hq, hkv, D, P = 64, 32, 4, 64, 16
    g = torch.Generator().manual_seed(3)
    lens = torch.randint(128, 2049, (B,), generator=g).numpy()
    pages = int(((lens + P - 1) // P).sum()) + 32
    cache = _cache_cls()(1, B, hkv, D, page_size=P, num_pages=pages, max_blocks=2048 // P + 1, kv_dtype="int4")
    model = O.PagedCacheModel(B, pages, P, hkv, D, kv_dtype="int4", staging_dtype=np.float16,
                              max_blocks=2048 // P + 1)
    _fill_in_chunks(cache, model, lens, g, hkv, D, chunk=2048, outliers=0.01)
    _check_state(cache, model)
    q = torch.randn(B, hq, D, generator=g).half()
    out = cache.attend(0, q.cuda())
    torch.cuda.synchronize()
    cache.check()
    assert _plan_mode(cache) == 1
    err = _excess(out, model.attend(q.float().numpy(), 1.0 / 8))
    assert err < TOL, err


def test_gpt2_shape_int8_full_size_matches_oracle():
    """B=32, 12 heads, 1024 tokens (64 committed pages, no tail), physical
    pages drawn from a shuffled free stack."""
    B, H, D, P, C = 32, 12, 64, 16, 1024
    g = torch.Generator().manual_seed(5)
    pages = B * C // P + 64
    cache = _cache_cls()(1, B, H, D, page_size=P, num_pages=pages, max_blocks=C // P + 4)
    model = O.PagedCacheModel(B, pages, P, H, D, staging_dtype=np.float16, max_blocks=C // P + 4)
    perm = torch.randperm(pages, generator=g).to(torch.int32)
    cache.allocator.free_stack.copy_(perm.cuda())
    model.free_list = perm.tolist()
    _fill_in_chunks(cache, model, np.full(B, C), g, H, D, chunk=C)
    _check_state(cache, model)
    q = torch.randn(B, H, D, generator=g).half()
    out = cache.attend(0, q.cuda())
    torch.cuda.synchronize()
    cache.check()
    err = _excess(out, model.attend(q.float().numpy(), 1.0 / 8))
    assert err < TOL, err
    # one more decode token per sequence: a staged tail of 1 row beside 64 pages
    k = torch.randn(B, 1, H, D, generator=g).half()
    v = torch.randn(B, 1, H, D, generator=g).half()
    cache.begin_step(1)
    cache.append(0, k.cuda(), v.cuda())
    model.append(k.numpy(), v.numpy())
    out = cache.attend(0, q.cuda())
    torch.cuda.synchronize()
    cache.check()
    err = _excess(out, model.attend(q.float().numpy(), 1.0 / 8))
    assert err < TOL, err


@pytest.mark.parametrize("kv", ["int8", "int4"])
def test_decode_graph_replays_match_eager_steps_and_oracle(kv):
    """24 replays of the captured decode step (2 layers, one token per
    sequence per step, contexts starting at 10..40 so every sequence commits
    at least one page on the way), with an eager truncation after replay 12;
    every step's outputs equal the eager steps' bit for bit and the oracle's
    within the bar, and the final pools, scales, block tables and free list
    are equal to both."""
    from metagross_b200.batched import DecodeGraph

    B, hq, hkv, D, P, Lyr = 6, 8, 4, 64, 16, 2
    g = torch.Generator().manual_seed(77)
    pages, mb = 64, 8
    mk = lambda: _cache_cls()(Lyr, B, hkv, D, page_size=P, num_pages=pages, max_blocks=mb, kv_dtype=kv)  # noqa: E731
    gc, ec = mk(), mk()
    models = [O.PagedCacheModel(B, pages, P, hkv, D, kv_dtype=kv, staging_dtype=np.float16, max_blocks=mb)
              for _ in range(Lyr)]
    lens = torch.randint(10, 41, (B,), generator=g, dtype=torch.int32)
    T = int(lens.max())
    for c in (gc, ec):
        c.begin_step(lens)
    for layer in range(Lyr):
        k = torch.randn(B, T, hkv, D, generator=g).half()
        v = torch.randn(B, T, hkv, D, generator=g).half()
        for c in (gc, ec):
            c.append(layer, k.cuda(), v.cuda())
        models[layer].append(k.numpy(), v.numpy(), lens.numpy())
    q = torch.zeros(Lyr, B, hq, D, dtype=torch.float16, device="cuda")
    kn = torch.zeros(Lyr, B, hkv, D, dtype=torch.float16, device="cuda")
    vn = torch.zeros_like(kn)
    out = torch.zeros_like(q)
    graph = DecodeGraph(gc, q, kn, vn, out, n_new=1)
    for step in range(24):
        qs = torch.randn(Lyr, B, hq, D, generator=g).half()
        ks = torch.randn(Lyr, B, hkv, D, generator=g).half()
        vs = torch.randn(Lyr, B, hkv, D, generator=g).half()
        q.copy_(qs.cuda())
        kn.copy_(ks.cuda())
        vn.copy_(vs.cuda())
        graph.replay()
        ec.begin_step(1)
        eager = []
        for layer in range(Lyr):
            ec.append(layer, ks[layer].cuda(), vs[layer].cuda())
            eager.append(ec.attend(layer, qs[layer].cuda()))
            models[layer].append(ks[layer].numpy()[:, None], vs[layer].numpy()[:, None])
        torch.cuda.synchronize()
        gc.check()
        ec.check()
        for layer in range(Lyr):
            assert torch.equal(out[layer], eager[layer]), (step, layer)
            ref = models[layer].attend(qs[layer].float().numpy(), 1.0 / 8)
            err = _excess(out[layer], ref)
            assert err < TOL, (step, layer, err)
        if step == 12:
            # eager truncation on both caches: a page boundary, inside the
            # staged tail, and to zero
            sl = gc.seq_lens.cpu().tolist()
            new = [(sl[0] // P - 1) * P, sl[1] - sl[1] % P + (sl[1] % P) // 2, 0, sl[3], sl[4], sl[5]]
            for c in (gc, ec):
                c.truncate(new)
            for m in models:
                for b, n in enumerate(new):
                    m.truncate(b, n)
    torch.cuda.synchronize()
    for layer in range(Lyr):
        for c in (gc, ec):
            np.testing.assert_array_equal(c.seq_lens.cpu().numpy(), models[layer].seq_lens)
            bt = c.block_tables.cpu().numpy()
            for b in range(B):
                nb = int(models[layer].num_blocks[b])
                np.testing.assert_array_equal(bt[b, :nb], models[layer].block_tables[b, :nb])
            used = sorted({int(models[layer].block_tables[b, j]) for b in range(B)
                           for j in range(int(models[layer].num_blocks[b]))})
            for p in used:
                np.testing.assert_array_equal(c.k_pool[layer, p].cpu().numpy(), models[layer].k_pool[p])
                np.testing.assert_array_equal(c.v_pool[layer, p].cpu().numpy(), models[layer].v_pool[p])
                assert c.k_scales[layer, p].item() == models[layer].k_scales[p]
                assert c.v_scales[layer, p].item() == models[layer].v_scales[p]
            assert c.allocator.free_list() == models[layer].free_list
