"""Host-side logic that needs no GPU: the reference's allocator tests
(tests/test_block_allocator.py of the reference), constructor and argument
validation of the cache and attention wrappers (tests/test_edge_cases.py of
the reference: ValueError from the wrappers), and the attention helpers
against the golden fixtures."""
import os

import numpy as np
import pytest
import torch

from metagross_b200.allocator import BlockAllocator
from metagross_b200.attention import _merge_unnormalized, _repeat_kv_heads, _staging_contribution, paged_attention
from metagross_b200.cache import LayerKVCache, PagedKVCache

GOLD = os.path.join(os.path.dirname(__file__), "golden")


# ---- allocator (reference tests/test_block_allocator.py) --------------------

def test_allocate_returns_distinct_pages():
    a = BlockAllocator(num_pages=4)
    assert {a.allocate() for _ in range(4)} == {0, 1, 2, 3}


def test_fresh_allocator_order_is_lifo_from_the_top():
    a = BlockAllocator(num_pages=5)
    assert [a.allocate() for _ in range(5)] == [4, 3, 2, 1, 0]


def test_allocate_raises_when_exhausted():
    a = BlockAllocator(num_pages=2)
    a.allocate()
    a.allocate()
    with pytest.raises(RuntimeError):
        a.allocate()


def test_free_makes_page_available_again():
    a = BlockAllocator(num_pages=1)
    p = a.allocate()
    with pytest.raises(RuntimeError):
        a.allocate()
    a.free(p)
    assert a.allocate() == p


def test_double_free_raises():
    a = BlockAllocator(num_pages=2)
    p = a.allocate()
    a.free(p)
    with pytest.raises(RuntimeError):
        a.free(p)


def test_free_out_of_range_raises():
    a = BlockAllocator(num_pages=2)
    with pytest.raises(ValueError):
        a.free(5)
    with pytest.raises(ValueError):
        a.free(-1)


def test_num_free_and_num_used_track_correctly():
    a = BlockAllocator(num_pages=3)
    assert (a.num_free, a.num_used) == (3, 0)
    p = a.allocate()
    assert (a.num_free, a.num_used) == (2, 1)
    a.free(p)
    assert (a.num_free, a.num_used) == (3, 0)


def test_zero_or_negative_num_pages_rejected():
    with pytest.raises(ValueError):
        BlockAllocator(num_pages=0)
    with pytest.raises(ValueError):
        BlockAllocator(num_pages=-1)


def test_allocator_matches_reference_script():
    z = np.load(os.path.join(GOLD, "allocator_script.npz"))
    for c in range(int(z["n"][0])):
        a = BlockAllocator(int(z[f"n{c}"][0]))
        for op, want in zip(z[f"ops{c}"], z[f"res{c}"]):
            op, want = int(op), int(want)
            if op == -1:
                try:
                    got = a.allocate()
                except RuntimeError:
                    got = -1
            else:
                try:
                    a.free(op)
                    got = op
                except RuntimeError:
                    got = -2
                except ValueError:
                    got = -3
            assert got == want
        assert a._free == list(z[f"free{c}"])


# ---- constructor / argument validation (ValueError, no device work) --------

@pytest.mark.parametrize("kw", [dict(num_heads=0), dict(num_heads=-1), dict(head_dim=0), dict(head_dim=-1),
                                dict(page_size=0), dict(page_size=-1), dict(max_pages=0), dict(max_pages=-1)])
def test_layer_cache_constructor_validation(kw):
    args = dict(num_heads=4, head_dim=8, page_size=16, max_pages=2, device="cpu")
    args.update(kw)
    with pytest.raises(ValueError):
        LayerKVCache(**args)


@pytest.mark.parametrize("n", [0, -1])
def test_paged_cache_rejects_bad_num_layers(n):
    with pytest.raises(ValueError):
        PagedKVCache(num_layers=n, num_heads=4, head_dim=8, page_size=16, max_pages=2, device="cpu")


def _cpu_cache():
    return PagedKVCache(num_layers=1, num_heads=4, head_dim=8, page_size=16, max_pages=2, device="cpu")


def test_append_shape_errors_are_value_errors():
    c = _cpu_cache()
    with pytest.raises(ValueError):
        c.append(0, torch.zeros(5, 4, 8), torch.zeros(6, 4, 8))
    with pytest.raises(ValueError):
        c.append(0, torch.zeros(5, 4, 8), torch.zeros(5, 3, 8))
    with pytest.raises(ValueError):
        c.append(0, torch.zeros(5, 4, 8), torch.zeros(5, 32))
    with pytest.raises(ValueError):
        c.append(0, torch.zeros(5, 99, 8), torch.zeros(5, 99, 8))
    with pytest.raises(ValueError):
        c.append(0, torch.zeros(5, 4, 99), torch.zeros(5, 4, 99))
    with pytest.raises(ValueError):
        c.append(5, torch.zeros(5, 4, 8), torch.zeros(5, 4, 8))
    with pytest.raises(ValueError):
        c.append(-1, torch.zeros(5, 4, 8), torch.zeros(5, 4, 8))


def test_staging_below_page_size_needs_no_kernel():
    c = _cpu_cache()
    c.append(0, torch.randn(10, 4, 8), torch.randn(10, 4, 8))
    assert c.seq_len == 10 and c.k_layers[0].block_table == [] and len(c.k_layers[0]._staging) == 10
    c.k_layers[0].append(torch.empty(0, 4, 8))
    assert c.k_layers[0].seq_len == 10


def test_paged_attention_validation():
    c = PagedKVCache(num_layers=1, num_heads=4, head_dim=64, page_size=16, max_pages=2, device="cpu")
    with pytest.raises(ValueError):  # empty cache
        paged_attention(c, 0, torch.randn(4, 64))
    c.append(0, torch.randn(3, 4, 64), torch.randn(3, 4, 64))
    with pytest.raises(ValueError):
        paged_attention(c, 0, torch.randn(4 * 64))
    for bad in [0.0, -1.0, float("nan"), float("inf"), float("-inf")]:
        with pytest.raises(ValueError):
            paged_attention(c, 0, torch.randn(4, 64), scale=bad)
    with pytest.raises(ValueError):
        paged_attention(c, 0, torch.randn(7, 64))


def test_memory_bytes_matches_shape_arithmetic():
    c = PagedKVCache(num_layers=2, num_heads=4, head_dim=8, page_size=16, max_pages=4, device="cpu")
    assert c.memory_bytes() == 2 * 2 * 4 * 16 * 4 * 8


# ---- attention helpers vs golden fixtures (torch, any device) ---------------

def test_helpers_match_golden():
    z = np.load(os.path.join(GOLD, "attention_helpers.npz"))
    for i in range(int(z["n"][0])):
        q = torch.from_numpy(z[f"q{i}"])
        hq, hkv = q.shape[0], z[f"k1{i}"].shape[1]
        rep = hq // hkv
        sc = float(z[f"scale{i}"][0])
        k1, v1 = torch.from_numpy(z[f"k1{i}"]), torch.from_numpy(z[f"v1{i}"])
        k2, v2 = torch.from_numpy(z[f"k2{i}"]), torch.from_numpy(z[f"v2{i}"])
        m1, s1, wv1 = _staging_contribution(q, _repeat_kv_heads(k1, rep), _repeat_kv_heads(v1, rep), sc)
        m2, s2, wv2 = _staging_contribution(q, _repeat_kv_heads(k2, rep), _repeat_kv_heads(v2, rep), sc)
        wv, l = _merge_unnormalized(m1, s1, wv1, m2, s2, wv2)
        torch.testing.assert_close(wv / l.unsqueeze(-1), torch.from_numpy(z[f"out{i}"]), atol=1e-5, rtol=1e-5)


def test_repeat_kv_heads_layout():
    x = torch.randn(5, 4, 3)
    out = _repeat_kv_heads(x, 8)
    assert out.shape == (5, 32, 3)
    for h in range(4):
        for r in range(8):
            assert torch.equal(out[:, h * 8 + r], x[:, h])


def test_empty_staging_is_identity():
    m, s, wv = _staging_contribution(torch.randn(4, 64), torch.empty(0, 4, 64), torch.empty(0, 4, 64), 0.125)
    assert torch.isinf(m).all() and (m < 0).all() and (s == 0).all() and (wv == 0).all()


def test_batched_cache_scale_granularity_arguments():
    """Rejected before anything is allocated (the cache itself lives on a GPU)."""
    from metagross_b200.batched import BatchedPagedKVCache

    with pytest.raises(ValueError):
        BatchedPagedKVCache(1, 1, 4, 64, device="cpu", scale_granularity="token")
    with pytest.raises(ValueError):  # per-vector absmax is reduced over a power-of-two head_dim
        BatchedPagedKVCache(1, 1, 4, 96, device="cpu", scale_granularity="token_head")


def test_bench_byte_counts_agree():
    """The append sweep's byte count for any step size reduces to the decode
    benchmark's one-token count, page commits included."""
    import bench

    for name in ("gpt2_int8", "tinyllama_int4"):
        w = bench.WORKLOADS[name]
        lens_after = [1, 15, 16, 17, 31, 32, 1024, 1009]
        one = bench.append_bytes(lens_after, w)
        many = bench.append_sweep_bytes([c - 1 for c in lens_after], lens_after, w)
        assert one == many
        # a 64-token step over one sequence: 4 page commits, no staged rows read or written
        P, row = w["page"], w["hkv"] * w["d"]
        bq = 1.0 if w["kv"] == "int8" else 0.5
        assert bench.append_sweep_bytes([0], [64], w) == 2 * 64 * row * 2 + 4 * (2 * P * row * bq + 8)
