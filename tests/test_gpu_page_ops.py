"""Single-page ops (``_C`` -> C ABI -> sm_100a kernels) against the oracle.

Bit-exact: INT8 codes, packed INT4 bytes, scales (the double the op returns and
the fp32 the kernel uses), dequantized values.  Ports the reference's
tests/test_quantize.py, tests/test_int4.py, the randomized round trips of
tests/test_cuda_stress.py and the op-level cases of tests/test_edge_cases.py.
"""
import math

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

BASE_SEED = 20260822
N_TRIALS = 25


def _C():
    from metagross_b200 import _C

    return _C


def _rng(off):
    return torch.Generator().manual_seed(BASE_SEED + off)


def _tokens(t, h=4, d=8, scale=3.0, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(t, h, d, generator=g) * scale).cuda()


@pytest.mark.parametrize("trial", range(N_TRIALS))
def test_int8_new_scale_bit_exact_random_shapes(trial):
    g = _rng(trial)
    t, h, d = int(torch.randint(1, 17, (1,), generator=g)), int(torch.randint(1, 9, (1,), generator=g)), int(
        torch.randint(1, 33, (1,), generator=g))
    sc = float(torch.rand((1,), generator=g)) * 10 + 0.01
    P = t + int(torch.randint(0, 8, (1,), generator=g))
    off = int(torch.randint(0, P - t + 1, (1,), generator=g))
    x = (torch.randn(t, h, d, generator=g) * sc).cuda()
    page = torch.zeros(P, h, d, dtype=torch.int8, device="cuda")
    s = _C().quantize_new_scale(x, page, off)
    ref_page, ref_s = O.quantize_int8(x.cpu().numpy(), np.zeros((P, h, d), np.int8), off)
    assert s == ref_s  # same double
    np.testing.assert_array_equal(page.cpu().numpy(), ref_page)
    deq = _C().dequantize_page(page, off, t, s)
    np.testing.assert_array_equal(deq.cpu().numpy(), O.dequantize_int8(ref_page, off, t, ref_s))
    assert (deq - x).abs().max().item() <= s / 2 + 1e-4


@pytest.mark.parametrize("trial", range(N_TRIALS))
def test_int4_new_scale_bit_exact_random_shapes(trial):
    g = _rng(1000 + trial)
    t, h = int(torch.randint(1, 17, (1,), generator=g)), int(torch.randint(1, 9, (1,), generator=g))
    d = int(torch.randint(1, 17, (1,), generator=g)) * 2
    sc = float(torch.rand((1,), generator=g)) * 10 + 0.01
    x = (torch.randn(t, h, d, generator=g) * sc).cuda()
    packed = torch.zeros(16, h, d // 2, dtype=torch.uint8, device="cuda")
    s = _C().quantize_int4_new_scale(x, packed, 0)
    ref, ref_s = O.quantize_int4(x.cpu().numpy(), np.zeros((16, h, d // 2), np.uint8), 0)
    assert s == ref_s
    np.testing.assert_array_equal(packed.cpu().numpy(), ref)
    deq = _C().dequantize_int4_page(packed, 0, t, s)
    np.testing.assert_array_equal(deq.cpu().numpy(), O.dequantize_int4(ref, 0, t, ref_s))
    assert (deq - x).abs().max().item() <= s / 2 + 1e-4


def test_fixed_scale_and_offsets():
    page = torch.zeros(16, 4, 8, dtype=torch.int8, device="cuda")
    a, b = _tokens(8, seed=2), _tokens(8, seed=3)
    s = _C().quantize_new_scale(a, page, 0)
    before = page.clone()
    _C().quantize_fixed_scale(b, page, 8, s)
    ref = np.zeros((16, 4, 8), np.int8)
    O.quantize_int8(a.cpu().numpy(), ref, 0)
    O.quantize_int8(b.cpu().numpy(), ref, 8, scale=s)
    np.testing.assert_array_equal(page.cpu().numpy(), ref)
    assert torch.equal(page[:8], before[:8])


def test_kat_exact_integers_scale_one():
    g = _rng(7100)
    for _ in range(5):
        x = torch.randint(-127, 128, (16, 4, 64), generator=g).float()
        x[0, 0, 0] = 127.0
        page = torch.zeros(16, 4, 64, dtype=torch.int8, device="cuda")
        s = _C().quantize_new_scale(x.cuda(), page, 0)
        assert s == 1.0
        torch.testing.assert_close(_C().dequantize_page(page, 0, 16, s).cpu(), x, atol=0, rtol=0)


@pytest.mark.parametrize("val,code", [(1e6, 127), (-1e6, -127)])
def test_clamp(val, code):
    page = torch.zeros(16, 2, 4, dtype=torch.int8, device="cuda")
    _C().quantize_fixed_scale(torch.full((1, 2, 4), val, device="cuda"), page, 0, 0.01)
    assert (page[0] == code).all() and (page[1:] == 0).all()


def test_nan_inf_edge_cases_match_oracle():
    x = torch.tensor([[[1.0, float("nan"), -2.0, 0.5], [float("inf"), -float("inf"), 3.0, 0.0]]])
    for t in (x[:, :1], x):
        page = torch.zeros(4, t.shape[1], 4, dtype=torch.int8, device="cuda")
        s = _C().quantize_new_scale(t.cuda(), page, 1)
        ref, rs = O.quantize_int8(t.numpy(), np.zeros((4, t.shape[1], 4), np.int8), 1)
        assert s == rs
        np.testing.assert_array_equal(page.cpu().numpy(), ref)
    page = torch.zeros(16, 2, 4, dtype=torch.int8, device="cuda")
    _C().quantize_fixed_scale(torch.full((1, 2, 4), 1e30, device="cuda"), page, 0, 1e-10)
    assert (page[0] == 127).all()
    _C().quantize_fixed_scale(torch.full((1, 2, 4), float("nan"), device="cuda"), page, 0, 0.1)
    assert (page[0] == 0).all()


def test_zero_tokens():
    page = torch.zeros(16, 2, 4, dtype=torch.int8, device="cuda")
    assert _C().quantize_new_scale(torch.empty(0, 2, 4, device="cuda"), page, 0) == pytest.approx(1e-8)
    out = _C().dequantize_page(page, 0, 0, 0.5)
    assert out.shape == (0, 2, 4) and out.dtype == torch.float32 and out.is_cuda
    packed = torch.zeros(16, 2, 2, dtype=torch.uint8, device="cuda")
    assert _C().quantize_int4_new_scale(torch.empty(0, 2, 4, device="cuda"), packed, 0) == pytest.approx(1e-8)
    assert _C().dequantize_int4_page(packed, 0, 0, 0.5).shape == (0, 2, 4)


def test_all_zeros_scale():
    page = torch.zeros(16, 2, 4, dtype=torch.int8, device="cuda")
    assert _C().quantize_new_scale(torch.zeros(4, 2, 4, device="cuda"), page, 0) == pytest.approx(1e-8)
    assert (page == 0).all()


def test_inf_in_new_scale_input_does_not_crash():
    x = _tokens(4, 2, 4, seed=50)
    x[0, 0, 0] = float("inf")
    page = torch.zeros(16, 2, 4, dtype=torch.int8, device="cuda")
    s = _C().quantize_new_scale(x, page, 0)
    assert math.isfinite(s) and s > 0
    assert torch.isfinite(_C().dequantize_page(page, 0, 4, s)).all()


def test_non_contiguous_input_accepted_storage_rejected():
    base = torch.randn(8, 4, 4, device="cuda")
    x = base.permute(2, 1, 0)
    assert not x.is_contiguous()
    page = torch.zeros(16, 4, 8, dtype=torch.int8, device="cuda")
    s = _C().quantize_new_scale(x, page, 0)
    ref, rs = O.quantize_int8(x.contiguous().cpu().numpy(), np.zeros((16, 4, 8), np.int8), 0)
    assert s == rs
    np.testing.assert_array_equal(page.cpu().numpy(), ref)
    bad = torch.zeros(8, 4, 16, dtype=torch.int8, device="cuda").permute(2, 1, 0)
    with pytest.raises(RuntimeError):
        _C().quantize_new_scale(_tokens(4, 4, 8), bad, 0)


def test_runtime_errors():
    C = _C()
    p8 = torch.zeros(16, 2, 4, dtype=torch.int8, device="cuda")
    p4 = torch.zeros(16, 2, 2, dtype=torch.uint8, device="cuda")
    t = _tokens(4, 2, 4)
    for fn in [lambda: C.quantize_new_scale(t, p8, -1), lambda: C.quantize_fixed_scale(t, p8, -1, 0.1),
               lambda: C.dequantize_page(p8, -1, 4, 0.1), lambda: C.dequantize_page(p8, 0, -1, 0.1),
               lambda: C.quantize_int4_new_scale(t, p4, -1), lambda: C.dequantize_int4_page(p4, -1, 4, 0.1),
               lambda: C.dequantize_int4_page(p4, 0, -1, 0.1),
               lambda: C.quantize_new_scale(torch.randn(4, 4, device="cuda"), p8, 0),
               lambda: C.quantize_new_scale(t, torch.zeros(16, 8, dtype=torch.int8, device="cuda"), 0),
               lambda: C.quantize_new_scale(t, torch.zeros(16, 3, 4, dtype=torch.int8, device="cuda"), 0),
               lambda: C.quantize_new_scale(t, torch.zeros(16, 2, 5, dtype=torch.int8, device="cuda"), 0),
               lambda: C.quantize_new_scale(_tokens(20, 2, 4), p8, 0),
               lambda: C.quantize_int4_new_scale(torch.randn(4, 2, 5, device="cuda"),
                                                 torch.zeros(16, 2, 3, dtype=torch.uint8, device="cuda"), 0),
               lambda: C.quantize_int4_new_scale(torch.randn(4, 2, 0, device="cuda"),
                                                 torch.zeros(16, 2, 0, dtype=torch.uint8, device="cuda"), 0),
               lambda: C.quantize_int4_new_scale(_tokens(4, 2, 8), torch.zeros(16, 2, 3, dtype=torch.uint8,
                                                                                device="cuda"), 0),
               lambda: C.quantize_int4_new_scale(_tokens(4, 2, 8), torch.zeros(16, 3, 4, dtype=torch.uint8,
                                                                                device="cuda"), 0),
               lambda: C.quantize_int4_new_scale(_tokens(17, 2, 8), torch.zeros(16, 2, 4, dtype=torch.uint8,
                                                                                 device="cuda"), 0),
               lambda: C.quantize_fixed_scale(t, p8, 0, 0.0), lambda: C.quantize_fixed_scale(t, p8, 0, float("nan")),
               lambda: C.dequantize_page(p8, 0, 4, float("inf"))]:
        with pytest.raises(RuntimeError):
            fn()


def test_sanity_add():
    import metagross_b200

    torch.manual_seed(0)
    a, b = torch.randn(10_000, device="cuda"), torch.randn(10_000, device="cuda")
    torch.testing.assert_close(metagross_b200.sanity_add(a, b), a + b, rtol=0, atol=0)
    with pytest.raises(RuntimeError):
        metagross_b200.sanity_add(torch.randn(10, device="cuda"), torch.randn(20, device="cuda"))
