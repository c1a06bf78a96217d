"""Pin the CPU oracle before trusting it.

Fixtures in tests/golden/ were produced by the reference's own Python
(tests/golden/make_golden.py): tests/reference.py's quantizers, the reference
BlockAllocator and the attention helpers of metagross/attention.py.  The
oracle (oracle/mg_oracle.c + oracle/oracle.py) must reproduce them:

  * INT8 / INT4 codes and packed nibbles: bit-exact, except where the two
    reference implementations themselves disagree (tests/reference.py rounds
    half-to-even and lets NaN poison the absmax; the CUDA ops -- the bit-exact
    target -- round half away from zero and ignore NaN).  Random float inputs
    never hit an exact .5 tie, which the test asserts rather than assumes.
  * scales: the oracle's double scale agrees with reference.py's float32 one
    to rel 1e-6 (the reference test uses rel 1e-5).
  * allocator replay: identical ids and identical error outcomes.
  * attention: float64 oracle within 1e-5 of the reference's fp32 torch math.
"""
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


def test_int8_codes_and_scales_match_reference_cpu_path():
    z = _load("int8_quant.npz")
    for i in range(int(z["n"][0])):
        x = z[f"x{i}"]
        page, s = O.quantize_int8(x)
        assert s == pytest.approx(float(z[f"s{i}"][0]), rel=1e-6)
        # no exact .5 ties in the quotient, so half-even == half-away here
        qf = x / np.float32(s)
        frac = np.abs(qf - np.trunc(qf))
        assert not np.any(frac == 0.5)
        np.testing.assert_array_equal(page, z[f"q{i}"], err_msg=f"case {i}")
        deq = O.dequantize_int8(page, 0, x.shape[0], s)
        np.testing.assert_allclose(deq, z[f"deq{i}"], rtol=1e-6, atol=0)


def test_int4_packed_bytes_match_reference_cpu_path():
    z = _load("int4_quant.npz")
    for i in range(int(z["n"][0])):
        x = z[f"x{i}"]
        packed, s = O.quantize_int4(x)
        assert s == pytest.approx(float(z[f"s{i}"][0]), rel=1e-6)
        np.testing.assert_array_equal(packed.reshape(-1), z[f"p{i}"], err_msg=f"case {i}")
        deq = O.dequantize_int4(packed, 0, x.shape[0], s)
        np.testing.assert_allclose(deq, z[f"deq{i}"], rtol=1e-6, atol=0)


def test_exact_kat_scale_one():
    """Integer inputs with absmax 127 give scale exactly 1.0 and codes == inputs
    (tests/test_cuda_stress.py:275-333)."""
    z = _load("int8_kat_scale1.npz")
    for i in range(5):
        x = z[f"x{i}"]
        page, s = O.quantize_int8(x)
        assert s == 1.0
        np.testing.assert_array_equal(page, z[f"q{i}"])
        np.testing.assert_array_equal(page.astype(np.float32), x)
        np.testing.assert_array_equal(O.dequantize_int8(page, 0, 16, s), x)


def test_allocator_replay_matches_reference_allocator():
    z = _load("allocator_script.npz")
    for c in range(int(z["n"][0])):
        n = int(z[f"n{c}"][0])
        res, free, nfree = O.allocator_replay(n, z[f"ops{c}"])
        np.testing.assert_array_equal(res, z[f"res{c}"], err_msg=f"script {c}")
        np.testing.assert_array_equal(free, z[f"free{c}"])


def test_attention_helpers_match_reference_torch_math():
    z = _load("attention_helpers.npz")
    for i in range(int(z["n"][0])):
        q, sc = z[f"q{i}"], float(z[f"scale{i}"][0])
        k1, v1, k2, v2 = z[f"k1{i}"], z[f"v1{i}"], z[f"k2{i}"], z[f"v2{i}"]
        wv1, l1, m1 = O.attention_unnormalized(q, k1, v1, sc)
        wv2, l2, m2 = O.attention_unnormalized(q, k2, v2, sc)
        if k1.shape[0]:
            np.testing.assert_allclose(m1, z[f"m1{i}"], rtol=1e-6, atol=1e-6)
            np.testing.assert_allclose(l1, z[f"s1{i}"], rtol=2e-6)
            np.testing.assert_allclose(wv1, z[f"wv1{i}"], rtol=2e-5, atol=2e-5)
        else:
            assert np.all(np.isneginf(z[f"m1{i}"])) and np.all(np.isneginf(m1))
        wv, l, m = O.merge_unnormalized(m1, l1, wv1, m2, l2, wv2)
        np.testing.assert_allclose(wv / l[:, None], z[f"out{i}"], rtol=0, atol=1e-5)
        full = O.attention(q, np.concatenate([k1, k2]), np.concatenate([v1, v2]), sc)
        np.testing.assert_allclose(full, z[f"out{i}"], rtol=0, atol=1e-5)


# ---- semantics the reference's CUDA ops define (read from csrc/*.cu) -------

def test_zero_input_scale_is_1e8():
    page, s = O.quantize_int8(np.zeros((4, 2, 4), np.float32))
    assert s == 1e-8 and not page.any()
    packed, s4 = O.quantize_int4(np.zeros((4, 2, 4), np.float32))
    assert s4 == 1e-8 and not packed.any()


def test_zero_tokens_returns_1e8_and_leaves_page():
    page = np.full((16, 2, 4), 7, np.int8)
    _, s = O.quantize_int8(np.zeros((0, 2, 4), np.float32), page, 0)
    assert s == 1e-8 and (page == 7).all()


def test_clamp_to_pm127_with_fixed_scale():
    page, _ = O.quantize_int8(np.full((1, 2, 4), 1e6, np.float32), np.zeros((16, 2, 4), np.int8), 0, scale=0.01)
    assert (page[0] == 127).all() and (page[1:] == 0).all()
    page, _ = O.quantize_int8(np.full((1, 2, 4), -1e6, np.float32), np.zeros((16, 2, 4), np.int8), 0, scale=0.01)
    assert (page[0] == -127).all()


def test_nan_is_zero_and_ignored_by_absmax():
    x = np.array([[[1.0, np.nan, -2.0, 0.5]]], np.float32)
    page, s = O.quantize_int8(x)
    assert s == pytest.approx(2.0 / 127.0)
    assert page[0, 0, 1] == 0 and page[0, 0, 2] == -127


def test_inf_makes_scale_1e8_and_codes_saturate():
    x = np.array([[[1.0, np.inf, -2.0, 0.5]]], np.float32)
    page, s = O.quantize_int8(x)
    assert s == 1e-8
    assert page[0, 0, 1] == 127 and page[0, 0, 2] == -127 and page[0, 0, 0] == 127


def test_round_half_away_from_zero():
    # x / s = k + 0.5 exactly: the CUDA op rounds away from zero (roundf)
    x = np.array([[[0.5, 1.5, 2.5, -0.5, -2.5, 127.0]]], np.float32)
    page, s = O.quantize_int8(x)
    assert s == 1.0
    np.testing.assert_array_equal(page[0, 0], [1, 2, 3, -1, -3, 127])


def test_int4_nibble_order_and_range():
    x = np.array([[[7.0, -7.0, 1.0, -1.0, 0.0, 3.0]]], np.float32)
    packed, s = O.quantize_int4(x)
    assert s == 1.0
    # element 2j in the low nibble of byte j, two's complement
    assert list(packed[0, 0]) == [0x97, 0xF1, 0x30]
    np.testing.assert_array_equal(O.dequantize_int4(packed, 0, 1, s)[0, 0], x[0, 0])


def test_offset_write_leaves_other_tokens():
    page = np.zeros((16, 2, 4), np.int8)
    a = np.random.default_rng(0).standard_normal((8, 2, 4)).astype(np.float32)
    O.quantize_int8(a, page, 0)
    before = page.copy()
    O.quantize_int8(a * 2, page, 8, scale=0.05)
    np.testing.assert_array_equal(page[:8], before[:8])
    assert (page[8:] != 0).any()


def _th_inputs():
    """The seeded inputs of token_head_int8.npz (recipe in tests/golden/make_golden.py)."""
    import sys

    if GOLD not in sys.path:
        sys.path.insert(0, GOLD)
    import make_golden

    return make_golden.th_inputs()


def test_token_head_int8_matches_reference_cpu_path():
    """Per-(token, head) INT8 scales on the GPT-2-small CPU-reference decode step
    (batch 4, 12 heads, head_dim 64, contexts U[1, 512], full pages quantized,
    the partial page exact): the oracle's codes and fp32 scales hash to the
    fixture's (the reference's CPU path, with the CUDA kernels'
    half-away-from-zero rounding at the listed ties), and its float64
    dequantize-then-attend is within 1e-5 of the reference's fp32 torch math."""
    import hashlib

    z = _load("token_head_int8.npz")
    lens, ks, vs, q = _th_inputs()
    assert lens.numpy().tolist() == z["lens"].tolist()
    for b in range(len(lens)):
        n = int(lens[b]) // 16 * 16
        deq = {}
        for name, x in (("k", ks[b]), ("v", vs[b])):
            codes, sc = O.quantize_token_head(x.numpy()[:n], "int8")
            s32 = sc.astype(np.float32)
            np.testing.assert_array_equal(codes[:16], z[f"{name}_codes_page0_{b}"])
            np.testing.assert_array_equal(s32[:16], z[f"{name}_scales_page0_{b}"])
            for t, h, d, _cpu_code, kernel_code in z[f"{name}_ties{b}"]:
                assert codes[t, h, d] == kernel_code
            assert hashlib.sha256(codes.tobytes()).digest() == z[f"{name}_codes_sha{b}"].tobytes()
            assert hashlib.sha256(s32.tobytes()).digest() == z[f"{name}_scales_sha{b}"].tobytes()
            deq[name] = np.concatenate([O.dequantize_token_head(codes, sc, "int8"), x.numpy()[n:]])
        out = O.attention(q[b].numpy(), deq["k"], deq["v"], 1.0 / 8)
        np.testing.assert_allclose(out, z[f"out{b}"], atol=1e-5, rtol=0)
