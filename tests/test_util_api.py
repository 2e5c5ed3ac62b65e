"""The host helpers of util.py that the reference's callers use, against
restatements of the reference functions written out in the tests
(util.py:61-166, 252-382, 497-539, 614-645, 833-861)."""
import math

import numpy as np
import pytest

from cross_b200 import util

Q = util.find_moduli_ntt(4, 28, 2 ** 17)              # NTT primes, 1 mod 2^17


def test_num_bits_to_tuple_and_slices():
    assert [util.num_bits(x) for x in (1, 2, 3, 4, 255, 256, 2 ** 40)] == [0, 1, 1, 2, 7, 8, 40]
    assert util.to_tuple(np.arange(6).reshape(2, 3)) == ((0, 1, 2), (3, 4, 5))
    assert util.to_tuple([[1, [2]], 3]) == ((1, (2,)), 3)
    arrs = ((1, 2, 3, 4), (5, 6, 7, 8))
    assert util.slice_first_k_along_axis0(arrs, 2) == ((1, 2), (5, 6))
    assert util.slice_k_to_end_along_axis0(arrs, 3) == ((4,), (8,))
    assert util.slice_kth_along_axis0(arrs, 1) == (2, 6)
    assert util.slice_k0_to_k1_axis0(arrs, 1, 3) == ((2, 3), (6, 7))
    assert util.slice_0_to_k0_to_k1_along_axis0(arrs, 1, 3) == ((1, 4), (5, 8))
    assert util.slice_0_to_k0_to_k1_along_axis0([[1, 2, 3], [4, 5, 6]], 0, 2) == [[3], [6]]
    got = util.slice_0_to_k0_to_k1_along_axis0((np.arange(5), np.arange(5, 10)), 1, 4)
    assert [g.tolist() for g in got] == [[0, 4], [5, 9]]
    with pytest.raises(ValueError):
        util.slice_0_to_k0_to_k1_along_axis0({0: (1, 2)}, 0, 1)


def test_extended_gcd_and_modinv_manual():
    for a, b in [(240, 46), (17, 5), (1, 1), (0, 7), (2 ** 61 - 1, 12345)]:
        g, x, y = util.extended_gcd(a, b)
        assert g == math.gcd(a, b) and a * x + b * y == g
    for q in Q:
        for x in (1, 2, 12345, q - 1):
            assert util.modinv_manual(x, q) == pow(x, -1, q)
    with pytest.raises(Exception, match="does not exist"):
        util.modinv_manual(6, 9)


def test_any_primitive_root_of_unity():
    for q in Q:
        for n in (2, 16, 1 << 17):
            w = util.any_primitive_root_of_unity(n, q)
            g = util.find_generator(q)
            assert w == pow(g, (q - 1) // n, q)
            assert pow(w, n, q) == 1 and (n == 1 or pow(w, n // 2, q) != 1)
    with pytest.raises(ValueError):
        util.any_primitive_root_of_unity(3, 17)


def test_compute_barrett_mu():
    for m in [17, 65537] + Q + [2 ** 31 - 1]:
        b = 2 ** (math.floor(math.log(m)) + 1)
        k = math.floor(math.log(m, b)) + 1
        assert util.compute_barrett_mu(m) == ((b ** (2 * k)) // m, k)


def test_approx_mod_down_control_generation():
    cur, tgt = Q[:2], Q[2:]
    p_inv, i0, i1, inv, qm = util.approx_mod_down_control_generation(cur, tgt)
    P = cur[0] * cur[1]
    assert p_inv == [pow(P, -1, q) for q in tgt]
    assert (i0, i1) == (2, 2)
    assert (inv, qm) == util.compute_QHatInvModq_QHatModp(cur, tgt)
    _, i0, i1, _, _ = util.approx_mod_down_control_generation(Q[:3], Q[3:])
    assert (i0, i1) == (3, 1)


def test_compute_powers_of_psi():
    ring = 64
    got = util.compute_powers_of_psi(ring, Q[:2])
    assert got.dtype == np.uint64 and got.shape == (2, ring)
    for row, q in zip(got, Q[:2]):
        psi = util.root_of_unity(2 * ring, q)
        assert row.tolist() == [pow(psi, i, q) for i in range(ring)]


def test_random_ciphertexts_stay_below_their_limb_modulus():
    x = util.random_batched_ciphertext((2, 4, 8, 4), Q, dtype=np.uint32)
    assert x.shape == (2, 4, 8, 4) and x.dtype == np.uint32
    assert (x.astype(np.uint64) < np.array(Q, np.uint64)).all()
    y = util.random_ciphertext((2, 16, 4), Q)
    assert y.shape == (2, 16, 4) and y.dtype == np.int32
    assert (y < np.array(Q)).all() and (y >= 0).all()
    np.testing.assert_array_equal(util.random_ciphertext((2, 16, 4), Q), y)     # seeded
    r = util.random_parameters((3, 5), Q, np.uint64)
    assert r.dtype == np.uint64 and (r < min(Q) - 1).all()
    with pytest.raises(AssertionError):
        util.random_ciphertext((2, 16, 3), Q)


def _swap_reverse(x):
    """util.py:623-630 restated: swap i and bitrev(i) for i < bitrev(i)."""
    x = list(x)
    bits = len(x).bit_length() - 1
    for i in range(len(x)):
        j = util.bit_reverse(i, bits)
        if i < j:
            x[i], x[j] = x[j], x[i]
    return x


@pytest.mark.parametrize("n", [1, 2, 8, 1024])
def test_bit_reverse_array(n):
    src = list(range(100, 100 + n))
    assert util.bit_reverse_array(src) == _swap_reverse(src)
    assert src == list(range(100, 100 + n))                       # input untouched
    arr = np.arange(n) * 3
    np.testing.assert_array_equal(util.bit_reverse_array(arr), np.array(_swap_reverse(arr.tolist())))
    assert util.bit_reverse_array(tuple(src)) == tuple(_swap_reverse(src))


def test_chunk_decomposition():
    x = 0x0123456789ABCDEF
    np.testing.assert_array_equal(util.chunk_decomposition(x), [0xEF, 0xCD, 0xAB, 0x89, 0x67, 0x45, 0x23, 0x01])
    d16 = util.chunk_decomposition(x, 16)
    assert d16.dtype == np.uint16 and d16.tolist() == [0xCDEF, 0x89AB, 0x4567, 0x0123]
    d32 = util.chunk_decomposition(x, 32)
    assert d32.dtype == np.uint32 and d32.tolist() == [0x89ABCDEF, 0x01234567]
    d4 = util.chunk_decomposition(0xAB, 4)
    assert d4.dtype == np.uint8 and d4.tolist() == [0xB, 0xA]
    assert util.chunk_decomposition(0).size == 0


def test_openfhe_text_round_trip():
    """format_ciphertext_string writes what parse_ciphertext_string (util.py:
    545-608) reads back, in the layout of the reference's test fixtures."""
    import json
    import os
    rng = np.random.default_rng(5)
    data = [[rng.integers(0, q, 16).tolist() for q in Q] for _ in range(2)]
    text = util.format_ciphertext_string(data, Q)
    assert text.startswith("Element 0: 0: EVAL: [") and "\nElement 1: 0: EVAL: [" in text
    assert util.parse_ciphertext_string(text) == (data, list(Q))
    # a fixture written by OpenFHE (rescale_test.py:19-45) survives parse -> format -> parse
    with open(os.path.join(os.path.dirname(__file__), "golden", "rescale.json")) as f:
        g = json.load(f)
    d, m = util.parse_ciphertext_string(g["in_ciphertexts_str"])
    assert util.parse_ciphertext_string(util.format_ciphertext_string(d, m)) == (d, m)
    with pytest.raises(ValueError):
        util.format_ciphertext_string([[[1, 2]]], Q)
