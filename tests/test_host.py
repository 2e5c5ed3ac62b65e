"""Host-side logic without a GPU: the library loads and exports the C ABI,
and the product's parameter math / tables equal the oracle's."""
import os
import re

import numpy as np
import pytest

from oracle import cross_oracle as O
from tests.conftest import ROOT


def _header_symbols():
    with open(os.path.join(ROOT, "include", "cross_b200.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|uint64_t|const char\*)\s+(cross_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    import ctypes

    from cross_b200 import _lib, build
    build.build(verbose=False)
    h = ctypes.CDLL(_lib.LIB_PATH)
    syms = _header_symbols()
    assert len(syms) >= 30
    missing = [s for s in syms if not hasattr(h, s)]
    assert not missing, missing
    assert set(syms) == set(_lib.exported_symbols())
    assert _lib.lib().cross_abi_version() == 1


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from cross_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()


def test_status_codes_raise_reference_exceptions():
    from cross_b200 import _lib
    _lib.lib()
    # cross_ntt with a null plan -> CROSS_ERR_INVALID_ARG -> ValueError
    rc = _lib.lib().cross_ntt(None, 0, None, None, 1, 0, None, 0, None)
    with pytest.raises(ValueError, match="cross_ntt"):
        _lib.check(rc, "cross_ntt")


@pytest.mark.parametrize("q", O.find_moduli_ntt(3, 28, 2 * 4096) + [134219681, 1073742881, 524353, 17, 29])
def test_barrett_constants_match(q):
    from cross_b200 import util
    s, w, sw, m = util.barrett_constants([q])
    b = O.Barrett([q])
    assert (s, w, sw, m) == (b.barrett_s, b.barrett_w, b.barrett_s_w, b.barrett_m)


@pytest.mark.parametrize("m,q", [(32, 134219681), (8192, O.find_moduli_ntt(1, 28, 8192)[0]),
                                 (32, 524353), (32, 1073741441)])
def test_root_of_unity_matches(m, q):
    from cross_b200 import util
    assert util.root_of_unity(m, q) == O.root_of_unity(m, q)


def test_util_tables_match():
    from cross_b200 import util
    q = O.find_moduli_ntt(1, 28, 2 * 4096)[0]
    np.testing.assert_array_equal(util.powers(12345, 4096, q), O.powers_mod(12345, 4096, q))
    np.testing.assert_array_equal(util.twiddle_matrix(64, 64, q, 3), O.twiddle_matrix(64, 64, q, 3).astype(np.uint64))
    for k in (1, 7, 100):
        n = 256
        g = util.find_automorphism_index_2n_complex(k, 2 * n)
        assert g == O.find_automorphism_index_2n_complex(k, 2 * n)
        assert util.precompute_auto_map(n, g) == O.precompute_auto_map(n, g)
    L = O.find_moduli_ntt(6, 28, 2 * 64)
    a, b = util.compute_QHatInvModq_QHatModp(L[:3], L[3:])
    c, d = O.compute_qhat(L[:3], L[3:])
    assert a == c and b == d
    ga, gb = util.gamma_beta_calculation(L)
    oa, ob = O.gamma_beta(L)
    np.testing.assert_array_equal(ga, oa)
    np.testing.assert_array_equal(gb, ob)


@pytest.mark.parametrize("n,r,c", [(16, 4, 4), (4096, 64, 64), (4096, 32, 128)])
def test_ntt_context_tables_match_oracle(n, r, c):
    from cross_b200 import ntt_mm
    q = O.find_moduli_ntt(3, 28, 2 * n)
    ctx = ntt_mm.NTTCiphertextBarrettContext(q, {"r": r, "c": c})
    ref = O.NTTBarrett(q, r, c)
    for name in ("ntt_tf_step1", "ntt_tf_step2", "ntt_tf_step3", "intt_tf_step1", "intt_tf_step2", "intt_tf_step3",
                 "ntt_bat_tf_step1", "ntt_bat_tf_step3", "intt_bat_tf_step1", "intt_bat_tf_step3"):
        np.testing.assert_array_equal(getattr(ctx, name), getattr(ref, name), err_msg=name)


def test_bconv_tables_match_oracle():
    from cross_b200 import bconv
    ov = O.find_moduli_ntt(9, 28, 2 * 64)
    b = bconv.BConvBarrett(ov)
    b.control_gen([([0, 1, 2, 3], [4, 5, 6, 7, 8]), ([4, 5], [0, 1, 2])])
    o = O.BConvBarrett(ov)
    o.control_gen([([0, 1, 2, 3], [4, 5, 6, 7, 8]), ([4, 5], [0, 1, 2])])
    for i in range(2):
        np.testing.assert_array_equal(b.QHatModpBAT[i], o.controls[i]["bat"])
        np.testing.assert_array_equal(b.QHatInvModq[i], o.controls[i]["qhat_inv"])


def test_digit_partition_matches():
    from cross_b200.hemul import digits
    for L, d in [(23, 3), (4, 3), (5, 3), (34, 5), (1, 1)]:
        a, p, g = digits(L, d)
        oa, op, og = O.digit_partition(L, d)
        assert (a, p, g) == (oa, op, og)
