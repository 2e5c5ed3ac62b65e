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


# ---------------------------------------------------------------------------
# Montgomery / Shoup / BAT-lazy variants: host-side tables equal the oracle's
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("reduction", ["montgomery", "shoup", "bat_lazy"])
def test_variant_ntt_tables_match_oracle(reduction):
    """ntt_mm.py:172-181 (computation format + BAT) and 457-469 (Shoup)."""
    from cross_b200 import ntt_mm
    from oracle import variants as V
    q = O.find_moduli_ntt(3, 28, 2 * 256)
    cls = {"montgomery": ntt_mm.NTTCiphertextMontgomeryContext, "shoup": ntt_mm.NTTCiphertextShoupContext,
           "bat_lazy": ntt_mm.NTTCiphertextBATLazyContext}[reduction]
    ctx = cls(q, {"r": 16, "c": 16})
    ref = V.NTTVariant(q, 16, 16, reduction)
    if reduction == "shoup":
        names = [n + s for n in cls._TABLES for s in ("", "_shoup")]
    else:
        names = ["ntt_bat_tf_step1", "ntt_tf_step2", "ntt_bat_tf_step3", "intt_bat_tf_step1", "intt_tf_step2",
                 "intt_bat_tf_step3"]
    for n in names:
        np.testing.assert_array_equal(np.asarray(getattr(ctx, n)).astype(np.uint64),
                                      np.asarray(getattr(ref, n)).astype(np.uint64), err_msg=n)


@pytest.mark.parametrize("reduction", ["montgomery", "shoup", "bat_lazy"])
def test_variant_bconv_constants_match_oracle(reduction):
    """bconv.py:67-97 in the contexts' computation formats; BConvShoup's
    companions (bconv.py:300-314) are 0: the reference shifts uint32 arrays by
    32 under JAX."""
    from cross_b200 import bconv
    from oracle import variants as V
    ov = O.find_moduli_ntt(9, 28, 64)
    ctl = [([0, 1, 2], [3, 4, 5, 6, 7, 8])]
    dev = {"montgomery": bconv.BConvMontgomery, "shoup": bconv.BConvShoup,
           "bat_lazy": bconv.BConvBATLazy}[reduction](ov)
    dev.control_gen(ctl)
    ref = V.BConvVariant(ov, reduction)
    ref.control_gen(ctl)
    c = ref.controls[0]
    np.testing.assert_array_equal(np.asarray(dev.QHatInvModq[0]).astype(np.uint64), c["qhat_inv"])
    np.testing.assert_array_equal(np.asarray(dev.QHatModp[0]).astype(np.uint64), c["qhat_modp"])
    np.testing.assert_array_equal(dev.QHatModpBAT[0], c["bat"])
    if reduction == "shoup":
        assert not np.asarray(dev.QHatInvModq_shoup[0]).any() and not np.asarray(dev.QHatModp_shoup[0]).any()
        np.testing.assert_array_equal(dev.QHatModp_shoup[0], c["qhat_modp_shoup"])


def test_single_modulus_contexts_expose_reference_tables():
    """ntt_sm.py:143-152,214-221: the single-modulus tables are the
    multi-modulus ones of one modulus."""
    from cross_b200 import finite_field as ff, ntt_sm
    q = O.find_moduli_ntt(1, 28, 2 * 256)[0]
    ctx = ntt_sm.NTTBarrettContext(q, {"r": 16, "c": 16, "finite_field_context": ff.BarrettContext(q)})
    ref = O.NTTBarrett([q], 16, 16)
    np.testing.assert_array_equal(ctx.ntt_tf_bat_mat_comp_step1, ref.ntt_bat_tf_step1[..., 0])
    np.testing.assert_array_equal(ctx.intt_tf_mat_comp_step2.astype(np.uint64), ref.intt_tf_step2[..., 0])
    sh = ntt_sm.NTTShoupContext(q, {"r": 16, "c": 16, "finite_field_context": ff.ShoupContext(q)})
    t = sh.ntt_tf_mat_step1
    np.testing.assert_array_equal(sh.to_shoup_computation_format(t), sh.ntt_tf_mat_step1_shoup)
    with pytest.raises(TypeError):
        ntt_sm.NTTContextBase(q, {"r": 16, "c": 16, "finite_field_context": ff.ShoupContext(q)})


def test_ckks_host_helpers_match_oracle():
    """ckks_ctx.py:113-153 and key_gen.py:77-105: the host helpers of the CKKS
    client equal the oracle's on edge values."""
    from cross_b200 import ckks_ctx, key_gen
    from oracle import ckks as K
    for x in (0.0, 0.5, -0.5, 1.5, -1.5, 2.4999999, -2.5000001, 1e17 + 0.5, -7.0):
        assert ckks_ctx.nearest_int(x) == K.nearest_int(x)
    q = 1073741441
    vals = [0, 1, 5, 2 ** 40, K.MAX_INT_64 - 3, (K.MAX_INT_64 >> 1) + 1, K.MAX_INT_64 >> 1]
    assert ckks_ctx.fit_to_native_vector(vals, K.MAX_INT_64, q, 14) == K.fit_to_native_vector(vals, K.MAX_INT_64, q, 14)
    y = [complex(1.5, -2.0), complex(0.0, 3.25)]
    assert ckks_ctx.slot_to_coeffs(y) == [1.5, 0.0, -2.0, 3.25]
    coeffs = [0, 1, 524352 // 2, 524353 // 2 + 1, 524352]
    assert key_gen.modulus_switch(coeffs, 524353, 1073740609) == K.modulus_switch(coeffs, 524353, 1073740609)
    # threshold (cur + 1) // 2 = 7: 6 stays, 7 and 12 become 101 + v - 13
    assert [key_gen.modulus_switch(v, 13, 101) for v in (6, 7, 12)] == [6, 95, 100]


def test_shoup_precompute_follows_the_reference_dtypes():
    """finite_field.py:295-297 under JAX: a uint32 operand shifted by 32 is 0
    (so BConvShoup's companions are 0); wider operands give floor(a 2^32 / q)."""
    from cross_b200 import finite_field as ff
    q = [1073741441, 1073740609]
    sh = ff.ShoupContext(q)
    a = np.array([5, 1073741440], np.uint32)
    assert not sh.precompute_constant_operand(a).any()
    np.testing.assert_array_equal(sh.precompute_constant_operand(a.astype(np.uint64)),
                                  (a.astype(np.uint64) << np.uint64(32)) // np.array(q, np.uint64))


def _twiddle(rows, cols, q, omega):
    """ntt_mm.py:75-97 restated: omega^(r c) mod q, one pow per entry."""
    return np.array([[pow(omega, r * c, q) for c in range(cols)] for r in range(rows)], np.int64)


def test_twiddle_matrix_functions_and_single_modulus_tables():
    """ntt_mm.py:75-119 and ntt_sm.py:143-221: the twiddle matrices, their
    memory-aligned forms and the BAT forms under the reference's names."""
    from cross_b200 import finite_field as ff, ntt_mm, ntt_sm, util
    q = O.find_moduli_ntt(1, 28, 2 * 256)[0]
    r = c = 16
    psi = util.root_of_unity(2 * r * c, q)
    om = psi * psi % q
    np.testing.assert_array_equal(ntt_mm.gen_twiddle_matrix(8, 4, q, om), _twiddle(8, 4, q, om))
    inv = ntt_mm.gen_twiddle_matrix_inv(4, 8, q, om)
    assert inv.dtype == np.int64
    np.testing.assert_array_equal(inv, _twiddle(4, 8, q, pow(om, -1, q)))
    for ffc, cls in ((ff.BarrettContext(q), ntt_sm.NTTBarrettContext),
                     (ff.MontgomeryContext(q), ntt_sm.NTTMontgomeryContext)):
        ctx = cls(q, {"r": r, "c": c, "finite_field_context": ffc})
        oc, orow = pow(om, c, q), pow(om, r, q)
        want = (_twiddle(r, r, q, oc), _twiddle(r, c, q, om), _twiddle(c, c, q, orow))
        for got, w in zip(ctx.ntt_coefficients_precompute(), want):
            assert got.dtype == np.int64
            np.testing.assert_array_equal(got, w)
        i1, i2, i3 = ctx.intt_coefficients_precompute()
        np.testing.assert_array_equal(i1, _twiddle(c, c, q, pow(orow, -1, q)))
        np.testing.assert_array_equal(i2, _twiddle(r, c, q, pow(om, -1, q)) * pow(c, -1, q) % q)
        np.testing.assert_array_equal(i3, _twiddle(r, r, q, pow(oc, -1, q)) * pow(r, -1, q) % q)
        perm = util.bit_reverse_indices(r)
        np.testing.assert_array_equal(ctx.ntt_tf_mat_step1, ctx.ntt_tf_step1[perm, :])
        np.testing.assert_array_equal(ctx.ntt_tf_mat_step3, ctx.ntt_tf_step3[:, perm])
        np.testing.assert_array_equal(ctx.intt_tf_mat_step3, ctx.intt_tf_step3[:, perm])
        # the BAT tables the device plan uses are those of the memory-aligned
        # tables in the computation format
        mm = ctx._mm
        np.testing.assert_array_equal(ctx.ntt_tf_bat_mat_comp_step1, mm.ntt_bat_tf_step1[..., 0])
        np.testing.assert_array_equal(ctx.intt_tf_bat_mat_comp_step3, mm.intt_bat_tf_step3[..., 0])
        np.testing.assert_array_equal(ctx.ntt_tf_mat_comp_step2, np.asarray(mm.ntt_tf_step2)[..., 0])
        bat = ctx.basis_aligned_transformation(ctx.ntt_tf_mat_step1)
        assert bat.shape == (r, 4, r, 4) and bat.dtype == np.uint8
        np.testing.assert_array_equal(mm.basis_aligned_transformation(ctx.ntt_tf_mat_step1[..., None])[..., 0], bat)
    sh = ntt_sm.NTTShoupContext(q, {"r": r, "c": c, "finite_field_context": ff.ShoupContext(q)})
    assert sh.moduli == [q]
    assert sh.ntt_tf_mat_step1_shoup.dtype == np.uint32 and sh.ntt_tf_mat_step2_shoup.dtype == np.uint64
    np.testing.assert_array_equal(sh.ntt_tf_step1, _twiddle(r, r, q, pow(om, c, q)))


def test_coefmap_factorisation_and_its_errors():
    """herot.py:15-53: row / column factors of a decomposable map, and the
    reference's ValueError for every malformed one."""
    from cross_b200 import herot
    row, col = herot.mat_1d_shuffle_to_2d(np.arange(16)[::-1].copy(), 4, 4)
    assert row.dtype == np.int32 and row.tolist() == [3, 2, 1, 0] and col.tolist() == [3, 2, 1, 0]
    row, col = herot.mat_1d_shuffle_to_2d(np.arange(16), 8, 2)
    assert row.tolist() == list(range(8)) and col.tolist() == [0, 1]
    swapped = np.arange(16)
    swapped[[0, 1]] = swapped[[1, 0]]
    for args, msg in (((np.arange(15), 4, 4), "1D of length"), ((np.arange(16).reshape(4, 4), 4, 4), "1D of length"),
                      ((np.arange(0), 0, 0), "positive"), ((np.arange(12), 4, 3), "powers of two"),
                      ((swapped, 4, 4), "NOT decomposable")):
        with pytest.raises(ValueError, match=msg):
            herot.mat_1d_shuffle_to_2d(*args)


def test_twiddle_table_cache():
    """The per-modulus twiddle tables are computed once per process and shared
    read-only by every context over the same (q, r, c); the reference-named
    gen_twiddle_matrix returns a fresh array each call, so a caller that
    writes into it cannot change what the next caller gets."""
    from cross_b200 import ntt_mm
    q = O.find_moduli_ntt(1, 28, 2 * 256)[0]
    a, b = ntt_mm._limb_tables(q, 16, 16), ntt_mm._limb_tables(q, 16, 16)
    assert a is b and all(not t.flags.writeable for t in a)
    assert ntt_mm._limb_bat(q, 16, 16) is ntt_mm._limb_bat(q, 16, 16)
    om = 3                                   # any residue: the helper takes its powers
    m1 = ntt_mm.gen_twiddle_matrix(8, 4, q, om)
    keep = m1.copy()
    m1[:] = 0
    np.testing.assert_array_equal(ntt_mm.gen_twiddle_matrix(8, 4, q, om), keep)
