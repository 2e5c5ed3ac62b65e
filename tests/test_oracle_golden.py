"""Pin the CPU oracle against the reference's own known-answer vectors.

Every case mirrors one reference test (cited) and compares bit-exactly, so a
GPU result that matches the oracle matches the reference.
"""
import numpy as np
import pytest

from oracle import cross_oracle as O
from tests.conftest import load_golden

U32 = np.uint32
parse = O.parse_ciphertext_string


def test_ntt_intt_golden():
    """ntt_mm_test.py:33-54 (test_NTT_Barrett)."""
    g = load_golden("ntt_mm")
    r, c, b = g["r"], g["c"], g["test_batch"]
    coef = np.concatenate([np.array(g["coef_in"], np.uint64).T.reshape(1, r * c, -1)] * b, 0).astype(U32)
    ev = np.concatenate([np.array(g["eval_in"], U32).T.reshape(1, r * c, -1)] * b, 0)
    ctx = O.NTTBarrett(g["moduli"], r, c)
    out = ctx.ntt(coef.reshape(b, r, c, -1))
    np.testing.assert_array_equal(out.reshape(b, r * c, -1), ev)
    np.testing.assert_array_equal(ctx.intt(out).reshape(b, r * c, -1), coef)


def test_bconv_golden():
    """bconv_test.py:28-48 (basis_change) and 138-158 (BAT congruent to plain)."""
    g = load_golden("bconv")
    x = np.array(g["in_tower"], np.uint64).T
    ref = np.array(g["reference_result"], np.uint64).T
    bc = O.BConvBarrett(g["original_moduli"] + g["target_moduli"])
    bc.control_gen([(list(range(2)), list(range(2, 7)))])
    assert bc.controls[0]["qhat_inv"].tolist() == g["QHatInvModq"]
    assert bc.controls[0]["qhat_modp"].tolist() == g["QHatModp"]
    np.testing.assert_array_equal(bc.basis_change(x), ref)
    diff = (bc.basis_change_bat(x).astype(np.int64) - ref.astype(np.int64)) % np.array(g["target_moduli"])
    assert not diff.any()


def test_bconv_multiple_control_gen():
    """bconv_test.py:78-120 (scalar known answers with primes 17/19/23/29)."""
    bc = O.BConvBarrett([17, 19, 23, 29])
    bc.control_gen([([0], [2]), ([1], [3])])
    assert bc.basis_change(np.array([[[15]]], np.uint64), 0)[0, 0, 0] == 15
    assert bc.basis_change(np.array([[[20]]], np.uint64), 1)[0, 0, 0] == 1
    assert bc.basis_change(np.array([[[20]]], np.uint64), 0)[0, 0, 0] == 3


def test_rescale_golden():
    """rescale_test.py:49-87 (batch 1 and batch 2)."""
    g = load_golden("rescale")
    inc = np.array(parse(g["in_ciphertexts_str"])[0], U32)
    fin = np.array(parse(g["final_result_str"])[0], U32)
    rp = O.RescalePlan(g["q_towers"], 4, 4)
    for b in (1, 2):
        x = np.tile(np.transpose(inc, (0, 2, 1))[None], (b, 1, 1, 1)).reshape(b, 2, 4, 4, 5)
        res = rp.rescale(x).reshape(b, 2, 16, 4)
        for i in range(b):
            np.testing.assert_array_equal(np.transpose(res[i], (0, 2, 1)), fin)


def _herot_inputs():
    g = load_golden("herot")
    r, c, dnum = g["r"], g["c"], g["dnum"]
    rin, rmod = parse(g["rotate_in_ciphertext_str"])
    eb, ebm = parse(g["evalkey_b_vector_str"])
    ea, _ = parse(g["evalkey_a_vector_str"])
    x = np.array(rin, U32).transpose(0, 2, 1).reshape(1, -1, r, c, len(rmod))
    evb = np.array(eb, np.uint64).transpose(0, 2, 1).reshape(dnum, r, c, len(ebm))
    eva = np.array(ea, np.uint64).transpose(0, 2, 1).reshape(dnum, r, c, len(ebm))
    fin = np.array(parse(g["final_result_str"])[0], U32).transpose(0, 2, 1).reshape(1, -1, r * c, len(rmod))
    return g, x, eva, evb, rmod, ebm[len(rmod):], fin


def test_herot_golden():
    """herot_test.py:229-251 (coefMap known answer + final result)."""
    g, x, eva, evb, q, p, fin = _herot_inputs()
    cm = O.precompute_auto_map(16, O.find_automorphism_index_2n_complex(1, 16))
    assert cm == g["coef_map"]
    h = O.HERot(4, 4, 3, q, p)
    h.control_gen(1)
    h.setup_rotate(eva, evb, cm)
    np.testing.assert_array_equal(h.rotate(x), fin)


def test_hemul_golden_and_e2e():
    """hemul_test.py:64-140: HE-Mult bit-exact, then decrypt bit-exact, then
    decode within decimal=3 (|err| < 1.5e-3)."""
    g = load_golden("hemul")
    he = O.HEMul(1, 4, 4, 3, 1, g["q_towers"], g["p_towers"])
    he.setup_relinearization(np.array(g["evalkey_a_vector"], U32), np.array(g["evalkey_b_vector"], U32))
    out = he.mul(np.array(g["input_ciphertext"], U32))
    np.testing.assert_array_equal(out, np.array(g["encrypted_mult_result_ref"], U32))
    enc = out.reshape(1, 2, 16, 4)
    dec = O.ckks_decrypt([enc[0, 0].tolist(), enc[0, 1].tolist()], g["secret_key"], g["q_towers"][:4])
    assert dec == g["decrypted_result_ref"]
    qt = g["q_towers"]
    vals = O.ckks_decode(dec, qt, (g["scalingFactor"] / qt[-1]) ** 2, g["num_slots"], g["p"])
    np.testing.assert_array_almost_equal(vals.real, g["real_values_multiply_result"], decimal=3)


def test_barrett_known_answer():
    """finite_field_test.py:51-55: Barrett(a*b) == a*b mod q for a 31-bit NTT prime."""
    q = O.find_moduli_ntt(1, 31, 16)[0]
    rng = np.random.default_rng(0)
    a = rng.integers(0, q - 1, 4096, dtype=np.uint64)
    b = rng.integers(0, q - 1, 4096, dtype=np.uint64)
    ff = O.Barrett(q)
    np.testing.assert_array_equal(ff.reduce((a * b)[:, None])[:, 0] % q, (a * b) % q)


def test_moduli_search_and_roots():
    """util.py:219-249 / 431-458 properties on the benchmark's 28-bit primes."""
    qs = O.find_moduli_ntt(8, 28, 2 * 4096)
    assert len(set(qs)) == 8 and all(q < 2 ** 28 and (q - 1) % 8192 == 0 for q in qs)
    for q in qs[:2]:
        psi = O.root_of_unity(8192, q)
        assert pow(psi, 4096, q) == q - 1


@pytest.mark.parametrize("n", [16, 64])
def test_ntt_matches_schoolbook_negacyclic(n):
    """Independent check: pre-twisted BAT NTT == bit-reversed negacyclic NTT
    evaluated by definition (util.py:763-798)."""
    q = O.find_moduli_ntt(1, 28, 2 * n)[0]
    r, c = O.default_rc(n)
    ctx = O.NTTBarrett([q], r, c)
    rng = np.random.default_rng(1)
    a = rng.integers(0, q, n, dtype=np.uint64)
    psi = ctx.psi_list[0]
    tw = (a * O.powers_mod(psi, n, q)) % q
    out = ctx.ntt(tw.astype(U32).reshape(1, r, c, 1)).reshape(-1).astype(np.int64) % q
    omega = psi * psi % q
    nat = [sum(int(tw[i]) * pow(omega, i * k, q) for i in range(n)) % q for k in range(n)]
    np.testing.assert_array_equal(out, np.array(O.bit_reverse_array(nat)))


# ---------------------------------------------------------------------------
# Montgomery / Shoup / BAT-lazy variants (oracle/variants.py)
# ---------------------------------------------------------------------------

def _ntt_golden_batch():
    g = load_golden("ntt_mm")
    r, c, b = g["r"], g["c"], g["test_batch"]
    coef = np.concatenate([np.array(g["coef_in"], np.uint64).T.reshape(1, r * c, -1)] * b, 0)
    ev = np.concatenate([np.array(g["eval_in"], U32).T.reshape(1, r * c, -1)] * b, 0)
    return g["moduli"], r, c, b, coef, ev


def test_ntt_montgomery_golden():
    """ntt_mm_test.py:56-90 (test_NTT_Montgomery): Montgomery-form input, NTT,
    back to the original format."""
    from oracle import variants as V
    q, r, c, b, coef, ev = _ntt_golden_batch()
    ctx = V.NTTVariant(q, r, c, "montgomery")
    y = ctx.ntt(ctx.mont.to_computation_format(coef).reshape(b, r, c, -1))
    np.testing.assert_array_equal(ctx.mont.to_original_format(y.reshape(b, r * c, -1)), ev)
    np.testing.assert_array_equal(ctx.mont.to_original_format(ctx.intt(y).reshape(b, r * c, -1)), coef)


def test_ntt_shoup_golden():
    """ntt_mm_test.py:92-114 (test_NTT_Shoup)."""
    from oracle import variants as V
    q, r, c, b, coef, ev = _ntt_golden_batch()
    ctx = V.NTTVariant(q, r, c, "shoup")
    y = ctx.ntt(coef.astype(U32).reshape(b, r, c, -1))
    np.testing.assert_array_equal(ctx.sh.to_original_format(y).reshape(b, r * c, -1), ev)
    np.testing.assert_array_equal(ctx.sh.to_original_format(ctx.intt(y)).reshape(b, r * c, -1), coef)


def test_ntt_bat_lazy_golden():
    """ntt_mm_test.py:116-133 (test_NTT_BATLazy): exact equality."""
    from oracle import variants as V
    q, r, c, b, coef, ev = _ntt_golden_batch()
    ctx = V.NTTVariant(q, r, c, "bat_lazy")
    y = ctx.ntt(coef.astype(U32).reshape(b, r, c, -1))
    np.testing.assert_array_equal(y.reshape(b, r * c, -1), ev)
    np.testing.assert_array_equal(ctx.intt(y).reshape(b, r * c, -1), coef)


@pytest.mark.parametrize("reduction", ["barrett", "montgomery", "bat_lazy", "shoup"])
def test_ntt_single_modulus_golden(reduction):
    """ntt_sm_test.py:28-107: the single-modulus contexts are the multi-modulus
    transform with one modulus."""
    from oracle import variants as V
    g = load_golden("ntt_sm")
    q, r, c = g["modulus"], g["r"], g["c"]
    coef = np.array(g["coef_in"], np.uint64).reshape(1, r, c, 1)
    ev = np.array(g["eval_in"], np.uint64)
    ctx = O.NTTBarrett([q], r, c) if reduction == "barrett" else V.NTTVariant([q], r, c, reduction)
    if reduction == "montgomery":
        y = ctx.ntt(ctx.mont.to_computation_format(coef))
        np.testing.assert_array_equal(ctx.mont.to_original_format(y).reshape(-1), ev)
        np.testing.assert_array_equal(ctx.mont.to_original_format(ctx.intt(y)).reshape(-1), coef.reshape(-1))
        return
    y = ctx.ntt(coef.astype(U32))
    np.testing.assert_array_equal(y.reshape(-1).astype(np.uint64) % q, ev)
    np.testing.assert_array_equal(ctx.intt(y).reshape(-1).astype(np.uint64) % q, coef.reshape(-1))


def test_bconv_bat_lazy_golden():
    """bconv_test.py:53-76 (test_bat_lazy_context): uint64 output congruent to
    the reference result."""
    from oracle import variants as V
    g = load_golden("bconv")
    x = np.array(g["in_tower"], np.uint64).T
    ref = np.array(g["reference_result"], np.uint64).T
    bc = V.BConvVariant(g["original_moduli"] + g["target_moduli"], "bat_lazy")
    bc.control_gen([(list(range(2)), list(range(2, 7)))])
    out = bc.basis_change(x)
    assert out.dtype == np.uint64
    diff = (out.astype(np.int64) - ref.astype(np.int64)) % np.array(g["target_moduli"])
    assert not diff.any()


def test_reduction_contexts_known_answers():
    """finite_field_test.py:40-80: Montgomery, Shoup and BAT-lazy single-modulus
    products reduce to a*b mod q; plus the reference's 16-bit-split Montgomery
    equals (z_hi + q - hi32(t q)) mod 2^32 on random 64-bit inputs."""
    from oracle import variants as V
    q = O.find_moduli_ntt(1, 31, 16)[0]
    rng = np.random.default_rng(0)
    a = rng.integers(0, q - 1, 4096, dtype=np.uint64)
    b = rng.integers(0, q - 1, 4096, dtype=np.uint64)
    ab_q = (a * b) % np.uint64(q)
    mo = V.Montgomery(q)
    res = mo.reduce(mo.to_computation_format(a).astype(np.uint64) * mo.to_computation_format(b).astype(np.uint64))
    np.testing.assert_array_equal(mo.to_original_format(res), ab_q)
    sh = V.Shoup(q)
    np.testing.assert_array_equal(sh.to_original_format(sh.reduce(a * b, sh.precompute_constant_operand(a) * b)), ab_q)
    lz = V.BATLazy(q)
    np.testing.assert_array_equal(lz.to_original_format(lz.reduce(a * b)), ab_q)
    z = rng.integers(0, 2 ** 63, 4096, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, 4096, dtype=np.uint64)
    qi = pow(q, -1, 1 << 32)
    want = [((int(v) >> 32) + q - (((int(v) & 0xFFFFFFFF) * qi & 0xFFFFFFFF) * q >> 32)) & 0xFFFFFFFF for v in z]
    np.testing.assert_array_equal(mo.reduce(z), np.array(want, np.uint64))


# ---------------------------------------------------------------------------
# CKKS client side (oracle/ckks.py)
# ---------------------------------------------------------------------------

CKKS_TEST = dict(degree=16, slots=8, q_towers=[1073742881, 1073742721, 1073741441, 1073741857, 524353],
                 p_towers=[1073740609, 1073739937, 1073739649], scale=563019763943521, p=30)
CKKS_IN1 = [complex(v, 0) for v in (0.25, 0.5, 0.75, 1, 2, 3, 4, 5)]


def _ckks_keys(rng):
    from oracle import ckks as K
    c = CKKS_TEST
    deg, mods = c["degree"], c["q_towers"] + c["p_towers"]
    s = [int(v) for v in rng.integers(0, 2, deg)]
    e = [int(v) for v in np.rint(rng.normal(0, 3.19, deg))]
    a = [[int(v) for v in rng.integers(0, q, deg)] for q in mods]
    return K.gen_pke_pair(c["q_towers"], c["p_towers"], deg, s, a, e)


def test_ckks_encode_decode_round_trip():
    """ckks_ctx_test.py:75-83 (decimal=3) on the oracle."""
    from oracle import ckks as K
    c = CKKS_TEST
    enc = K.ckks_encode(CKKS_IN1, 2 * c["degree"], c["q_towers"], c["scale"])
    dec = K.decode_rns(enc, c["q_towers"], c["scale"], c["slots"], c["p"], is_ntt=True)
    np.testing.assert_array_almost_equal([d.real for d in dec], [v.real for v in CKKS_IN1], decimal=3)


def test_ckks_encrypt_decrypt_round_trip():
    """ckks_ctx_test.py:85-97 (decimal=3) on the oracle, with seeded keys and noise."""
    from oracle import ckks as K
    c = CKKS_TEST
    deg, qt = c["degree"], c["q_towers"]
    rng = np.random.default_rng(3)
    kp = _ckks_keys(rng)
    ev = lambda co, q: O.bit_reverse_array(K.ntt_negacyclic([x % q for x in co], q, O.root_of_unity(2 * deg, q)))  # noqa: E731
    vco = [int(v) for v in rng.integers(0, 2, deg)]
    e0 = [int(v) for v in np.rint(rng.normal(0, 3.19, deg))]
    e1 = [int(v) for v in np.rint(rng.normal(0, 3.19, deg))]
    enc = K.ckks_encode(CKKS_IN1, 2 * deg, qt, c["scale"])
    ctx = K.ckks_encrypt(enc, kp["public_key"], qt, [ev(vco, q) for q in qt],
                         ([ev(e0, q) for q in qt], [ev(e1, q) for q in qt]))
    dec = K.decode_rns(O.ckks_decrypt(ctx, kp["secret_key"], qt), qt, c["scale"], c["slots"], c["p"])
    np.testing.assert_array_almost_equal([d.real for d in dec], [v.real for v in CKKS_IN1], decimal=3)


def test_ckks_decode_of_the_hemul_golden():
    """hemul_test.py:100-140: the decrypted HE-Mult result decodes (CRT +
    special FFT of oracle/ckks.py) to the reference's slot values."""
    from oracle import ckks as K
    g = load_golden("hemul")
    qt = g["q_towers"][:4]
    vals = K.decode_rns(g["decrypted_result_ref"], qt, (g["scalingFactor"] / g["q_towers"][-1]) ** 2,
                        g["num_slots"], g["p"])
    np.testing.assert_array_almost_equal([v.real for v in vals], g["real_values_multiply_result"], decimal=3)


def test_negacyclic_transform_round_trip():
    """util.py:763-827: intt_negacyclic inverts ntt_negacyclic."""
    from oracle import ckks as K
    q = O.find_moduli_ntt(1, 28, 64)[0]
    psi = O.root_of_unity(64, q)
    a = [int(v) for v in np.random.default_rng(0).integers(0, q, 32)]
    assert O.intt_negacyclic(K.ntt_negacyclic(a, q, psi), q, psi) == a
