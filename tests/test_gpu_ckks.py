"""GPU parity of the CKKS client side (ckks_ctx.py, key_gen.py): the special
FFTs, encode, encrypt, decrypt, CRT and decode against the oracle
(oracle/ckks.py) -- bit-exact, doubles included -- and the reference's own
round trips (ckks_ctx_test.py:75-97, decimal=3)."""
import math

import numpy as np
import pytest

from oracle import ckks as K
from oracle import cross_oracle as O
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu
U32 = np.uint32

CKKS_TEST = dict(degree=16, slots=8, q_towers=[1073742881, 1073742721, 1073741441, 1073741857, 524353],
                 p_towers=[1073740609, 1073739937, 1073739649], scale=563019763943521, p=30)
CKKS_IN1 = [complex(v, 0) for v in (0.25, 0.5, 0.75, 1, 2, 3, 4, 5)]


def _np(t):
    return t.cpu().numpy()


def _slots(n, seed):
    rng = np.random.default_rng(seed)
    return [complex(a, b) for a, b in zip(rng.uniform(-1, 1, n), rng.uniform(-1, 1, n))]


def _ev(coeffs, q, deg):
    return O.bit_reverse_array(K.ntt_negacyclic([int(x) % q for x in coeffs], q, O.root_of_unity(2 * deg, q)))


@pytest.mark.parametrize("nh", [1, 8, 64, 2048])
def test_fft_special_bit_exact(nh):
    """ckks_ctx.py:48-110: the device FFTs equal CPython's complex arithmetic bit for bit."""
    from cross_b200 import ckks_ctx
    x = _slots(nh, nh)
    a, b = list(x), list(x)
    ckks_ctx.FFTSpecialInv(a, 4 * nh)
    K.fft_special_inv(b, 4 * nh)
    assert a == b
    ckks_ctx.FFTSpecial(a, 4 * nh)
    K.fft_special(b, 4 * nh)
    assert a == b


@pytest.mark.parametrize("deg,towers,scale", [(16, None, None), (1024, 4, 2.0 ** 40), (4096, 6, 2.0 ** 45)])
def test_encode_bit_exact(deg, towers, scale):
    """ckks_ctx.py:331-404 against the oracle (exact residues)."""
    from cross_b200 import ckks_ctx
    if towers is None:
        qt, scale, x = CKKS_TEST["q_towers"], CKKS_TEST["scale"], CKKS_IN1
    else:
        qt, x = O.find_moduli_ntt(towers, 30, 2 * deg), _slots(deg // 2, deg)
    got = _np(ckks_ctx.ckks_encode(x, 2 * deg, qt, [], scale))
    want = np.array(K.ckks_encode(x, 2 * deg, qt, scale), np.uint64)
    np.testing.assert_array_equal(got.astype(np.uint64), want)


def test_encode_large_values_and_noise_scale_degree():
    """The approx-factor path (logc > max_bits_in_word, ckks_ctx.py:366-380)
    and noise_scale_degree > 1 (ckks_ctx.py:382-387)."""
    from cross_b200 import ckks_ctx
    deg = 64
    qt = O.find_moduli_ntt(3, 30, 2 * deg)
    x = [v * 1000 for v in _slots(deg // 2, 5)]
    got = _np(ckks_ctx.ckks_encode(x, 2 * deg, qt, [], 2.0 ** 60, max_bits_in_word=50))
    np.testing.assert_array_equal(got.astype(np.uint64),
                                  np.array(K.ckks_encode(x, 2 * deg, qt, 2.0 ** 60, max_bits_in_word=50), np.uint64))
    got = _np(ckks_ctx.ckks_encode(x, 2 * deg, qt, [], 2.0 ** 20, noise_scale_degree=3))
    np.testing.assert_array_equal(got.astype(np.uint64),
                                  np.array(K.ckks_encode(x, 2 * deg, qt, 2.0 ** 20, noise_scale_degree=3), np.uint64))


def test_decrypt_and_decode_of_the_hemul_golden():
    """hemul_test.py:100-140: decrypt bit-exact to the reference's result, the
    CRT integers equal, the slot values equal the oracle's bit for bit and the
    reference's within decimal=3."""
    from cross_b200 import ckks_ctx
    g = load_golden("hemul")
    enc = np.array(g["encrypted_mult_result_ref"], U32).reshape(1, 2, 16, 4)
    qt = g["q_towers"][:4]
    dec = _np(ckks_ctx.ckks_decrypt([enc[0, 0].tolist(), enc[0, 1].tolist()], g["secret_key"], qt))
    assert dec.tolist() == g["decrypted_result_ref"]
    assert ckks_ctx._crt_combine_rns_plaintext(dec, qt) == K.crt_combine(g["decrypted_result_ref"], qt)
    big_q = math.prod(qt)
    sf = (g["scalingFactor"] / g["q_towers"][-1]) ** 2
    plain = K.crt_combine(g["decrypted_result_ref"], qt)
    got = ckks_ctx.ckks_decode(plain, sf, g["num_slots"], big_q, g["p"])
    assert got == K.ckks_decode(plain, sf, g["num_slots"], big_q, g["p"])
    np.testing.assert_array_almost_equal([v.real for v in got], g["real_values_multiply_result"], decimal=3)


@pytest.mark.parametrize("deg,towers", [(1024, 5), (4096, 8)])
def test_decrypt_crt_decode_vs_oracle(deg, towers):
    from cross_b200 import ckks_ctx
    qt = O.find_moduli_ntt(towers, 30, 2 * deg)
    rng = np.random.default_rng(deg)
    c = [rng.integers(0, 2 ** 30, size=(deg, towers)).astype(np.uint64) % np.array(qt, np.uint64) for _ in range(3)]
    s = (rng.integers(0, 2 ** 30, size=(towers, deg)).astype(np.uint64) % np.array(qt, np.uint64)[:, None])
    got = _np(ckks_ctx.ckks_decrypt([x.astype(U32) for x in c], s.astype(U32), qt))
    want = O.ckks_decrypt([x.tolist() for x in c], s.tolist(), qt)
    np.testing.assert_array_equal(got.astype(np.int64), np.array(want, np.int64))
    ints = ckks_ctx._crt_combine_rns_plaintext(got, qt)
    assert ints == K.crt_combine(want, qt)


@pytest.mark.parametrize("slots", [1, 2, 4, 6, 4096, 32768])
def test_decode_stddev_vs_oracle(slots):
    """ckks_ctx.py:448-481: the device's approximation-error estimate (parallel
    sums) against the oracle's sequential one at a relative tolerance of 1e-12;
    the reference's sum() compensates, so no summation order is bit for bit."""
    import torch
    from cross_b200 import _lib, _tensor
    rng = np.random.default_rng(slots)
    cur = rng.normal(0.0, 3.0, size=(slots, 2)) + 0.25
    want = K.decode_stddev([complex(a, b) for a, b in cur])
    dev = torch.from_numpy(cur).cuda()
    out = torch.empty(1, dtype=torch.float64, device="cuda")
    _tensor.call("cross_ckks_decode_stddev", dev.data_ptr(), slots, out.data_ptr(), _lib.cuda_stream())
    assert float(out.cpu()[0]) == pytest.approx(want, rel=1e-12)


def test_decode_bit_exact_random():
    """ckks_ctx.py:407-514 on an encoded (noise-free) plaintext of N = 2^12:
    the device slot values equal the oracle's exactly."""
    from cross_b200 import ckks_ctx
    deg, towers, scale = 4096, 4, 2.0 ** 40
    qt = O.find_moduli_ntt(towers, 30, 2 * deg)
    x = _slots(deg // 2, 1)
    enc = K.ckks_encode(x, 2 * deg, qt, scale)
    coefs = [[0] * towers for _ in range(deg)]
    for t, q in enumerate(qt):
        col = O.intt_negacyclic(O.bit_reverse_array([enc[d][t] for d in range(deg)]), q, O.root_of_unity(2 * deg, q))
        for d in range(deg):
            coefs[d][t] = col[d]
    plain = K.crt_combine(coefs, qt)
    big_q = math.prod(qt)
    got = ckks_ctx.ckks_decode(plain, scale, deg // 2, big_q, 40)
    assert got == K.ckks_decode(plain, scale, deg // 2, big_q, 40)
    np.testing.assert_array_almost_equal([v.real for v in got], [v.real for v in x], decimal=3)


def test_encrypt_with_given_noise_bit_exact():
    """ckks_ctx.py:156-235 with v and e given, and gen_pke_pair (key_gen.py:299-347)
    with s, a, e given: both equal the oracle."""
    from cross_b200 import ckks_ctx, key_gen
    c = CKKS_TEST
    deg, qt, pt = c["degree"], c["q_towers"], c["p_towers"]
    mods = qt + pt
    rng = np.random.default_rng(9)
    s = [int(v) for v in rng.integers(0, 2, deg)]
    e = [int(v) for v in np.rint(rng.normal(0, 3.19, deg))]
    a = [[int(v) for v in rng.integers(0, q, deg)] for q in mods]
    kp_ref = K.gen_pke_pair(qt, pt, deg, s, a, e)
    kp = key_gen.gen_pke_pair(qt, pt, deg, s_ref=[_ev(s, q, deg) for q in mods],
                              a_ref=[_ev(a[i], q, deg) for i, q in enumerate(mods)],
                              e_ref=[_ev(e, q, deg) for q in mods])
    np.testing.assert_array_equal(_np(kp["public_key"][0]).astype(np.int64), np.array(kp_ref["public_key"][0]))
    np.testing.assert_array_equal(_np(kp["secret_key"]).astype(np.int64), np.array(kp_ref["secret_key"]))
    enc = K.ckks_encode(CKKS_IN1, 2 * deg, qt, c["scale"])
    v = [_ev([int(x) for x in rng.integers(0, 2, deg)], q, deg) for q in qt]
    e0 = [_ev([int(x) for x in np.rint(rng.normal(0, 3.19, deg))], q, deg) for q in qt]
    e1 = [_ev([int(x) for x in np.rint(rng.normal(0, 3.19, deg))], q, deg) for q in qt]
    got = ckks_ctx.ckks_encrypt(enc, kp_ref["public_key"], qt, v=v, e=(e0, e1))
    want = K.ckks_encrypt(enc, kp_ref["public_key"], qt, v, (e0, e1))
    for g_, w_ in zip(got, want):
        np.testing.assert_array_equal(_np(g_).astype(np.int64), np.array(w_, np.int64))


@pytest.mark.parametrize("deg,slots_n", [(16, 8), (4096, 2048)])
def test_ckks_context_round_trips(deg, slots_n):
    """ckks_ctx_test.py:75-97 on the GPU: encode -> decode(is_ntt) and
    encode -> encrypt (device key pair, sampled noise) -> decrypt -> decode."""
    from cross_b200 import ckks_ctx, key_gen
    if deg == 16:
        c = CKKS_TEST
        qt, pt, scale, p, x = c["q_towers"], c["p_towers"], c["scale"], c["p"], CKKS_IN1
    else:
        qt, pt = O.find_moduli_ntt(8, 30, 2 * deg)[:6], O.find_moduli_ntt(8, 30, 2 * deg)[6:]
        scale, p, x = 2.0 ** 40, 40, [complex(v.real, 0) for v in _slots(slots_n, 2)]
    kp = key_gen.gen_pke_pair(qt, pt, deg)
    params = {"degree": deg, "num_slots": slots_n, "scalingFactor": scale, "output_scale": scale, "q_towers": qt,
              "p_towers": pt, "p": p, "CKKS_M_FACTOR": 1, "max_bits_in_word": 61, "noise_scale_degree": 1,
              "public_key": kp["public_key"], "secret_key": kp["secret_key"]}
    ctx = ckks_ctx.CKKSContext(params)
    enc = ctx.encode(x)
    np.testing.assert_array_almost_equal(ctx.decode(enc, is_ntt=True).real, [v.real for v in x], decimal=3)
    dec = ctx.decode(ctx.decrypt(ctx.encrypt(enc)))
    np.testing.assert_array_almost_equal(dec.real, [v.real for v in x], decimal=3)


def test_ckks_round_trip_full_size():
    """N = 2^16 with 24 towers: encode -> encrypt -> decrypt -> decode on the GPU."""
    from cross_b200 import ckks_ctx, key_gen
    deg = 65536
    mods = O.find_moduli_ntt(32, 28, 2 * deg)
    qt, pt = mods[:24], mods[24:]
    kp = key_gen.gen_pke_pair(qt, pt, deg)
    x = [complex(v.real, 0) for v in _slots(deg // 2, 4)]
    params = {"degree": deg, "num_slots": deg // 2, "scalingFactor": 2.0 ** 40, "output_scale": 2.0 ** 40,
              "q_towers": qt, "p_towers": pt, "p": 40, "public_key": kp["public_key"], "secret_key": kp["secret_key"]}
    ctx = ckks_ctx.CKKSContext(params)
    dec = ctx.decode(ctx.decrypt(ctx.encrypt(ctx.encode(x))))
    np.testing.assert_array_almost_equal(dec.real, [v.real for v in x], decimal=3)


# ---------------------------------------------------------------------------
# key-switching keys and the reference's end-to-end tests
# ---------------------------------------------------------------------------

def _seeded_parts(mods, deg, parts, rng):
    a = [[_ev([int(v) for v in rng.integers(0, 2, deg)], q, deg) for q in mods] for _ in range(parts)]
    e = [[_ev([int(v) for v in np.rint(rng.normal(0, 3.19, deg))], q, deg) for q in mods] for _ in range(parts)]
    return a, e


def test_evaluation_and_rotation_keys_bit_exact():
    """key_gen.py:108-297 with a and e given: b equals the oracle's for the
    relinearisation key and a rotation key."""
    from cross_b200 import key_gen
    c = CKKS_TEST
    deg, qt, pt = c["degree"], c["q_towers"], c["p_towers"]
    mods = qt + pt
    rng = np.random.default_rng(21)
    sk = [_ev([int(v) for v in rng.integers(0, 2, deg)], q, deg) for q in qt]
    a, e = _seeded_parts(mods, deg, 3, rng)
    got = key_gen.gen_evaluation_key(sk, qt, pt, a=a, e=e, dnum=3)
    want = K.gen_evaluation_key(sk, qt, pt, a, e, dnum=3)
    np.testing.assert_array_equal(_np(got["b"]).astype(np.int64), np.array(want["b"], np.int64))
    for rot in (1, 3, -1):
        got = key_gen.gen_rotation_key(sk, qt, pt, rot, dnum=3, a=a, e=e)
        want = K.gen_rotation_key(sk, qt, pt, rot, a, e, dnum=3)
        np.testing.assert_array_equal(_np(got["b"]).astype(np.int64), np.array(want["b"], np.int64))


def _e2e_params(kp, scale_out=None):
    c = CKKS_TEST
    return {"degree": c["degree"], "num_slots": c["slots"], "scalingFactor": c["scale"],
            "output_scale": c["scale"] if scale_out is None else scale_out, "q_towers": c["q_towers"],
            "p_towers": c["p_towers"], "p": c["p"], "CKKS_M_FACTOR": 1, "max_bits_in_word": 61,
            "noise_scale_degree": 1, "public_key": kp["public_key"], "secret_key": kp["secret_key"]}


def test_ckks_encrypt_multiply_decrypt():
    """ckks_ctx_test.py:152-190 on the GPU: device keys (public and
    relinearisation), encode, encrypt, HE-Mult, decrypt, decode."""
    from cross_b200 import ckks_ctx, hemul, key_gen
    c = CKKS_TEST
    qt, pt = c["q_towers"], c["p_towers"]
    kp = key_gen.gen_pke_pair(qt, pt, c["degree"])
    ek = key_gen.gen_evaluation_key(kp["secret_key"], q=qt, P=pt, noise_std=3.19, noise_scale=1, dnum=3)
    eva, evb = (_np(ek[k]).transpose(0, 2, 1).astype(U32) for k in ("a", "b"))
    ctx = ckks_ctx.CKKSContext(_e2e_params(kp, (c["scale"] / qt[-1]) ** 2))
    he = hemul.HEMul(1, 4, 4, 3, 1, qt, pt)
    he.control_gen(degree_layout=(4, 4))
    he.setup_relinearization(eva, evb)
    in2 = [complex(v, 0) for v in (5, 4, 3, 2, 1, 0.75, 0.5, 0.25)]
    e1, e2 = ctx.encrypt(ctx.encode(CKKS_IN1)), ctx.encrypt(ctx.encode(in2))
    ins = np.concatenate([_np(e1.ciphertext), _np(e2.ciphertext)], 1).reshape(1, 4, 4, 4, len(qt)).astype(U32)
    res = _np(he.mul(ins))
    e1.drop_last_modulus()
    e1.set_batch_ciphertext(res.reshape(1, 2, c["degree"], len(qt) - 1))
    dec = ctx.decode(ctx.decrypt(e1))
    np.testing.assert_array_almost_equal(dec.real, [1.25, 2, 2.25, 2, 2, 2.25, 2, 1.25], decimal=3)


def test_ckks_encrypt_rotate_decrypt():
    """ckks_ctx_test.py:99-121 on the GPU with a device rotation key."""
    from cross_b200 import ckks_ctx, herot, key_gen, util
    c = CKKS_TEST
    qt, pt, deg = c["q_towers"], c["p_towers"], c["degree"]
    kp = key_gen.gen_pke_pair(qt, pt, deg)
    coef_map = util.precompute_auto_map(deg, key_gen.find_automorphism_index_2n_complex(1, deg))
    ek = key_gen.gen_rotation_key(kp["secret_key"], qt, pt, rot_index=1, dnum=3, noise_std=3.19, noise_scale=1)
    hr = herot.HERot(4, 4, 3, qt, pt)
    hr.setup_rotate(_np(ek["a"]).astype(np.uint64).transpose(0, 2, 1).reshape(3, 4, 4, -1),
                    _np(ek["b"]).astype(np.uint64).transpose(0, 2, 1).reshape(3, 4, 4, -1), coef_map)
    hr.control_gen(batch=1, degree_layout=(4, 4))
    ctx = ckks_ctx.CKKSContext(_e2e_params(kp))
    enc = ctx.encrypt(ctx.encode(CKKS_IN1))
    res = _np(hr.rotate(_np(enc.ciphertext).reshape(1, 2, 4, 4, len(qt))))
    enc.set_batch_ciphertext(res.reshape(1, 2, deg, len(qt)))
    dec = ctx.decode(ctx.decrypt(enc))
    np.testing.assert_array_almost_equal(dec.real, [0.5, 0.75, 1, 2, 3, 4, 5, 0.25], decimal=3)


def test_ckks_encrypt_rescale_decrypt():
    """ckks_ctx_test.py:123-150 on the GPU: Ciphertext.rescale between encrypt and decrypt."""
    from cross_b200 import ciphertext, ckks_ctx, key_gen
    c = CKKS_TEST
    qt, pt, deg = c["q_towers"], c["p_towers"], c["degree"]
    kp = key_gen.gen_pke_pair(qt, pt, deg)
    ctx = ckks_ctx.CKKSContext(_e2e_params(kp, c["scale"] / qt[-1]))
    ct = ciphertext.Ciphertext({"batch": 1, "num_elements": 2, "degree": deg, "num_moduli": 5, "precision": 32,
                                "degree_layout": (4, 4)}, {"moduli": qt, "r": 4, "c": 4})
    ct.modulus_switch_control_gen(degree_layout=(4, 4))
    enc = ctx.encrypt(ctx.encode(CKKS_IN1))
    ct.set_batch_ciphertext(_np(enc.ciphertext).reshape(1, 2, 4, 4, 5))
    ct.rescale()
    ct.ciphertext = ct.ciphertext.reshape(1, 2, deg, 4)
    dec = ctx.decode(ctx.decrypt(ct))
    np.testing.assert_array_almost_equal(dec.real, [v.real for v in CKKS_IN1], decimal=3)
