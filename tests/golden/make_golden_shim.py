"""Runs the reference's own operators (jaxite_word, read where it lies) on the
numpy stand-in for jax in tests/golden/jax_shim, and writes
tests/golden/shim_digests.json: for every case of shim_cases.py the moduli
and the sha256 of the reference's output on the seeded inputs.

The stand-in is first held to the reference's own golden vectors at N = 16
(ntt_mm_test.py, bconv_test.py, rescale_test.py, hemul_test.py,
herot_test.py, as extracted into tests/golden/*.json): if the reference run
through it does not reproduce them, nothing is written.

    python tests/golden/make_golden_shim.py <path of the reference's jaxite_word directory> [--regenerate]
"""
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "jax_shim"))
sys.path.insert(0, HERE)

import shim_cases as S  # noqa: E402

U32 = np.uint32


def load(name):
    with open(os.path.join(HERE, f"{name}.json")) as f:
        return json.load(f)


def check_stand_in(util, ntt, ff, bconv, Ciphertext, HEMul, HERot):
    """The reference through the stand-in reproduces its N = 16 goldens."""
    g = load("ntt_mm")
    q, r, c = g["moduli"], g["r"], g["c"]
    coef = np.array(g["coef_in"], np.uint64).T.reshape(1, r, c, -1).astype(U32)
    ev = np.array(g["eval_in"], np.uint64).T.reshape(1, r, c, -1).astype(U32)
    ctx = ntt.NTTCiphertextBarrettContext(moduli=q, parameters={"r": r, "c": c,
                                                                "finite_field_context": ff.BarrettContext(moduli=q)})
    out = np.asarray(ctx.ntt(coef))
    assert np.array_equal(out, ev), "NTT golden"
    assert np.array_equal(np.asarray(ctx.intt(out)), coef), "INTT golden"
    # ntt_mm_test.py:86-121: the Shoup transform (byte convolutions)
    sh = ntt.NTTCiphertextShoupContext(moduli=q, parameters={"r": r, "c": c,
                                                              "finite_field_context": ff.ShoupContext(moduli=q)})
    sh_ev = sh.ntt(coef)
    assert np.array_equal(np.asarray(sh.to_original_format(sh_ev)), ev), "Shoup NTT golden"
    assert np.array_equal(np.asarray(sh.to_original_format(sh.intt(sh_ev))), coef), "Shoup INTT golden"

    g = load("bconv")
    bc = bconv.BConvBarrett(g["original_moduli"] + g["target_moduli"])
    bc.control_gen([(list(range(2)), list(range(2, 7)))])
    x = np.array(g["in_tower"], np.uint64).T.astype(U32)
    assert np.array_equal(np.asarray(bc.basis_change(x)), np.array(g["reference_result"], np.uint64).T), "BConv golden"

    g = load("rescale")
    inc = np.array(util.parse_ciphertext_string(g["in_ciphertexts_str"])[0], U32)
    fin = np.array(util.parse_ciphertext_string(g["final_result_str"])[0], U32)
    ct = Ciphertext({"batch": 1, "num_elements": 2, "degree": 16, "num_moduli": 5, "precision": 32},
                    {"moduli": g["q_towers"], "r": 4, "c": 4})
    ct.modulus_switch_control_gen(degree_layout=(4, 4))
    ct.set_batch_ciphertext(np.transpose(inc, (0, 2, 1))[None].reshape(1, 2, 4, 4, 5))
    ct.rescale()
    res = np.asarray(ct.get_batch_ciphertext()).reshape(1, 2, 16, 4)
    assert np.array_equal(np.transpose(res[0], (0, 2, 1)), fin), "rescale golden"

    g = load("hemul")
    he = HEMul(1, 4, 4, 3, 1, g["q_towers"], g["p_towers"])
    he.control_gen(degree_layout=(4, 4))
    he.setup_relinearization(np.array(g["evalkey_a_vector"], U32), np.array(g["evalkey_b_vector"], U32))
    out = np.asarray(he.mul(np.array(g["input_ciphertext"], U32)))
    assert np.array_equal(out, np.array(g["encrypted_mult_result_ref"], U32)), "HE-Mult golden"

    g = load("herot")
    par = util.parse_ciphertext_string
    rin, rmod = par(g["rotate_in_ciphertext_str"])
    eb, pmods = par(g["evalkey_b_vector_str"])
    ea, _ = par(g["evalkey_a_vector_str"])
    n_q = len(rmod)
    # herot_test.py:237-250
    x = np.array(rin, U32).transpose(0, 2, 1).reshape(1, -1, 4, 4, n_q)
    fin = np.array(par(g["final_result_str"])[0], U32).transpose(0, 2, 1).reshape(1, -1, 16, n_q)
    evb = np.array(eb, np.uint64).transpose(0, 2, 1).reshape(3, 4, 4, len(pmods))
    eva = np.array(ea, np.uint64).transpose(0, 2, 1).reshape(3, 4, 4, len(pmods))
    h = HERot(4, 4, 3, rmod, pmods[n_q:])
    h.control_gen(batch=1, degree_layout=(4, 4))
    h.setup_rotate(eva, evb, np.array(g["coef_map"]))
    assert np.array_equal(np.asarray(h.rotate(x)), fin), "HE-Rotate golden"


def run_case(name, kind, p, util, ntt, ff, bconv, Ciphertext, HEMul, HERot):
    if kind == "ntt":
        n = p["r"] * p["c"]
        q = util.find_moduli_ntt(p["limbs"], 28, 2 * n)
        x = S.inputs(name, kind, p, q)["x"]
        # the finite-field contexts of ntt_mm_test.py:43-135 (the BAT-lazy
        # transform reduces steps 2 and 3 with a BarrettContext)
        ctx_cls, ff_cls = {"barrett": (ntt.NTTCiphertextBarrettContext, ff.BarrettContext),
                           "montgomery": (ntt.NTTCiphertextMontgomeryContext, ff.MontgomeryContext),
                           "bat_lazy": (ntt.NTTCiphertextBATLazyContext, ff.BarrettContext),
                           "shoup": (ntt.NTTCiphertextShoupContext, ff.ShoupContext)}[p["reduction"]]
        ctx = ctx_cls(moduli=q, parameters={"r": p["r"], "c": p["c"], "finite_field_context": ff_cls(moduli=q)})
        out = np.asarray(ctx.ntt(x))
        if p["reduction"] == "barrett":
            assert np.array_equal(np.asarray(ctx.intt(out)), x), f"{name}: INTT(NTT(x)) != x"
        return q, out
    if kind == "ff":
        import jax.numpy as jnp
        q = util.find_moduli_ntt(p["limbs"], 28, 2 * 4096)
        ins = {k: jnp.asarray(v) for k, v in S.inputs(name, kind, p, q).items()}
        cls = {"barrett": ff.BarrettContext, "montgomery": ff.MontgomeryContext, "shoup": ff.ShoupContext,
               "bat_lazy": ff.BATLazyContext}[p["reduction"]]
        ctx = cls(moduli=q)
        out = ctx.modular_reduction(ins["z"], ins["z_s"]) if p["reduction"] == "shoup" else \
            ctx.modular_reduction(ins["z"])
        return q, np.asarray(out)
    if kind == "ntt_sm":
        import ntt_sm
        q = util.find_moduli_ntt(1, 28, 2 * p["r"] * p["c"])
        x = S.inputs(name, kind, p, q)["x"]
        # the finite-field contexts of ntt_sm_test.py (the BAT-lazy one is
        # the lazy context; the transform adds its own Barrett context)
        ctx_cls, ff_cls = {"barrett": (ntt_sm.NTTBarrettContext, ff.BarrettContext),
                           "montgomery": (ntt_sm.NTTMontgomeryContext, ff.MontgomeryContext),
                           "bat_lazy": (ntt_sm.NTTBATLazyContext, ff.BATLazyContext),
                           "shoup": (ntt_sm.NTTShoupContext, ff.ShoupContext)}[p["reduction"]]
        ctx = ctx_cls(q[0], {"r": p["r"], "c": p["c"], "finite_field_context": ff_cls(moduli=q[0])})
        return q, np.asarray(ctx.ntt(x))
    if kind == "bconv":
        ov = util.find_moduli_ntt(p["sq"] + p["sp"], 28, 2 * p["n"])
        x = S.inputs(name, kind, p, ov)["x"]
        cls = {"barrett": bconv.BConvBarrett, "montgomery": bconv.BConvMontgomery, "bat_lazy": bconv.BConvBATLazy,
               "shoup": bconv.BConvShoup}[p.get("reduction", "barrett")]
        bc = cls(ov)
        bc.control_gen([(list(range(p["sq"])), list(range(p["sq"], p["sq"] + p["sp"])))])
        return ov, np.asarray(bc.basis_change_bat(x) if p["bat"] else bc.basis_change(x))
    if kind == "rescale":
        r, c, L, B = p["r"], p["c"], p["limbs"], p["batch"]
        q = util.find_moduli_ntt(L, 28, 2 * r * c)
        x = S.inputs(name, kind, p, q)["x"]
        ct = Ciphertext({"batch": B, "num_elements": 2, "degree": r * c, "num_moduli": L, "precision": 32},
                        {"moduli": q, "r": r, "c": c})
        ct.modulus_switch_control_gen(degree_layout=(r, c))
        ct.set_batch_ciphertext(x)
        ct.rescale()
        return q, np.asarray(ct.get_batch_ciphertext())
    if kind.startswith("ckks"):
        return run_ckks(name, kind, p, util)
    if kind == "evk":
        import key_gen
        ov = util.find_moduli_ntt(p["limbs"] + p["special"], 28, 2 * p["degree"])
        sk, a, e = S.evk_operands(name, p, ov)
        key = key_gen.gen_evaluation_key(sk, ov[:p["limbs"]], ov[p["limbs"]:], a=a, e=e, dnum=p["dnum"])
        return ov, np.array(key["b"], np.uint64)
    r, c, L, K, d, B = p["r"], p["c"], p["limbs"], p["special"], p["dnum"], p["batch"]
    n = r * c
    ov = util.find_moduli_ntt(L + K, 28, 2 * n)
    import jax.numpy as jnp
    # as jax arrays, like the reference's callers pass them (hemul.py:137
    # indexes the keys with an out-of-range index that jax clamps)
    ins = {k: jnp.asarray(v) for k, v in S.inputs(name, kind, p, ov).items()}
    if kind == "hemul":
        he = HEMul(B, r, c, d, 1, ov[:L], ov[L:])
        he.control_gen(degree_layout=(r, c))
        he.setup_relinearization(ins["evk_a"], ins["evk_b"])
        return ov, np.asarray(he.mul(ins["x"]))
    cm = np.array(util.precompute_auto_map(n, util.find_automorphism_index_2n_complex(p["rotation"], 2 * n)))
    h = HERot(r, c, d, ov[:L], ov[L:])
    h.control_gen(batch=B, degree_layout=(r, c))
    h.setup_rotate(ins["evk_a"], ins["evk_b"], cm)
    return ov, np.asarray(h.rotate(ins["x"]))


def run_ckks(name, kind, p, util):
    """ckks_ctx.py:156-236 (encrypt with given v, e), 331-404 (encode),
    407-514 (decode of the encoded plaintext in coefficient form, CRT-combined
    by ckks_ctx.py:517-545)."""
    import ckks_ctx
    n, t = p["degree"], p["towers"]
    q = util.find_moduli_ntt(t, 28, 2 * n)
    enc = ckks_ctx.ckks_encode(S.ckks_slots(name, p), 2 * n, q, [], p["scale"])
    if kind == "ckks_encode":
        return q, np.array(enc, np.uint64)
    if kind == "ckks_encrypt":
        pk, v, e = S.ckks_encrypt_operands(name, p, q)
        return q, np.array(ckks_ctx.ckks_encrypt(enc, pk, q, v=v, e=e), np.uint64)
    coefs = [[0] * t for _ in range(n)]
    for j, qj in enumerate(q):
        col = util.intt_negacyclic_bit_reverse(util.bit_reverse_array([enc[d][j] for d in range(n)]), qj,
                                               util.root_of_unity(2 * n, qj))
        for d in range(n):
            coefs[d][j] = col[d]
    plain = ckks_ctx._crt_combine_rns_plaintext(coefs, q)
    big_q = 1
    for qj in q:
        big_q *= qj
    vals = ckks_ctx.ckks_decode(plain, p["scale"], n // 2, big_q, p["p"])
    return q, np.array(vals, np.complex128)


def main(ref_dir, regenerate=False):
    """Cases already in shim_digests.json with the same parameters are kept
    unless regenerate (the benchmark-point ones take minutes each)."""
    sys.path.insert(0, ref_dir)
    import util
    import ntt_mm as ntt
    import finite_field as ff
    import bconv
    from ciphertext import Ciphertext
    from hemul import HEMul
    from herot import HERot
    mods = (util, ntt, ff, bconv, Ciphertext, HEMul, HERot)
    check_stand_in(*mods)
    print("stand-in reproduces the reference's N = 16 golden vectors")
    out = {"source": "jaxite_word operators run on tests/golden/jax_shim (make_golden_shim.py)", "cases": {}}
    path = os.path.join(HERE, "shim_digests.json")
    old = {}
    if os.path.exists(path) and not regenerate:
        with open(path) as f:
            old = json.load(f)["cases"]
    for name, kind, p in S.CASES:
        if name in old and old[name]["kind"] == kind and old[name]["params"] == p:
            out["cases"][name] = old[name]          # recorded earlier with the same parameters
            continue
        t0 = time.time()
        moduli, res = run_case(name, kind, p, *mods)
        out["cases"][name] = {"kind": kind, "params": p, "moduli": [int(m) for m in moduli],
                              "dtype": str(res.dtype), "shape": list(res.shape), "sha256": S.digest(res)}
        print(f"{name}: {res.dtype}{list(res.shape)} in {time.time() - t0:.1f} s")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if a != "--regenerate"]
    if len(args) != 1:
        sys.exit("usage: python tests/golden/make_golden_shim.py <jaxite_word directory of the reference> [--regenerate]")
    main(args[0], regenerate="--regenerate" in sys.argv)
