"""The oracle against the reference's own operators at sizes beyond the
reference's N = 16 golden vectors: tests/golden/shim_digests.json holds the
sha256 of jaxite_word's outputs (run by tests/golden/make_golden_shim.py on a
numpy stand-in for jax, itself checked on those N = 16 goldens) on seeded
inputs at N = 2^12 and 2^16, the CKKS client's encode / encrypt / decode
included; the oracle must produce the same bytes (doubles too)."""
import json
import os
import sys

import numpy as np
import pytest

from oracle import ckks as K
from oracle import cross_oracle as O
from oracle import variants as V

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import shim_cases as S  # noqa: E402

with open(os.path.join(HERE, "golden", "shim_digests.json")) as f:
    DIGESTS = json.load(f)["cases"]


def _oracle_ckks(name, kind, p, q):
    n = p["degree"]
    enc = K.ckks_encode(S.ckks_slots(name, p), 2 * n, q, p["scale"])
    if kind == "ckks_encode":
        return np.array(enc, np.uint64)
    if kind == "ckks_encrypt":
        pk, v, e = S.ckks_encrypt_operands(name, p, q)
        return np.array(K.ckks_encrypt(enc, pk, q, v, e), np.uint64)
    coefs = [[0] * len(q) for _ in range(n)]
    for j, qj in enumerate(q):
        col = O.intt_negacyclic(O.bit_reverse_array([enc[d][j] for d in range(n)]), qj, O.root_of_unity(2 * n, qj))
        for d in range(n):
            coefs[d][j] = col[d]
    big_q = 1
    for qj in q:
        big_q *= qj
    return np.array(K.ckks_decode(K.crt_combine(coefs, q), p["scale"], n // 2, big_q, p["p"]), np.complex128)


def _oracle(name, kind, p, moduli):
    if kind.startswith("ckks"):
        return _oracle_ckks(name, kind, p, moduli)
    if kind == "evk":
        sk, a, e = S.evk_operands(name, p, moduli)
        key = K.gen_evaluation_key(sk, moduli[:p["limbs"]], moduli[p["limbs"]:], a, e, dnum=p["dnum"])
        return np.array(key["b"], np.uint64)
    ins = S.inputs(name, kind, p, moduli)
    x = ins.get("x")
    if kind == "ntt":
        if p["reduction"] == "barrett":
            return O.NTTBarrett(moduli, p["r"], p["c"]).ntt(x)
        return V.NTTVariant(moduli, p["r"], p["c"], p["reduction"]).ntt(x)
    if kind == "ff":
        red = p["reduction"]
        if red == "barrett":
            return O.Barrett(moduli).reduce(ins["z"])
        if red == "shoup":
            return V.Shoup(moduli).reduce(ins["z"], ins["z_s"])
        return {"montgomery": V.Montgomery, "bat_lazy": V.BATLazy}[red](moduli).reduce(ins["z"])
    if kind == "ntt_sm":
        # one modulus: the multi-modulus transform with M = 1 (Shoup on one matrix)
        red, r, c = p["reduction"], p["r"], p["c"]
        ctx = O.NTTBarrett(moduli, r, c) if red == "barrett" else V.NTTVariant(moduli, r, c, red)
        y = ctx.ntt(x[..., None] if p["batch"] else x[None, ..., None])[..., 0]
        return y if p["batch"] else y[0]
    if kind == "bconv":
        red = p.get("reduction", "barrett")
        bc = O.BConvBarrett(moduli) if red == "barrett" else V.BConvVariant(moduli, red)
        bc.control_gen([(list(range(p["sq"])), list(range(p["sq"], p["sq"] + p["sp"])))])
        return bc.basis_change_bat(x) if p["bat"] else bc.basis_change(x)
    if kind == "rescale":
        return O.RescalePlan(moduli, p["r"], p["c"]).rescale(x)
    L, r, c, d = p["limbs"], p["r"], p["c"], p["dnum"]
    if kind == "hemul":
        he = O.HEMul(p["batch"], r, c, d, 1, moduli[:L], moduli[L:])
        he.setup_relinearization(ins["evk_a"], ins["evk_b"])
        return he.mul(x)
    n = r * c
    h = O.HERot(r, c, d, moduli[:L], moduli[L:])
    h.control_gen(p["batch"])
    h.setup_rotate(ins["evk_a"], ins["evk_b"],
                   O.precompute_auto_map(n, O.find_automorphism_index_2n_complex(p["rotation"], 2 * n)))
    return h.rotate(x)


def test_every_case_is_recorded():
    assert sorted(DIGESTS) == sorted(name for name, _, _ in S.CASES)


@pytest.mark.parametrize("name,kind,p", S.CASES, ids=[c[0] for c in S.CASES])
def test_oracle_matches_the_reference_run(name, kind, p):
    rec = DIGESTS[name]
    assert rec["kind"] == kind and rec["params"] == p
    out = np.asarray(_oracle(name, kind, p, rec["moduli"]))
    assert list(out.shape) == rec["shape"]
    assert S.digest(out.astype(rec["dtype"])) == rec["sha256"], f"{name}: oracle differs from the reference"
