"""The device against the reference's own operators: every case of
tests/golden/shim_digests.json (jaxite_word run by make_golden_shim.py on a
numpy stand-in for jax, on seeded inputs up to the benchmark point) recomputed
through this library's operator API on the GPU must give the same bytes."""
import json
import math
import os
import sys

import numpy as np
import pytest

from oracle import ckks as K
from oracle import cross_oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import shim_cases as S  # noqa: E402

with open(os.path.join(HERE, "golden", "shim_digests.json")) as f:
    DIGESTS = json.load(f)["cases"]


def _np(t):
    return t.cpu().numpy() if hasattr(t, "cpu") else np.asarray(t)


def _ckks(name, kind, p, q):
    from cross_b200 import ckks_ctx
    n = p["degree"]
    slots = S.ckks_slots(name, p)
    if kind == "ckks_encode":
        return _np(ckks_ctx.ckks_encode(slots, 2 * n, q, [], p["scale"]))
    enc = K.ckks_encode(slots, 2 * n, q, p["scale"])       # the input, from the oracle
    if kind == "ckks_encrypt":
        pk, v, e = S.ckks_encrypt_operands(name, p, q)
        return np.stack([_np(c) for c in ckks_ctx.ckks_encrypt(enc, pk, q, v=v, e=e)])
    coefs = [[0] * len(q) for _ in range(n)]
    for j, qj in enumerate(q):
        col = O.intt_negacyclic(O.bit_reverse_array([enc[d][j] for d in range(n)]), qj, O.root_of_unity(2 * n, qj))
        for d in range(n):
            coefs[d][j] = col[d]
    plain = K.crt_combine(coefs, q)
    return np.array(ckks_ctx.ckks_decode(plain, p["scale"], n // 2, math.prod(q), p["p"]), np.complex128)


def _device(name, kind, p, moduli):
    from cross_b200 import bconv, finite_field, hemul, herot, key_gen, ntt_mm, util
    from cross_b200.ciphertext import Ciphertext
    if kind.startswith("ckks"):
        return _ckks(name, kind, p, moduli)
    if kind == "evk":
        sk, a, e = S.evk_operands(name, p, moduli)
        return _np(key_gen.gen_evaluation_key(sk, moduli[:p["limbs"]], moduli[p["limbs"]:], a=a, e=e,
                                              dnum=p["dnum"])["b"])
    ins = S.inputs(name, kind, p, moduli)
    x = ins.get("x")
    if kind == "ntt":
        ctx_cls, ff_cls = {"barrett": (ntt_mm.NTTCiphertextBarrettContext, finite_field.BarrettContext),
                           "montgomery": (ntt_mm.NTTCiphertextMontgomeryContext, finite_field.MontgomeryContext),
                           "bat_lazy": (ntt_mm.NTTCiphertextBATLazyContext, finite_field.BarrettContext),
                           "shoup": (ntt_mm.NTTCiphertextShoupContext, finite_field.ShoupContext)}[p["reduction"]]
        ctx = ctx_cls(moduli, {"r": p["r"], "c": p["c"], "finite_field_context": ff_cls(moduli)})
        return _np(ctx.ntt(x))
    if kind == "ff":
        red = p["reduction"]
        ctx = {"barrett": finite_field.BarrettContext, "montgomery": finite_field.MontgomeryContext,
               "shoup": finite_field.ShoupContext, "bat_lazy": finite_field.BATLazyContext}[red](moduli)
        return _np(ctx.modular_reduction(ins["z"], ins["z_s"]) if red == "shoup" else ctx.modular_reduction(ins["z"]))
    if kind == "ntt_sm":
        from cross_b200 import ntt_sm
        ctx_cls, ff_cls = {"barrett": (ntt_sm.NTTBarrettContext, finite_field.BarrettContext),
                           "montgomery": (ntt_sm.NTTMontgomeryContext, finite_field.MontgomeryContext),
                           "bat_lazy": (ntt_sm.NTTBATLazyContext, finite_field.BATLazyContext),
                           "shoup": (ntt_sm.NTTShoupContext, finite_field.ShoupContext)}[p["reduction"]]
        ctx = ctx_cls(moduli[0], {"r": p["r"], "c": p["c"], "finite_field_context": ff_cls(moduli[0])})
        return _np(ctx.ntt(x))
    if kind == "bconv":
        b = {"barrett": bconv.BConvBarrett, "montgomery": bconv.BConvMontgomery, "bat_lazy": bconv.BConvBATLazy,
             "shoup": bconv.BConvShoup}[p.get("reduction", "barrett")](moduli)
        b.control_gen([(list(range(p["sq"])), list(range(p["sq"], p["sq"] + p["sp"])))])
        return _np(b.basis_change_bat(x) if p["bat"] else b.basis_change(x))
    r, c = p["r"], p["c"]
    if kind == "rescale":
        ct = Ciphertext({"batch": p["batch"], "num_elements": 2, "degree": r * c, "num_moduli": p["limbs"],
                         "precision": 32, "degree_layout": (r, c)}, {"moduli": moduli})
        ct.modulus_switch_control_gen(degree_layout=(r, c))
        ct.set_batch_ciphertext(x)
        return _np(ct.rescale())
    L, d = p["limbs"], p["dnum"]
    if kind == "hemul":
        he = hemul.HEMul(p["batch"], r, c, d, 1, moduli[:L], moduli[L:])
        he.control_gen(degree_layout=(r, c))
        he.setup_relinearization(ins["evk_a"], ins["evk_b"])
        return _np(he.mul(x))
    n = r * c
    h = herot.HERot(r, c, d, moduli[:L], moduli[L:])
    h.control_gen(batch=p["batch"], degree_layout=(r, c))
    h.setup_rotate(ins["evk_a"], ins["evk_b"],
                   util.precompute_auto_map(n, util.find_automorphism_index_2n_complex(p["rotation"], 2 * n)))
    return _np(h.rotate(x))


@pytest.mark.parametrize("name,kind,p", S.CASES, ids=[c[0] for c in S.CASES])
def test_device_matches_the_reference_run(name, kind, p):
    rec = DIGESTS[name]
    out = np.asarray(_device(name, kind, p, rec["moduli"]))
    assert list(out.shape) == rec["shape"], f"{name}: shape {out.shape}"
    assert S.digest(out.astype(rec["dtype"])) == rec["sha256"], f"{name}: device output differs from the reference"
