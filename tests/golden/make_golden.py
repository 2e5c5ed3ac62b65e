"""Extract the reference's golden vectors into JSON fixtures.

The reference (EfficientPPML/CROSS, jaxite_word) embeds OpenFHE-produced
known-answer vectors as literals in its test files.  This script reads those
files as TEXT (``ast.literal_eval`` of the literal assignments; nothing of the
reference is imported or executed) and writes one JSON file per test into this
directory.  The committed JSON files are what the tests use; this script only
needs the reference checkout when the fixtures are regenerated:

    python tests/golden/make_golden.py <path of the reference's jaxite_word directory>

Sources:
  ntt_mm_test.py:13-24      NTT / INTT, N=16 (4x4), 3 x 134219681
  ntt_sm_test.py:11-22      single-modulus NTT / INTT, N=16 (4x4), 134219681
  bconv_test.py:13-23       basis change 2 -> 5 moduli, N=16
  rescale_test.py:19-46     rescale 5 -> 4 moduli, N=16, OpenFHE text format
  herot_test.py:75-222      HE-Rotate, N=16, dnum=3, with stage references
  hemul_test.py:16-87       HE-Mult + relinearisation, N=16, dnum=3, with keys,
                            encrypt inputs, decrypt and decode references
"""

from __future__ import annotations

import ast
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def _module(path):
    with open(path) as f:
        return ast.parse(f.read(), filename=path)


def _top_assign(tree, name):
    for node in tree.body:
        if isinstance(node, ast.Assign):
            for t in node.targets:
                if isinstance(t, ast.Name) and t.id == name:
                    return ast.literal_eval(node.value)
    raise KeyError(name)


def _method(tree, cls, meth):
    for node in ast.walk(tree):
        if isinstance(node, ast.ClassDef) and node.name == cls:
            for item in node.body:
                if isinstance(item, ast.FunctionDef) and item.name == meth:
                    return item
    raise KeyError(f"{cls}.{meth}")


def _assigns(func):
    """Literal assignments `x = <literal>` and `self.x = <literal>` in a function body."""
    out = {}
    for node in ast.walk(func):
        if isinstance(node, ast.Assign) and len(node.targets) == 1:
            t = node.targets[0]
            key = t.id if isinstance(t, ast.Name) else (t.attr if isinstance(t, ast.Attribute) else None)
            if key is None:
                continue
            try:
                out[key] = ast.literal_eval(node.value)
            except (ValueError, SyntaxError):
                pass
    return out


def _dump(name, obj):
    path = os.path.join(HERE, name)
    with open(path, "w") as f:
        json.dump(obj, f, separators=(",", ":"))
    print("wrote", path, os.path.getsize(path), "bytes")


def main(ref_dir):
    # ntt_mm_test.py:13-24 -- (name, moduli, psi, batch, r, c, coef_in, eval_in)
    ntt = _top_assign(_module(os.path.join(ref_dir, "ntt_mm_test.py")), "NTT")
    name, q, _psi, _batch, r, c, coef_in, eval_in = ntt[0]
    _dump("ntt_mm.json", dict(source="ntt_mm_test.py:13-24", moduli=q, r=r, c=c,
                              test_batch=2, coef_in=coef_in, eval_in=eval_in))

    # ntt_sm_test.py:11-22 -- (name, modulus, psi, batch, r, c, coef_in, eval_in)
    ntt = _top_assign(_module(os.path.join(ref_dir, "ntt_sm_test.py")), "NTT")
    name, q, _psi, batch, r, c, coef_in, eval_in = ntt[0]
    _dump("ntt_sm.json", dict(source="ntt_sm_test.py:11-22", modulus=q, r=r, c=c, batch=batch,
                              coef_in=coef_in, eval_in=eval_in))

    # bconv_test.py:13-23
    tp = _top_assign(_module(os.path.join(ref_dir, "bconv_test.py")), "TEST_PARAMS")[0]
    _, part, orig, target, qhat_inv, qhat_modp, ref = tp
    _dump("bconv.json", dict(source="bconv_test.py:13-23", in_tower=part, original_moduli=orig,
                             target_moduli=target, QHatInvModq=qhat_inv, QHatModp=qhat_modp,
                             reference_result=ref))

    # rescale_test.py:19-46
    tree = _module(os.path.join(ref_dir, "rescale_test.py"))
    a = _assigns(_method(tree, "RescaleJaxTest", "setUp"))
    _dump("rescale.json", dict(source="rescale_test.py:19-46", q_towers=a["q_towers"],
                               p_towers=a["p_towers"], r=4, c=4,
                               in_ciphertexts_str=a["in_ciphertexts_str"],
                               final_result_str=a["final_result_str"]))

    # herot_test.py:75-222, 230-235
    tree = _module(os.path.join(ref_dir, "herot_test.py"))
    a = _assigns(_method(tree, "HERotTest", "setUp"))
    keys = ["rotate_in_ciphertext_str", "evalkey_a_vector_str", "evalkey_b_vector_str",
            "ks_precompute_ref_str", "ks_core_ext_result_str", "approx_mod_down_result_str",
            "ks_results_ref_str", "final_result_str"]
    _dump("herot.json", dict(source="herot_test.py:75-235", batch=1, r=4, c=4, dnum=3, rotation=1,
                             coef_map=[4, 5, 6, 7, 3, 2, 0, 1, 14, 15, 13, 12, 8, 9, 10, 11],
                             **{k: a[k] for k in keys}))

    # hemul_test.py:16-87
    tree = _module(os.path.join(ref_dir, "hemul_test.py"))
    s = _assigns(_method(tree, "HEMulTest", "setUp"))
    t = _assigns(_method(tree, "HEMulTest", "test_ckks_context_encrypt_multiply_decrypt_debug"))
    keep = ["secret_key", "evalkey_a_vector", "evalkey_b_vector", "input_ciphertext",
            "encrypted_mult_result_ref", "decrypted_result_ref"]
    setup = {k: s[k] for k in ["degree", "num_slots", "scalingFactor", "q_towers", "p_towers", "p",
                               "CKKS_M_FACTOR"]}
    _dump("hemul.json", dict(source="hemul_test.py:16-140", r=4, c=4, batch=1, dnum=3, num_eval_mult=1,
                             real_values_multiply_result=[1.25, 2, 2.25, 2, 2, 2.25, 2, 1.25],
                             decode_decimal=3, **setup, **{k: t[k] for k in keep}))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <jaxite_word directory of the reference>")
    main(sys.argv[1])
