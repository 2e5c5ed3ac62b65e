"""Key generation (jaxite_word key_gen.py) on the GPU: the public key, the
relinearisation and rotation keys, and the polynomial samplers: coefficients are sampled on the host (ternary {0, 1} and rounded
Gaussian, as the reference samples them, from the OS's CSPRNG), mapped into
every modulus and brought to the reference's evaluation form (psi twist, BAT
NTT, bit-reversed order) by the CUDA kernels; ``b`` is combined on the device.
"""
from __future__ import annotations

import secrets
from typing import Any, Dict, List

import numpy as np

from . import _lib, _tensor
from .ckks_ctx import _negacyclic, _rns_of, _rows, _sample_coeffs, sigma

MAX_INT_64 = 9223372036854775295


class RnsPolynomial:
    """The fields of rns.RnsPolynomial that the samplers fill (coefficient form)."""

    def __init__(self, degree: int, moduli, coeffs, is_ntt: bool = False):
        self.degree, self.moduli, self.coeffs, self.is_ntt = degree, list(moduli), coeffs, is_ntt


def gen_ternary_uniform_polynomial(degree: int, moduli) -> RnsPolynomial:
    """key_gen.py:18-21: coefficients uniform in {0, 1}."""
    return RnsPolynomial(degree, moduli, _rns_of(_sample_coeffs(degree, "ternary"), moduli))


def gen_uniform_polynomial(degree: int, moduli) -> RnsPolynomial:
    """key_gen.py:24-29: every residue uniform in [0, q)."""
    rng = np.random.Generator(np.random.PCG64(secrets.randbits(128)))
    return RnsPolynomial(degree, moduli, np.stack([rng.integers(0, q, size=degree) for q in moduli]).astype(np.uint32))


def gen_gaussian_polynomial(degree: int, moduli, sigma: float) -> RnsPolynomial:
    """key_gen.py:32-50: coefficients round(N(0, sigma))."""
    return RnsPolynomial(degree, moduli, _rns_of(_sample_coeffs(degree, "gauss", sigma), moduli))


def gen_pke_pair(q_towers, p_towers, degree: int, noise_std: float = sigma, noise_scale: int = 1,
                 a_ref=None, s_ref=None, e_ref=None) -> Dict[str, Any]:
    """key_gen.py:299-347: {"public_key": [b, a], "secret_key": s} with every
    array (moduli, degree) in evaluation form on the device; b = e ns - a s."""
    moduli = list(q_towers) + list(p_towers)
    neg = _negacyclic(moduli, degree)
    s = neg.forward(gen_ternary_uniform_polynomial(degree, moduli).coeffs)
    s = _rows(s_ref) if s_ref is not None else s
    a = neg.forward(gen_uniform_polynomial(degree, moduli).coeffs)
    a = _rows(a_ref) if a_ref is not None else a
    e = neg.forward(gen_gaussian_polynomial(degree, moduli, noise_std).coeffs)
    e = _rows(e_ref) if e_ref is not None else e
    if any(tuple(x.shape) != (len(moduli), degree) for x in (s, a, e)):
        raise ValueError(f"gen_pke_pair: s, a, e must be ({len(moduli)}, {degree})")
    b = _tensor.empty_u32((len(moduli), degree))
    _tensor.call("cross_pke_b", neg.ff.handle(), e.data_ptr(), a.data_ptr(), s.data_ptr(), int(noise_scale),
                 b.data_ptr(), degree, _lib.cuda_stream())
    return {"public_key": [b, a], "secret_key": s[:len(q_towers)]}


def ntt_form(coeffs, moduli, degree: int):
    """Integer coefficients (one vector, or (moduli, degree) residues) in the
    reference's evaluation form: bit_reverse_array(ntt_negacyclic_bit_reverse(.))
    per modulus (key_gen.py:323-327)."""
    c = np.asarray(coeffs)
    x = _rns_of(c, moduli) if c.ndim == 1 else c.astype(np.uint32)
    return _negacyclic(list(moduli), degree).forward(x)


def modulus_switch(coefficient, cur_moduli: int = 524353, target_moduli: int = 1152921504606845473):
    """key_gen.py:77-105 (host helper on Python integers)."""
    thr = (cur_moduli + 1) // 2

    def one(v):
        v = int(v)
        return v if v < thr else target_moduli + v - cur_moduli
    return [one(c) for c in coefficient] if isinstance(coefficient, list) else one(coefficient)


def _ff(moduli):
    from .ckks_ctx import _negacyclic_ff
    return _negacyclic_ff(moduli)


def key_switch_gen(sOld, sNew, q_list, p_list, noise_std: float = sigma, noise_scale: int = 1, a=None, e=None,
                   dnum: int = 3) -> Dict[str, Any]:
    """key_gen.py:147-254 on the GPU.  sOld, sNew: (Q, N) evaluations; a, e
    (optional): parts x (Q + P) x N evaluations.  Returns the reference's dict
    with "a" and "b" as (parts, Q + P, N) CUDA tensors (a as given when given)."""
    t = _tensor.torch()
    q_list, p_list = [int(q) for q in q_list], [int(p) for p in p_list]
    s_new = _rows(sNew).contiguous()
    size_q, size_p = len(q_list), len(p_list)
    degree = s_new.shape[1]
    moduli = q_list + p_list
    if tuple(s_new.shape) != (size_q, degree):
        raise ValueError(f"key_switch_gen: sNew must be ({size_q}, N)")
    s_old = _rows(sOld).contiguous()
    if tuple(s_old.shape) != (size_q, degree):
        raise ValueError(f"key_switch_gen: sOld must be ({size_q}, N)")
    neg_q, neg_qp = _negacyclic(q_list, degree), _negacyclic(moduli, degree)
    s_out = neg_q.inverse(s_new)                                       # coefficients over Q (key_gen.py:176-181)
    s_p = _tensor.empty_u32((size_p, degree))
    if size_p:
        _tensor.call("cross_mod_switch_lift", s_out[0].contiguous().data_ptr(), degree, q_list[0],
                     _ff(p_list).handle(), s_p.data_ptr(), _lib.cuda_stream())
    s_eva = neg_qp.forward(t.cat([s_out, s_p], 0))                     # key_gen.py:183-195
    P = 1
    for p in p_list:
        P *= p
    pmq = t.from_numpy(np.array([P % q for q in q_list], np.uint32)).to(_tensor.device())
    per = (size_q + dnum - 1) // dnum
    parts = -(-size_q // per)
    a_parts, b_parts = [], []
    for part in range(parts):
        start, end = per * part, min(size_q, per * part + per)
        a_rows = neg_qp.forward(_rns_of(_sample_coeffs(degree, "ternary"), moduli))   # key_gen.py:211-214
        e_rows = neg_qp.forward(_rns_of(_sample_coeffs(degree, "gauss", noise_std), moduli))
        a_use = _rows(a[part]) if a is not None else a_rows
        e_use = _rows(e[part]) if e is not None else e_rows
        if any(tuple(x.shape) != (size_q + size_p, degree) for x in (a_use, e_use)):
            raise ValueError(f"key_switch_gen: a and e parts must be ({size_q + size_p}, N)")
        b = _tensor.empty_u32((size_q + size_p, degree))
        _tensor.call("cross_ks_key_b", neg_qp.ff.handle(), a_use.data_ptr(), e_use.data_ptr(), s_eva.data_ptr(),
                     s_old.data_ptr(), pmq.data_ptr(), start, end, int(noise_scale), b.data_ptr(), degree,
                     _lib.cuda_stream())
        a_parts.append(a_rows)
        b_parts.append(b)
    return {"a": t.stack(a_parts) if a is None else a, "b": t.stack(b_parts), "modulus": {"Q": q_list, "P": p_list},
            "P": p_list, "shape": (parts, size_q + size_p, degree)}


def gen_evaluation_key(private_key, q, P=1, noise_std: float = sigma, noise_scale: int = 1, a=None, e=None,
                       dnum: int = 3) -> Dict[str, Any]:
    """key_gen.py:108-144: the relinearisation key, from s^2 (evaluation form) to s."""
    q_list = list(q) if not isinstance(q, int) else [q]
    p_list = list(P) if isinstance(P, (list, tuple)) else [int(P)]
    s = _rows(private_key).contiguous()
    if s.shape[0] != len(q_list):
        raise ValueError("private_key must have one row per q modulus (len(q))")
    s_old = _tensor.empty_u32(tuple(s.shape))
    _tensor.call("cross_mul_reduce_lm", _ff(q_list).handle(), s.data_ptr(), s.data_ptr(), s_old.data_ptr(),
                 s.shape[1], _lib.cuda_stream())
    return key_switch_gen(s_old, s, q_list, p_list, noise_std, noise_scale, a, e, dnum)


def find_automorphism_index_2n_complex(i: int, m: int) -> int:
    """key_gen.py:257-270."""
    from . import util
    return util.find_automorphism_index_2n_complex(i, m)


def precompute_rotation_key_map(n: int, k: int) -> List[int]:
    """key_gen.py:273-285 (vectorised)."""
    from . import util
    logm = (2 * n).bit_length() - 1
    j = np.arange(n, dtype=np.int64)
    mul = ((j << 1) + 1) * k
    idx = (mul - ((mul >> logm) << logm)) >> 1
    rev = util.bit_reverse_indices(n)
    out = np.zeros(n, np.int64)
    out[rev] = rev[idx]
    return out.tolist()


def gen_rotation_key(sk, original_moduli, extend_moduli, rot_index, dnum: int = 3, noise_std: float = sigma,
                     noise_scale: int = 1, a=None, e=None) -> Dict[str, Any]:
    """key_gen.py:288-296: the key from s to s permuted by the rotation map."""
    s = _rows(sk).contiguous()
    n = s.shape[1]
    k = find_automorphism_index_2n_complex(rot_index, 2 * n)
    order = precompute_rotation_key_map(n, pow(k, -1, 2 * n))
    idx = _tensor.torch().tensor(order, dtype=_tensor.torch().int64, device=_tensor.device())
    t = _tensor.torch()
    sk_rot = s.view(t.int32).index_select(1, idx).contiguous().view(t.uint32)
    return key_switch_gen(s, sk_rot, original_moduli, extend_moduli, noise_std, noise_scale, a, e, dnum)
