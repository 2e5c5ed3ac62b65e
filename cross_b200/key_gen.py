"""Public-key generation and the polynomial samplers (jaxite_word key_gen.py)
on the GPU: coefficients are sampled on the host (ternary {0, 1} and rounded
Gaussian, as the reference samples them, from the OS's CSPRNG), mapped into
every modulus and brought to the reference's evaluation form (psi twist, BAT
NTT, bit-reversed order) by the CUDA kernels; ``b`` is combined on the device.
"""
from __future__ import annotations

import secrets
from typing import Any, Dict

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
