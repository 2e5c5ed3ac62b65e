"""Modular addition (jaxite_word add.py) on the GPU."""
from __future__ import annotations

import numpy as np

from . import _lib, _tensor
from . import finite_field as ff_context

_CTX = {}


def _ctx(moduli):
    key = tuple(int(q) for q in np.asarray(_tensor.to_numpy(moduli)).reshape(-1))
    if key not in _CTX:
        _CTX[key] = ff_context.BarrettContext(list(key))
    return _CTX[key]


def jax_add(value_a, value_b, modulus_list):
    """add.py:7-27: (E, L, N) + (E, L, N) -> a + b, minus q where the sum is
    strictly greater than q (the reference keeps results equal to q)."""
    a, b = _tensor.to_u32(value_a), _tensor.to_u32(value_b)
    if a.shape != b.shape or a.dim() != 3:
        raise ValueError("value_a and value_b must have the same (elements, limbs, degree) shape")
    ctx = _ctx(modulus_list)
    E, L, N = a.shape
    if L != len(ctx.moduli):
        raise ValueError(f"{L} limbs but {len(ctx.moduli)} moduli")
    out = _tensor.empty_u32(a.shape)
    _tensor.call("cross_add_mod", ctx.handle(), a.data_ptr(), b.data_ptr(), out.data_ptr(), E, N, _lib.cuda_stream())
    return out


def vmap_add(value_a, value_b, modulus_list):
    """add.py:30-57: same result as jax_add (subtract q when a+b > q)."""
    return jax_add(value_a, value_b, modulus_list)
