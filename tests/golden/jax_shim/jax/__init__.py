"""A numpy stand-in for the part of jax that jaxite_word's operators use, so
that the reference's own code runs in a container without jax to generate
golden vectors (tests/golden/make_golden_shim.py).  Test infrastructure only.

Semantics kept: x64 integer dtypes with wrap-around, einsum accumulated in
preferred_element_type (exactly), bitcast_convert_type little-endian byte
views, functional .at[].set updates.  jit / named_call / vmap run eagerly;
random draws come from numpy (the reference uses them only for perf_test
constants and random inputs, which the generator supplies itself).
"""
import numpy as _np

from . import numpy  # noqa: F401
from . import lax  # noqa: F401
from . import random  # noqa: F401
from . import sharding  # noqa: F401
from .numpy import ndarray as Array  # noqa: F401


class _Config:
    def update(self, *args, **kwargs):
        pass


config = _Config()


def jit(fun=None, **kwargs):
    if fun is None:
        return lambda f: f
    return fun


def named_call(fun, name=None):
    return fun


def device_get(x):
    return x


def device_put(x, *args, **kwargs):
    return x


def block_until_ready(x):
    return x


def devices(*args):
    return [_Device()]


def device_count():
    return 1


class _Device:
    device_kind = "cpu"
    platform = "cpu"


def vmap(fun, in_axes=0, out_axes=0):
    """Eager vmap: fun applied to every slice along the mapped axes, results
    stacked on out_axes (int or None per argument in in_axes)."""
    def mapped(*args):
        axes = in_axes if isinstance(in_axes, (tuple, list)) else (in_axes,) * len(args)
        n = None
        for a, ax in zip(args, axes):
            if ax is not None:
                n = _np.shape(a)[ax]
                break
        outs = []
        for i in range(n):
            sl = [a if ax is None else _np.take(a, i, axis=ax) for a, ax in zip(args, axes)]
            outs.append(fun(*sl))
        if isinstance(outs[0], tuple):
            return tuple(numpy.stack([o[k] for o in outs], axis=out_axes) for k in range(len(outs[0])))
        return numpy.stack(outs, axis=out_axes)
    return mapped


def make_mesh(*args, **kwargs):
    return None
