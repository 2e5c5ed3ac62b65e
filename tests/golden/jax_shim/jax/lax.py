"""jax.lax subset: bitcast_convert_type and rev."""
import numpy as _np

from .numpy import _wrap


def bitcast_convert_type(x, new_dtype):
    x = _np.ascontiguousarray(_np.asarray(x))
    new = _np.dtype(new_dtype)
    old = x.dtype
    if new.itemsize == old.itemsize:
        return _wrap(x.view(new))
    if new.itemsize < old.itemsize:
        ratio = old.itemsize // new.itemsize
        return _wrap(x.view(new).reshape(x.shape + (ratio,)))
    ratio = new.itemsize // old.itemsize
    assert x.shape[-1] == ratio, "the last axis must hold the bytes of one wider element"
    return _wrap(x.view(new).reshape(x.shape[:-1]))


def rev(x, dimensions):
    return _wrap(_np.flip(_np.asarray(x), axis=tuple(dimensions)))
