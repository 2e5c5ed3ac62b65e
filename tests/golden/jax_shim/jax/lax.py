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


def conv_general_dilated(lhs, rhs, window_strides, padding, lhs_dilation=None, rhs_dilation=None,
                         dimension_numbers=None, feature_group_count=1, batch_group_count=1, precision=None,
                         preferred_element_type=None):
    """1-D convolution in XLA's convention (a cross-correlation), for the
    dimension-number strings of ntt_mm.py / ntt_sm.py ("NCW", "IOW", "NCW" and
    permutations), exact in the accumulator type."""
    assert feature_group_count == 1 and batch_group_count == 1
    assert lhs_dilation in (None, (1,)) and rhs_dilation in (None, (1,))
    lhs_spec, rhs_spec, out_spec = dimension_numbers
    acc = _np.dtype(preferred_element_type) if preferred_element_type is not None else _np.result_type(lhs, rhs)
    x = _np.asarray(lhs).transpose([lhs_spec.index(ch) for ch in "NCW"]).astype(acc)     # (N, C, W)
    k = _np.asarray(rhs).transpose([rhs_spec.index(ch) for ch in "OIW"]).astype(acc)     # (O, I, K)
    (lo, hi), = padding
    (s,) = window_strides
    x = _np.pad(x, ((0, 0), (0, 0), (lo, hi)))
    n_out = (x.shape[2] - k.shape[2]) // s + 1
    out = _np.zeros((x.shape[0], k.shape[0], n_out), acc)
    for t in range(k.shape[2]):
        out += _np.einsum("ncw,oc->now", x[:, :, t:t + s * (n_out - 1) + 1:s], k[:, :, t])
    return _wrap(out.transpose([("NCW").index(ch) for ch in out_spec]))
