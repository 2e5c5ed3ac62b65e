"""jax.numpy over numpy: arrays are an ndarray subclass with jax's
functional ``.at[idx].set(v)``; reductions keep the input dtype as jax does
(numpy widens small integer sums); einsum accumulates exactly in
preferred_element_type.  Anything not defined here is numpy's function with
its array results wrapped."""
import numpy as _np

uint8, uint16, uint32, uint64 = _np.uint8, _np.uint16, _np.uint32, _np.uint64
int8, int16, int32, int64 = _np.int8, _np.int16, _np.int32, _np.int64
float16, float32, float64 = _np.float16, _np.float32, _np.float64
complex64, complex128 = _np.complex64, _np.complex128
bool_ = _np.bool_
dtype = _np.dtype
iinfo = _np.iinfo
pi = _np.pi


class _At:
    def __init__(self, arr):
        self._arr = arr

    def __getitem__(self, idx):
        return _AtIndex(self._arr, idx)


class _AtIndex:
    def __init__(self, arr, idx):
        self._arr, self._idx = arr, idx

    def _apply(self, fn):
        out = _np.array(self._arr, copy=True)
        fn(out)
        return _wrap(out)

    def set(self, v):
        def f(o):
            o[self._idx] = _np.asarray(v)
        return self._apply(f)

    def add(self, v):
        def f(o):
            o[self._idx] += _np.asarray(v).astype(o.dtype)
        return self._apply(f)

    def multiply(self, v):
        def f(o):
            o[self._idx] *= _np.asarray(v).astype(o.dtype)
        return self._apply(f)

    def get(self):
        return _wrap(_np.asarray(self._arr)[self._idx])


class ndarray(_np.ndarray):
    """jax array stand-in.  Binary operations promote as numpy does; for the
    integer operands the reference mixes this is jax's lattice too (int64
    with uint64 gives float64 in both)."""

    @property
    def at(self):
        return _At(self)

    def __array_ufunc__(self, ufunc, method, *inputs, **kwargs):
        args = [_np.asarray(x) if isinstance(x, ndarray) else x for x in inputs]
        if "out" in kwargs:
            kwargs["out"] = tuple(_np.asarray(o) if isinstance(o, ndarray) else o for o in kwargs["out"])
        res = getattr(ufunc, method)(*args, **kwargs)
        if isinstance(res, tuple):
            return tuple(_wrap(r) for r in res)
        return _wrap(res)

    def sum(self, axis=None, dtype=None, **kwargs):
        return sum(self, axis=axis, dtype=dtype, **kwargs)

    def __getitem__(self, key):
        try:
            return super().__getitem__(key)
        except IndexError:
            # jax clamps out-of-range integer indices instead of raising
            return super().__getitem__(_clamp(key, self.shape))


def _clamp(key, shape):
    key = key if isinstance(key, tuple) else (key,)
    n_axes = sum_axes = len([k for k in key if k is not None and k is not Ellipsis])
    out, axis = [], 0
    for k in key:
        if k is None:
            out.append(k)
        elif k is Ellipsis:
            axis += len(shape) - n_axes
            out.append(k)
        else:
            if isinstance(k, (int, _np.integer)):
                d = shape[axis]
                k = int(k) + d if k < 0 else int(k)
                k = min(max(k, 0), d - 1)
            out.append(k)
            axis += 1
    del sum_axes
    return tuple(out)


def _wrap(x):
    if isinstance(x, _np.ndarray) and not isinstance(x, ndarray):
        return x.view(ndarray)
    return x


def array(obj, dtype=None, copy=True, **kwargs):
    if isinstance(obj, (list, tuple)) and obj and all(isinstance(o, _np.ndarray) for o in obj):
        obj = _np.stack([_np.asarray(o) for o in obj])
    return _wrap(_np.array(obj, dtype=dtype))


def asarray(obj, dtype=None, **kwargs):
    return array(obj, dtype=dtype)


def sum(a, axis=None, dtype=None, keepdims=False, **kwargs):
    a = _np.asarray(a)
    dt = dtype if dtype is not None else (a.dtype if a.dtype.kind in "uib" and a.dtype != _np.bool_ else None)
    if a.dtype == _np.bool_ and dtype is None:
        dt = _np.int32
    return _wrap(_np.asarray(_np.sum(a, axis=axis, dtype=dt, keepdims=keepdims)))


def prod(a, axis=None, dtype=None, keepdims=False, **kwargs):
    a = _np.asarray(a)
    dt = dtype if dtype is not None else (a.dtype if a.dtype.kind in "ui" else None)
    return _wrap(_np.asarray(_np.prod(a, axis=axis, dtype=dt, keepdims=keepdims)))


def einsum(subscripts, *operands, preferred_element_type=None, optimize=True, **kwargs):
    ops = [_np.asarray(o) for o in operands]
    out_dt = _np.dtype(preferred_element_type) if preferred_element_type is not None else _np.result_type(*ops)
    if (len(ops) == 2 and all(o.dtype == _np.uint8 for o in ops) and out_dt.kind == "u" and out_dt.itemsize >= 4):
        # u8 x u8 products summed over fewer than 2^37 terms stay below 2^53:
        # float64 (BLAS) is exact, then the accumulator type as jax has it
        res = _np.einsum(subscripts, *[o.astype(_np.float64) for o in ops], optimize=optimize)
        return _wrap(res.astype(_np.uint64).astype(out_dt))
    # exact: every operand widened to the accumulation type, integer einsum
    # (wraps modulo 2^bits in that type, as the accumulator does)
    ops = [o.astype(out_dt) for o in ops]
    return _wrap(_np.einsum(subscripts, *ops, optimize=optimize))


def take(a, indices, axis=None, **kwargs):
    return _wrap(_np.take(_np.asarray(a), _np.asarray(indices), axis=axis))


def __getattr__(name):
    fn = getattr(_np, name)
    if not callable(fn) or isinstance(fn, type):
        return fn

    def wrapped(*args, **kwargs):
        args = [_np.asarray(a) if isinstance(a, ndarray) else a for a in args]
        res = fn(*args, **kwargs)
        if isinstance(res, (list, tuple)):
            return type(res)(_wrap(r) for r in res)
        return _wrap(res)
    wrapped.__name__ = name
    return wrapped
