"""jax.random subset backed by numpy generators (values differ from jax's)."""
import numpy as _np

from .numpy import _wrap


def key(seed):
    return _np.random.default_rng(int(seed))


PRNGKey = key


def split(k, num=2):
    return [k for _ in range(num)]


def bits(k, shape=(), dtype=_np.uint32):
    dt = _np.dtype(dtype)
    return _wrap(k.integers(0, 2 ** (8 * dt.itemsize), size=shape, dtype=_np.uint64).astype(dt))


def randint(k, shape, minval, maxval, dtype=_np.int32):
    return _wrap(k.integers(int(minval), int(maxval), size=shape, dtype=_np.int64).astype(dtype))
