"""Device-array plumbing for the operator API (torch is only the allocator)."""
from __future__ import annotations

import numpy as np

from . import _lib


def torch():
    import torch as _t
    if not _t.cuda.is_available():
        raise RuntimeError("cross_b200 operators need a CUDA device (there is no CPU fallback)")
    return _t


def device():
    t = torch()
    return t.device("cuda", t.cuda.current_device())


def to_u32(x):
    """A contiguous uint32 CUDA tensor holding x (numpy, list or torch)."""
    t = torch()
    if isinstance(x, t.Tensor):
        if x.dtype != t.uint32:
            if x.dtype in (t.uint64, t.int64, t.int32):
                x = x.to(t.int64).to(t.uint32) if x.dtype != t.uint64 else _u64_to_u32(x)
            else:
                raise TypeError(f"unsupported dtype {x.dtype}")
        return x.to(device()).contiguous()
    a = np.ascontiguousarray(np.asarray(x).astype(np.uint32))
    return t.from_numpy(a).to(device())


def _u64_to_u32(x):
    # truncating cast (jnp .astype(uint32) semantics)
    t = torch()
    lo = x.contiguous().view(t.int32).reshape(*x.shape, 2)[..., 0]
    return lo.contiguous().view(t.uint32)


def to_u64(x):
    """A contiguous uint64 CUDA tensor holding x (values zero-extended)."""
    t = torch()
    if isinstance(x, t.Tensor):
        if x.dtype == t.uint64:
            return x.to(device()).contiguous()
        if x.dtype == t.uint32:
            x = x.to(device()).contiguous()
            lo = x.view(t.int32).to(t.int64) & 0xFFFFFFFF
            return lo.view(t.uint64)
        if x.dtype in (t.int64, t.int32):
            return x.to(device()).to(t.int64).contiguous().view(t.uint64)
        raise TypeError(f"unsupported dtype {x.dtype}")
    a = np.ascontiguousarray(np.asarray(x).astype(np.uint64))
    return t.from_numpy(a).to(device())


def to_any(x):
    """(tensor, is_u64) for an operand that may be uint32 or uint64."""
    t = torch()
    if isinstance(x, t.Tensor):
        if x.dtype == t.uint64:
            return x.to(device()).contiguous(), True
        return to_u32(x), False
    a = np.asarray(x)
    if a.dtype == np.uint64 or a.dtype == np.int64 and a.size and a.max() >= 2 ** 32:
        return t.from_numpy(np.ascontiguousarray(a.astype(np.uint64))).to(device()), True
    return to_u32(a), False


def empty_u32(shape):
    return torch().empty(tuple(shape), dtype=torch().uint32, device=device())


def workspace(nbytes: int):
    t = torch()
    return t.empty(max(int(nbytes), 1), dtype=t.uint8, device=device())


def to_numpy(x):
    """Host numpy view of a tensor (device tensors are copied) or array."""
    if hasattr(x, "detach") and hasattr(x, "cpu"):
        return x.detach().cpu().numpy()
    return np.asarray(x)


def call(name, *args):
    _lib.check(getattr(_lib.lib(), name)(*args), name)
