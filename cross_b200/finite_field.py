"""Finite-field contexts (jaxite_word finite_field.py).

BarrettContext is the reduction of the whole HE pipeline.  The Montgomery,
Shoup and BAT-lazy contexts back the variant NTT / BConv classes.  Every
``modular_reduction`` runs a CUDA kernel; the format conversions
(``to_computation_format`` / ``to_original_format`` / Shoup's
``precompute_constant_operand``) prepare constant tables on the host, as the
reference's offline functions do.
"""
from __future__ import annotations

from typing import List, Union

import numpy as np

from . import _lib, _tensor, util

U32, U64 = np.uint32, np.uint64


class FiniteFieldContextBase:
    """finite_field.py:35-52."""

    def __init__(self, moduli):
        self.moduli = moduli

    def to_computation_format(self, a):
        return a

    def to_original_format(self, a):
        return a

    def get_jax_parameters(self):
        return {}

    def modular_reduction(self, a):
        raise NotImplementedError("Subclasses must implement this method")

    def drop_last_modulus(self):
        raise NotImplementedError("Subclasses must implement this method")


class BarrettContext(FiniteFieldContextBase):
    """finite_field.py:170-272."""

    def __init__(self, moduli: Union[List[int], int]):
        super().__init__(moduli)
        self.moduli = [moduli] if isinstance(moduli, int) else list(moduli)
        s, w, sw, m = util.barrett_constants(self.moduli)
        self.barrett_s, self.barrett_w, self.barrett_s_w, self.barrett_m = s, w, sw, m
        self.m = np.array(m, U64)
        self.moduli_reduction = np.array(self.moduli, U64)
        self.w = np.array(w, np.uint16)
        self.s_w = np.array(sw, np.uint16)
        self._handle = None
        self._active = len(self.moduli)

    # -- device modulus set -------------------------------------------------
    def handle(self):
        """cross_moduli handle for the active moduli (created lazily)."""
        if self._handle is None:
            n = self._active
            q = np.array(self.moduli[:n], U32)
            mm = np.array(self.barrett_m[:n], U64)
            w = np.array(self.barrett_w[:n], U32)
            sw = np.array(self.barrett_s_w[:n], U32)
            out = _lib.vp()
            _lib.check(_lib.lib().cross_moduli_create(n, q.ctypes.data, mm.ctypes.data, w.ctypes.data,
                                                      sw.ctypes.data, _lib.C.byref(out)), "cross_moduli_create")
            self._handle = out
        return self._handle

    def __del__(self):
        if getattr(self, "_handle", None) is not None and getattr(_lib, "_lib", None) is not None:
            _lib._lib.cross_moduli_destroy(self._handle)
            self._handle = None

    def get_jax_parameters(self):
        return {"barrett_m": tuple(self.barrett_m), "moduli": tuple(self.moduli),
                "barrett_w": tuple(self.barrett_w), "barrett_s_w": tuple(self.barrett_s_w)}

    def modular_reduction(self, z):
        """finite_field.py:201-230 on the GPU: z (..., M) uint64/uint32 -> uint32."""
        t, is64 = _tensor.to_any(z)
        M = self._active
        if t.shape[-1] != M:
            raise ValueError(f"last axis {t.shape[-1]} != number of moduli {M}")
        out = _tensor.empty_u32(t.shape)
        _tensor.call("cross_mod_reduce", self.handle(), t.data_ptr(), int(is64), out.data_ptr(),
                     t.numel() // M, _lib.cuda_stream())
        return out

    def modular_reduction_single_modulus(self, z, modulus_index: int):
        """finite_field.py:233-262."""
        sub = BarrettContext([self.moduli[modulus_index]])
        t, _ = _tensor.to_any(z)
        return sub.modular_reduction(t.reshape(*t.shape, 1)).reshape(t.shape)

    def drop_last_modulus(self):
        """finite_field.py:265-272 (moduli list kept, active constants sliced)."""
        self._active -= 1
        self.m = self.m[:-1]
        self.moduli_reduction = self.moduli_reduction[:-1]
        self.w = self.w[:-1]
        self.s_w = self.s_w[:-1]
        if self._handle is not None:
            _lib.lib().cross_moduli_destroy(self._handle)
            self._handle = None


class _DeviceModuli:
    """A cross_moduli handle over the context's active moduli (Barrett constants
    of finite_field.py:177-180; the device derives the Montgomery, Shoup and
    BAT-lazy constants from the same moduli)."""

    _handle = None

    def _active_moduli(self):
        return self.moduli[: len(self.moduli_reduction)]

    def handle(self):
        if self._handle is None:
            mods = self._active_moduli()
            _, w, sw, m = util.barrett_constants(mods)
            q = np.array(mods, U32)
            mm, w, sw = np.array(m, U64), np.array(w, U32), np.array(sw, U32)
            out = _lib.vp()
            _lib.check(_lib.lib().cross_moduli_create(len(mods), q.ctypes.data, mm.ctypes.data, w.ctypes.data,
                                                      sw.ctypes.data, _lib.C.byref(out)), "cross_moduli_create")
            self._handle = out
        return self._handle

    def _drop_handle(self):
        if self._handle is not None and getattr(_lib, "_lib", None) is not None:
            _lib._lib.cross_moduli_destroy(self._handle)
        self._handle = None

    def __del__(self):
        self._drop_handle()

    def _reduce_device(self, reduction, z, z_s=None):
        """cross_mod_reduce_ex over the last axis (one modulus: every element)."""
        t = _tensor.torch()
        zt = _tensor.to_u64(z)
        M = len(self.moduli_reduction)
        shape = tuple(zt.shape)
        if M == 1:
            zt = zt.reshape(-1, 1)
        elif zt.dim() == 0 or shape[-1] != M:
            raise ValueError(f"last axis {shape[-1] if shape else None} != number of moduli {M}")
        zs = None
        if reduction == _lib.REDUCTION_SHOUP:
            zs = _tensor.to_u64(z_s).reshape(zt.shape)
        dt = t.uint64 if reduction == _lib.REDUCTION_BAT_LAZY else t.uint32
        out = t.empty(tuple(zt.shape), dtype=dt, device=_tensor.device())
        _tensor.call("cross_mod_reduce_ex", self.handle(), reduction, zt.data_ptr(),
                     zs.data_ptr() if zs is not None else None, out.data_ptr(), zt.numel() // zt.shape[-1],
                     _lib.cuda_stream())
        return out.reshape(shape)


class MontgomeryContext(_DeviceModuli, FiniteFieldContextBase):
    """finite_field.py:58-164."""

    def __init__(self, moduli):
        super().__init__(moduli)
        self.moduli = [moduli] if isinstance(moduli, int) else list(moduli)
        self.w = 32
        self.w_inv = [util.modinv(1 << self.w, m) for m in self.moduli]
        self.w_inv_reduction = np.array(self.w_inv, U64)
        self.moduli_reduction = np.array(self.moduli, U64)
        self.moduli_inv_32 = [util.modinv(m, 2 ** 32) for m in self.moduli]
        self.moduli_low16 = [m & 0xFFFF for m in self.moduli]
        self.moduli_high16 = [m >> 16 for m in self.moduli]

    def to_computation_format(self, a):
        """finite_field.py:78-81 (host: table preparation)."""
        return ((np.asarray(a).astype(U64) << U64(self.w)) % self.moduli_reduction).astype(U32)

    def to_original_format(self, a):
        """finite_field.py:83-84 (host)."""
        return (np.asarray(a).astype(U64) * self.w_inv_reduction) % self.moduli_reduction

    def get_jax_parameters(self):
        return {"moduli": tuple(self.moduli), "moduli_inv_32": tuple(self.moduli_inv_32),
                "moduli_low": tuple(self.moduli_low16), "moduli_high": tuple(self.moduli_high16)}

    def modular_reduction(self, z):
        """finite_field.py:94-154 on the GPU: uint64 -> uint32 (lazy)."""
        return self._reduce_device(_lib.REDUCTION_MONTGOMERY, z)

    def drop_last_modulus(self):
        """finite_field.py:156-164 (w_inv sliced as well, so that
        to_original_format keeps working on the shorter basis)."""
        self.moduli_reduction = self.moduli_reduction[:-1]
        self.w_inv_reduction = self.w_inv_reduction[:-1]
        self._drop_handle()


class ShoupContext(_DeviceModuli, FiniteFieldContextBase):
    """finite_field.py:278-338."""

    def __init__(self, moduli):
        super().__init__(moduli)
        self.moduli = [moduli] if isinstance(moduli, int) else list(moduli)
        self.moduli_reduction = np.array(self.moduli, U64)
        self.q = np.array(self.moduli, U64)
        self.w = 32

    def to_computation_format(self, a):
        """finite_field.py:289-291."""
        return (np.asarray(a).astype(U64) % self.moduli_reduction).astype(U32)

    def to_original_format(self, a):
        """finite_field.py:293-294."""
        return (np.asarray(a).astype(U64) % self.moduli_reduction).astype(U32)

    def precompute_constant_operand(self, a):
        """finite_field.py:295-297: (a << 32) // q.  The reference runs this
        under JAX, where a uint32 array shifted by 32 is 0 (XLA's shift
        semantics): a uint32 input gives 0, as in BConvShoup.control_gen
        (bconv.py:313-314); wider inputs give floor(a 2^32 / q)."""
        a = np.asarray(a)
        if a.dtype == np.uint32:
            return np.zeros(a.shape, U64)
        return (a.astype(U64) << U64(self.w)) // self.moduli_reduction

    def get_jax_parameters(self):
        return {"moduli": tuple(self.moduli)}

    def modular_reduction(self, z, z_s):
        """finite_field.py:300-330 on the GPU: (z - (z_s >> 32) q) cast to uint32."""
        return self._reduce_device(_lib.REDUCTION_SHOUP, z, z_s)

    def drop_last_modulus(self):
        """finite_field.py:332-338."""
        self.moduli_reduction = self.moduli_reduction[:-1]
        self.q = self.q[:-1]
        self._drop_handle()


class BATLazyContext(_DeviceModuli, FiniteFieldContextBase):
    """finite_field.py:344-428."""

    def __init__(self, moduli):
        super().__init__(moduli)
        self.moduli = [moduli] if isinstance(moduli, int) else list(moduli)
        self.L = 4
        qa = np.array(self.moduli, U64)
        r_vals = (U64(1) << (np.arange(4, 8, dtype=U64) * U64(8)))[None, :] % qa[:, None]
        self.R = ((r_vals[:, :, None] >> (np.arange(4, dtype=U64) * U64(8))[None, None, :]) & U64(0xFF)).astype(np.uint8)
        self.moduli_reduction = qa

    def to_computation_format(self, a):
        return a

    def to_original_format(self, a):
        """finite_field.py:375-376."""
        return (np.asarray(a).astype(U64) % self.moduli_reduction).astype(U32)

    def get_jax_parameters(self):
        return {"moduli": tuple(self.moduli), "R": self.R}

    def modular_reduction(self, z):
        """finite_field.py:378-425 on the GPU: uint64 -> uint64 congruent to z."""
        return self._reduce_device(_lib.REDUCTION_BAT_LAZY, z)

    def drop_last_modulus(self):
        """finite_field.py:427-428."""
        self.moduli = self.moduli[:-1]
        self.R = self.R[:-1]
        self.moduli_reduction = self.moduli_reduction[:-1]
        self._drop_handle()
