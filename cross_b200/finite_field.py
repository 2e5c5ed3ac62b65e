"""Finite-field contexts (jaxite_word finite_field.py).

BarrettContext is the reduction of the whole HE pipeline; its
``modular_reduction`` runs the CUDA kernel.  The Montgomery, Shoup and
BAT-lazy contexts keep the reference's constructors and host-side formats
(``to_computation_format`` / ``to_original_format`` / constants); their
device reductions are not part of the HE-Mult / HE-Rotate path.
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


class MontgomeryContext(FiniteFieldContextBase):
    """finite_field.py:58-164 (host-side formats)."""

    def __init__(self, moduli):
        super().__init__(moduli)
        self.moduli = [moduli] if isinstance(moduli, int) else list(moduli)
        self.w = 32
        self.w_inv = [util.modinv(1 << self.w, m) for m in self.moduli]
        self.moduli_reduction = np.array(self.moduli, U64)
        self.moduli_inv_32 = [util.modinv(m, 2 ** 32) for m in self.moduli]
        self.moduli_low16 = [m & 0xFFFF for m in self.moduli]
        self.moduli_high16 = [m >> 16 for m in self.moduli]

    def to_computation_format(self, a):
        return ((np.asarray(a).astype(U64) << U64(self.w)) % self.moduli_reduction).astype(U32)

    def to_original_format(self, a):
        return (np.asarray(a).astype(U64) * np.array(self.w_inv, U64)) % self.moduli_reduction

    def modular_reduction(self, z):
        """finite_field.py:94-154 (host numpy; not on the HE path)."""
        z = np.asarray(z).astype(U64)
        q = np.array(self.moduli, U32)
        zl, zh = z.astype(U32), (z >> U64(32)).astype(U32)
        t = (zl * np.array(self.moduli_inv_32, U32)) & U32(0xFFFFFFFF)
        prod = (t.astype(U64) * q.astype(U64)) >> U64(32)
        return (zh.astype(U64) + q - prod).astype(U32)


class ShoupContext(FiniteFieldContextBase):
    """finite_field.py:278-338 (host-side formats)."""

    def __init__(self, moduli):
        super().__init__(moduli)
        self.moduli = [moduli] if isinstance(moduli, int) else list(moduli)
        self.moduli_reduction = np.array(self.moduli, U64)
        self.q = np.array(self.moduli, U64)
        self.w = 32

    def to_computation_format(self, a):
        return (np.asarray(a).astype(U64) % self.moduli_reduction).astype(U32)

    def to_original_format(self, a):
        return (np.asarray(a).astype(U64) % self.moduli_reduction).astype(U32)

    def precompute_constant_operand(self, a):
        return (np.asarray(a).astype(U64) << U64(self.w)) // self.moduli_reduction

    def modular_reduction(self, z, z_s):
        t = np.asarray(z_s).astype(U64) >> U64(32)
        return (np.asarray(z).astype(U64) - t * self.q).astype(U32)


class BATLazyContext(FiniteFieldContextBase):
    """finite_field.py:344-428 (host-side formats)."""

    def __init__(self, moduli):
        super().__init__(moduli)
        self.moduli = [moduli] if isinstance(moduli, int) else list(moduli)
        self.L = 4
        qa = np.array(self.moduli, U64)
        r_vals = (U64(1) << (np.arange(4, 8, dtype=U64) * U64(8)))[None, :] % qa[:, None]
        self.R = ((r_vals[:, :, None] >> (np.arange(4, dtype=U64) * U64(8))[None, None, :]) & U64(0xFF)).astype(np.uint8)
        self.moduli_reduction = qa

    def to_original_format(self, a):
        return (np.asarray(a).astype(U64) % self.moduli_reduction).astype(U32)

    def modular_reduction(self, z):
        zb = np.ascontiguousarray(np.asarray(z).astype(U64)).view(np.uint8).reshape(*np.shape(z), 8)
        A, B = zb[..., :4].astype(np.int64), zb[..., 4:].astype(np.int64)
        R = self.R[0] if len(self.moduli) == 1 else self.R
        res = np.einsum("...i,...ij->...j", B, R.astype(np.int64)) + A
        return np.sum(res.astype(U64) << np.array([0, 8, 16, 24], U64), axis=-1)
