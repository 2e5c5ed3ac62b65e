"""Basis conversion (jaxite_word bconv.py) on the GPU.

BConvBarrett is the conversion of the HE pipeline (tensor cores for the BAT
form); BConvMontgomery, BConvShoup and BConvBATLazy (bconv.py:261-390) run the
reference's variant arithmetic on the CUDA cores.
"""
from __future__ import annotations

import numpy as np

from . import _lib, _tensor, util
from . import finite_field as ff_context

U32, U64 = np.uint32, np.uint64


def qhat_modp_bat(qhat_modp: np.ndarray, target_moduli) -> np.ndarray:
    """bconv.py:93-97,157-170: (sizeQ, sizeP) -> (4*sizeQ, sizeP, 4) uint8 with
    [(i, a), j, b] = byte_b((QHatModp[i, j] << 8a) mod p_j)."""
    qm = np.asarray(qhat_modp).astype(U64)
    ps = np.array(target_moduli, U64)
    red = np.stack([((qm << U64(8 * a)) % ps).astype(U32) for a in range(4)], 0)   # (4, sq, sp)
    u8 = np.ascontiguousarray(red).view(np.uint8).reshape(*red.shape, 4)          # (4, sq, sp, 4)
    return np.ascontiguousarray(u8.transpose(1, 0, 2, 3).reshape(-1, qm.shape[1], 4))


class BConv:
    """bconv.py:40-252."""

    _reduction = _lib.REDUCTION_BARRETT

    def __init__(self, overall_moduli):
        self.overall_moduli = list(overall_moduli)
        self.original_moduli, self.target_moduli = [], []
        self.ff_ctx_origin, self.ff_ctx_target = [], []
        self.QHatInvModq, self.QHatModp, self.QHatModpBAT = [], [], []
        self._plans = []

    def _create_contexts(self, original_moduli, target_moduli):
        raise NotImplementedError

    def control_gen(self, control_indices_list, perf_test: bool = False):
        """bconv.py:101-155 (perf_test keeps the real constants: same cost)."""
        self.__init__(self.overall_moduli)
        for original_index, target_index in control_indices_list:
            om = [self.overall_moduli[i] for i in original_index]
            tm = [self.overall_moduli[i] for i in target_index]
            self.original_moduli.append(om)
            self.target_moduli.append(tm)
            co, ct = self._create_contexts(om, tm)
            self.ff_ctx_origin.append(co)
            self.ff_ctx_target.append(ct)
            inv, qm = util.compute_QHatInvModq_QHatModp(om, tm)
            # bconv.py:79-91: the constants in the contexts' computation format
            inv = np.asarray(co.to_computation_format(np.array(inv, U64)))
            qm = np.asarray(ct.to_computation_format(np.array(qm, U64).reshape(len(om), len(tm))))
            self.QHatInvModq.append(inv)
            self.QHatModp.append(qm)
            self.QHatModpBAT.append(qhat_modp_bat(qm, tm))
            self._plans.append(None)
        self._after_control_gen()

    def _after_control_gen(self):
        pass

    def _shoup_tables(self, control_index):
        return None, None

    def plan(self, control_index: int = 0):
        if self._plans[control_index] is None:
            inv = np.ascontiguousarray(np.asarray(self.QHatInvModq[control_index]).astype(U32))
            qm = np.ascontiguousarray(np.asarray(self.QHatModp[control_index]).astype(U32))
            bat = np.ascontiguousarray(self.QHatModpBAT[control_index])
            inv_s, qm_s = self._shoup_tables(control_index)
            out = _lib.vp()
            _lib.check(_lib.lib().cross_bconv_plan_create_ex(
                self.ff_ctx_origin[control_index].handle(), self.ff_ctx_target[control_index].handle(),
                self._reduction, inv.ctypes.data, inv_s.ctypes.data if inv_s is not None else None, qm.ctypes.data,
                qm_s.ctypes.data if qm_s is not None else None, bat.ctypes.data, _lib.C.byref(out)),
                "cross_bconv_plan_create")
            self._plans[control_index] = out
        return self._plans[control_index]

    def __del__(self):
        if getattr(_lib, "_lib", None) is not None:
            for p in getattr(self, "_plans", []):
                if p is not None:
                    _lib._lib.cross_bconv_plan_destroy(p)

    def check_device(self):
        """Raise TimeoutError if a tensor-core kernel of these plans hit a bounded wait."""
        for p in self._plans:
            if p is not None:
                _lib.check(_lib.lib().cross_bconv_plan_check(p), "cross_bconv_plan_check")

    def _run(self, in_tower, control_index, bat):
        t = _tensor.torch()
        x = _tensor.to_u32(in_tower)
        sq = len(self.original_moduli[control_index])
        sp = len(self.target_moduli[control_index])
        if x.shape[-1] != sq:
            raise ValueError(f"last axis {x.shape[-1]} != sizeQ {sq}")
        plan = self.plan(control_index)
        dt = t.uint64 if _lib.lib().cross_bconv_output_bytes(plan) == 8 else t.uint32
        out = t.empty((*x.shape[:-1], sp), dtype=dt, device=_tensor.device())
        rows = x.numel() // sq
        _tensor.call("cross_bconv_ex", plan, int(bat), x.data_ptr(), out.data_ptr(), 1, rows,
                     _lib.LAYOUT_REFERENCE, _lib.cuda_stream())
        return out

    def basis_change_bat(self, in_tower, control_index: int = 0):
        """bconv.py:215-252: (..., N, sizeQ) -> (..., N, sizeP) uint32."""
        return self._run(in_tower, control_index, True)

    def basis_change(self, in_tower, control_index: int = 0):
        """bconv.py:173-212 (uint64 multiply-accumulate form)."""
        return self._run(in_tower, control_index, False)


class BConvBarrett(BConv):
    """bconv.py:255-258."""

    def _create_contexts(self, original_moduli, target_moduli):
        return ff_context.BarrettContext(original_moduli), ff_context.BarrettContext(target_moduli)


class BConvMontgomery(BConv):
    """bconv.py:261-288: Montgomery contexts; basis_change re-encodes source
    limb i with target modulus i (the reference broadcasts size_q against
    size_p), so it needs size_q == size_p or size_p == 1."""

    _reduction = _lib.REDUCTION_MONTGOMERY

    def _create_contexts(self, original_moduli, target_moduli):
        return ff_context.MontgomeryContext(original_moduli), ff_context.MontgomeryContext(target_moduli)


class BConvShoup(BConv):
    """bconv.py:291-339: Shoup contexts with the companions of
    BConvShoup.control_gen (bconv.py:300-314), computed from the uint32
    tables exactly as the reference does (ShoupContext.precompute_constant_operand);
    basis_change_bat is not defined for Shoup (bconv.py:244 calls the
    two-operand reduction with one operand) and raises TypeError."""

    _reduction = _lib.REDUCTION_SHOUP

    def __init__(self, overall_moduli):
        super().__init__(overall_moduli)
        self.QHatInvModq_shoup, self.QHatModp_shoup = [], []

    def _create_contexts(self, original_moduli, target_moduli):
        return ff_context.ShoupContext(original_moduli), ff_context.ShoupContext(target_moduli)

    def _after_control_gen(self):
        self.QHatInvModq_shoup, self.QHatModp_shoup = [], []
        for i in range(len(self.QHatInvModq)):
            self.QHatInvModq_shoup.append(self.ff_ctx_origin[i].precompute_constant_operand(self.QHatInvModq[i]))
            self.QHatModp_shoup.append(self.ff_ctx_target[i].precompute_constant_operand(self.QHatModp[i]))

    def _shoup_tables(self, control_index):
        return (np.ascontiguousarray(np.asarray(self.QHatInvModq_shoup[control_index]).astype(U32)),
                np.ascontiguousarray(np.asarray(self.QHatModp_shoup[control_index]).astype(U32)))

    def basis_change_bat(self, in_tower, control_index: int = 0):
        raise TypeError("ShoupContext.modular_reduction() missing 1 required positional argument: 'z_s' "
                        "(BConvShoup has no BAT path, bconv.py:244)")


class BConvBATLazy(BConv):
    """bconv.py:341-390: BAT-lazy contexts; the outputs are uint64 (lazy,
    congruent to the converted value)."""

    _reduction = _lib.REDUCTION_BAT_LAZY

    def _create_contexts(self, original_moduli, target_moduli):
        return ff_context.BATLazyContext(original_moduli), ff_context.BATLazyContext(target_moduli)
