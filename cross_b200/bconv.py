"""Basis conversion (jaxite_word bconv.py) on the GPU."""
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
            qm = np.array(qm, U64).reshape(len(om), len(tm))
            self.QHatInvModq.append(np.array(inv, U64))
            self.QHatModp.append(qm)
            self.QHatModpBAT.append(qhat_modp_bat(qm, tm))
            self._plans.append(None)

    def plan(self, control_index: int = 0):
        if self._plans[control_index] is None:
            inv = np.ascontiguousarray(self.QHatInvModq[control_index].astype(U32))
            qm = np.ascontiguousarray(self.QHatModp[control_index].astype(U32))
            bat = np.ascontiguousarray(self.QHatModpBAT[control_index])
            out = _lib.vp()
            _lib.check(_lib.lib().cross_bconv_plan_create(
                self.ff_ctx_origin[control_index].handle(), self.ff_ctx_target[control_index].handle(),
                inv.ctypes.data, qm.ctypes.data, bat.ctypes.data, _lib.C.byref(out)), "cross_bconv_plan_create")
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
        x = _tensor.to_u32(in_tower)
        sq = len(self.original_moduli[control_index])
        sp = len(self.target_moduli[control_index])
        if x.shape[-1] != sq:
            raise ValueError(f"last axis {x.shape[-1]} != sizeQ {sq}")
        out = _tensor.empty_u32((*x.shape[:-1], sp))
        rows = x.numel() // sq
        _tensor.call("cross_bconv", self.plan(control_index), int(bat), x.data_ptr(), out.data_ptr(), 1, rows,
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
