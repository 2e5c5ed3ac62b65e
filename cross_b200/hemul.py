"""HE-Mult with relinearisation (jaxite_word hemul.py) as one fused GPU chain.

``HEMul.mul`` issues the whole chain -- rescale, tensor product, hybrid key
switch (ModUp BConv + NTTs + inner product), ModDown and the final add -- as
kernels of libcross_b200.so on the current CUDA stream.
"""
from __future__ import annotations

import numpy as np

from . import _lib, _tensor, util
from ._pipeline import HostPipeline
from .bconv import BConvBarrett
from .finite_field import BarrettContext
from .ntt_mm import NTTCiphertextBarrettContext

U32, U64 = np.uint32, np.uint64


def psi_tables(moduli, n):
    """(M, N) tables psi_i^t and psi_i^{-t} mod q_i (hemul.py:86-95)."""
    psi = [util.root_of_unity(2 * n, q) for q in moduli]
    fwd = np.stack([util.powers(p, n, q) for p, q in zip(psi, moduli)], 0).astype(U32)
    inv = np.stack([util.powers(pow(p, -1, q), n, q) for p, q in zip(psi, moduli)], 0).astype(U32)
    return fwd, inv


def rescale_tables(moduli, n):
    """ciphertext.py:229-262: inv_psi_last (N), gamma_i psi_i^t (L-1, N), betas (L-1)."""
    fwd, inv = psi_tables(moduli, n)
    gammas, betas = util.gamma_beta_calculation(moduli)
    qs = np.array(moduli[:-1], U64)[:, None]
    gpsi = ((gammas[:, None].astype(U64) * fwd[:-1].astype(U64)) % qs).astype(U32)
    return np.ascontiguousarray(inv[-1]), np.ascontiguousarray(gpsi), betas.astype(U32), fwd, inv


def digits(size_q: int, dnum: int):
    """ciphertext.py:353-379: alpha, number of parts, consecutive digit groups."""
    alpha = (size_q + dnum - 1) // dnum
    parts = (size_q + alpha - 1) // alpha
    groups = [list(range(j * alpha, min((j + 1) * alpha, size_q))) for j in range(parts)]
    return alpha, parts, groups


class HEMul:
    """hemul.py:11-217."""

    def __init__(self, batch, r, c, dnum, num_eval_mult, original_moduli, extend_moduli):
        self.batch, self.r, self.c, self.dnum = batch, r, c, dnum
        self.num_eval_mult = num_eval_mult
        self.original_moduli = list(original_moduli)
        self.drop_last_extend_moduli = self.original_moduli[:-1] + list(extend_moduli)
        self.drop_last_moduli = self.original_moduli[:-1]
        self.extend_moduli = list(extend_moduli)
        self.last_tower_moduli = self.original_moduli[-1]
        self._plan = None
        self._host = None
        self._host_ws = None

    def control_gen(self, degree_layout=None, perf_test=False):
        """hemul.py:24-132 (perf_test keeps the real constants: same cost)."""
        if self.num_eval_mult != 1:
            raise ValueError("HEMul supports num_eval_mult == 1 (one rescale per multiplication)")
        self.degree_layout = tuple(degree_layout) if degree_layout is not None else (self.r, self.c)
        self.perf_test = perf_test
        n = self.r * self.c
        Q, P = self.original_moduli, self.extend_moduli
        L, K = len(Q), len(P)
        L1 = L - 1
        self.overall_sizeQ_in, self.overall_sizeP_in = L, K
        # transforms over Q then P with the HEMul factorisation; ct_extend uses
        # the default factorisation (hemul.py:76-77, ciphertext.py:69-70)
        self.ntt_qp = NTTCiphertextBarrettContext(Q + P, {"r": self.r, "c": self.c,
                                                          "finite_field_context": BarrettContext(Q + P)})
        rd, cd = util.default_rc(n)
        if (rd, cd) == (self.r, self.c):
            self.ntt_p, self.ntt_p_offset = self.ntt_qp, L
        else:
            self.ntt_p = NTTCiphertextBarrettContext(P, {"r": rd, "c": cd, "finite_field_context": BarrettContext(P)})
            self.ntt_p_offset = 0
        (self.power_of_last_tower_inv_psi, self.gammas_power_of_psi_no_last, self.betas, _,
         _) = rescale_tables(Q, n)
        self.moduli_threshold = (self.last_tower_moduli + 1) // 2
        dle = self.drop_last_extend_moduli
        fwd, inv = psi_tables(dle, n)
        self.power_of_psi = np.ascontiguousarray(fwd)                 # (L1+K, N) limb-major
        self.power_of_inv_psi = np.ascontiguousarray(inv[:L1])        # (L1, N)
        self.power_of_inv_psi_approx_down = np.ascontiguousarray(inv[L1:])  # (K, N)
        Pp = 1
        for p in P:
            Pp *= p
        self.PInvModq = np.array([util.modinv(Pp, q) for q in self.drop_last_moduli if q not in P], U32)
        self.alpha, self.num_parts, self.digit_groups = digits(L1, self.dnum)
        self.ks_bconv = BConvBarrett(dle)
        self.ks_bconv.control_gen([(g, [i for i in range(L1 + K) if i not in g]) for g in self.digit_groups])
        self.bconv = BConvBarrett(dle)                                 # hemul.py:98-103
        self.bconv.control_gen([(list(range(L1, L1 + K)), list(range(L1)))])
        self.q_correction = np.array(self.drop_last_moduli, U32)
        self._free_plan()

    def setup_relinearization(self, evalkey_a_vector, evalkey_b_vector):
        """hemul.py:134-151: evk (dnum, N, L + K) in the reference layout."""
        ea = np.ascontiguousarray(_tensor.to_numpy(evalkey_a_vector).astype(U32))
        eb = np.ascontiguousarray(_tensor.to_numpy(evalkey_b_vector).astype(U32))
        n = self.r * self.c
        ea, eb = ea.reshape(ea.shape[0], n, -1), eb.reshape(eb.shape[0], n, -1)
        if ea.shape[0] < self.num_parts:
            raise ValueError(f"evaluation key has {ea.shape[0]} digits, need {self.num_parts}")
        self._free_plan()
        L, K = len(self.original_moduli), len(self.extend_moduli)
        ks = [self.ks_bconv.plan(j) for j in range(self.num_parts)]
        self._ks_arr = (_lib.vp * len(ks))(*ks)
        self._keep = [np.ascontiguousarray(a) for a in (
            self.power_of_last_tower_inv_psi, self.gammas_power_of_psi_no_last, self.betas,
            self.power_of_inv_psi, self.power_of_psi, self.power_of_inv_psi_approx_down, self.PInvModq)]
        k = self._keep
        desc = _lib.HemulDesc(self.r, self.c, L, K, self.dnum, self.ntt_qp.plan(), self.ntt_p.plan(), self.ntt_p_offset,
                              self._ks_arr, self.bconv.plan(0), *[a.ctypes.data for a in k])
        out = _lib.vp()
        _lib.check(_lib.lib().cross_hemul_plan_create(_lib.C.byref(desc), _lib.C.byref(out)), "cross_hemul_plan_create")
        self._plan = out
        _lib.check(_lib.lib().cross_hemul_set_keys(out, ea.ctypes.data,
                                                   eb.ctypes.data, ea.shape[-1]), "cross_hemul_set_keys")

    def _free_plan(self):
        if getattr(self, "_plan", None) is not None and getattr(_lib, "_lib", None) is not None:
            _lib._lib.cross_hemul_plan_destroy(self._plan)
        self._plan = None

    def __del__(self):
        self._free_plan()

    def check_device(self):
        """Raise TimeoutError if a tensor-core kernel of this operator's plans hit
        a bounded wait (its output is then invalid).  Synchronises the device."""
        for name in ('ntt_qp', 'ntt_p', 'ks_bconv', 'bconv'):
            obj = getattr(self, name, None)
            if obj is not None and hasattr(obj, "check_device"):
                obj.check_device()

    def workspace_size(self, batch: int, layout: int = _lib.LAYOUT_REFERENCE) -> int:
        return int(_lib.lib().cross_hemul_workspace_size(self._plan, batch, layout))

    def mul(self, in_ciphertexts, out=None, workspace=None, layout: int = _lib.LAYOUT_REFERENCE, chunk: int = 4,
            sync: bool = True):
        """hemul.py:153-217: (B, 4, r, c, L) uint32 -> (B, 2, r, c, L-1) uint32.

        With layout=LAYOUT_LIMB_MAJOR the input is (B, 4, L, N) and the output
        (B, 2, L-1, N).  `out` and `workspace` may be passed to reuse buffers.
        A CPU uint32 tensor input (pinned for asynchronous copies) returns a CPU
        result (or fills a CPU `out`): the batch runs in chunks of `chunk`
        ciphertexts with host-device copies overlapped with compute; the result
        is ready on return unless sync=False (then the current stream orders it)."""
        if self._plan is None:
            raise RuntimeError("call control_gen() and setup_relinearization() first")
        t = _tensor.torch()
        if isinstance(in_ciphertexts, t.Tensor) and in_ciphertexts.device.type == "cpu":
            return self._mul_host(in_ciphertexts, out, layout, chunk, sync)
        x = _tensor.to_u32(in_ciphertexts)
        B = x.shape[0]
        L = len(self.original_moduli)
        n = self.r * self.c
        if x.numel() != B * 4 * n * L:
            raise ValueError(f"expected {B} x 4 x {n} x {L} residues, got shape {tuple(x.shape)}")
        if out is None:
            shape = (B, 2, *self.degree_layout, L - 1) if layout == _lib.LAYOUT_REFERENCE else (B, 2, L - 1, n)
            out = _tensor.empty_u32(shape)
        need = self.workspace_size(B, layout)
        if workspace is None or workspace.numel() < need:
            workspace = _tensor.workspace(need)
        _tensor.call("cross_hemul", self._plan, x.data_ptr(), out.data_ptr(), B, layout, workspace.data_ptr(),
                     workspace.numel(), _lib.cuda_stream())
        return out

    def _mul_host(self, x, out, layout, chunk, sync):
        t = _tensor.torch()
        if x.dtype != t.uint32:
            raise TypeError(f"host input must be uint32, got {x.dtype}")
        x = x.contiguous()
        B, L, n = x.shape[0], len(self.original_moduli), self.r * self.c
        if x.numel() != B * 4 * n * L:
            raise ValueError(f"expected {B} x 4 x {n} x {L} residues, got shape {tuple(x.shape)}")
        oshape = (B, 2, *self.degree_layout, L - 1) if layout == _lib.LAYOUT_REFERENCE else (B, 2, L - 1, n)
        if out is None:
            out = t.empty(oshape, dtype=t.uint32, pin_memory=x.is_pinned())
        if out.device.type != "cpu" or tuple(out.shape) != oshape or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous CPU tensor of shape {oshape}")
        if self._host is None:
            self._host = HostPipeline()
        cb = max(1, min(chunk, B))
        need = self.workspace_size(cb, layout)
        if self._host_ws is None or self._host_ws.numel() < need:
            self._host_ws = _tensor.workspace(need)
        ws = self._host_ws

        def compute(xd, od, nb, stream):
            _tensor.call("cross_hemul", self._plan, xd.data_ptr(), od.data_ptr(), nb, layout, ws.data_ptr(),
                         ws.numel(), stream.cuda_stream)

        return self._host.run(x.reshape(B, -1), out.reshape(B, -1), cb, compute, sync).reshape(oshape)
