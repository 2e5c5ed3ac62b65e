"""HE-Rotate (jaxite_word herot.py) as one fused GPU chain."""
from __future__ import annotations

import numpy as np

from . import _lib, _tensor, util
from ._pipeline import HostPipeline
from .bconv import BConvBarrett
from .finite_field import BarrettContext
from .hemul import digits, psi_tables
from .ntt_mm import NTTCiphertextBarrettContext

U32 = np.uint32


def is_power_of_two(x: int) -> bool:
    """herot.py:11-13."""
    return x > 0 and (x & (x - 1)) == 0


def mat_1d_shuffle_to_2d(coefMap, r, c):
    """herot.py:15-53: factor a 1-D permutation into row and column permutations."""
    cm = np.asarray(_tensor.to_numpy(coefMap))
    if cm.ndim != 1 or cm.shape[0] != r * c:
        raise ValueError(f"coefMap must be 1D of length r*c. Got shape {cm.shape}, r*c={r * c}.")
    if r <= 0 or c <= 0:
        raise ValueError("r and c must be positive.")
    if not (is_power_of_two(r) and is_power_of_two(c)):
        raise ValueError("For your setting, r and c should be powers of two.")
    c2 = cm.reshape(r, c)
    row = (c2[:, 0] // c).astype(np.int32)
    col = (c2[0, :] % c).astype(np.int32)
    if not np.array_equal(c2, row[:, None] * c + col[None, :]):
        raise ValueError("coefMap is NOT decomposable into a single global row permutation + column permutation "
                         f"for r={r}, c={c}.")
    return row, col


class HERot:
    """herot.py:55-302."""

    def __init__(self, r, c, dnum, rotate_in_ciphertext_moduli, extend_moduli):
        self.r, self.c, self.dnum = r, c, dnum
        self.rotate_in_ciphertext_moduli = list(rotate_in_ciphertext_moduli)
        self.extend_moduli = list(extend_moduli)
        self.overall_moduli_init = self.rotate_in_ciphertext_moduli + self.extend_moduli
        self.bconv = BConvBarrett(self.overall_moduli_init)
        self._plan = None

    def control_gen(self, batch=1, degree_layout=None, perf_test=False):
        """herot.py:66-175.  Every transform uses the default (r, c) split,
        as the reference's internal Ciphertext objects do (herot.py:160-175)."""
        n = self.r * self.c
        self.degree_layout = tuple(degree_layout) if degree_layout is not None else (n,)
        self.perf_test = perf_test
        self.batch = batch
        Q, P = self.rotate_in_ciphertext_moduli, self.extend_moduli
        L, K = len(Q), len(P)
        ov = Q + P
        self.overall_moduli = ov
        self.sizeQlP, self.sizeQl = L + K, L
        fwd, inv = psi_tables(ov, n)
        self.power_of_psi = np.ascontiguousarray(fwd)                   # (L+K, N)
        self.power_of_inv_psi = np.ascontiguousarray(inv[:L])           # (L, N)
        self.power_of_inv_psi_approx_down = np.ascontiguousarray(inv[L:])
        Pp = 1
        for p in P:
            Pp *= p
        self.PInvModq = np.array([util.modinv(Pp, q) for q in ov if q not in P], U32)
        self.alpha, self.num_parts, groups = digits(L, self.dnum)
        self.select_tower_index = groups
        self.non_select_tower_index = [[i for i in range(L + K) if i not in g] for g in groups]
        ctl = list(zip(self.select_tower_index, self.non_select_tower_index))
        ctl.append((list(range(L, L + K)), list(range(L))))
        self.bconv.control_gen(ctl)
        rd, cd = util.default_rc(n)
        self.ntt_qp = NTTCiphertextBarrettContext(ov, {"r": rd, "c": cd, "finite_field_context": BarrettContext(ov)})
        self._free_plan()
        if getattr(self, "_pending_keys", None) is not None:
            # the reference stores the keys in setup_rotate and uses them at rotate
            # time, so setup_rotate may come first (ckks_ctx_test.py:104-106)
            keys, self._pending_keys = self._pending_keys, None
            self.setup_rotate(*keys)

    def setup_rotate(self, evalkey_a_vector, evalkey_b_vector, coefMap):
        """herot.py:178-181: evk (dnum, N, L + K) (or (dnum, r, c, L + K)).
        Before control_gen the keys are kept and installed by control_gen."""
        if not hasattr(self, "sizeQlP"):
            self._pending_keys = (evalkey_a_vector, evalkey_b_vector, coefMap)
            return
        n = self.r * self.c
        ea = np.ascontiguousarray(_tensor.to_numpy(evalkey_a_vector).astype(U32)).reshape(-1, n, self.sizeQlP)
        eb = np.ascontiguousarray(_tensor.to_numpy(evalkey_b_vector).astype(U32)).reshape(-1, n, self.sizeQlP)
        cm = np.ascontiguousarray(np.asarray(_tensor.to_numpy(coefMap)).astype(np.int32))
        if cm.shape != (n,):
            raise ValueError(f"coefMap must have {n} entries")
        if ea.shape[0] < self.dnum:
            raise ValueError(f"evaluation key has {ea.shape[0]} digits, need {self.dnum}")
        self.coefMap = cm
        self._free_plan()
        if self.num_parts < self.dnum:
            # herot.py:212-213 indexes select_tower_index[part] for part < dnum
            raise IndexError(f"dnum={self.dnum} exceeds the {self.num_parts} digits of {self.sizeQl} limbs")
        ks = [self.bconv.plan(j) for j in range(self.dnum)]
        self._ks_arr = (_lib.vp * len(ks))(*ks)
        self._keep = [self.power_of_inv_psi, self.power_of_psi, self.power_of_inv_psi_approx_down, self.PInvModq]
        desc = _lib.HerotDesc(self.r, self.c, self.sizeQl, self.sizeQlP - self.sizeQl, self.dnum, self.ntt_qp.plan(),
                              self._ks_arr, self.bconv.plan(self.dnum), *[a.ctypes.data for a in self._keep])
        out = _lib.vp()
        _lib.check(_lib.lib().cross_herot_plan_create(_lib.C.byref(desc), _lib.C.byref(out)), "cross_herot_plan_create")
        self._plan = out
        _lib.check(_lib.lib().cross_herot_set_keys(out, ea.ctypes.data, eb.ctypes.data, cm.ctypes.data),
                   "cross_herot_set_keys")

    def _free_plan(self):
        if getattr(self, "_plan", None) is not None and getattr(_lib, "_lib", None) is not None:
            _lib._lib.cross_herot_plan_destroy(self._plan)
        self._plan = None

    def __del__(self):
        self._free_plan()

    def check_device(self):
        """Raise TimeoutError if a tensor-core kernel of this operator's plans hit
        a bounded wait (its output is then invalid).  Synchronises the device."""
        for name in ('ntt_qp', 'bconv'):
            obj = getattr(self, name, None)
            if obj is not None and hasattr(obj, "check_device"):
                obj.check_device()

    def workspace_size(self, batch: int, layout: int = _lib.LAYOUT_REFERENCE) -> int:
        return int(_lib.lib().cross_herot_workspace_size(self._plan, batch, layout))

    def rotate(self, in_ciphertexts, out=None, workspace=None, layout: int = _lib.LAYOUT_REFERENCE, chunk: int = 4,
               sync: bool = True):
        """herot.py:183-302: (B, 2, r, c, L) -> (B, 2, N, L) uint32
        (LAYOUT_LIMB_MAJOR: (B, 2, L, N) -> (B, 2, L, N)).  A CPU uint32 tensor
        input runs in chunks with host-device copies overlapped with compute
        and returns a CPU result (ready on return unless sync=False)."""
        if self._plan is None:
            raise RuntimeError("call control_gen() and setup_rotate() first")
        t = _tensor.torch()
        if isinstance(in_ciphertexts, t.Tensor) and in_ciphertexts.device.type == "cpu":
            return self._rotate_host(in_ciphertexts, out, layout, chunk, sync)
        x = _tensor.to_u32(in_ciphertexts)
        B = x.shape[0]
        n, L = self.r * self.c, self.sizeQl
        if x.numel() != B * 2 * n * L:
            raise ValueError(f"expected {B} x 2 x {n} x {L} residues, got shape {tuple(x.shape)}")
        if out is None:
            out = _tensor.empty_u32((B, 2, n, L) if layout == _lib.LAYOUT_REFERENCE else (B, 2, L, n))
        need = self.workspace_size(B, layout)
        if workspace is None or workspace.numel() < need:
            workspace = _tensor.workspace(need)
        _tensor.call("cross_herot", self._plan, x.data_ptr(), out.data_ptr(), B, layout, workspace.data_ptr(),
                     workspace.numel(), _lib.cuda_stream())
        return out

    def _rotate_host(self, x, out, layout, chunk, sync):
        t = _tensor.torch()
        if x.dtype != t.uint32:
            raise TypeError(f"host input must be uint32, got {x.dtype}")
        x = x.contiguous()
        B, n, L = x.shape[0], self.r * self.c, self.sizeQl
        if x.numel() != B * 2 * n * L:
            raise ValueError(f"expected {B} x 2 x {n} x {L} residues, got shape {tuple(x.shape)}")
        oshape = (B, 2, n, L) if layout == _lib.LAYOUT_REFERENCE else (B, 2, L, n)
        if out is None:
            out = t.empty(oshape, dtype=t.uint32, pin_memory=x.is_pinned())
        if out.device.type != "cpu" or tuple(out.shape) != oshape or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous CPU tensor of shape {oshape}")
        if getattr(self, "_host", None) is None:
            self._host, self._host_ws = HostPipeline(), None
        cb = max(1, min(chunk, B))
        need = self.workspace_size(cb, layout)
        if self._host_ws is None or self._host_ws.numel() < need:
            self._host_ws = _tensor.workspace(need)
        ws = self._host_ws

        def compute(xd, od, nb, stream):
            _tensor.call("cross_herot", self._plan, xd.data_ptr(), od.data_ptr(), nb, layout, ws.data_ptr(),
                         ws.numel(), stream.cuda_stream)

        return self._host.run(x.reshape(B, -1), out.reshape(B, -1), cb, compute, sync).reshape(oshape)
