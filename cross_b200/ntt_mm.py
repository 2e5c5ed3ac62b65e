"""Multi-modulus BAT 3-step NTT (jaxite_word ntt_mm.py) on the GPU.

The constructors precompute exactly the reference's tables (same names,
shapes and values, ntt_mm.py:136-255, in the context's computation format);
``ntt`` / ``intt`` run the CUDA kernels of libcross_b200.so through the C ABI.
The reduction follows the reference: the finite-field context's type for the
base / Barrett / Montgomery classes (ntt_mm.py:351-407 call
``self.ff_ctx.modular_reduction``), BAT-lazy then Barrett for
NTTCiphertextBATLazyContext, Shoup's for NTTCiphertextShoupContext.
"""
from __future__ import annotations

import functools

import numpy as np

from . import _lib, _tensor, util
from . import finite_field as ff_context

U32, U64 = np.uint32, np.uint64


def get_bit_reverse_perm(n: int):
    """ntt_mm.py:261-274."""
    bits = n.bit_length() - 1
    return [util.bit_reverse(i, bits) for i in range(n)] if n > 0 else []


def basis_aligned_transformation(matrix: np.ndarray, moduli) -> np.ndarray:
    """ntt_mm.py:248-255: (rows, cols, M) -> (rows, 4, cols, 4, M) uint8 with
    [x, q, y, p, m] = byte_p((T[x, y, m] << 8q) mod q_m)."""
    mu = np.asarray(matrix).astype(U64)
    qs = np.array(moduli, U64)
    red = np.stack([((mu << U64(8 * i)) % qs).astype(U32) for i in range(4)], 0)
    u8 = np.ascontiguousarray(red).view(np.uint8).reshape(*red.shape, 4)
    return np.ascontiguousarray(u8.transpose(1, 0, 2, 4, 3))


def gen_twiddle_matrix(rows: int, cols: int, q: int, omega: int) -> np.ndarray:
    """ntt_mm.py:75-97: T[r, c] = omega^(r c) mod q (int64)."""
    return util.twiddle_matrix(rows, cols, q, omega).astype(np.int64)


def gen_twiddle_matrix_inv(rows: int, cols: int, q: int, omega: int) -> np.ndarray:
    """ntt_mm.py:100-119: T[r, c] = omega^-(r c) mod q (int64)."""
    return util.twiddle_matrix(rows, cols, q, pow(omega, -1, q)).astype(np.int64)


@functools.lru_cache(maxsize=512)
def _limb_tables(q: int, r: int, c: int):
    """The six raw twiddle tables of one modulus (ntt_mm.py:186-240), shared
    by every context that uses (q, r, c): HE-Mult, HE-Rotate and ciphertext
    objects over overlapping moduli compute each limb once per process.
    Read-only arrays."""
    n = r * c
    om = pow(util.root_of_unity(2 * n, q), 2, q)
    perm_r, perm_c = get_bit_reverse_perm(r), get_bit_reverse_perm(c)
    t1 = util.twiddle_matrix(r, r, q, pow(om, c, q))[perm_r, :]
    t2 = util.twiddle_matrix(r, c, q, om)[perm_r, :]
    t3 = util.twiddle_matrix(c, c, q, pow(om, r, q))[:, perm_c]
    inv_col = pow(pow(om, c, q), -1, q)
    inv_row = pow(pow(om, r, q), -1, q)
    a = util.twiddle_matrix(c, c, q, inv_row)[perm_c, :]
    b = util.twiddle_matrix(r, c, q, pow(om, -1, q))[perm_r, :]
    d = util.twiddle_matrix(r, r, q, inv_col)[:, perm_r]
    b = (b * U64(pow(c, -1, q))) % U64(q)
    d = (d * U64(pow(r, -1, q))) % U64(q)
    out = tuple(np.ascontiguousarray(t.astype(U32)) for t in (t1, t2, t3, a, b, d))
    for t in out:
        t.flags.writeable = False
    return out


@functools.lru_cache(maxsize=512)
def _limb_bat(q: int, r: int, c: int):
    """basis_aligned_transformation of the four contraction tables of one
    modulus in the Barrett (identity) computation format (ntt_mm.py:172-181),
    shared like _limb_tables.  Read-only arrays."""
    t1, _, t3, it1, _, it3 = _limb_tables(q, r, c)
    out = tuple(np.ascontiguousarray(basis_aligned_transformation(t[..., None], [q])[..., 0])
                for t in (t1, t3, it1, it3))
    for t in out:
        t.flags.writeable = False
    return out


class NTTCiphertextContextBase:
    """ntt_mm.py:125-419."""

    def _default_ff_ctx(self):
        return ff_context.BarrettContext(self.moduli)

    def __init__(self, moduli, parameters: dict, perf_test: bool = False):
        self.ff_ctx = parameters.get("finite_field_context", None)
        self.num_bytes = 4
        self.moduli = [moduli] if isinstance(moduli, int) else list(moduli)
        self.parameters = parameters
        assert all(q < 2 ** 31 for q in self.moduli), "moduli must be less than 2**31"
        self.r = parameters.get("r", 0)
        self.c = parameters.get("c", 0)
        assert self.r != 0, "r must be non-zero"
        assert self.c != 0, "c must be non-zero"
        self.transform_length = self.r * self.c
        self.psi_list = [util.root_of_unity(2 * self.transform_length, q) for q in self.moduli]
        self.omega_list = [(psi * psi) % q for psi, q in zip(self.psi_list, self.moduli)]
        # perf_test replaced the tables by random bits in the reference
        # (ntt_mm.py:150-171); the real tables cost the same here, so they are
        # always used and results stay checkable.
        self.perf_test = perf_test
        if self.ff_ctx is None:
            self.ff_ctx = self._default_ff_ctx()
        self.memory_aligned_transformation()
        self.ntt_tf_step1, self.ntt_tf_step2, self.ntt_tf_step3 = self.ntt_coefficients_precompute()
        self.intt_tf_step1, self.intt_tf_step2, self.intt_tf_step3 = self.intt_coefficients_precompute()
        self._format_tables()
        self._plan = None
        self._plan_barrett = None

    def _format_tables(self):
        """ntt_mm.py:172-181: BAT of the tables in the computation format."""
        if type(self.ff_ctx) is ff_context.BarrettContext:
            # identity format: the per-modulus BAT tables are shared
            per = [_limb_bat(int(q), self.r, self.c) for q in self.moduli]
            st = lambda k: np.stack([p[k] for p in per], -1)  # noqa: E731
            self.ntt_bat_tf_step1, self.ntt_bat_tf_step3 = st(0), st(1)
            self.intt_bat_tf_step1, self.intt_bat_tf_step3 = st(2), st(3)
            self.ntt_tf_step2 = self.ntt_tf_step2.astype(U64)
            self.intt_tf_step2 = self.intt_tf_step2.astype(U64)
            return
        fmt = self.to_computation_format
        self.ntt_bat_tf_step1 = basis_aligned_transformation(fmt(self.ntt_tf_step1), self.moduli)
        self.ntt_tf_step2 = fmt(self.ntt_tf_step2).astype(U64)
        self.ntt_bat_tf_step3 = basis_aligned_transformation(fmt(self.ntt_tf_step3), self.moduli)
        self.intt_bat_tf_step1 = basis_aligned_transformation(fmt(self.intt_tf_step1), self.moduli)
        self.intt_tf_step2 = fmt(self.intt_tf_step2).astype(U64)
        self.intt_bat_tf_step3 = basis_aligned_transformation(fmt(self.intt_tf_step3), self.moduli)

    def _reduction(self) -> int:
        """The reduction ntt / intt apply: that of the finite-field context."""
        if isinstance(self.ff_ctx, ff_context.MontgomeryContext):
            return _lib.REDUCTION_MONTGOMERY
        if isinstance(self.ff_ctx, ff_context.BarrettContext):
            return _lib.REDUCTION_BARRETT
        if isinstance(self.ff_ctx, ff_context.ShoupContext):
            # ntt_mm.py:372 calls modular_reduction(z); Shoup's takes (z, z_s)
            raise TypeError("ShoupContext.modular_reduction() needs z_s: use NTTCiphertextShoupContext")
        raise NotImplementedError(f"{type(self).__name__}: no device transform for {type(self.ff_ctx).__name__}")

    # -- offline --------------------------------------------------------------
    def memory_aligned_transformation(self):
        """ntt_mm.py:257-277."""
        self.perm_r = get_bit_reverse_perm(self.r)
        self.perm_c = get_bit_reverse_perm(self.c)

    def _tables(self, first: int):
        per = [_limb_tables(int(q), self.r, self.c) for q in self.moduli]
        return tuple(np.stack([t[first + k] for t in per], -1) for k in range(3))

    def ntt_coefficients_precompute(self):
        """ntt_mm.py:186-209 (per-modulus tables cached by _limb_tables)."""
        return self._tables(0)

    def intt_coefficients_precompute(self):
        """ntt_mm.py:211-240 (per-modulus tables cached by _limb_tables)."""
        return self._tables(3)

    def to_computation_format(self, a):
        """ntt_mm.py:242-243 (host)."""
        return np.asarray(self.ff_ctx.to_computation_format(_tensor.to_numpy(a).astype(U64))).astype(U32)

    def to_original_format(self, a):
        """ntt_mm.py:245-246 (host)."""
        return np.asarray(self.ff_ctx.to_original_format(_tensor.to_numpy(a).astype(U64))).astype(U32)

    def basis_aligned_transformation(self, matrix):
        """ntt_mm.py:248-255: (rows, 4, cols, 4, M) uint8, the bytes of
        (matrix << 8 i) mod q_m for a (rows, cols, M) table."""
        m = np.asarray(matrix)
        return basis_aligned_transformation(m, self.moduli[: m.shape[-1]])

    def get_jax_parameters(self):
        return {"rows": self.r, "cols": self.c, "finite_field_parameters": self.ff_ctx.get_jax_parameters()}

    # -- device plan ----------------------------------------------------------
    def _moduli_ctx(self) -> ff_context.BarrettContext:
        M = self.ntt_tf_step2.shape[-1]
        if self._plan_barrett is None or len(self._plan_barrett.moduli) != M:
            self._plan_barrett = ff_context.BarrettContext(self.moduli[:M])
        return self._plan_barrett

    def plan(self):
        """The cross_ntt_plan of the current (possibly dropped) moduli."""
        if self._plan is None:
            c = lambda a: np.ascontiguousarray(a)  # noqa: E731
            arrs = [c(self.ntt_bat_tf_step1), c(self.ntt_tf_step2.astype(U32)), c(self.ntt_bat_tf_step3),
                    c(self.intt_bat_tf_step1), c(self.intt_tf_step2.astype(U32)), c(self.intt_bat_tf_step3)]
            out = _lib.vp()
            _lib.check(_lib.lib().cross_ntt_plan_create_ex(self._moduli_ctx().handle(), self.r, self.c,
                                                           self._reduction(), *[a.ctypes.data for a in arrs],
                                                           _lib.C.byref(out)),
                       "cross_ntt_plan_create")
            self._plan = out
        return self._plan

    def __del__(self):
        if getattr(self, "_plan", None) is not None and getattr(_lib, "_lib", None) is not None:
            _lib._lib.cross_ntt_plan_destroy(self._plan)
            self._plan = None

    def check_device(self):
        """Raise TimeoutError if a tensor-core kernel of this plan hit a bounded wait."""
        if self._plan is not None:
            _lib.check(_lib.lib().cross_ntt_plan_check(self._plan), "cross_ntt_plan_check")

    # -- online ---------------------------------------------------------------
    def _run(self, v, inverse: bool):
        x = _tensor.to_u32(v)
        M = self.ntt_tf_step2.shape[-1]
        if x.dim() != 4 or tuple(x.shape[1:]) != (self.r, self.c, M):
            raise ValueError(f"expected (B, {self.r}, {self.c}, {M}), got {tuple(x.shape)}")
        out = _tensor.empty_u32(x.shape)
        B = x.shape[0]
        L = _lib.lib()
        ws = _tensor.workspace(L.cross_ntt_workspace_size(self.plan(), B, _lib.LAYOUT_REFERENCE))
        _tensor.call("cross_ntt", self.plan(), int(inverse), x.data_ptr(), out.data_ptr(), B,
                     _lib.LAYOUT_REFERENCE, ws.data_ptr(), ws.numel(), _lib.cuda_stream())
        return out

    def ntt(self, v):
        """ntt_mm.py:351-378: (B, R, C, M) uint32 -> bit-reversed evaluations."""
        return self._run(v, False)

    def intt(self, v):
        """ntt_mm.py:380-407."""
        return self._run(v, True)

    def ntt_limb(self, v, limb_index: int):
        """ntt_mm.py:295-321: (B, R, C) for one limb."""
        return self._single(limb_index).ntt(_tensor.to_u32(v).unsqueeze(-1))[..., 0]

    def intt_limb(self, v, limb_index: int):
        """ntt_mm.py:323-349."""
        return self._single(limb_index).intt(_tensor.to_u32(v).unsqueeze(-1))[..., 0]

    def _single(self, i):
        # ntt_limb uses BarrettContext.modular_reduction_single_modulus (ntt_mm.py:316-320),
        # which only the Barrett context has
        if self._reduction() != _lib.REDUCTION_BARRETT:
            raise AttributeError(f"{type(self.ff_ctx).__name__} has no modular_reduction_single_modulus")
        return NTTCiphertextBarrettContext([self.moduli[i]], {"r": self.r, "c": self.c})

    def drop_last_modulus(self):
        """ntt_mm.py:412-419."""
        for name in ("ntt_bat_tf_step1", "ntt_tf_step2", "ntt_bat_tf_step3",
                     "intt_bat_tf_step1", "intt_tf_step2", "intt_bat_tf_step3"):
            setattr(self, name, np.ascontiguousarray(getattr(self, name)[..., :-1]))
        self.ff_ctx.drop_last_modulus()
        if self._plan is not None:
            _lib.lib().cross_ntt_plan_destroy(self._plan)
            self._plan = None


class NTTCiphertextBarrettContext(NTTCiphertextContextBase):
    """ntt_mm.py:421-429."""

    def __init__(self, moduli, parameters: dict, perf_test: bool = False):
        super().__init__(moduli, parameters, perf_test=perf_test)
        if self.ff_ctx is None:
            self.ff_ctx = ff_context.BarrettContext(self.moduli)
        assert self.ff_ctx is not None, "finite_field_context must be provided"
        assert self.moduli == list(self.ff_ctx.moduli), "moduli must be the same as the moduli of the finite_field_context"


class NTTCiphertextMontgomeryContext(NTTCiphertextContextBase):
    """ntt_mm.py:432-440: Montgomery-form tables, Montgomery reductions."""

    def _default_ff_ctx(self):
        return ff_context.MontgomeryContext(self.moduli)

    def __init__(self, moduli, parameters: dict, perf_test: bool = False):
        super().__init__(moduli, parameters, perf_test=perf_test)
        assert self.moduli == list(self.ff_ctx.moduli), "moduli must be the same as the moduli of the finite_field_context"


class NTTCiphertextBATLazyContext(NTTCiphertextContextBase):
    """ntt_mm.py:590-658: step 1 reduced by BATLazyContext (a uint64 value),
    the step-2 product taken in uint64 and Barrett-reduced, step 3 Barrett."""

    def __init__(self, moduli, parameters: dict, perf_test: bool = False):
        super().__init__(moduli, parameters, perf_test=perf_test)
        assert self.moduli == list(self.ff_ctx.moduli), "moduli must be the same as the moduli of the finite_field_context"
        self.ff_ctx_bat_lazy = ff_context.BATLazyContext(self.moduli)

    def _reduction(self) -> int:
        if not isinstance(self.ff_ctx, ff_context.BarrettContext):
            raise NotImplementedError("NTTCiphertextBATLazyContext runs steps 2 and 3 with a BarrettContext")
        return _lib.REDUCTION_BAT_LAZY


class NTTCiphertextShoupContext(NTTCiphertextContextBase):
    """ntt_mm.py:443-587: uint32 tables with their Shoup companions; every
    matrix product is the exact uint64 (wrapping) sum, reduced by Shoup's
    method and cast to uint32.  Runs on the CUDA cores."""

    _TABLES = ("ntt_tf_step1", "ntt_tf_step2", "ntt_tf_step3", "intt_tf_step1", "intt_tf_step2", "intt_tf_step3")

    def _default_ff_ctx(self):
        return ff_context.ShoupContext(self.moduli)

    def __init__(self, moduli, parameters: dict, perf_test: bool = False):
        super().__init__(moduli, parameters, perf_test=perf_test)
        assert self.moduli == list(self.ff_ctx.moduli), "moduli must be the same as the moduli of the finite_field_context"

    def _format_tables(self):
        """ntt_mm.py:457-469: computation format (a mod q) and the companions
        floor(T 2^32 / q), computed from uint64 (ntt_mm.py:475-476)."""
        ff = self.ff_ctx
        for name in self._TABLES:
            t = np.asarray(getattr(self, name))
            setattr(self, name, self.to_computation_format(t).astype(U64 if name.endswith("step2") else U32))
            setattr(self, name + "_shoup", np.asarray(ff.precompute_constant_operand(t.astype(U64))).astype(U64))
        self.ntt_bat_tf_step1 = self.ntt_tf_step1
        self.ntt_bat_tf_step3 = self.ntt_tf_step3
        self.intt_bat_tf_step1 = self.intt_tf_step1
        self.intt_bat_tf_step3 = self.intt_tf_step3

    def to_computation_format(self, a):
        """ntt_mm.py:471-472."""
        return self.ff_ctx.to_computation_format(_tensor.to_numpy(a).astype(U64))

    def to_shoup_computation_format(self, a):
        """ntt_mm.py:474-475."""
        return self.ff_ctx.precompute_constant_operand(np.asarray(a).astype(U64))

    def to_original_format(self, a):
        """ntt_mm.py:477-478."""
        return self.ff_ctx.to_original_format(_tensor.to_numpy(a).astype(U64))

    def _reduction(self) -> int:
        return _lib.REDUCTION_SHOUP

    def plan(self):
        if self._plan is None:
            names = list(self._TABLES) + [n + "_shoup" for n in self._TABLES]
            arrs = [np.ascontiguousarray(np.asarray(getattr(self, n)).astype(U32)) for n in names]
            ptrs = (_lib.vp * 12)(*[a.ctypes.data for a in arrs])
            out = _lib.vp()
            _lib.check(_lib.lib().cross_ntt_plan_create_shoup(self._moduli_ctx().handle(), self.r, self.c, ptrs,
                                                              _lib.C.byref(out)), "cross_ntt_plan_create_shoup")
            self._plan = out
        return self._plan

    def drop_last_modulus(self):
        """ntt_mm.py:412-419; the Shoup tables the transform reads are sliced too."""
        for name in list(self._TABLES) + [n + "_shoup" for n in self._TABLES]:
            setattr(self, name, np.ascontiguousarray(getattr(self, name)[..., :-1]))
        for name in ("ntt_bat_tf_step1", "ntt_bat_tf_step3", "intt_bat_tf_step1", "intt_bat_tf_step3"):
            setattr(self, name, np.ascontiguousarray(getattr(self, name)[..., :-1]))
        self.ff_ctx.drop_last_modulus()
        if self._plan is not None:
            _lib.lib().cross_ntt_plan_destroy(self._plan)
            self._plan = None
