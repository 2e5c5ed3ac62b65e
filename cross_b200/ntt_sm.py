"""Single-modulus BAT 3-step NTT (jaxite_word ntt_sm.py) on the GPU.

The single-modulus transform is the multi-modulus one with one modulus: the
same twiddle tables (ntt_sm.py:156-177 equal ntt_mm.py:186-240 for M = 1),
the same Memory- and Basis-Aligned Transformations (ntt_sm.py:185-221), the
same three reductions (ntt_sm.py:275-328).  Each context here holds the
matching ``ntt_mm`` context over ``[q]`` and runs its device plan on
(B, R, C) arrays (the Shoup context, like the reference's, on one (R, C)
matrix).  Table attributes keep the reference's names and shapes.
"""
from __future__ import annotations

import numpy as np

from . import _tensor, ntt_mm
from . import finite_field as ff_context
# ntt_sm.py:75-119 repeat ntt_mm.py's twiddle-matrix functions
from .ntt_mm import gen_twiddle_matrix, gen_twiddle_matrix_inv  # noqa: F401

U32, U64 = np.uint32, np.uint64


class NTTContextBase:
    """ntt_sm.py:116-328.  The reduction is that of the finite-field context
    (ntt_sm.py:295-300 call ``self.ff_ctx.modular_reduction``): Barrett or
    Montgomery."""

    _mm_class = None   # set per subclass; None: chosen from the context type

    def __init__(self, moduli: int, parameters: dict):
        self.ff_ctx = parameters.get("finite_field_context", None)
        self.num_bytes = 4
        self.moduli = moduli
        self.parameters = parameters
        assert self.moduli < 2 ** 31, "moduli must be less than 2**32"
        self.r = parameters.get("r", 0)
        self.c = parameters.get("c", 0)
        assert self.r != 0, "r must be non-zero"
        assert self.c != 0, "c must be non-zero"
        assert self.ff_ctx is not None, "finite_field_context must be provided"
        self.transform_length = self.r * self.c
        self._q = int(moduli)
        self._mm = self._make_mm()
        self.psi = self._mm.psi_list[0]
        self.omega = self._mm.omega_list[0]
        self._expose_tables()

    # -- the multi-modulus context with one modulus ----------------------------
    def _mm_ff_ctx(self):
        return self.ff_ctx

    def _make_mm(self):
        cls = self._mm_class
        if cls is None:
            if isinstance(self.ff_ctx, ff_context.MontgomeryContext):
                cls = ntt_mm.NTTCiphertextMontgomeryContext
            elif isinstance(self.ff_ctx, ff_context.BarrettContext):
                cls = ntt_mm.NTTCiphertextBarrettContext
            elif isinstance(self.ff_ctx, ff_context.ShoupContext):
                # ntt_sm.py:296 calls modular_reduction(z); Shoup's takes (z, z_s)
                raise TypeError("ShoupContext.modular_reduction() needs z_s: use NTTShoupContext")
            else:
                # a BAT-lazy context reduces step 2 to uint64, which the step-3
                # BAT contraction (a uint32 byte view) cannot take: use NTTBATLazyContext
                raise NotImplementedError(f"NTTContextBase has no transform for {type(self.ff_ctx).__name__}")
        return cls([self.moduli], {"r": self.r, "c": self.c, "finite_field_context": self._mm_ff_ctx()})

    def _expose_tables(self):
        """ntt_sm.py:143-152 with the reference's names for the one modulus:
        the twiddle matrices (``*_tf_step*``, int64), their memory-aligned
        forms (``*_tf_mat_step*``) and those in the computation format, BAT
        for steps 1 and 3 (``*_tf_bat_mat_comp_step*``)."""
        self._raw_tables()
        self.memory_aligned_transformation()
        fmt = self.to_computation_format
        self.ntt_tf_bat_mat_comp_step1 = self.basis_aligned_transformation(fmt(self.ntt_tf_mat_step1))
        self.ntt_tf_mat_comp_step2 = np.asarray(fmt(self.ntt_tf_mat_step2)).astype(U64)
        self.ntt_tf_bat_mat_comp_step3 = self.basis_aligned_transformation(fmt(self.ntt_tf_mat_step3))
        self.intt_tf_bat_mat_comp_step1 = self.basis_aligned_transformation(fmt(self.intt_tf_mat_step1))
        self.intt_tf_mat_comp_step2 = np.asarray(fmt(self.intt_tf_mat_step2)).astype(U64)
        self.intt_tf_bat_mat_comp_step3 = self.basis_aligned_transformation(fmt(self.intt_tf_mat_step3))

    def _raw_tables(self):
        """The twiddle matrices of ntt_sm.py:156-177 (not memory-aligned),
        from the multi-modulus context's memory-aligned ones: the
        bit-reversal permutation is its own inverse."""
        q = self._q
        pr, pc = np.array(ntt_mm.get_bit_reverse_perm(self.r)), np.array(ntt_mm.get_bit_reverse_perm(self.c))
        t1, t2, t3, a, b, d = (t.astype(np.int64) for t in ntt_mm._limb_tables(q, self.r, self.c))
        self.ntt_tf_step1, self.ntt_tf_step2, self.ntt_tf_step3 = t1[pr, :], t2[pr, :], t3[:, pc]
        self.intt_tf_step1, self.intt_tf_step2, self.intt_tf_step3 = a[pc, :], b[pr, :], d[:, pr]

    # -- offline (the reference's public table functions) ---------------------
    def ntt_coefficients_precompute(self):
        """ntt_sm.py:156-162: (step 1, step 2, step 3) twiddle matrices."""
        return self.ntt_tf_step1.copy(), self.ntt_tf_step2.copy(), self.ntt_tf_step3.copy()

    def intt_coefficients_precompute(self):
        """ntt_sm.py:164-177: the inverse matrices, 1/C and 1/R folded into
        steps 2 and 3."""
        return self.intt_tf_step1.copy(), self.intt_tf_step2.copy(), self.intt_tf_step3.copy()

    def memory_aligned_transformation(self):
        """ntt_sm.py:195-221: bit-reversal row / column permutations of the
        twiddle matrices into the ``*_tf_mat_step*`` attributes."""
        pr, pc = np.array(ntt_mm.get_bit_reverse_perm(self.r)), np.array(ntt_mm.get_bit_reverse_perm(self.c))
        self.ntt_tf_mat_step1 = self.ntt_tf_step1[pr, :]
        self.ntt_tf_mat_step2 = self.ntt_tf_step2[pr, :]
        self.ntt_tf_mat_step3 = self.ntt_tf_step3[:, pc]
        self.intt_tf_mat_step1 = self.intt_tf_step1[pc, :]
        self.intt_tf_mat_step2 = self.intt_tf_step2[pr, :]
        self.intt_tf_mat_step3 = self.intt_tf_step3[:, pr]

    def basis_aligned_transformation(self, matrix):
        """ntt_sm.py:185-193: (rows, 4, cols, 4) uint8, the bytes of
        (matrix << 8 i) mod q for i < 4."""
        return ntt_mm.basis_aligned_transformation(np.asarray(matrix)[..., None], [self._q])[..., 0]

    def to_computation_format(self, a):
        """ntt_sm.py:179-180."""
        return self.ff_ctx.to_computation_format(_tensor.to_numpy(a))

    def to_original_format(self, a):
        """ntt_sm.py:182-183."""
        return self.ff_ctx.to_original_format(_tensor.to_numpy(a))

    def check_device(self):
        self._mm.check_device()

    def _run(self, v, inverse: bool):
        x = _tensor.to_u32(v)
        if x.dim() != 3 or tuple(x.shape[1:]) != (self.r, self.c):
            raise ValueError(f"expected (B, {self.r}, {self.c}), got {tuple(x.shape)}")
        y = self._mm.intt(x.unsqueeze(-1)) if inverse else self._mm.ntt(x.unsqueeze(-1))
        return y[..., 0]

    def ntt(self, v):
        """ntt_sm.py:275-300: (B, R, C) uint32 -> bit-reversed evaluations."""
        return self._run(v, False)

    def intt(self, v):
        """ntt_sm.py:302-328."""
        return self._run(v, True)


class NTTBarrettContext(NTTContextBase):
    """ntt_sm.py:330-337."""

    def __init__(self, moduli: int, parameters: dict):
        super().__init__(moduli, parameters)
        assert [self.moduli] == list(self.ff_ctx.moduli), "moduli must be the same as the moduli of the finite_field_context"


class NTTMontgomeryContext(NTTContextBase):
    """ntt_sm.py:339-346."""

    def __init__(self, moduli: int, parameters: dict):
        super().__init__(moduli, parameters)
        assert [self.moduli] == list(self.ff_ctx.moduli), "moduli must be the same as the moduli of the finite_field_context"


class NTTBATLazyContext(NTTContextBase):
    """ntt_sm.py:348-412: step 1 reduced by the BAT-lazy context given as
    finite_field_context, steps 2 and 3 by a Barrett context over the same
    modulus (``ff_ctx_full``)."""

    _mm_class = ntt_mm.NTTCiphertextBATLazyContext

    def __init__(self, moduli: int, parameters: dict):
        self.ff_ctx_full = ff_context.BarrettContext(moduli)
        super().__init__(moduli, parameters)

    def _mm_ff_ctx(self):
        return self.ff_ctx_full


class NTTShoupContext(NTTContextBase):
    """ntt_sm.py:415-494: one (R, C) matrix, uint32 tables with Shoup
    companions (computed from the integers, ntt_sm.py:440-447)."""

    _mm_class = ntt_mm.NTTCiphertextShoupContext

    def __init__(self, moduli: int, parameters: dict):
        super().__init__(moduli, parameters)
        if type(self.moduli) is int:
            self.moduli = [self.moduli]                 # ntt_sm.py:422-423
        assert self.moduli == list(self.ff_ctx.moduli), "moduli must be the same as the moduli of the finite_field_context"

    def _expose_tables(self):
        """ntt_sm.py:420-437: the base tables, then the memory-aligned ones in
        the computation format with their Shoup companions."""
        super()._expose_tables()
        m = self._mm
        for name in ("ntt_tf", "intt_tf"):
            for k in (1, 2, 3):
                setattr(self, f"{name}_mat_step{k}", np.asarray(getattr(m, f"{name}_step{k}"))[..., 0])
                # companions as the reference stores them: uint32 for steps 1
                # and 3 (below 2^32 since T < q), uint64 for step 2
                setattr(self, f"{name}_mat_step{k}_shoup",
                        np.asarray(getattr(m, f"{name}_step{k}_shoup"))[..., 0].astype(U64 if k == 2 else U32))

    def to_shoup_computation_format(self, a):
        """ntt_sm.py:440-447."""
        return np.array([self.ff_ctx.precompute_constant_operand(np.uint64(int(x)))
                         for x in np.asarray(a).reshape(-1)], U64).reshape(np.shape(a))

    def _run(self, v, inverse: bool):
        x = _tensor.to_u32(v)
        if x.dim() != 2 or tuple(x.shape) != (self.r, self.c):
            raise ValueError(f"expected ({self.r}, {self.c}), got {tuple(x.shape)}")
        y = self._mm.intt(x[None, ..., None]) if inverse else self._mm.ntt(x[None, ..., None])
        return y[0, ..., 0]
