"""Numpy restatement of jaxite_word's Montgomery, Shoup and BAT-lazy variants
of the NTT and the basis conversion (the oracle for those paths).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

The Barrett hot path lives in ``cross_oracle``; this module restates the
other reduction contexts of finite_field.py and the NTT / BConv classes built
on them, with the reference's integer semantics (uint32 / uint64 wrap-around,
the same lazy representatives, the same truncating casts):

  finite_field.py:58-164   MontgomeryContext      -> Montgomery
  finite_field.py:278-338  ShoupContext           -> Shoup
  finite_field.py:344-428  BATLazyContext         -> BATLazy
  ntt_mm.py:432-440        NTTCiphertextMontgomeryContext  -> NTTVariant("montgomery")
  ntt_mm.py:443-587        NTTCiphertextShoupContext       -> NTTVariant("shoup")
  ntt_mm.py:590-658        NTTCiphertextBATLazyContext     -> NTTVariant("bat_lazy")
  ntt_sm.py:116-494        single-modulus contexts         -> the same with one modulus
  bconv.py:261-390         BConvMontgomery / BConvShoup / BConvBATLazy
"""

from __future__ import annotations

from typing import Sequence

import numpy as np

from .cross_oracle import (U32, U64, Barrett, NTTBarrett, _combine_bytes, _exact_u8_matmul,
                           basis_aligned_transformation, compute_qhat)

MASK32 = U64(0xFFFFFFFF)


def _as_list(moduli) -> list:
    return [moduli] if isinstance(moduli, (int, np.integer)) else [int(q) for q in moduli]


# ---------------------------------------------------------------------------
# finite_field.py: the three other reduction contexts
# ---------------------------------------------------------------------------

class Montgomery:
    """finite_field.py:58-164 (MontgomeryContext), w = 32."""

    def __init__(self, moduli):
        self.moduli = _as_list(moduli)
        self.q = np.array(self.moduli, U64)
        self.w_inv = np.array([pow(1 << 32, -1, q) for q in self.moduli], U64)           # :67-68
        self.q_inv_32 = np.array([pow(q, -1, 1 << 32) for q in self.moduli], U64)        # :72
        self.q_low = self.q & U64(0xFFFF)                                                 # :73
        self.q_high = self.q >> U64(16)                                                   # :74

    def to_computation_format(self, a, moduli_axis=None):
        """finite_field.py:82-84: (a << 32) mod q, moduli on the last axis."""
        return ((np.asarray(a).astype(U64) << U64(32)) % self.q).astype(U32)

    def to_original_format(self, a):
        """finite_field.py:86-87: a * 2^-32 mod q (uint64)."""
        return (np.asarray(a).astype(U64) * self.w_inv) % self.q

    def reduce_with(self, z, q, q_inv, q_low, q_high) -> np.ndarray:
        """finite_field.py:126-154 with explicit constants (uint32 wrap-around,
        the 16-bit split of t * q)."""
        z = np.asarray(z).astype(U64)
        m16 = U64(0xFFFF)
        z_low = z & MASK32
        z_high = z >> U64(32)
        t = (z_low * q_inv) & MASK32
        t_low, t_high = t & m16, (t >> U64(16)) & m16
        prod_high = t_high * q_high
        prod_mid_high = t_high * q_low
        prod_mid_low = t_low * q_high
        prod_low = t_low * q_low
        mid_low = (prod_mid_high & m16) + (prod_mid_low & m16) + (prod_low >> U64(16))
        mid_high = (prod_mid_high >> U64(16)) + (prod_mid_low >> U64(16)) + (mid_low >> U64(16))
        t_final = prod_high + mid_high
        return ((z_high + q - t_final) & MASK32).astype(U32)                            # u32 arithmetic

    def reduce(self, z) -> np.ndarray:
        """finite_field.py:94-154, moduli on the last axis."""
        return self.reduce_with(z, self.q, self.q_inv_32, self.q_low, self.q_high)

    def reduce_limb(self, z, i: int) -> np.ndarray:
        return self.reduce_with(z, self.q[i], self.q_inv_32[i], self.q_low[i], self.q_high[i])


class Shoup:
    """finite_field.py:278-338 (ShoupContext)."""

    def __init__(self, moduli):
        self.moduli = _as_list(moduli)
        self.q = np.array(self.moduli, U64)

    def to_computation_format(self, a):
        """finite_field.py:289-291."""
        return (np.asarray(a).astype(U64) % self.q).astype(U32)

    def to_original_format(self, a):
        """finite_field.py:293-294."""
        return (np.asarray(a).astype(U64) % self.q).astype(U32)

    def precompute_constant_operand(self, a):
        """finite_field.py:296-298: floor(a 2^32 / q) (uint64)."""
        return (np.asarray(a).astype(U64) << U64(32)) // self.q

    @staticmethod
    def reduce_with(z, z_s, q) -> np.ndarray:
        """finite_field.py:305-330: (z - (z_s >> 32) q) in uint64, cast to uint32."""
        t = np.asarray(z_s).astype(U64) >> U64(32)
        return (np.asarray(z).astype(U64) - t * np.asarray(q, U64)).astype(U32)

    def reduce(self, z, z_s) -> np.ndarray:
        return self.reduce_with(z, z_s, self.q)

    def reduce_limb(self, z, z_s, i: int) -> np.ndarray:
        return self.reduce_with(z, z_s, self.q[i])


class BATLazy:
    """finite_field.py:344-428 (BATLazyContext).  R[m, i, j] = byte j of
    (256^(i+4) mod q_m); reduction = B @ R + A over the byte split of z."""

    def __init__(self, moduli):
        self.moduli = _as_list(moduli)
        qa = np.array(self.moduli, U64)
        r_vals = (U64(1) << (np.arange(4, 8, dtype=U64) * U64(8)))[None, :] % qa[:, None]       # :363-365
        shifts = np.arange(4, dtype=U64) * U64(8)
        self.R = ((r_vals[:, :, None] >> shifts[None, None, :]) & U64(0xFF)).astype(np.uint8)    # :369-370
        self.q = qa

    def to_computation_format(self, a):
        return a

    def to_original_format(self, a):
        """finite_field.py:375-376."""
        return (np.asarray(a).astype(U64) % self.q).astype(U32)

    @staticmethod
    def reduce_with(z, R) -> np.ndarray:
        """finite_field.py:384-425: bytes 0-3 (A) plus bytes 4-7 (B) times R,
        each byte lane summed exactly, recombined in uint64."""
        z = np.asarray(z).astype(U64)
        zb = np.ascontiguousarray(z).view(np.uint8).reshape(*z.shape, 8)
        A, B = zb[..., :4].astype(np.int64), zb[..., 4:].astype(np.int64)
        res = np.einsum("...i,...ij->...j", B, np.asarray(R).astype(np.int64)) + A
        return np.sum(res.astype(U64) << np.array([0, 8, 16, 24], U64), axis=-1)

    def reduce(self, z) -> np.ndarray:
        """Moduli on the last axis (one modulus: every element)."""
        R = self.R[0] if len(self.moduli) == 1 else self.R
        return self.reduce_with(z, R)

    def reduce_limb(self, z, i: int) -> np.ndarray:
        return self.reduce_with(z, self.R[i])


# ---------------------------------------------------------------------------
# ntt_mm.py / ntt_sm.py: NTT with the other reductions
# ---------------------------------------------------------------------------

def _u64_matmul_wrap(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """sum_k a[..., i, k] * b[k, j] in uint64 with wrap-around: every product of
    two uint32 values is exact in uint64, and numpy's uint64 sums wrap like the
    reference's byte-convolution sums recombined in uint64 (ntt_mm.py:40-65)."""
    a = a.astype(U64)
    b = b.astype(U64)
    out = np.zeros(a.shape[:-1] + (b.shape[-1],), U64)
    for k in range(a.shape[-1]):
        out += a[..., k:k + 1] * b[k][None, :]
    return out


class NTTVariant(NTTBarrett):
    """The 3-step NTT of ntt_mm.py:351-407 with another reduction.

    montgomery (ntt_mm.py:432-440): tables in Montgomery form
        (ntt_mm.py:172-181), all three reductions Montgomery.
    bat_lazy (ntt_mm.py:590-658, ntt_sm.py:348-412): step 1 BAT-lazy (uint64
        out), step 2 Barrett of the uint64 (wrapping) product, step 3 Barrett.
    shoup (ntt_mm.py:443-587, ntt_sm.py:415-494): plain uint32 tables, uint64
        matrix products (byte convolutions recombined in uint64), Shoup's
        reduction with the precomputed floor(T 2^32 / q) tables.
    """

    def __init__(self, moduli, r: int, c: int, reduction: str):
        super().__init__(moduli, r, c)
        self.reduction = reduction
        if reduction == "montgomery":
            self.mont = Montgomery(self.moduli)
            fmt = self.mont.to_computation_format
            self.ntt_bat_tf_step1 = basis_aligned_transformation(fmt(self.ntt_tf_step1), self.moduli)
            self.ntt_bat_tf_step3 = basis_aligned_transformation(fmt(self.ntt_tf_step3), self.moduli)
            self.intt_bat_tf_step1 = basis_aligned_transformation(fmt(self.intt_tf_step1), self.moduli)
            self.intt_bat_tf_step3 = basis_aligned_transformation(fmt(self.intt_tf_step3), self.moduli)
            self.ntt_tf_step2 = fmt(self.ntt_tf_step2)
            self.intt_tf_step2 = fmt(self.intt_tf_step2)
        elif reduction == "bat_lazy":
            self.lazy = BATLazy(self.moduli)
        elif reduction == "shoup":
            self.sh = Shoup(self.moduli)
            # ntt_mm.py:457-469: computation format (a mod q) and the Shoup companions
            for name in ("ntt_tf_step1", "ntt_tf_step2", "ntt_tf_step3",
                         "intt_tf_step1", "intt_tf_step2", "intt_tf_step3"):
                t = self.sh.to_computation_format(getattr(self, name))
                setattr(self, name, t)
                setattr(self, name + "_shoup", self.sh.precompute_constant_operand(t))
        else:
            raise ValueError(f"unknown reduction {reduction!r}")

    # one limb ---------------------------------------------------------------
    def _step(self, s, m, kind):
        if self.reduction == "montgomery":
            return self.mont.reduce_limb(s, m)
        if self.reduction == "bat_lazy" and kind == 1:
            return self.lazy.reduce_limb(s, m)                       # uint64
        return self.ff.reduce_limb(s, m)                             # Barrett

    def _limb(self, v, m, inverse):
        if self.reduction == "shoup":
            return self._limb_shoup(v, m, inverse)
        if not inverse:
            s1 = self._bat_col(v, self.ntt_bat_tf_step1[..., m])
            t2, t3 = self.ntt_tf_step2[..., m], self.ntt_bat_tf_step3[..., m]
        else:
            s1 = self._bat_row(v, self.intt_bat_tf_step1[..., m])
            t2, t3 = self.intt_tf_step2[..., m], self.intt_bat_tf_step3[..., m]
        r1 = self._step(s1, m, 1)
        r2 = self._step(r1.astype(U64) * t2.astype(U64), m, 2)       # uint64 product, wraps
        s3 = self._bat_row(r2, t3) if not inverse else self._bat_col(r2, t3)
        return self._step(s3, m, 3)

    @staticmethod
    def _bat_col(x, t):
        from .cross_oracle import bat_col
        return bat_col(x, t)

    @staticmethod
    def _bat_row(x, t):
        from .cross_oracle import bat_row
        return bat_row(x, t)

    def _limb_shoup(self, v, m, inverse):
        sh = self.sh
        q = sh.q[m]
        v = v.astype(U64)
        if not inverse:
            # ntt_mm.py:500-542: Z = T1 V, (.) T2, W = Z T3 (all uint64 wrap)
            t1, t1s = self.ntt_tf_step1[..., m], self.ntt_tf_step1_shoup[..., m]
            t2, t2s = self.ntt_tf_step2[..., m], self.ntt_tf_step2_shoup[..., m]
            t3, t3s = self.ntt_tf_step3[..., m], self.ntt_tf_step3_shoup[..., m]
            vt = np.swapaxes(v, -1, -2)                                   # (B, C, R)
            z = np.swapaxes(_u64_matmul_wrap(vt, t1.T), -1, -2)           # sum_r T1[z, r] V[r, c]
            zs = np.swapaxes(_u64_matmul_wrap(vt, t1s.T), -1, -2)
            r1 = Shoup.reduce_with(z, zs, q)
            r2 = Shoup.reduce_with(r1.astype(U64) * t2.astype(U64), r1.astype(U64) * t2s.astype(U64), q)
            z3 = _u64_matmul_wrap(r2, t3)                                 # sum_c R2[r, c] T3[c, n]
            z3s = _u64_matmul_wrap(r2, t3s)
            return Shoup.reduce_with(z3, z3s, q)
        # ntt_mm.py:544-587: Y = V iT1, (.) iT2, X = iT3 Y
        t1, t1s = self.intt_tf_step1[..., m], self.intt_tf_step1_shoup[..., m]
        t2, t2s = self.intt_tf_step2[..., m], self.intt_tf_step2_shoup[..., m]
        t3, t3s = self.intt_tf_step3[..., m], self.intt_tf_step3_shoup[..., m]
        z = _u64_matmul_wrap(v, t1)
        zs = _u64_matmul_wrap(v, t1s)
        r1 = Shoup.reduce_with(z, zs, q)
        r2 = Shoup.reduce_with(r1.astype(U64) * t2.astype(U64), r1.astype(U64) * t2s.astype(U64), q)
        r2t = np.swapaxes(r2.astype(U64), -1, -2)                        # (B, C, R)
        z3 = np.swapaxes(_u64_matmul_wrap(r2t, t3.T), -1, -2)            # sum_r iT3[l, r] R2[r, c]
        z3s = np.swapaxes(_u64_matmul_wrap(r2t, t3s.T), -1, -2)
        return Shoup.reduce_with(z3, z3s, q)

    def _run(self, v, inverse):
        v = np.asarray(v).astype(U32)
        B = v.shape[0]
        dt = U32
        outs = [self._limb(v[..., m], m, inverse) for m in range(len(self.moduli))]
        out = np.empty((B, self.r, self.c, len(self.moduli)), dt)
        for m, o in enumerate(outs):
            out[..., m] = o
        return out

    def ntt(self, v: np.ndarray) -> np.ndarray:
        return self._run(v, False)

    def intt(self, v: np.ndarray) -> np.ndarray:
        return self._run(v, True)


# ---------------------------------------------------------------------------
# bconv.py:261-390: basis conversion with the other reductions
# ---------------------------------------------------------------------------

def _bat_bytes(qhat_modp: np.ndarray, dst: Sequence[int]) -> np.ndarray:
    """bconv.py:93-97,157-170: (sizeQ, sizeP) -> (4 sizeQ, sizeP, 4) uint8."""
    shifted = np.array([qhat_modp.astype(U64) << U64(8 * a) for a in range(4)], U64)
    red = (shifted % np.array(dst, U64)).astype(U32)
    u8 = np.ascontiguousarray(red).view(np.uint8).reshape(4, qhat_modp.shape[0], len(dst), 4)
    return np.ascontiguousarray(u8.transpose(1, 0, 2, 3).reshape(-1, len(dst), 4))


def _bat_contract(c: np.ndarray, bat: np.ndarray, sq: int, sp: int) -> np.ndarray:
    """matmul_bat_einsum(c, QHatModpBAT, '...q,qpb->...pb') (bconv.py:19-37)."""
    lead = c.shape[:-1]
    a = np.ascontiguousarray(c.astype(U32)).view(np.uint8).reshape(-1, 4 * sq)
    p = _exact_u8_matmul(a, bat.reshape(4 * sq, sp * 4)).reshape(*lead, sp, 4)
    return _combine_bytes(p)


def _sum_products(c: np.ndarray, tab: np.ndarray) -> np.ndarray:
    """sum_i c[..., i] * tab[i, j] in uint64 with wrap-around (bconv.py:199-204)."""
    c = c.astype(U64)
    acc = np.zeros(c.shape[:-1] + (tab.shape[1],), U64)
    for i in range(tab.shape[0]):
        acc = acc + c[..., i:i + 1] * tab[i].astype(U64)[None, :]
    return acc


def jax_precompute_u32(a, moduli) -> np.ndarray:
    """ShoupContext.precompute_constant_operand (finite_field.py:295-297) as
    BConvShoup.control_gen calls it (bconv.py:313-314): on the uint32 arrays that
    ShoupContext.to_computation_format returns (finite_field.py:289-291).  The
    reference runs under JAX, whose uint32 shift by 32 saturates to 0 (XLA
    shift semantics), so (a << 32) // q is 0 for every entry."""
    a = np.asarray(a)
    return np.zeros(a.shape, U64)


class BConvVariant:
    """BConvMontgomery / BConvShoup / BConvBATLazy (bconv.py:261-390) with the
    base-class constant generation (bconv.py:67-155)."""

    def __init__(self, overall_moduli, reduction: str):
        if reduction not in ("montgomery", "shoup", "bat_lazy"):
            raise ValueError(f"unknown reduction {reduction!r}")
        self.overall_moduli = list(overall_moduli)
        self.reduction = reduction
        self.controls = []

    def _ctx(self, moduli):
        return {"montgomery": Montgomery, "shoup": Shoup, "bat_lazy": BATLazy}[self.reduction](moduli)

    def control_gen(self, control_indices_list):
        self.controls = []
        for src_idx, dst_idx in control_indices_list:
            src = [self.overall_moduli[i] for i in src_idx]
            dst = [self.overall_moduli[i] for i in dst_idx]
            o, t = self._ctx(src), self._ctx(dst)
            qhat_inv, qhat_modp = compute_qhat(src, dst)
            qhat_inv = np.array(qhat_inv, U64)
            qhat_modp = np.array(qhat_modp, U64).reshape(len(src), len(dst))
            if self.reduction == "montgomery":                                   # bconv.py:85-91
                qhat_inv = o.to_computation_format(qhat_inv).astype(U64)
                qhat_modp = t.to_computation_format(qhat_modp).astype(U64)
            elif self.reduction == "shoup":
                qhat_inv = o.to_computation_format(qhat_inv).astype(U64)
                qhat_modp = t.to_computation_format(qhat_modp).astype(U64)
            ctl = dict(src=src, dst=dst, o=o, t=t, qhat_inv=qhat_inv, qhat_modp=qhat_modp,
                       bat=_bat_bytes(qhat_modp, dst))
            if self.reduction == "shoup":                                        # bconv.py:300-314
                ctl["qhat_inv_shoup"] = jax_precompute_u32(qhat_inv, src)
                ctl["qhat_modp_shoup"] = jax_precompute_u32(qhat_modp, dst)
            self.controls.append(ctl)

    def basis_change(self, x, control_index: int = 0) -> np.ndarray:
        ctl = self.controls[control_index]
        o, t = ctl["o"], ctl["t"]
        x = np.asarray(x).astype(U64)
        cu = x * ctl["qhat_inv"]
        if self.reduction == "montgomery":                                       # bconv.py:266-287
            c = o.reduce(cu)
            back = o.to_original_format(c)
            if len(ctl["src"]) != len(ctl["dst"]) and len(ctl["dst"]) != 1:
                raise ValueError("BConvMontgomery.basis_change: the target-basis format broadcasts "
                                 "source limbs against target moduli (size_q must equal size_p, or size_p 1)")
            c = t.to_computation_format(back)
            return t.reduce(_sum_products(c, ctl["qhat_modp"]))
        if self.reduction == "shoup":                                            # bconv.py:315-339
            c = o.reduce(cu, x * ctl["qhat_inv_shoup"])
            z = _sum_products(c, ctl["qhat_modp"])
            zs = _sum_products(c, ctl["qhat_modp_shoup"].astype(U32))
            return t.reduce(z, zs)
        c = o.reduce(cu)                                                          # bconv.py:347-368
        c = o.to_original_format(c)
        return t.reduce(_sum_products(c, ctl["qhat_modp"]))                      # uint64 out

    def basis_change_bat(self, x, control_index: int = 0) -> np.ndarray:
        ctl = self.controls[control_index]
        o, t = ctl["o"], ctl["t"]
        sq, sp = len(ctl["src"]), len(ctl["dst"])
        x = np.asarray(x).astype(U64)
        cu = x * ctl["qhat_inv"]
        if self.reduction == "shoup":
            # the base-class path calls the two-operand Shoup reduction with one operand
            raise TypeError("BConvShoup.basis_change_bat: ShoupContext.modular_reduction needs z_s")
        if self.reduction == "montgomery":                                       # bconv.py:234-252
            c = o.reduce(cu)
            return t.reduce(_bat_contract(c, ctl["bat"], sq, sp))
        c = o.reduce(cu).astype(U32)                                             # bconv.py:370-390
        c = o.to_original_format(c)
        return t.reduce(_bat_contract(c, ctl["bat"], sq, sp))                    # uint64 out
