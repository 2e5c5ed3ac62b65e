"""RNS ciphertext object (jaxite_word ciphertext.py) backed by CUDA tensors.

Layout (batch, elements, *degree_layout, limbs), limb-innermost, as the
reference.  Transforms, modular reductions, the tensor product, the basis
conversions and rescale run the kernels of libcross_b200.so.  ``add``,
``sub`` and ``mul`` are the reference's raw (unreduced, wrapping) integer
operations.
"""
from __future__ import annotations

import math
from typing import List, Optional, Union

import numpy as np

from . import _lib, _tensor, util
from . import finite_field as ff_context
from . import ntt_mm as ntt
from .bconv import BConvBarrett

U32, U64 = np.uint32, np.uint64


def _t():
    return _tensor.torch()


def _u64(x):
    """x as a CUDA uint64 tensor (zero-extended from uint32)."""
    t = _t()
    if isinstance(x, t.Tensor) and x.dtype == t.uint64:
        return x.to(_tensor.device())
    if isinstance(x, t.Tensor):
        return _tensor.to_u32(x).view(t.int32).to(t.int64).bitwise_and(0xFFFFFFFF).view(t.uint64)
    return t.from_numpy(np.ascontiguousarray(np.asarray(x).astype(U64))).to(_tensor.device())


def _low32(r):
    """Low 32 bits of an int64 tensor as uint32 (two's-complement wrap)."""
    t = _t()
    lo = r.bitwise_and(0xFFFFFFFF)
    return (lo - ((lo >> 31) << 32)).to(t.int32).view(t.uint32)


def _bcast(x, shape):
    """Materialise the numpy-style broadcast of x to shape (any 32/64-bit dtype)."""
    t = _t()
    if x.dtype == t.uint32:
        return x.view(t.int32).broadcast_to(shape).contiguous().view(t.uint32)
    if x.dtype == t.uint64:
        return x.view(t.int64).broadcast_to(shape).contiguous().view(t.uint64)
    return x.broadcast_to(shape).contiguous()


def _wrap_op(a, b, op):
    """uint64 (or uint32) add/sub/mul with wrap-around, result dtype as numpy promotion."""
    t = _t()
    a_is64 = isinstance(a, t.Tensor) and a.dtype == t.uint64 or isinstance(a, np.ndarray) and a.dtype == U64
    b_is64 = isinstance(b, t.Tensor) and b.dtype == t.uint64 or isinstance(b, np.ndarray) and b.dtype == U64
    A, B = _u64(a).view(t.int64), _u64(b).view(t.int64)
    r = op(A, B)
    return r.view(t.uint64) if (a_is64 or b_is64) else _low32(r)


def gen_power_of_inv_psi_arr(moduli, ring_dim):
    """ciphertext.py:13-20."""
    q_list = [moduli] if not isinstance(moduli, list) else moduli
    arr = np.stack([util.powers(pow(util.root_of_unity(2 * ring_dim, q), -1, q), ring_dim, q) for q in q_list], -1)
    return arr.reshape(1, 1, ring_dim, -1)


class Ciphertext:
    """ciphertext.py:23-519."""

    def __init__(self, shapes: dict, parameters: Optional[dict] = None):
        self.batch = shapes["batch"]
        self.num_elements = shapes["num_elements"]
        self.num_moduli = shapes["num_moduli"]
        self.degree = shapes["degree"]
        self.precision = shapes["precision"]
        self.degree_layout = tuple(shapes["degree_layout"]) if "degree_layout" in shapes else (self.degree,)
        self.modulus_dtype = U32 if self.precision <= 32 else U64
        if parameters is not None and "moduli" in parameters:
            self.moduli = list(parameters["moduli"])
        else:
            self.moduli = util.find_moduli_ntt(self.num_moduli, self.precision, 2 * self.degree)
        log_degree = int(math.log2(self.degree))
        if parameters is not None and "finite_field_context" in parameters:
            self.r, self.c = parameters["r"], parameters["c"]
            ffc = parameters["finite_field_context"](moduli=self.moduli)
        else:
            self.r = 1 << (log_degree // 2)
            self.c = self.degree // self.r
            ffc = ff_context.BarrettContext(moduli=self.moduli)
        ntt_params = {"r": self.r, "c": self.c, "finite_field_context": ffc}
        self.bit_reverse_indices = util.bit_reverse_indices(self.degree)
        self.shape_in_ntt_all_limbs = (-1, self.r, self.c, self.num_moduli)
        if parameters is not None and parameters.get("BAT_lazy", False):
            self._ntt_cls = ntt.NTTCiphertextBATLazyContext
        elif isinstance(ffc, ff_context.BarrettContext):
            self._ntt_cls = ntt.NTTCiphertextBarrettContext
        elif isinstance(ffc, ff_context.MontgomeryContext):
            self._ntt_cls = ntt.NTTCiphertextMontgomeryContext
        elif isinstance(ffc, ff_context.ShoupContext):
            self._ntt_cls = ntt.NTTCiphertextShoupContext
        else:
            raise ValueError(f"Unsupported finite field context type: {type(ffc)}")
        # the NTT context (ciphertext.py:98-107) is built at its first use:
        # objects that only carry data (the CKKS context's results) skip the
        # table precompute
        self._ntt_args = (list(self.moduli), ntt_params)
        self._ntt_ctx = None
        self.moduli_array = np.array(self.moduli, dtype=self.modulus_dtype)
        self.ciphertext = _tensor.torch().zeros((self.batch, self.num_elements, self.degree, self.num_moduli),
                                                dtype=_tensor.torch().uint32 if self.precision <= 32 else _tensor.torch().uint64,
                                                device=_tensor.device())
        self.bconv = None
        self.bconv_indices_list = []

    @property
    def ntt_ctx(self):
        if self._ntt_ctx is None:
            self._ntt_ctx = self._ntt_cls(*self._ntt_args)
        return self._ntt_ctx

    @ntt_ctx.setter
    def ntt_ctx(self, value):
        self._ntt_ctx = value

    def _create_bconv(self, moduli):
        if self.bconv is None:
            self.bconv = BConvBarrett(moduli)
        return self.bconv

    def random_init(self, seed: int = 0):
        shape = (self.batch, self.num_elements, *self.degree_layout, self.num_moduli)
        rng = np.random.default_rng(seed)
        q = np.array(self.moduli, U64)
        self.ciphertext = _tensor.to_u32((rng.integers(0, 2 ** 62, size=shape, dtype=np.uint64) % q).astype(U32))

    # -- getters / setters (ciphertext.py:110-149) ---------------------------
    @property
    def shape(self):
        return tuple(self.ciphertext.shape)

    def get_batch_ciphertext(self):
        return self.ciphertext

    def get_ciphertext(self, batch_index):
        return self.ciphertext[batch_index]

    def get_element(self, element_index):
        return self.ciphertext[:, element_index]

    def get_limb(self, limb_index):
        return self.ciphertext[..., limb_index]

    def set_batch_ciphertext(self, batch_ciphertext):
        t = _t()
        self.ciphertext = batch_ciphertext if isinstance(batch_ciphertext, t.Tensor) and batch_ciphertext.is_cuda \
            else _tensor.to_any(batch_ciphertext)[0]

    def set_ciphertext(self, batch_index, ciphertext):
        self.ciphertext = self.ciphertext.clone()
        self.ciphertext[batch_index] = _tensor.to_any(ciphertext)[0].to(self.ciphertext.dtype)

    def set_element(self, element_index, element):
        self.ciphertext = self.ciphertext.clone()
        self.ciphertext[:, element_index] = _tensor.to_any(element)[0].to(self.ciphertext.dtype)

    def set_limb(self, limb_index, limb):
        self.ciphertext = self.ciphertext.clone()
        self.ciphertext[..., limb_index] = _tensor.to_any(limb)[0].to(self.ciphertext.dtype)

    def get_moduli_array(self):
        return self.moduli_array

    def get_moduli(self) -> Union[List[int], int]:
        return self.moduli

    def get_modulus(self, index: int) -> int:
        return self.moduli[index]

    # -- domain conversion (ciphertext.py:154-170) ---------------------------
    def to_ntt_form(self):
        shape = self.ciphertext.shape
        self.ciphertext = self.ntt_ctx.ntt(_tensor.to_u32(self.ciphertext).reshape(self.shape_in_ntt_all_limbs)).reshape(shape)

    def to_coeffs_form(self):
        shape = self.ciphertext.shape
        self.ciphertext = self.ntt_ctx.intt(_tensor.to_u32(self.ciphertext).reshape(self.shape_in_ntt_all_limbs)).reshape(shape)

    def to_compute_format(self):
        self.ciphertext = _tensor.to_u32(self.ntt_ctx.to_computation_format(_tensor.to_numpy(self.ciphertext)))

    def to_original_format(self):
        self.ciphertext = _tensor.to_u32(self.ntt_ctx.to_original_format(_tensor.to_numpy(self.ciphertext)))

    # -- arithmetic (ciphertext.py:175-197) ----------------------------------
    def _other(self, other):
        return other.ciphertext if isinstance(other, Ciphertext) else other

    def add(self, other):
        self.ciphertext = _wrap_op(self.ciphertext, self._other(other), lambda a, b: a + b)

    def sub(self, other):
        self.ciphertext = _wrap_op(self.ciphertext, self._other(other), lambda a, b: a - b)

    def mul(self, other):
        t = _t()
        r = _wrap_op(self.ciphertext, self._other(other), lambda a, b: a * b)
        self.ciphertext = r if r.dtype == t.uint64 else _u64(r)

    def modmul(self, other):
        a, a64 = _tensor.to_any(self.ciphertext)
        b, b64 = _tensor.to_any(self._other(other))
        shape = _t().broadcast_shapes(a.shape, b.shape)
        a, b = _bcast(a, shape), _bcast(b, shape)
        ff = self.ntt_ctx.ff_ctx
        out = _tensor.empty_u32(shape)
        _tensor.call("cross_modmul", ff.handle(), a.data_ptr(), int(a64), b.data_ptr(), int(b64), a.numel() // shape[-1],
                     out.data_ptr(), a.numel() // shape[-1], _lib.cuda_stream())
        self.ciphertext = out

    def mod_reduce(self):
        self.ciphertext = self.ntt_ctx.ff_ctx.modular_reduction(self.ciphertext)

    # -- modulus dropping (ciphertext.py:203-217) ----------------------------
    def drop_last_modulus(self):
        if self.num_moduli <= 1:
            raise ValueError("Cannot drop modulus from a single-limb ciphertext.")
        self.ciphertext = self.ciphertext[..., :-1].contiguous() if self.ciphertext.dtype != _t().uint32 else \
            self.ciphertext.view(_t().int32)[..., :-1].contiguous().view(_t().uint32)
        self.moduli = self.moduli[:-1]
        self.moduli_array = self.moduli_array[:-1]
        self.num_moduli -= 1
        self.shape_in_ntt_all_limbs = (-1, self.r, self.c, self.num_moduli)
        self.shape_in_ntt_last_limb = (-1, self.r, self.c)
        self.ntt_ctx.drop_last_modulus()
        return self.ciphertext

    # -- rescale (ciphertext.py:223-303) -------------------------------------
    def modulus_switch_control_gen(self, degree_layout: tuple = None, perf_test: bool = False):
        if self.num_moduli <= 1:
            raise ValueError("Cannot perform modulus switch with fewer than two moduli.")
        from .hemul import rescale_tables
        n = self.degree
        inv_last, gpsi, betas, _, _ = rescale_tables(self.moduli, n)
        self.power_of_last_tower_inv_psi = inv_last
        self.gammas_power_of_psi_no_last = gpsi
        self.betas = betas
        self.moduli_threshold = (self.moduli[-1] + 1) // 2
        self.last_tower_moduli = self.moduli[-1]
        self._rs_ntt = ntt.NTTCiphertextBarrettContext(self.moduli, {"r": self.r, "c": self.c})
        self._rs_keep = [np.ascontiguousarray(a) for a in (inv_last, gpsi, betas)]
        desc = _lib.RescaleDesc(self.r, self.c, self.num_moduli, self._rs_ntt.plan(),
                                *[a.ctypes.data for a in self._rs_keep])
        out = _lib.vp()
        _lib.check(_lib.lib().cross_rescale_plan_create(_lib.C.byref(desc), _lib.C.byref(out)),
                   "cross_rescale_plan_create")
        self._rs_plan = out
        self._rs_L = self.num_moduli
        self.mod_switch_params = True
        self.drop_last_modulus()

    def rescale(self):
        """ciphertext.py:267-303 as one kernel chain (cross_rescale)."""
        if not hasattr(self, "mod_switch_params"):
            self.modulus_switch_control_gen(degree_layout=self.degree_layout)
        x = _tensor.to_u32(self.ciphertext)
        L = self._rs_L
        if x.shape[-1] != L:
            raise ValueError(f"rescale expects {L} limbs, got {x.shape[-1]}")
        polys = x.numel() // (self.degree * L)
        out = _tensor.empty_u32((*x.shape[:-1], L - 1))
        L_ = _lib.lib()
        ws = _tensor.workspace(L_.cross_rescale_workspace_size(self._rs_plan, polys, _lib.LAYOUT_REFERENCE))
        _tensor.call("cross_rescale", self._rs_plan, x.data_ptr(), out.data_ptr(), polys, _lib.LAYOUT_REFERENCE,
                     ws.data_ptr(), ws.numel(), _lib.cuda_stream())
        self.ciphertext = out
        return out

    def __del__(self):
        if getattr(self, "_rs_plan", None) is not None and getattr(_lib, "_lib", None) is not None:
            _lib._lib.cross_rescale_plan_destroy(self._rs_plan)

    # -- HE kernels (ciphertext.py:309-519) ----------------------------------
    def ciphertext_mult(self):
        """ciphertext.py:309-324."""
        x = _tensor.to_u32(self.ciphertext)
        B, M = x.shape[0], x.shape[-1]
        n = x.numel() // (B * 4 * M)
        rest = tuple(x.shape[2:])
        o01 = _tensor.empty_u32((B, 2, *rest))
        o2 = _tensor.empty_u32((B, 1, *rest))
        _tensor.call("cross_tensor_product", self.ntt_ctx.ff_ctx.handle(), x.data_ptr(), o01.data_ptr(),
                     o2.data_ptr(), B, n, _lib.cuda_stream())
        return o01, o2

    def key_switch_control_gen(self, extend_moduli, dnum, evalkey_a, evalkey_b, perf_test=False,
                               selected_moduli=None, degree_layout=None):
        """ciphertext.py:329-453."""
        from .hemul import digits, psi_tables
        cur = list(self.moduli if selected_moduli is None else selected_moduli)
        dle = cur + list(extend_moduli)
        n = self.degree
        self.ks_params = {"drop_last_extend_moduli": dle}
        fwd, inv = psi_tables(dle, n)
        self.ks_params["drop_last_power_of_psi"] = fwd.T.reshape(*self.degree_layout, len(dle))
        alpha, parts, groups = digits(len(cur), dnum)
        self.ks_params.update(alpha=alpha, numPartQl=parts)
        sel = groups
        non = [[i for i in range(len(dle)) if i not in g] for g in sel]
        rest = []
        for s, ns in zip(sel, non):
            order = s + ns
            ri = [0] * len(order)
            for pos, v in enumerate(order):
                ri[v] = pos
            rest.append(ri)
        self.ks_params.update(select_tower_index_overall=sel, non_select_tower_index_overall=non, restore_indices=rest)
        inv_cur = np.stack([util.powers(pow(util.root_of_unity(2 * n, q), -1, q), n, q) for q in cur], -1)
        self.ks_params["power_of_inv_psi_arr_drop_last"] = inv_cur.reshape(1, 1, *self.degree_layout, len(cur))
        self.ks_params["ks_control_start_idx"] = len(self.bconv_indices_list)
        self.bconv_indices_list.extend(list(zip(sel, non)))
        self._create_bconv(dle)
        self.bconv.control_gen(self.bconv_indices_list)
        common = {"batch": self.batch, "num_elements": 2, "degree": n, "precision": self.precision,
                  "degree_layout": self.degree_layout}
        pc = {"r": self.r, "c": self.c, "finite_field_context": ff_context.BarrettContext}
        self.ks_params["ct_ks_parts"] = [Ciphertext({**common, "num_moduli": len(ns)}, {**pc, "moduli": [dle[i] for i in ns]})
                                         for ns in non]
        self.ks_params["ct_drop_last_extend"] = Ciphertext({**common, "num_moduli": len(dle)}, {**pc, "moduli": dle})
        ea = np.asarray(_tensor.to_numpy(evalkey_a)).astype(U32)
        eb = np.asarray(_tensor.to_numpy(evalkey_b)).astype(U32)
        K = len(extend_moduli)
        Lc = len(cur)
        cat = lambda e: np.ascontiguousarray(np.concatenate([e[..., :Lc], e[..., e.shape[-1] - K:]], -1).reshape(  # noqa: E731
            -1, *self.degree_layout, len(dle)))
        self.ks_params["evk_a_precomp"] = _tensor.torch().from_numpy(cat(ea)).to(_tensor.device())
        self.ks_params["evk_b_precomp"] = _tensor.torch().from_numpy(cat(eb)).to(_tensor.device())
        self.ks_params["ff_drop_last_extend"] = ff_context.BarrettContext(moduli=dle)

    def key_switch(self):
        """ciphertext.py:455-519; the inner product with the evaluation key
        (:506-518) is cross_ks_inner_product."""
        if not hasattr(self, "ks_params"):
            raise RuntimeError("Key switch parameters not initialized. Call key_switch_control_gen first.")
        t = _t()
        p = self.ks_params
        input_ntt = _tensor.to_u32(self.ciphertext)
        self.to_coeffs_form()
        self.modmul(p["power_of_inv_psi_arr_drop_last"])
        coef = self.ciphertext
        take = lambda x, idx: x.view(t.int32)[..., list(idx)].contiguous().view(t.uint32)  # noqa: E731
        exts = []
        for part in range(p["numPartQl"]):
            sel, ns = p["select_tower_index_overall"][part], p["non_select_tower_index_overall"][part]
            tw = np.ascontiguousarray(p["drop_last_power_of_psi"][..., ns])
            ev = self.bconv.basis_change_bat(take(coef, sel), control_index=p["ks_control_start_idx"] + part)
            cp = p["ct_ks_parts"][part]
            cp.ciphertext = ev
            cp.modmul(tw)
            cp.to_ntt_form()
            ext = t.cat([take(input_ntt, sel).view(t.int32), cp.ciphertext.view(t.int32)], -1)
            exts.append(ext[..., list(p["restore_indices"][part])].contiguous().view(t.uint32))
        # res0 = sum_j ext_j evk_b[j], res1 = sum_j ext_j evk_a[j] in uint64, then
        # mod_reduce of the concatenation (ciphertext.py:508-518)
        B = exts[0].shape[0]
        LT = exts[0].shape[-1]
        n = exts[0].numel() // (B * LT)
        result = _tensor.empty_u32((B, 2, *exts[0].shape[2:]))
        ptrs = (_lib.vp * len(exts))(*[e.data_ptr() for e in exts])
        _tensor.call("cross_ks_inner_product", p["ff_drop_last_extend"].handle(), ptrs, len(exts),
                     p["evk_a_precomp"].data_ptr(), p["evk_b_precomp"].data_ptr(), result.data_ptr(), B, n,
                     _lib.LAYOUT_REFERENCE, _lib.cuda_stream())
        cd = p["ct_drop_last_extend"]
        cd.set_batch_ciphertext(result)
        self.set_batch_ciphertext(cd.get_batch_ciphertext())
