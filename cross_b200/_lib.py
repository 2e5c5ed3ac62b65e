"""ctypes binding of libcross_b200.so (the C ABI declared in include/cross_b200.h).

The library is built in-tree by ``cross_b200.build`` (or
``__graft_entry__.build()``).  There is no fallback: importing an operator
without the library, or without a CUDA device, raises.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcross_b200.so")

LAYOUT_REFERENCE = 0
LAYOUT_LIMB_MAJOR = 1
LAYOUT_LIMB_MAJOR_TRANSPOSED = 2   # cross_ntt only: coefficients (M, c, r), evaluations (M, r, c)

# cross_reduction (include/cross_b200.h): the finite_field.py context of a plan
REDUCTION_BARRETT = 0
REDUCTION_MONTGOMERY = 1
REDUCTION_SHOUP = 2
REDUCTION_BAT_LAZY = 3

_STATUS = {-1: ValueError, -2: RuntimeError, -3: NotImplementedError, -4: MemoryError, -5: TimeoutError}

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_int64
sz = C.c_size_t


class HemulDesc(C.Structure):
    _fields_ = [("r", i32), ("c", i32), ("L", i32), ("K", i32), ("dnum", i32),
                ("ntt_qp", vp), ("ntt_p", vp), ("ntt_p_limb_offset", i32),
                ("ks_bconv", C.POINTER(vp)), ("down_bconv", vp),
                ("inv_psi_last", vp), ("gamma_psi", vp), ("betas", vp), ("inv_psi_q", vp),
                ("psi_qp", vp), ("inv_psi_p", vp), ("p_inv_mod_q", vp)]


class RescaleDesc(C.Structure):
    _fields_ = [("r", i32), ("c", i32), ("L", i32), ("ntt_q", vp),
                ("inv_psi_last", vp), ("gamma_psi", vp), ("betas", vp)]


class HemulShardDesc(C.Structure):
    _fields_ = [("plan", vp), ("q_begin", i32), ("q_end", i32), ("p_begin", i32), ("p_end", i32),
                ("ks_bconv", C.POINTER(vp)), ("down_bconv", vp)]


class HerotDesc(C.Structure):
    _fields_ = [("r", i32), ("c", i32), ("L", i32), ("K", i32), ("dnum", i32),
                ("ntt_qp", vp), ("ks_bconv", C.POINTER(vp)), ("down_bconv", vp),
                ("inv_psi_q", vp), ("psi_qp", vp), ("inv_psi_p", vp), ("p_inv_mod_q", vp)]


_SIGS = {
    "cross_abi_version": (i32, []),
    "cross_last_error": (C.c_char_p, []),
    "cross_launch_count": (C.c_uint64, []),
    "cross_tc_i8_probe": (i32, [i32, i64, vp, vp, vp]),
    "cross_wait_selftest": (i32, [C.c_uint64, vp]),
    "cross_moduli_create": (i32, [i32, vp, vp, vp, vp, C.POINTER(vp)]),
    "cross_moduli_destroy": (i32, [vp]),
    "cross_mod_reduce": (i32, [vp, vp, i32, vp, i64, vp]),
    "cross_mod_reduce_ex": (i32, [vp, i32, vp, vp, vp, i64, vp]),
    "cross_modmul": (i32, [vp, vp, i32, vp, i32, i64, vp, i64, vp]),
    "cross_tensor_product": (i32, [vp, vp, vp, vp, i64, i64, vp]),
    "cross_add_mod": (i32, [vp, vp, vp, vp, i64, i64, vp]),
    "cross_ks_inner_product": (i32, [vp, C.POINTER(vp), i32, vp, vp, vp, i64, i64, i32, vp]),
    "cross_moddown_sub_mul": (i32, [vp, vp, vp, vp, vp, vp, i64, vp]),
    "cross_rescale_lift": (i32, [vp, vp, C.c_uint32, vp, vp, i64, i64, i32, vp]),
    "cross_automorphism": (i32, [vp, vp, vp, i64, i64, i32, vp]),
    "cross_to_limb_major": (i32, [vp, vp, i64, i64, i32, vp]),
    "cross_to_reference": (i32, [vp, vp, i64, i64, i32, vp]),
    "cross_ntt_plan_create": (i32, [vp, i32, i32, vp, vp, vp, vp, vp, vp, C.POINTER(vp)]),
    "cross_ntt_plan_create_ex": (i32, [vp, i32, i32, i32, vp, vp, vp, vp, vp, vp, C.POINTER(vp)]),
    "cross_ntt_plan_create_shoup": (i32, [vp, i32, i32, C.POINTER(vp), C.POINTER(vp)]),
    "cross_ntt_plan_reduction": (i32, [vp]),
    "cross_ntt_plan_destroy": (i32, [vp]),
    "cross_ntt_workspace_size": (sz, [vp, i64, i32]),
    "cross_ntt": (i32, [vp, i32, vp, vp, i64, i32, vp, sz, vp]),
    "cross_ntt_noalloc": (i32, [vp, i32, vp, vp, i64, vp]),
    "cross_ntt_plan_check": (i32, [vp]),
    "cross_bconv_plan_create": (i32, [vp, vp, vp, vp, vp, C.POINTER(vp)]),
    "cross_bconv_plan_create_ex": (i32, [vp, vp, i32, vp, vp, vp, vp, vp, C.POINTER(vp)]),
    "cross_bconv_output_bytes": (i32, [vp]),
    "cross_bconv_ex": (i32, [vp, i32, vp, vp, i64, i64, i32, vp]),
    "cross_bconv_plan_destroy": (i32, [vp]),
    "cross_bconv_plan_check": (i32, [vp]),
    "cross_bconv": (i32, [vp, i32, vp, vp, i64, i64, i32, vp]),
    "cross_fft_special": (i32, [vp, i64, i32, i32, vp, vp, i32, C.c_double, vp]),
    "cross_ckks_max_abs_scaled": (i32, [vp, i64, C.c_double, vp, vp]),
    "cross_ckks_quantize": (i32, [vp, vp, i32, C.c_double, i32, vp, vp, vp]),
    "cross_mul_reduce_lm": (i32, [vp, vp, vp, vp, i64, vp]),
    "cross_rns_from_signed": (i32, [vp, vp, i64, vp, vp]),
    "cross_ckks_decrypt_sum": (i32, [vp, vp, i32, vp, vp, i64, vp]),
    "cross_ckks_encrypt": (i32, [vp, vp, vp, vp, vp, vp, vp, C.c_uint64, vp, vp, i64, vp]),
    "cross_pke_b": (i32, [vp, vp, vp, vp, C.c_uint64, vp, i64, vp]),
    "cross_mod_switch_lift": (i32, [vp, i64, C.c_uint32, vp, vp, vp]),
    "cross_ks_key_b": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, C.c_uint64, vp, i64, vp]),
    "cross_crt_combine": (i32, [vp, vp, i64, vp, vp, vp, i32, vp, vp]),
    "cross_ckks_decode_scale": (i32, [vp, i32, vp, vp, C.c_double, i32, i32, vp, vp, vp]),
    "cross_ckks_decode_stddev": (i32, [vp, i32, vp, vp]),
    "cross_ckks_decode_combine": (i32, [vp, vp, i32, C.c_double, vp]),
    "cross_rescale_plan_create": (i32, [C.POINTER(RescaleDesc), C.POINTER(vp)]),
    "cross_rescale_plan_destroy": (i32, [vp]),
    "cross_rescale_workspace_size": (sz, [vp, i64, i32]),
    "cross_rescale": (i32, [vp, vp, vp, i64, i32, vp, sz, vp]),
    "cross_hemul_plan_create": (i32, [C.POINTER(HemulDesc), C.POINTER(vp)]),
    "cross_hemul_set_keys": (i32, [vp, vp, vp, i32]),
    "cross_hemul_plan_destroy": (i32, [vp]),
    "cross_hemul_workspace_size": (sz, [vp, i64, i32]),
    "cross_hemul": (i32, [vp, vp, vp, i64, i32, vp, sz, vp]),
    "cross_hemul_shard_create": (i32, [C.POINTER(HemulShardDesc), C.POINTER(vp)]),
    "cross_hemul_shard_destroy": (i32, [vp]),
    "cross_hemul_shard_workspace_size": (sz, [vp, i64]),
    "cross_hemul_shard_modup_input": (i32, [vp, vp, i64, vp, vp, sz, vp]),
    "cross_hemul_shard_keyswitch": (i32, [vp, vp, i64, vp, vp, sz, vp]),
    "cross_hemul_shard_moddown": (i32, [vp, vp, i64, vp, vp, sz, vp]),
    "cross_herot_plan_create": (i32, [C.POINTER(HerotDesc), C.POINTER(vp)]),
    "cross_herot_set_keys": (i32, [vp, vp, vp, vp]),
    "cross_herot_plan_destroy": (i32, [vp]),
    "cross_herot_workspace_size": (sz, [vp, i64, i32]),
    "cross_herot": (i32, [vp, vp, vp, i64, i32, vp, sz, vp]),
}

_lib = None


def lib():
    """Load libcross_b200.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m cross_b200.build` "
                "(there is no CPU fallback for the CROSS operators)")
        h = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _lib = h
    return _lib


def exported_symbols():
    return list(_SIGS)


def check(rc: int, what: str = ""):
    """Raise the reference-style Python exception for a nonzero status."""
    if rc != 0:
        msg = lib().cross_last_error().decode(errors="replace")
        raise _STATUS.get(rc, RuntimeError)(f"{what}: {msg}" if what else msg)


def ptr(a) -> int:
    """Raw device/host address of a torch tensor or numpy array."""
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


def cuda_stream():
    import torch
    return torch.cuda.current_stream().cuda_stream
