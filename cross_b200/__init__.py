"""cross_b200: B200-native (sm_100a) CKKS hot path of EfficientPPML/CROSS.

Drop-in for the jaxite_word operator API:

    finite_field  BarrettContext, MontgomeryContext, ShoupContext, BATLazyContext
    ntt_mm        NTTCiphertext{Barrett,Montgomery,Shoup,BATLazy}Context(moduli, {"r", "c", ...}).ntt / .intt
    ntt_sm        NTT{Barrett,Montgomery,BATLazy,Shoup}Context(q, {"r", "c", ...}): one modulus
    bconv         BConv{Barrett,Montgomery,Shoup,BATLazy}(overall).control_gen(...).basis_change_bat / .basis_change
    ciphertext    Ciphertext(shapes, parameters) with rescale / key_switch / ...
    hemul         HEMul(batch, r, c, dnum, 1, Q, P).control_gen / setup_relinearization / mul
    herot         HERot(r, c, dnum, Q, P).control_gen / setup_rotate / rotate
    add           jax_add / vmap_add
    util          parameter math

Every operator runs hand-written CUDA kernels of libcross_b200.so through
the C ABI of include/cross_b200.h; tensors are CUDA torch tensors (numpy
inputs are copied to the device).
"""
from ._lib import LAYOUT_LIMB_MAJOR, LAYOUT_REFERENCE, LIB_PATH, lib  # noqa: F401

__version__ = "0.1.0"
