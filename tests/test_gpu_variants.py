"""GPU parity of the Montgomery / Shoup / BAT-lazy variants (ntt_mm.py:432-658,
ntt_sm.py:116-494, bconv.py:261-390, finite_field.py:58-428): every device
result against the oracle (oracle/variants.py), bit-exact, and against the
reference's golden vectors."""
import numpy as np
import pytest

from oracle import cross_oracle as O
from oracle import variants as V
from tests.conftest import load_golden, rng_residues

pytestmark = pytest.mark.gpu
U32, U64 = np.uint32, np.uint64

NTT_CLASSES = {"montgomery": "NTTCiphertextMontgomeryContext", "shoup": "NTTCiphertextShoupContext",
               "bat_lazy": "NTTCiphertextBATLazyContext"}
BCONV_CLASSES = {"montgomery": "BConvMontgomery", "shoup": "BConvShoup", "bat_lazy": "BConvBATLazy"}


def _np(t):
    return t.cpu().numpy()


def _ctx(reduction, q, r, c):
    from cross_b200 import ntt_mm
    return getattr(ntt_mm, NTT_CLASSES[reduction])(q, {"r": r, "c": c})


def _golden_batch():
    g = load_golden("ntt_mm")
    r, c, b = g["r"], g["c"], g["test_batch"]
    coef = np.concatenate([np.array(g["coef_in"], np.uint64).T.reshape(1, r * c, -1)] * b, 0)
    ev = np.concatenate([np.array(g["eval_in"], U32).T.reshape(1, r * c, -1)] * b, 0)
    return g["moduli"], r, c, b, coef, ev


# ---------------------------------------------------------------------------
# multi-modulus NTT (ntt_mm.py)
# ---------------------------------------------------------------------------

def test_ntt_montgomery_golden():
    """ntt_mm_test.py:56-90."""
    from cross_b200 import finite_field, ntt_mm
    q, r, c, b, coef, ev = _golden_batch()
    ctx = ntt_mm.NTTCiphertextMontgomeryContext(q, {"r": r, "c": c,
                                                    "finite_field_context": finite_field.MontgomeryContext(q)})
    x = ctx.to_computation_format(coef).reshape(b, r, c, -1)
    y = ctx.ntt(x)
    np.testing.assert_array_equal(ctx.to_original_format(_np(y).reshape(b, r * c, -1)), ev)
    np.testing.assert_array_equal(ctx.to_original_format(_np(ctx.intt(y)).reshape(b, r * c, -1)), coef)


def test_ntt_shoup_golden():
    """ntt_mm_test.py:92-114."""
    from cross_b200 import finite_field, ntt_mm
    q, r, c, b, coef, ev = _golden_batch()
    ctx = ntt_mm.NTTCiphertextShoupContext(q, {"r": r, "c": c, "finite_field_context": finite_field.ShoupContext(q)})
    y = ctx.ntt(coef.astype(U32).reshape(b, r, c, -1))
    np.testing.assert_array_equal(ctx.to_original_format(y).reshape(b, r * c, -1), ev)
    np.testing.assert_array_equal(ctx.to_original_format(ctx.intt(y)).reshape(b, r * c, -1), coef)


def test_ntt_bat_lazy_golden():
    """ntt_mm_test.py:116-133 (exact equality)."""
    from cross_b200 import finite_field, ntt_mm
    q, r, c, b, coef, ev = _golden_batch()
    ctx = ntt_mm.NTTCiphertextBATLazyContext(q, {"r": r, "c": c,
                                                 "finite_field_context": finite_field.BarrettContext(q)})
    y = ctx.ntt(coef.astype(U32).reshape(b, r, c, -1))
    np.testing.assert_array_equal(_np(y).reshape(b, r * c, -1), ev)
    np.testing.assert_array_equal(_np(ctx.intt(y)).reshape(b, r * c, -1), coef)


# (r, c): dp4a CUDA-core path below 128, two-SM tensor-core kernel for 128..256,
# the one-SM kernel for a K extent of 512
SIZES = [(16, 16, 3, 2), (64, 64, 4, 3), (32, 128, 2, 2), (128, 128, 3, 2), (256, 256, 2, 2), (512, 128, 2, 1)]


@pytest.mark.parametrize("reduction", ["montgomery", "bat_lazy", "shoup"])
@pytest.mark.parametrize("r,c,L,B", SIZES)
def test_ntt_variant_vs_oracle(reduction, r, c, L, B):
    if reduction == "shoup" and r * c > 32768:
        pytest.skip("the uint64 oracle of the Shoup transform is slow above N = 2^15")
    n = r * c
    q = O.find_moduli_ntt(L, 28, 2 * n)
    x = rng_residues(np.random.default_rng(n + L), (B, r, c, L), q)
    ctx = _ctx(reduction, q, r, c)
    ref = V.NTTVariant(q, r, c, reduction)
    y = _np(ctx.ntt(x))
    yr = ref.ntt(x)
    np.testing.assert_array_equal(y, yr)
    np.testing.assert_array_equal(_np(ctx.intt(y)), ref.intt(yr))
    ctx.check_device()


@pytest.mark.parametrize("reduction", ["montgomery", "bat_lazy", "shoup"])
@pytest.mark.parametrize("r,c", [(64, 64), (128, 256)])
def test_ntt_variant_full_range_inputs(reduction, r, c):
    """Any uint32 input (not only residues) follows the reference's integer
    arithmetic: the byte contraction and the reductions wrap identically."""
    if reduction == "shoup" and r * c > 16384:
        pytest.skip("the uint64 oracle of the Shoup transform is slow above N = 2^14")
    q = O.find_moduli_ntt(2, 28, 2 * r * c)
    x = np.random.default_rng(7).integers(0, 2 ** 32, size=(2, r, c, 2), dtype=np.uint64).astype(U32)
    ctx = _ctx(reduction, q, r, c)
    ref = V.NTTVariant(q, r, c, reduction)
    np.testing.assert_array_equal(_np(ctx.ntt(x)), ref.ntt(x))
    np.testing.assert_array_equal(_np(ctx.intt(x)), ref.intt(x))


def test_ntt_variant_drop_last_modulus():
    """ntt_mm.py:412-419 on a Montgomery context: the dropped plan equals a
    fresh plan over the remaining moduli."""
    q = O.find_moduli_ntt(3, 28, 2 * 4096)
    x = rng_residues(np.random.default_rng(3), (2, 64, 64, 2), q[:2])
    ctx = _ctx("montgomery", q, 64, 64)
    ctx.drop_last_modulus()
    np.testing.assert_array_equal(_np(ctx.ntt(x)), V.NTTVariant(q[:2], 64, 64, "montgomery").ntt(x))


# ---------------------------------------------------------------------------
# single-modulus NTT (ntt_sm.py)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("reduction", ["barrett", "montgomery", "bat_lazy", "shoup"])
def test_ntt_single_modulus_golden(reduction):
    """ntt_sm_test.py:28-107."""
    from cross_b200 import finite_field as ff, ntt_sm
    g = load_golden("ntt_sm")
    q, r, c = g["modulus"], g["r"], g["c"]
    coef = np.array(g["coef_in"], np.uint64)
    ev = np.array(g["eval_in"], np.uint64)
    if reduction == "barrett":
        ctx = ntt_sm.NTTContextBase(q, {"r": r, "c": c, "finite_field_context": ff.BarrettContext(q)})
        y = ctx.ntt(coef.astype(U32).reshape(-1, r, c))
        np.testing.assert_array_equal(_np(y).reshape(-1), ev)
        np.testing.assert_array_equal(_np(ctx.intt(y))[0].reshape(-1), coef)
    elif reduction == "montgomery":
        ctx = ntt_sm.NTTContextBase(q, {"r": r, "c": c, "finite_field_context": ff.MontgomeryContext(q)})
        y = ctx.ntt(ctx.to_computation_format(coef).reshape(-1, r, c))
        np.testing.assert_array_equal(ctx.to_original_format(_np(y).astype(np.uint64).reshape(-1)), ev)
        np.testing.assert_array_equal(ctx.to_original_format(_np(ctx.intt(y)).astype(np.uint64))[0].reshape(-1), coef)
    elif reduction == "bat_lazy":
        ctx = ntt_sm.NTTBATLazyContext(q, {"r": r, "c": c, "finite_field_context": ff.BATLazyContext(q)})
        y = ctx.ntt(coef.astype(U32).reshape(-1, r, c))
        np.testing.assert_array_equal(_np(y).reshape(-1).astype(np.uint64) % q, ev)
        x = ctx.to_original_format(_np(ctx.intt(y)))
        np.testing.assert_array_equal(x[0].reshape(-1).astype(np.uint64) % q, coef)
    else:
        ctx = ntt_sm.NTTShoupContext(q, {"r": r, "c": c, "finite_field_context": ff.ShoupContext(q)})
        y = ctx.ntt(coef.astype(U32).reshape(r, c))
        np.testing.assert_array_equal(ctx.to_original_format(_np(y).reshape(-1)), ev)
        np.testing.assert_array_equal(ctx.to_original_format(_np(ctx.intt(y))).reshape(-1), coef)


@pytest.mark.parametrize("reduction", ["barrett", "montgomery", "bat_lazy"])
def test_ntt_single_modulus_vs_oracle(reduction):
    from cross_b200 import finite_field as ff, ntt_sm
    r, c = 128, 128
    q = O.find_moduli_ntt(1, 28, 2 * r * c)[0]
    x = rng_residues(np.random.default_rng(11), (3, r, c, 1), [q])[..., 0]
    if reduction == "barrett":
        ctx = ntt_sm.NTTBarrettContext(q, {"r": r, "c": c, "finite_field_context": ff.BarrettContext(q)})
        ref = O.NTTBarrett([q], r, c)
    elif reduction == "montgomery":
        ctx = ntt_sm.NTTMontgomeryContext(q, {"r": r, "c": c, "finite_field_context": ff.MontgomeryContext(q)})
        ref = V.NTTVariant([q], r, c, "montgomery")
    else:
        ctx = ntt_sm.NTTBATLazyContext(q, {"r": r, "c": c, "finite_field_context": ff.BATLazyContext(q)})
        ref = V.NTTVariant([q], r, c, "bat_lazy")
    y = _np(ctx.ntt(x))
    np.testing.assert_array_equal(y, ref.ntt(x[..., None])[..., 0])
    np.testing.assert_array_equal(_np(ctx.intt(y)), ref.intt(y[..., None])[..., 0])


# ---------------------------------------------------------------------------
# basis conversion (bconv.py)
# ---------------------------------------------------------------------------

def test_bconv_bat_lazy_golden():
    """bconv_test.py:53-76: uint64 output congruent to the reference result."""
    from cross_b200 import bconv
    g = load_golden("bconv")
    x = np.array(g["in_tower"], np.uint64).T
    ref = np.array(g["reference_result"], np.uint64).T
    bc = bconv.BConvBATLazy(g["original_moduli"] + g["target_moduli"])
    bc.control_gen([(list(range(2)), list(range(2, 7)))])
    out = _np(bc.basis_change(x))
    assert out.dtype == np.uint64
    diff = (out.astype(np.int64) - ref.astype(np.int64)) % np.array(g["target_moduli"])
    assert not diff.any()


@pytest.mark.parametrize("reduction,bat,sq,sp,n", [
    ("montgomery", True, 8, 23, 4096), ("montgomery", False, 4, 4, 4096), ("montgomery", False, 3, 1, 1024),
    ("montgomery", True, 24, 25, 256), ("shoup", False, 5, 9, 4096), ("shoup", False, 24, 8, 512),
    ("bat_lazy", True, 8, 23, 4096), ("bat_lazy", False, 8, 23, 4096), ("bat_lazy", True, 40, 12, 256),
    ("bat_lazy", False, 2, 5, 16)])
def test_bconv_variant_vs_oracle(reduction, bat, sq, sp, n):
    from cross_b200 import bconv
    ov = O.find_moduli_ntt(sq + sp, 28, 2 * max(n, 16))
    x = rng_residues(np.random.default_rng(sq * 100 + sp), (2, n, sq), ov[:sq])
    ctl = [(list(range(sq)), list(range(sq, sq + sp)))]
    dev = getattr(bconv, BCONV_CLASSES[reduction])(ov)
    dev.control_gen(ctl)
    ref = V.BConvVariant(ov, reduction)
    ref.control_gen(ctl)
    got = _np(dev.basis_change_bat(x) if bat else dev.basis_change(x))
    want = ref.basis_change_bat(x) if bat else ref.basis_change(x)
    assert got.dtype == want.dtype
    np.testing.assert_array_equal(got, want)


def test_bconv_variant_limb_major_layout():
    """cross_bconv_ex with the limb-major layout equals the reference layout."""
    from cross_b200 import _lib, bconv
    import torch
    sq, sp, n, B = 8, 23, 4096, 2
    ov = O.find_moduli_ntt(sq + sp, 28, 2 * n)
    x = rng_residues(np.random.default_rng(5), (B, n, sq), ov[:sq])
    for cls in ("BConvMontgomery", "BConvBATLazy"):
        dev = getattr(bconv, cls)(ov)
        dev.control_gen([(list(range(sq)), list(range(sq, sq + sp)))])
        ref = _np(dev.basis_change_bat(x))
        xl = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1))).cuda()
        yl = torch.empty((B, sp, n), dtype=torch.uint64 if cls == "BConvBATLazy" else torch.uint32, device="cuda")
        _lib.check(_lib.lib().cross_bconv_ex(dev.plan(0), 1, xl.data_ptr(), yl.data_ptr(), B, n,
                                             _lib.LAYOUT_LIMB_MAJOR, None), "cross_bconv_ex")
        np.testing.assert_array_equal(_np(yl), ref.transpose(0, 2, 1))


def test_bconv_variant_reference_errors():
    """The reference's undefined cases stay errors: Montgomery basis_change with
    size_q != size_p (a broadcast error in bconv.py:278-280) and Shoup's BAT
    path (bconv.py:244)."""
    from cross_b200 import bconv
    ov = O.find_moduli_ntt(7, 28, 64)
    x = rng_residues(np.random.default_rng(1), (1, 16, 2), ov[:2])
    m = bconv.BConvMontgomery(ov)
    m.control_gen([([0, 1], [2, 3, 4, 5, 6])])
    with pytest.raises(ValueError):
        m.basis_change(x)
    s = bconv.BConvShoup(ov)
    s.control_gen([([0, 1], [2, 3, 4, 5, 6])])
    with pytest.raises(TypeError):
        s.basis_change_bat(x)


# ---------------------------------------------------------------------------
# elementwise reductions (finite_field.py)
# ---------------------------------------------------------------------------

def test_variant_modular_reductions_vs_oracle():
    from cross_b200 import finite_field as ff
    q = O.find_moduli_ntt(5, 30, 64)
    rng = np.random.default_rng(9)
    z = rng.integers(0, 2 ** 63, size=(1000, 5), dtype=np.uint64) * np.uint64(2) + \
        rng.integers(0, 2, size=(1000, 5), dtype=np.uint64)
    zs = rng.integers(0, 2 ** 63, size=(1000, 5), dtype=np.uint64)
    np.testing.assert_array_equal(_np(ff.MontgomeryContext(q).modular_reduction(z)), V.Montgomery(q).reduce(z))
    np.testing.assert_array_equal(_np(ff.ShoupContext(q).modular_reduction(z, zs)), V.Shoup(q).reduce(z, zs))
    got = _np(ff.BATLazyContext(q).modular_reduction(z))
    assert got.dtype == np.uint64
    np.testing.assert_array_equal(got, V.BATLazy(q).reduce(z))
    # one modulus reduces every element of any shape (finite_field.py:408-411)
    z1 = z[:, :3].reshape(10, 100, 3)
    np.testing.assert_array_equal(_np(ff.MontgomeryContext(q[0]).modular_reduction(z1)),
                                  V.Montgomery(q[0]).reduce(z1))
