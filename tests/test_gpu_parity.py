"""GPU parity: every operator through the C ABI against the CPU oracle
(bit-exact) and against the reference's golden vectors."""
import numpy as np
import pytest

from oracle import cross_oracle as O
from tests.conftest import load_golden, rng_residues

pytestmark = pytest.mark.gpu
U32 = np.uint32
parse = O.parse_ciphertext_string


def _np(t):
    return t.cpu().numpy()


# ---------------------------------------------------------------------------
# NTT
# ---------------------------------------------------------------------------

def test_ntt_golden():
    """ntt_mm_test.py:33-54."""
    from cross_b200 import ntt_mm, finite_field
    g = load_golden("ntt_mm")
    r, c, b = g["r"], g["c"], 2
    coef = np.concatenate([np.array(g["coef_in"], np.uint64).T.reshape(1, r * c, -1)] * b, 0).astype(U32)
    ev = np.concatenate([np.array(g["eval_in"], U32).T.reshape(1, r * c, -1)] * b, 0)
    ctx = ntt_mm.NTTCiphertextBarrettContext(g["moduli"], {"r": r, "c": c,
                                                           "finite_field_context": finite_field.BarrettContext(g["moduli"])})
    out = ctx.ntt(coef.reshape(b, r, c, -1))
    np.testing.assert_array_equal(_np(out).reshape(b, r * c, -1), ev)
    np.testing.assert_array_equal(_np(ctx.intt(out)).reshape(b, r * c, -1), coef)


@pytest.mark.parametrize("n,r,c,limbs,batch", [(4096, 64, 64, 8, 16), (4096, 32, 128, 3, 2), (1024, 32, 32, 5, 3),
                                               (65536, 256, 256, 4, 2), (65536, 128, 512, 2, 1),
                                               (16384, 128, 128, 3, 3), (32768, 128, 256, 2, 1)])
def test_ntt_intt_vs_oracle(n, r, c, limbs, batch):
    from cross_b200 import ntt_mm
    q = O.find_moduli_ntt(limbs, 28, 2 * n)
    x = rng_residues(np.random.default_rng(n + limbs), (batch, r, c, limbs), q)
    ctx = ntt_mm.NTTCiphertextBarrettContext(q, {"r": r, "c": c})
    ref = O.NTTBarrett(q, r, c)
    y = ctx.ntt(x)
    yr = ref.ntt(x)
    np.testing.assert_array_equal(_np(y), yr)
    np.testing.assert_array_equal(_np(ctx.intt(y)), ref.intt(yr))


def test_tensor_core_path_matches_cuda_core_path(monkeypatch):
    """The tcgen05 contraction (r, c multiples of 128) and the dp4a contraction
    are both exact: their NTT / INTT outputs must be identical."""
    from cross_b200 import ntt_mm
    n, L, B = 65536, 8, 6
    q = O.find_moduli_ntt(L, 28, 2 * n)
    x = rng_residues(np.random.default_rng(42), (B, 256, 256, L), q)
    tc = ntt_mm.NTTCiphertextBarrettContext(q, {"r": 256, "c": 256})
    y_tc = _np(tc.ntt(x))
    z_tc = _np(tc.intt(y_tc))
    tc.check_device()
    monkeypatch.setenv("CROSS_B200_DISABLE_TC", "1")
    cc = ntt_mm.NTTCiphertextBarrettContext(q, {"r": 256, "c": 256})
    np.testing.assert_array_equal(y_tc, _np(cc.ntt(x)))
    np.testing.assert_array_equal(z_tc, _np(cc.intt(y_tc)))


@pytest.mark.parametrize("B,L", [(16, 8), (3, 5), (300, 1), (40, 8)])
def test_ntt64_single_launch_vs_oracle(monkeypatch, B, L):
    """N = 2^12 (64 x 64): the single-launch tensor-core transform (one
    limb-polynomial at a time per CTA, its rows in both halves of the 128-row
    tiles) against the oracle and against the CUDA-core path, for the
    benchmark shape (16 x 8), an odd batch (3 x 5), CTAs that walk several
    polynomials of one limb (300 x 1: more items than CTAs) and CTAs whose
    items cross a limb boundary (40 x 8); limb-major through the C ABI, in
    place, and in the reference layout through the context."""
    import torch
    from cross_b200 import _lib, ntt_mm
    n = 4096
    q = O.find_moduli_ntt(L, 28, 2 * n)
    x = rng_residues(np.random.default_rng(B * 10 + L), (B, 64, 64, L), q)
    ref = O.NTTBarrett(q, 64, 64)
    yr = ref.ntt(x)
    ctx = ntt_mm.NTTCiphertextBarrettContext(q, {"r": 64, "c": 64})
    np.testing.assert_array_equal(_np(ctx.ntt(x)), yr)
    np.testing.assert_array_equal(_np(ctx.intt(yr)), ref.intt(yr))
    lib = _lib.lib()
    xl = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 3, 1, 2))).cuda()     # (B, L, 64, 64)
    ws = torch.empty(lib.cross_ntt_workspace_size(ctx.plan(), B, _lib.LAYOUT_LIMB_MAJOR), dtype=torch.uint8,
                     device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.cross_ntt(ctx.plan(), 0, xl.data_ptr(), xl.data_ptr(), B, _lib.LAYOUT_LIMB_MAJOR, ws.data_ptr(),
                             ws.numel(), st), "cross_ntt")
    np.testing.assert_array_equal(_np(xl), yr.transpose(0, 3, 1, 2))
    _lib.check(lib.cross_ntt(ctx.plan(), 1, xl.data_ptr(), xl.data_ptr(), B, _lib.LAYOUT_LIMB_MAJOR, ws.data_ptr(),
                             ws.numel(), st), "cross_ntt")
    np.testing.assert_array_equal(_np(xl), ref.intt(yr).transpose(0, 3, 1, 2))
    ctx.check_device()
    monkeypatch.setenv("CROSS_B200_DISABLE_TC", "1")
    cc = ntt_mm.NTTCiphertextBarrettContext(q, {"r": 64, "c": 64})
    np.testing.assert_array_equal(_np(cc.ntt(x)), yr)


@pytest.mark.parametrize("r,c,L,B", [(256, 256, 5, 5), (128, 128, 3, 5), (128, 256, 4, 3), (512, 128, 2, 3)])
def test_two_sm_kernel_matches_one_sm_kernel(monkeypatch, r, c, L, B):
    """The cta_group::2 contraction (B half resident per CTA, K extent <= 256
    words) and the one-SM contraction give identical NTT / INTT outputs, for
    even and odd numbers of 128-row blocks (odd: the last pair's second CTA
    repeats the first CTA's rows and stores nothing)."""
    from cross_b200 import ntt_mm
    n = r * c
    q = O.find_moduli_ntt(L, 28, 2 * n)
    x = rng_residues(np.random.default_rng(r + c + L), (B, r, c, L), q)
    two = ntt_mm.NTTCiphertextBarrettContext(q, {"r": r, "c": c})
    y2 = _np(two.ntt(x))
    z2 = _np(two.intt(y2))
    two.check_device()
    monkeypatch.setenv("CROSS_B200_TC_1SM", "1")
    one = ntt_mm.NTTCiphertextBarrettContext(q, {"r": r, "c": c})
    np.testing.assert_array_equal(y2, _np(one.ntt(x)))
    np.testing.assert_array_equal(z2, _np(one.intt(y2)))
    one.check_device()
    assert not ((z2.astype(np.int64) - x) % np.array(q, np.int64)).any()


@pytest.mark.parametrize("r,c", [(256, 256), (64, 64), (128, 512)])
def test_ntt_transposed_coefficient_layout(r, c):
    """CROSS_LAYOUT_LIMB_MAJOR_TRANSPOSED: ntt of the transposed coefficients
    equals ntt of the natural ones, intt returns transposed coefficients."""
    import torch
    from cross_b200 import ntt_mm, _lib
    n, L, B = r * c, 3, 2
    q = O.find_moduli_ntt(L, 28, 2 * n)
    x = np.ascontiguousarray(rng_residues(np.random.default_rng(r + c), (B, r, c, L), q).transpose(0, 3, 1, 2))
    ctx = ntt_mm.NTTCiphertextBarrettContext(q, {"r": r, "c": c})
    lib = _lib.lib()

    def run(inv, src, layout):
        d = torch.from_numpy(np.ascontiguousarray(src)).cuda()
        o = torch.empty_like(d)
        ws = torch.empty(lib.cross_ntt_workspace_size(ctx.plan(), B, layout), dtype=torch.uint8, device="cuda")
        _lib.check(lib.cross_ntt(ctx.plan(), inv, d.data_ptr(), o.data_ptr(), B, layout, ws.data_ptr(), ws.numel(),
                                 None), "cross_ntt")
        return _np(o)

    xt = x.transpose(0, 1, 3, 2)
    y = run(0, x, _lib.LAYOUT_LIMB_MAJOR)
    np.testing.assert_array_equal(run(0, xt, _lib.LAYOUT_LIMB_MAJOR_TRANSPOSED).reshape(y.shape), y)
    z = run(1, y, _lib.LAYOUT_LIMB_MAJOR)
    np.testing.assert_array_equal(run(1, y, _lib.LAYOUT_LIMB_MAJOR_TRANSPOSED).reshape(xt.shape),
                                  z.transpose(0, 1, 3, 2))


def test_ntt_round_trip_and_linearity_full_size():
    """Size-independent properties at N = 2^16, 24 limbs: INTT(NTT(x)) == x mod q
    and NTT(x + y) == NTT(x) + NTT(y) mod q."""
    from cross_b200 import ntt_mm
    n, L, B = 65536, 24, 2
    q = O.find_moduli_ntt(L, 28, 2 * n)
    qa = np.array(q, np.int64)
    rng = np.random.default_rng(7)
    x = rng_residues(rng, (B, 256, 256, L), q)
    y = rng_residues(rng, (B, 256, 256, L), q)
    ctx = ntt_mm.NTTCiphertextBarrettContext(q, {"r": 256, "c": 256})
    fx, fy = _np(ctx.ntt(x)).astype(np.int64), _np(ctx.ntt(y)).astype(np.int64)
    back = _np(ctx.intt(ctx.ntt(x))).astype(np.int64)
    assert not ((back - x) % qa).any()
    s = ((x.astype(np.int64) + y) % qa).astype(U32)
    fs = _np(ctx.ntt(s)).astype(np.int64)
    assert not ((fs - fx - fy) % qa).any()


# ---------------------------------------------------------------------------
# BConv
# ---------------------------------------------------------------------------

def test_bconv_golden():
    """bconv_test.py:28-48 (+ BAT congruence)."""
    from cross_b200 import bconv
    g = load_golden("bconv")
    x = np.array(g["in_tower"], np.uint64).T.astype(U32)
    ref = np.array(g["reference_result"], np.uint64).T
    b = bconv.BConvBarrett(g["original_moduli"] + g["target_moduli"])
    b.control_gen([(list(range(2)), list(range(2, 7)))])
    np.testing.assert_array_equal(_np(b.basis_change(x)), ref)
    o = O.BConvBarrett(g["original_moduli"] + g["target_moduli"])
    o.control_gen([(list(range(2)), list(range(2, 7)))])
    np.testing.assert_array_equal(_np(b.basis_change_bat(x)), o.basis_change_bat(x))


def test_bconv_small_primes():
    """bconv_test.py:78-120."""
    from cross_b200 import bconv
    b = bconv.BConvBarrett([17, 19, 23, 29])
    b.control_gen([([0], [2]), ([1], [3])])
    assert int(_np(b.basis_change(np.array([[[15]]], U32), 0))[0, 0, 0]) == 15
    assert int(_np(b.basis_change(np.array([[[20]]], U32), 1))[0, 0, 0]) == 1
    assert int(_np(b.basis_change(np.array([[[20]]], U32), 0))[0, 0, 0]) == 3


@pytest.mark.parametrize("n,sq,sp,batch", [(4096, 24, 25, 2), (256, 8, 23, 3), (65536, 24, 25, 1)])
def test_bconv_vs_oracle(n, sq, sp, batch):
    from cross_b200 import bconv
    ov = O.find_moduli_ntt(sq + sp, 28, 2 * n)
    x = rng_residues(np.random.default_rng(sq), (batch, n, sq), ov[:sq])
    b = bconv.BConvBarrett(ov)
    b.control_gen([(list(range(sq)), list(range(sq, sq + sp)))])
    o = O.BConvBarrett(ov)
    o.control_gen([(list(range(sq)), list(range(sq, sq + sp)))])
    np.testing.assert_array_equal(_np(b.basis_change_bat(x)), o.basis_change_bat(x))
    np.testing.assert_array_equal(_np(b.basis_change(x)), o.basis_change(x))


@pytest.mark.parametrize("n,sq,sp,batch", [(4096, 8, 23, 3), (1024, 7, 24, 2), (128, 8, 8, 5), (4096, 16, 40, 2),
                                           (256, 3, 5, 4), (1024, 32, 64, 1), (65536, 8, 23, 2)])
def test_bconv_limb_major_tensor_core(monkeypatch, n, sq, sp, batch):
    """Limb-major BConv with contiguous coefficients (n % 128 == 0) runs the
    tcgen05 kernel: bit-exact against the oracle and the dp4a kernel."""
    import torch
    from cross_b200 import bconv, _lib
    ov = O.find_moduli_ntt(sq + sp, 28, 2 * n)
    x = rng_residues(np.random.default_rng(n + sq + sp), (batch, n, sq), ov[:sq])
    o = O.BConvBarrett(ov)
    o.control_gen([(list(range(sq)), list(range(sq, sq + sp)))])
    want = o.basis_change_bat(x).transpose(0, 2, 1)
    xl = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1))).cuda()

    def run():
        b = bconv.BConvBarrett(ov)
        b.control_gen([(list(range(sq)), list(range(sq, sq + sp)))])
        out = torch.empty((batch, sp, n), dtype=xl.dtype, device="cuda")
        _lib.check(_lib.lib().cross_bconv(b.plan(0), 1, xl.data_ptr(), out.data_ptr(), batch, n,
                                          _lib.LAYOUT_LIMB_MAJOR, None), "cross_bconv")
        got = _np(out)
        b.check_device()
        return got

    np.testing.assert_array_equal(run(), want)
    monkeypatch.setenv("CROSS_B200_DISABLE_TC", "1")
    np.testing.assert_array_equal(run(), want)


# ---------------------------------------------------------------------------
# Elementwise
# ---------------------------------------------------------------------------

def test_elementwise_vs_oracle():
    from cross_b200 import add, finite_field
    from cross_b200.ciphertext import Ciphertext
    q = O.find_moduli_ntt(5, 30, 2 * 64)
    rng = np.random.default_rng(3)
    z = rng.integers(0, 2 ** 64 - 1, size=(7, 5), dtype=np.uint64)
    ff = finite_field.BarrettContext(q)
    np.testing.assert_array_equal(_np(ff.modular_reduction(z)), O.Barrett(q).reduce(z))
    a = rng_residues(rng, (3, 64, 5), q).transpose(0, 2, 1).copy()    # (E, L, N) as add.py
    b = rng_residues(rng, (3, 64, 5), q).transpose(0, 2, 1).copy()
    a[0, 0, :4] = np.uint32(q[0]) - b[0, 0, :4]  # sums equal to q stay (add.py uses >)
    np.testing.assert_array_equal(_np(add.jax_add(a, b, np.array(q))), O.jax_add(a, b, q))
    ct = Ciphertext({"batch": 2, "num_elements": 4, "degree": 64, "num_moduli": 5, "precision": 32,
                     "degree_layout": (8, 8)}, {"moduli": q})
    x = rng_residues(rng, (2, 4, 8, 8, 5), q)
    ct.set_batch_ciphertext(x)
    m01, m2 = ct.ciphertext_mult()
    r01, r2 = O.ciphertext_mult(x, O.Barrett(q))
    np.testing.assert_array_equal(_np(m01), r01)
    np.testing.assert_array_equal(_np(m2), r2)
    tab = rng_residues(rng, (8, 8, 5), q).astype(np.uint64)
    ct.set_batch_ciphertext(x)
    ct.modmul(tab)
    np.testing.assert_array_equal(_np(ct.ciphertext), O._modmul(O.Barrett(q), x, tab))


# ---------------------------------------------------------------------------
# Ciphertext: rescale and key switch
# ---------------------------------------------------------------------------

def test_rescale_golden():
    """rescale_test.py:49-87."""
    from cross_b200.ciphertext import Ciphertext
    g = load_golden("rescale")
    inc = np.array(parse(g["in_ciphertexts_str"])[0], U32)
    fin = np.array(parse(g["final_result_str"])[0], U32)
    for b in (1, 2):
        x = np.tile(np.transpose(inc, (0, 2, 1))[None], (b, 1, 1, 1)).reshape(b, 2, 4, 4, 5)
        ct = Ciphertext({"batch": b, "num_elements": 2, "degree": 16, "num_moduli": 5, "precision": 32},
                        {"moduli": g["q_towers"], "r": 4, "c": 4})
        ct.modulus_switch_control_gen(degree_layout=(4, 4))
        ct.set_batch_ciphertext(x)
        ct.rescale()
        res = _np(ct.get_batch_ciphertext()).reshape(b, 2, 16, 4)
        for i in range(b):
            np.testing.assert_array_equal(np.transpose(res[i], (0, 2, 1)), fin)


def test_rescale_vs_oracle_n4096():
    from cross_b200.ciphertext import Ciphertext
    q = O.find_moduli_ntt(6, 28, 2 * 4096)
    x = rng_residues(np.random.default_rng(11), (2, 2, 64, 64, 6), q)
    ct = Ciphertext({"batch": 2, "num_elements": 2, "degree": 4096, "num_moduli": 6, "precision": 32,
                     "degree_layout": (64, 64)}, {"moduli": q})
    ct.modulus_switch_control_gen(degree_layout=(64, 64))
    ct.set_batch_ciphertext(x)
    np.testing.assert_array_equal(_np(ct.rescale()), O.RescalePlan(q, 64, 64).rescale(x))


def test_key_switch_vs_oracle():
    from cross_b200.ciphertext import Ciphertext
    from cross_b200 import finite_field
    n, L, K, dnum = 256, 5, 2, 3
    q = O.find_moduli_ntt(L + K, 28, 2 * n)
    rng = np.random.default_rng(5)
    evk_a = rng_residues(rng, (dnum, n, L + K), q)
    evk_b = rng_residues(rng, (dnum, n, L + K), q)
    x = rng_residues(rng, (2, 1, 16, 16, L), q[:L])
    ct = Ciphertext({"batch": 2, "num_elements": 1, "degree": n, "num_moduli": L, "precision": 32,
                     "degree_layout": (16, 16)},
                    {"moduli": q[:L], "r": 16, "c": 16, "finite_field_context": finite_field.BarrettContext})
    ct.key_switch_control_gen(q[L:], dnum, evk_a, evk_b)
    ct.set_batch_ciphertext(x)
    ct.key_switch()
    ref = O.KeySwitchPlan(q[:L], q[L:], dnum, evk_a, evk_b, 16, 16).key_switch(x)
    np.testing.assert_array_equal(_np(ct.get_batch_ciphertext()), ref)


def _lm(a):
    """(..., n, M) -> (..., M, n)."""
    return np.ascontiguousarray(np.swapaxes(a, -1, -2))


@pytest.mark.parametrize("layout,full", [(0, False), (1, False), (0, True)])
def test_ks_inner_product_entry_point(layout, full):
    """cross_ks_inner_product (ciphertext.py:506-518): Barrett of the uint64
    sums of digit-wise products; full-range words make the sums wrap as the
    reference's uint64 arithmetic does."""
    import torch
    from cross_b200 import _lib, finite_field
    n, M, dnum, B = 1024, 7, 5, 2
    q = O.find_moduli_ntt(M, 28, 2 * n)
    rng = np.random.default_rng(31 + layout + 2 * full)
    draw = (lambda shape: rng.integers(0, 2 ** 32, size=shape, dtype=np.uint64).astype(U32)) if full else \
        (lambda shape: rng_residues(rng, shape, q))
    ext = [draw((B, n, M)) for _ in range(dnum)]
    ea, eb = draw((dnum, n, M)), draw((dnum, n, M))
    bar = O.Barrett(q)
    s0 = sum(e.astype(np.uint64) * eb[j].astype(np.uint64) for j, e in enumerate(ext))
    s1 = sum(e.astype(np.uint64) * ea[j].astype(np.uint64) for j, e in enumerate(ext))
    want = np.stack([bar.reduce(s0), bar.reduce(s1)], 1)                          # (B, 2, n, M)
    if layout == _lib.LAYOUT_LIMB_MAJOR:
        ext, ea, eb, want = [_lm(e) for e in ext], _lm(ea), _lm(eb), _lm(want)
    dev = [torch.from_numpy(e).cuda() for e in ext]
    a, b = torch.from_numpy(ea).cuda(), torch.from_numpy(eb).cuda()
    out = torch.empty(want.shape, dtype=torch.uint32, device="cuda")
    ptrs = (_lib.vp * dnum)(*[d.data_ptr() for d in dev])
    ff = finite_field.BarrettContext(q)
    _lib.check(_lib.lib().cross_ks_inner_product(ff.handle(), ptrs, dnum, a.data_ptr(), b.data_ptr(), out.data_ptr(),
                                                 B, n, layout, None), "cross_ks_inner_product")
    np.testing.assert_array_equal(_np(out), want)


@pytest.mark.parametrize("with_base", [False, True])
def test_moddown_sub_mul_entry_point(with_base):
    """cross_moddown_sub_mul (hemul.py:199-207, 214-215): the uint32 subtract,
    the P^-1 modmul and the final add with its >= q correction."""
    import torch
    from cross_b200 import _lib, finite_field
    rows, M = 4096, 6
    q = O.find_moduli_ntt(M, 28, 2 * 1024)
    rng = np.random.default_rng(41 + with_base)
    x = (rng.integers(0, 2 ** 31, size=(rows, M), dtype=np.uint64)).astype(U32)
    y = rng_residues(rng, (rows, M), q)
    pinv = rng_residues(rng, (1, M), q)[0]
    base = rng_residues(rng, (rows, M), q)
    qa = np.array(q, U32)
    sub = np.where(x < y, x + qa - y, x - y)
    t = O.Barrett(q).reduce(sub.astype(np.uint64) * pinv.astype(np.uint64)).astype(U32)
    want = np.where(base + t >= qa, base + t - qa, base + t) if with_base else t
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    out = torch.empty((rows, M), dtype=torch.uint32, device="cuda")
    xd, yd, pd, bd = d(x), d(y), d(pinv), d(base)
    ff = finite_field.BarrettContext(q)          # owns the modulus set for the whole call
    _lib.check(_lib.lib().cross_moddown_sub_mul(ff.handle(), xd.data_ptr(), yd.data_ptr(), pd.data_ptr(),
                                                bd.data_ptr() if with_base else None, out.data_ptr(), rows, None),
               "cross_moddown_sub_mul")
    np.testing.assert_array_equal(_np(out), want)


@pytest.mark.parametrize("layout", [0, 1])
def test_rescale_lift_entry_point(layout):
    """cross_rescale_lift (ciphertext.py:279-295): the centred lift of the last
    limb (lazy Barrett values below 2 q_last) into every remaining modulus times
    gamma_i psi_i^t."""
    import torch
    from cross_b200 import _lib, finite_field
    n, L, polys = 2048, 6, 3
    mods = O.find_moduli_ntt(L, 28, 2 * n)
    qs, ql = mods[:-1], mods[-1]
    rng = np.random.default_rng(51 + layout)
    last = (rng.integers(0, 2 * ql, size=(polys, n), dtype=np.uint64)).astype(U32)
    gpsi = rng_residues(rng, (n, L - 1), qs)
    lifted = np.where(last[..., None] < (ql + 1) // 2, last[..., None].astype(np.uint64),
                      np.array(qs, np.uint64) - np.uint64(ql) + last[..., None].astype(np.uint64))
    want = O.Barrett(qs).reduce(lifted * gpsi.astype(np.uint64))                     # (polys, n, L - 1)
    if layout == _lib.LAYOUT_LIMB_MAJOR:
        gpsi, want = _lm(gpsi), _lm(want)
    out = torch.empty(want.shape, dtype=torch.uint32, device="cuda")
    ld, gd = torch.from_numpy(last).cuda(), torch.from_numpy(np.ascontiguousarray(gpsi)).cuda()
    ff = finite_field.BarrettContext(qs)         # owns the modulus set for the whole call
    _lib.check(_lib.lib().cross_rescale_lift(ff.handle(), ld.data_ptr(), ql, gd.data_ptr(), out.data_ptr(), polys,
                                             n, layout, None), "cross_rescale_lift")
    np.testing.assert_array_equal(_np(out), want)


# ---------------------------------------------------------------------------
# HE-Mult / HE-Rotate
# ---------------------------------------------------------------------------

def test_hemul_golden_e2e():
    """hemul_test.py:64-140: bit-exact HE-Mult, decrypt bit-exact, decode within
    an absolute tolerance of 1.5e-3 (decimal=3)."""
    from cross_b200 import hemul
    g = load_golden("hemul")
    he = hemul.HEMul(1, 4, 4, 3, 1, g["q_towers"], g["p_towers"])
    he.control_gen(degree_layout=(4, 4))
    he.setup_relinearization(np.array(g["evalkey_a_vector"], U32), np.array(g["evalkey_b_vector"], U32))
    out = _np(he.mul(np.array(g["input_ciphertext"], U32)))
    np.testing.assert_array_equal(out, np.array(g["encrypted_mult_result_ref"], U32))
    enc = out.reshape(1, 2, 16, 4)
    dec = O.ckks_decrypt([enc[0, 0].tolist(), enc[0, 1].tolist()], g["secret_key"], g["q_towers"][:4])
    assert dec == g["decrypted_result_ref"]
    qt = g["q_towers"]
    vals = O.ckks_decode(dec, qt, (g["scalingFactor"] / qt[-1]) ** 2, g["num_slots"], g["p"])
    assert np.max(np.abs(vals.real - np.array(g["real_values_multiply_result"]))) < 1.5e-3


def test_herot_golden():
    """herot_test.py:229-251."""
    from cross_b200 import herot, util
    g = load_golden("herot")
    r, c, dnum = 4, 4, 3
    rin, rmod = parse(g["rotate_in_ciphertext_str"])
    eb, ebm = parse(g["evalkey_b_vector_str"])
    ea, _ = parse(g["evalkey_a_vector_str"])
    x = np.array(rin, U32).transpose(0, 2, 1).reshape(1, -1, r, c, len(rmod))
    evb = np.array(eb, np.uint64).transpose(0, 2, 1).reshape(dnum, r, c, len(ebm))
    eva = np.array(ea, np.uint64).transpose(0, 2, 1).reshape(dnum, r, c, len(ebm))
    fin = np.array(parse(g["final_result_str"])[0], U32).transpose(0, 2, 1).reshape(1, -1, 16, len(rmod))
    cm = util.precompute_auto_map(16, util.find_automorphism_index_2n_complex(1, 16))
    assert cm == g["coef_map"]
    h = herot.HERot(r, c, dnum, rmod, ebm[len(rmod):])
    h.control_gen(batch=1, degree_layout=(r, c))
    h.setup_rotate(eva, evb, cm)
    np.testing.assert_array_equal(_np(h.rotate(x)), fin)


@pytest.mark.parametrize("n,r,c,L,K,dnum,batch", [(4096, 64, 64, 8, 3, 3, 2), (4096, 32, 128, 6, 2, 2, 1),
                                                  (1024, 32, 32, 5, 2, 3, 3)])
def test_hemul_vs_oracle(n, r, c, L, K, dnum, batch):
    from cross_b200 import hemul
    ov = O.find_moduli_ntt(L + K, 28, 2 * n)
    Q, P = ov[:L], ov[L:]
    rng = np.random.default_rng(n + L)
    ct = rng_residues(rng, (batch, 4, r, c, L), Q)
    evk_a = rng_residues(rng, (dnum, n, L + K), ov)
    evk_b = rng_residues(rng, (dnum, n, L + K), ov)
    he = hemul.HEMul(batch, r, c, dnum, 1, Q, P)
    he.control_gen(degree_layout=(r, c))
    he.setup_relinearization(evk_a, evk_b)
    ref = O.HEMul(batch, r, c, dnum, 1, Q, P)
    ref.setup_relinearization(evk_a, evk_b)
    np.testing.assert_array_equal(_np(he.mul(ct)), ref.mul(ct))


@pytest.mark.parametrize("n,L,K,dnum,batch,k", [(4096, 6, 2, 3, 2, 3), (1024, 4, 2, 2, 1, 100)])
def test_herot_vs_oracle(n, L, K, dnum, batch, k):
    from cross_b200 import herot, util
    ov = O.find_moduli_ntt(L + K, 28, 2 * n)
    Q, P = ov[:L], ov[L:]
    r, c = util.default_rc(n)
    rng = np.random.default_rng(k)
    ct = rng_residues(rng, (batch, 2, r, c, L), Q)
    evk_a = rng_residues(rng, (dnum, n, L + K), ov)
    evk_b = rng_residues(rng, (dnum, n, L + K), ov)
    cm = util.precompute_auto_map(n, util.find_automorphism_index_2n_complex(k, 2 * n))
    h = herot.HERot(r, c, dnum, Q, P)
    h.control_gen(batch=batch, degree_layout=(r, c))
    h.setup_rotate(evk_a, evk_b, cm)
    ref = O.HERot(r, c, dnum, Q, P)
    ref.control_gen(batch)
    ref.setup_rotate(evk_a.reshape(dnum, r, c, -1), evk_b.reshape(dnum, r, c, -1), cm)
    np.testing.assert_array_equal(_np(h.rotate(ct)), ref.rotate(ct))


@pytest.mark.parametrize("L,K,dnum", [(24, 8, 3), (35, 7, 5)])
def test_hemul_full_size_vs_oracle(L, K, dnum):
    """N = 2^16 parameter sets for one ciphertext, bit-exact against the oracle:
    the benchmark point (L = 24, K = 8, dnum = 3) and the eight-GPU configuration
    (L = 35, K = 7, dnum = 5)."""
    from cross_b200 import hemul
    n = 65536
    ov = O.find_moduli_ntt(L + K, 28, 2 * n)
    Q, P = ov[:L], ov[L:]
    rng = np.random.default_rng(2024)
    ct = rng_residues(rng, (1, 4, 256, 256, L), Q)
    evk_a = rng_residues(rng, (dnum, n, L + K), ov)
    evk_b = rng_residues(rng, (dnum, n, L + K), ov)
    he = hemul.HEMul(1, 256, 256, dnum, 1, Q, P)
    he.control_gen(degree_layout=(256, 256))
    he.setup_relinearization(evk_a, evk_b)
    got = _np(he.mul(ct))
    he.check_device()
    ref = O.HEMul(1, 256, 256, dnum, 1, Q, P)
    ref.setup_relinearization(evk_a, evk_b)
    np.testing.assert_array_equal(got, ref.mul(ct))


def test_herot_full_size_vs_oracle():
    """HE-Rotate at N = 2^16, L = 24, K = 8, dnum = 3 for one ciphertext and a
    seeded rotation index, bit-exact against the oracle."""
    from cross_b200 import herot, util
    n, L, K, dnum = 65536, 24, 8, 3
    ov = O.find_moduli_ntt(L + K, 28, 2 * n)
    Q, P = ov[:L], ov[L:]
    rng = np.random.default_rng(0)
    k = int(rng.integers(1, n // 2))
    ct = rng_residues(rng, (1, 2, 256, 256, L), Q)
    evk_a = rng_residues(rng, (dnum, n, L + K), ov)
    evk_b = rng_residues(rng, (dnum, n, L + K), ov)
    cm = util.precompute_auto_map(n, util.find_automorphism_index_2n_complex(k, 2 * n))
    h = herot.HERot(256, 256, dnum, Q, P)
    h.control_gen(batch=1, degree_layout=(256, 256))
    h.setup_rotate(evk_a, evk_b, cm)
    got = _np(h.rotate(ct))
    h.check_device()
    ref = O.HERot(256, 256, dnum, Q, P)
    ref.control_gen(1)
    ref.setup_rotate(evk_a.reshape(dnum, 256, 256, -1), evk_b.reshape(dnum, 256, 256, -1), cm)
    np.testing.assert_array_equal(got, ref.rotate(ct))


@pytest.mark.parametrize("pinned", [True, False])
def test_host_buffer_pipeline_matches_device_call(pinned):
    """HEMul.mul / HERot.rotate on CPU tensors (chunked, copies overlapped with
    compute, ragged last chunk) return exactly the device-call results."""
    import torch
    from cross_b200 import hemul, herot, util
    n, L, K, dnum, B = 4096, 6, 2, 3, 5
    ov = O.find_moduli_ntt(L + K, 28, 2 * n)
    Q, P = ov[:L], ov[L:]
    rng = np.random.default_rng(11)
    ct = rng_residues(rng, (B, 4, 64, 64, L), Q)
    ek = [rng_residues(rng, (dnum, n, L + K), ov) for _ in range(2)]
    he = hemul.HEMul(B, 64, 64, dnum, 1, Q, P)
    he.control_gen(degree_layout=(64, 64))
    he.setup_relinearization(*ek)
    want = _np(he.mul(ct))
    host = torch.from_numpy(ct)
    host = host.pin_memory() if pinned else host
    got = he.mul(host, chunk=2)
    torch.cuda.synchronize()
    assert got.device.type == "cpu"
    np.testing.assert_array_equal(got.numpy(), want)
    np.testing.assert_array_equal(he.mul(host, chunk=2).numpy(), want)   # buffers reused across calls
    r, c = util.default_rc(n)
    x2 = rng_residues(rng, (B, 2, r, c, L), Q)
    cm = util.precompute_auto_map(n, util.find_automorphism_index_2n_complex(5, 2 * n))
    h = herot.HERot(r, c, dnum, Q, P)
    h.control_gen(batch=B, degree_layout=(r, c))
    h.setup_rotate(*ek, cm)
    want_r = _np(h.rotate(x2))
    hx = torch.from_numpy(x2)
    hx = hx.pin_memory() if pinned else hx
    got_r = h.rotate(hx, chunk=3)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got_r.numpy(), want_r)


def test_unreduced_inputs_stay_bit_exact():
    """Full-range uint32 inputs and keys (not reduced mod q) drive the epilogue
    and BConv operands outside the lazy-residue range; the guarded fast Barrett
    forms must still return the reference's values (tensor-core path, N = 2^14)."""
    import torch
    from cross_b200 import hemul, bconv, _lib
    n, L, K, dnum, B = 16384, 6, 2, 3, 2
    ov = O.find_moduli_ntt(L + K, 28, 2 * n)
    Q, P = ov[:L], ov[L:]
    rng = np.random.default_rng(99)
    ct = rng.integers(0, 2 ** 32, size=(B, 4, 128, 128, L), dtype=np.uint64).astype(U32)
    ek = [rng.integers(0, 2 ** 32, size=(dnum, n, L + K), dtype=np.uint64).astype(U32) for _ in range(2)]
    he = hemul.HEMul(B, 128, 128, dnum, 1, Q, P)
    he.control_gen(degree_layout=(128, 128))
    he.setup_relinearization(*ek)
    got = _np(he.mul(ct))
    ref = O.HEMul(B, 128, 128, dnum, 1, Q, P)
    ref.setup_relinearization(*ek)
    np.testing.assert_array_equal(got, ref.mul(ct))
    # BConv 8 -> 23 (tensor-core kernel, limb-major) on full-range inputs
    mv = O.find_moduli_ntt(31, 28, 2 * 4096)
    x = rng.integers(0, 2 ** 32, size=(2, 4096, 8), dtype=np.uint64).astype(U32)
    ob = O.BConvBarrett(mv)
    ob.control_gen([(list(range(8)), list(range(8, 31)))])
    b = bconv.BConvBarrett(mv)
    b.control_gen([(list(range(8)), list(range(8, 31)))])
    xl = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1))).cuda()
    yl = torch.empty((2, 23, 4096), dtype=xl.dtype, device="cuda")
    _lib.check(_lib.lib().cross_bconv(b.plan(0), 1, xl.data_ptr(), yl.data_ptr(), 2, 4096, _lib.LAYOUT_LIMB_MAJOR,
                                      None), "cross_bconv")
    np.testing.assert_array_equal(_np(yl), ob.basis_change_bat(x).transpose(0, 2, 1))
    b.check_device()


def test_limb_major_layout_matches_reference_layout():
    import torch
    from cross_b200 import hemul, LAYOUT_LIMB_MAJOR
    n, L, K, dnum, B = 1024, 5, 2, 3, 2
    ov = O.find_moduli_ntt(L + K, 28, 2 * n)
    rng = np.random.default_rng(1)
    ct = rng_residues(rng, (B, 4, 32, 32, L), ov[:L])
    ek = [rng_residues(rng, (dnum, n, L + K), ov) for _ in range(2)]
    he = hemul.HEMul(B, 32, 32, dnum, 1, ov[:L], ov[L:])
    he.control_gen()
    he.setup_relinearization(*ek)
    ref_layout = _np(he.mul(ct))
    lm_in = torch.from_numpy(np.ascontiguousarray(ct.reshape(B, 4, n, L).transpose(0, 1, 3, 2))).cuda()
    lm = _np(he.mul(lm_in, layout=LAYOUT_LIMB_MAJOR))
    np.testing.assert_array_equal(lm.transpose(0, 1, 3, 2).reshape(ref_layout.shape), ref_layout)


@pytest.mark.parametrize("polys,n,L", [(3, 128, 1), (2, 4096, 24), (5, 1024, 7), (1, 256, 64),
                                        (2, 256, 65), (3, 96, 5), (2, 65536, 24)])
def test_layout_conversions(polys, n, L):
    """cross_to_limb_major / cross_to_reference are exact permutations (coalesced
    tile kernel for L <= 64 and n % 128 == 0, generic tile transpose otherwise)."""
    import torch
    from cross_b200 import _lib
    rng = np.random.default_rng(n + L)
    x = rng.integers(0, 2 ** 32, size=(polys, n, L), dtype=np.uint64).astype(U32)
    xd = torch.from_numpy(x).cuda()
    lm = torch.empty((polys, L, n), dtype=xd.dtype, device="cuda")
    back = torch.empty_like(xd)
    lib = _lib.lib()
    _lib.check(lib.cross_to_limb_major(xd.data_ptr(), lm.data_ptr(), polys, n, L, None), "cross_to_limb_major")
    _lib.check(lib.cross_to_reference(lm.data_ptr(), back.data_ptr(), polys, n, L, None), "cross_to_reference")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(lm.cpu().numpy(), x.transpose(0, 2, 1))
    np.testing.assert_array_equal(back.cpu().numpy(), x)
    # buffers offset by one word (not 16-byte aligned) take the generic kernel
    xo = torch.zeros(polys * n * L + 1, dtype=xd.dtype, device="cuda")
    xo[1:] = xd.reshape(-1)
    lo = torch.zeros(polys * n * L + 1, dtype=xd.dtype, device="cuda")
    _lib.check(lib.cross_to_limb_major(xo.data_ptr() + 4, lo.data_ptr() + 4, polys, n, L, None), "cross_to_limb_major")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(lo[1:].cpu().numpy().reshape(polys, L, n), x.transpose(0, 2, 1))


def test_errors_are_reference_exceptions():
    from cross_b200 import hemul, ntt_mm
    q = O.find_moduli_ntt(2, 28, 2 * 16)
    ctx = ntt_mm.NTTCiphertextBarrettContext(q, {"r": 4, "c": 4})
    with pytest.raises(ValueError):
        ctx.ntt(np.zeros((1, 4, 4, 3), U32))
    he = hemul.HEMul(1, 4, 4, 2, 1, q, O.find_moduli_ntt(3, 28, 32)[2:])
    he.control_gen()
    with pytest.raises(RuntimeError):
        he.mul(np.zeros((1, 4, 4, 4, 2), U32))


def test_empty_batches_are_no_ops():
    """Batch 0 through every operator returns empty results without launching."""
    import torch
    from cross_b200 import hemul, herot, ntt_mm, bconv, _lib, util
    n, L, K, dnum = 4096, 4, 2, 2
    ov = O.find_moduli_ntt(L + K, 28, 2 * n)
    Q, P = ov[:L], ov[L:]
    ctx = ntt_mm.NTTCiphertextBarrettContext(Q, {"r": 64, "c": 64})
    assert tuple(ctx.ntt(np.zeros((0, 64, 64, L), U32)).shape) == (0, 64, 64, L)
    b = bconv.BConvBarrett(ov)
    b.control_gen([(list(range(L)), list(range(L, L + K)))])
    assert tuple(b.basis_change_bat(np.zeros((0, n, L), U32)).shape) == (0, n, K)
    rng = np.random.default_rng(5)
    ek = [rng_residues(rng, (dnum, n, L + K), ov) for _ in range(2)]
    he = hemul.HEMul(1, 64, 64, dnum, 1, Q, P)
    he.control_gen(degree_layout=(64, 64))
    he.setup_relinearization(*ek)
    assert tuple(he.mul(np.zeros((0, 4, 64, 64, L), U32)).shape) == (0, 2, 64, 64, L - 1)
    r, c = util.default_rc(n)
    h = herot.HERot(r, c, dnum, Q, P)
    h.control_gen(batch=1, degree_layout=(r, c))
    h.setup_rotate(*ek, util.precompute_auto_map(n, util.find_automorphism_index_2n_complex(3, 2 * n)))
    assert tuple(h.rotate(np.zeros((0, 2, r, c, L), U32)).shape) == (0, 2, n, L)


def test_hemul_non_square_tensor_core_vs_oracle():
    """HE-Mult on the tensor-core path with r != c (N = 2^15, 128 x 256; the
    default (r, c) of the ModDown and key-switch transforms differs from the
    input layout's), bit-exact against the oracle."""
    from cross_b200 import hemul
    n, L, K, dnum, B = 32768, 5, 2, 3, 2
    ov = O.find_moduli_ntt(L + K, 28, 2 * n)
    Q, P = ov[:L], ov[L:]
    rng = np.random.default_rng(31)
    ct = rng_residues(rng, (B, 4, 128, 256, L), Q)
    ek = [rng_residues(rng, (dnum, n, L + K), ov) for _ in range(2)]
    he = hemul.HEMul(B, 128, 256, dnum, 1, Q, P)
    he.control_gen(degree_layout=(128, 256))
    he.setup_relinearization(*ek)
    got = _np(he.mul(ct))
    he.check_device()
    ref = O.HEMul(B, 128, 256, dnum, 1, Q, P)
    ref.setup_relinearization(*ek)
    np.testing.assert_array_equal(got, ref.mul(ct))


def test_ntt_refuses_unaligned_row_major_output():
    """The row-major contraction stages write their outputs with 16-byte
    stores; an output pointer off a 16-byte boundary through the C ABI is
    refused with CROSS_ERR_INVALID_ARG before the row stage launches, and the
    context keeps computing bit-exact results."""
    import torch
    from cross_b200 import _lib, ntt_mm
    q = O.find_moduli_ntt(2, 28, 2 * 65536)
    ctx = ntt_mm.NTTCiphertextBarrettContext(q, {"r": 256, "c": 256})
    lib = _lib.lib()
    B, M, n = 1, 2, 65536
    x = rng_residues(np.random.default_rng(5), (B, 256, 256, M), q)
    xl = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 3, 1, 2))).cuda()
    buf = torch.zeros(B * M * n + 4, dtype=torch.uint32, device="cuda")
    ws = torch.empty(lib.cross_ntt_workspace_size(ctx.plan(), B, _lib.LAYOUT_LIMB_MAJOR), dtype=torch.uint8,
                     device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.cross_ntt(ctx.plan(), 0, xl.data_ptr(), buf.data_ptr() + 4, B, _lib.LAYOUT_LIMB_MAJOR, ws.data_ptr(),
                       ws.numel(), st)
    assert rc == -1, lib.cross_last_error()                        # CROSS_ERR_INVALID_ARG
    assert b"16-byte aligned" in lib.cross_last_error()
    torch.cuda.synchronize()
    assert int(buf.count_nonzero()) == 0                           # nothing was written
    np.testing.assert_array_equal(_np(ctx.ntt(x)), O.NTTBarrett(q, 256, 256).ntt(x))
    ctx.check_device()


@pytest.mark.parametrize("a64,b64", [(False, False), (True, False), (False, True), (True, True)])
def test_elementwise_index_forms(a64, b64):
    """The element-wise kernels' index arithmetic (32-bit forms below 2^31
    elements) on shapes that exercise every split: cross_modmul with a table
    broadcast over rows (b_rows not dividing rows) and every operand width
    (ciphertext.py:189-193; products wrap in uint64), cross_add_mod at a
    ring dimension that is not a power of two (add.py:7-27), cross_automorphism
    with negative and out-of-range map entries (jnp.take's default mode,
    herot.py:300), and cross_mod_reduce of uint32 and uint64 input."""
    import torch
    from cross_b200 import _lib, finite_field
    lib = _lib.lib()
    q = O.find_moduli_ntt(5, 28, 2 * 64)
    M = len(q)
    ff = finite_field.BarrettContext(q)
    bar = O.Barrett(q)
    rng = np.random.default_rng(11 + 2 * a64 + b64)
    rows, b_rows = 105, 7
    a = rng.integers(0, 2 ** 63, size=(rows, M), dtype=np.uint64) if a64 else rng_residues(rng, (rows, M), q)
    b = rng.integers(0, 2 ** 63, size=(b_rows, M), dtype=np.uint64) if b64 else rng_residues(rng, (b_rows, M), q)
    want = bar.reduce(a.astype(np.uint64) * b.astype(np.uint64)[np.arange(rows) % b_rows])
    da, db = torch.from_numpy(a.view(np.int64) if a64 else a.view(np.int32)).cuda(), \
        torch.from_numpy(b.view(np.int64) if b64 else b.view(np.int32)).cuda()
    out = torch.empty((rows, M), dtype=torch.int32, device="cuda")
    _lib.check(lib.cross_modmul(ff.handle(), da.data_ptr(), int(a64), db.data_ptr(), int(b64), b_rows,
                                out.data_ptr(), rows, None), "cross_modmul")
    np.testing.assert_array_equal(out.cpu().numpy().view(U32), want)
    # add at n = 24 on (E, M, n): the sum minus q where it is strictly above q
    E, n = 3, 24
    x = rng_residues(rng, (E, n, M), q).transpose(0, 2, 1).copy()
    y = rng_residues(rng, (E, n, M), q).transpose(0, 2, 1).copy()
    x[1, 2, :5] = np.uint32(q[2]) - y[1, 2, :5]
    dx, dy = torch.from_numpy(x.view(np.int32)).cuda(), torch.from_numpy(y.view(np.int32)).cuda()
    dz = torch.empty_like(dx)
    _lib.check(lib.cross_add_mod(ff.handle(), dx.data_ptr(), dy.data_ptr(), dz.data_ptr(), E, n, None),
               "cross_add_mod")
    np.testing.assert_array_equal(dz.cpu().numpy().view(U32), O.jax_add(x, y, q))
    # automorphism at n = 24 with a map holding negative and out-of-range entries
    polys = 3
    src = rng.integers(0, 2 ** 32, size=(polys, n, M), dtype=np.uint64).astype(U32)
    cmap = rng.integers(-30, 30, size=n).astype(np.int32)
    idx = np.where(cmap < 0, cmap + n, cmap)
    ok = (idx >= 0) & (idx < n)
    ref = np.where(ok[None, :, None], src[:, np.clip(idx, 0, n - 1)], np.uint32(0xFFFFFFFF))
    ds = torch.from_numpy(src.view(np.int32)).cuda()
    dm = torch.from_numpy(cmap).cuda()
    do = torch.empty_like(ds)
    _lib.check(lib.cross_automorphism(ds.data_ptr(), dm.data_ptr(), do.data_ptr(), polys, n, M, None),
               "cross_automorphism")
    np.testing.assert_array_equal(do.cpu().numpy().view(U32), ref)
    # Barrett of uint32 and uint64 input
    z = rng.integers(0, 2 ** 63, size=(rows, M), dtype=np.uint64)
    dz64 = torch.from_numpy(z.view(np.int64)).cuda()
    dr = torch.empty((rows, M), dtype=torch.int32, device="cuda")
    _lib.check(lib.cross_mod_reduce(ff.handle(), dz64.data_ptr(), 1, dr.data_ptr(), rows, None), "cross_mod_reduce")
    np.testing.assert_array_equal(dr.cpu().numpy().view(U32), bar.reduce(z))
    z32 = (z & np.uint64(0xFFFFFFFF)).astype(U32)
    dz32 = torch.from_numpy(z32.view(np.int32)).cuda()
    _lib.check(lib.cross_mod_reduce(ff.handle(), dz32.data_ptr(), 0, dr.data_ptr(), rows, None), "cross_mod_reduce")
    np.testing.assert_array_equal(dr.cpu().numpy().view(U32), bar.reduce(z32.astype(np.uint64)))


@pytest.mark.parametrize("b_rows,offset,full", [(8, 0, False), (112, 0, False), (112, 0, True), (8, 1, False),
                                                (7, 0, False)])
def test_elementwise_vector_forms(b_rows, offset, full):
    """The 16-byte forms of cross_modmul (uint32 operands, sizes and the table
    period multiples of 4; residue operands take the exact 32-bit remainder
    form, full-range words the 64-bit one) and cross_add_mod (ring dimension a
    multiple of 4), and their fallbacks: buffers one word off a 16-byte
    boundary, a table period of 35 words, a ring dimension of 26."""
    import torch
    from cross_b200 import _lib, finite_field
    lib = _lib.lib()
    q = O.find_moduli_ntt(5, 28, 2 * 64)
    M = len(q)
    ff = finite_field.BarrettContext(q)
    rng = np.random.default_rng(100 + b_rows + offset + 7 * full)
    rows = 112
    draw = (lambda shape: rng.integers(0, 2 ** 32, size=shape, dtype=np.uint64).astype(U32)) if full else \
        (lambda shape: rng_residues(rng, shape, q))
    a, b = draw((rows, M)), draw((b_rows, M))
    want = O.Barrett(q).reduce(a.astype(np.uint64) * b.astype(np.uint64)[np.arange(rows) % b_rows])

    def dev(x):   # device copy starting `offset` words into a buffer
        t = torch.zeros(x.size + 4, dtype=torch.int32, device="cuda")
        t[offset:offset + x.size] = torch.from_numpy(x.reshape(-1).view(np.int32)).cuda()
        return t

    da, db, do = dev(a), dev(b), dev(np.zeros((rows, M), U32))
    _lib.check(lib.cross_modmul(ff.handle(), da.data_ptr() + 4 * offset, 0, db.data_ptr() + 4 * offset, 0, b_rows,
                                do.data_ptr() + 4 * offset, rows, None), "cross_modmul")
    got = do.cpu().numpy().view(U32)
    np.testing.assert_array_equal(got[offset:offset + rows * M].reshape(rows, M), want)
    assert not got[:offset].any() and not got[offset + rows * M:].any()     # nothing written outside
    for E, n in ((3, 24), (2, 26)):
        x = rng_residues(rng, (E, n, M), q).transpose(0, 2, 1).copy()
        y = rng_residues(rng, (E, n, M), q).transpose(0, 2, 1).copy()
        x[0, 1, :3] = np.uint32(q[1]) - y[0, 1, :3]
        dx, dy, dz = dev(x), dev(y), dev(np.zeros_like(x))
        _lib.check(lib.cross_add_mod(ff.handle(), dx.data_ptr() + 4 * offset, dy.data_ptr() + 4 * offset,
                                     dz.data_ptr() + 4 * offset, E, n, None), "cross_add_mod")
        z = dz.cpu().numpy().view(U32)
        np.testing.assert_array_equal(z[offset:offset + x.size].reshape(x.shape), O.jax_add(x, y, q))
