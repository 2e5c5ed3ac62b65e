"""CKKS client side (jaxite_word ckks_ctx.py) on the GPU: encode, encrypt,
decrypt and decode.

The special FFTs, the quantisation, the negacyclic transforms (psi twist and
the BAT NTT), the encryption and decryption sums, the CRT recombination and
the decode scaling all run as CUDA kernels.  Doubles are computed as CPython
computes them (no fused multiply-adds, the reference's twiddle values), so the
results equal the reference's bit for bit; integers are fully reduced as the
reference's Python ``%`` leaves them.  Functions take the reference's
arguments and return CUDA tensors in the reference's shapes ((degree, moduli)
residues; ``ckks_decode`` returns the list of complex slot values).
"""
from __future__ import annotations

import cmath
import math
import secrets
from typing import List

import numpy as np

from . import _lib, _tensor, util
from . import ciphertext as ct
from . import finite_field as ff_context

MAX_INT_64 = 9223372036854775295                 # ckks_ctx.py:14
sigma = 3.190000057220458984375                  # ckks_ctx.py:15
U32, U64 = np.uint32, np.uint64

_FFT_TABLES = {}
_NEGACYCLIC = {}


def _fft_tables(m: int, nh: int):
    """_roots(m) (ckks_ctx.py:23-24, the same cmath values) and _rot_group
    (ckks_ctx.py:27-32) as device arrays."""
    t = _tensor.torch()
    key = (m, nh, t.cuda.current_device())
    if key not in _FFT_TABLES:
        roots = np.array([cmath.exp(1j * 2 * math.pi * k / m) for k in range(m)], np.complex128)
        rg = [1]
        for _ in range(1, nh):
            rg.append((rg[-1] * 5) % m)
        _FFT_TABLES[key] = (t.from_numpy(roots).to(_tensor.device()),
                            t.from_numpy(np.array(rg, U32)).to(_tensor.device()))
    return _FFT_TABLES[key]


def _fft_dev(y, m: int, inverse: bool):
    """In-place special FFT of a (batch, nh) complex128 CUDA tensor."""
    nh = y.shape[-1]
    roots, rot = _fft_tables(m, nh)
    _tensor.call("cross_fft_special", y.data_ptr(), y.numel() // nh, nh, m, roots.data_ptr(), rot.data_ptr(),
                 int(inverse), 1.0 / nh, _lib.cuda_stream())
    return y


def _to_complex_dev(vals):
    t = _tensor.torch()
    if isinstance(vals, t.Tensor):
        return vals.to(device=_tensor.device(), dtype=t.complex128).contiguous().clone()
    return t.from_numpy(np.asarray(vals, np.complex128).copy()).to(_tensor.device())


def _fft_inplace(vals, cycl_order: int, inverse: bool):
    y = _fft_dev(_to_complex_dev(vals).reshape(1, -1), cycl_order, inverse)[0]
    t = _tensor.torch()
    if isinstance(vals, t.Tensor):
        vals.copy_(y.to(vals.device))
    else:
        out = y.cpu().numpy()
        vals[:] = [complex(v) for v in out] if isinstance(vals, list) else out


def FFTSpecialInv(vals, cycl_order: int) -> None:
    """ckks_ctx.py:48-80 on the GPU, in place (list, numpy array or tensor)."""
    _fft_inplace(vals, cycl_order, True)


def FFTSpecial(vals, cycl_order: int) -> None:
    """ckks_ctx.py:83-110 on the GPU, in place."""
    _fft_inplace(vals, cycl_order, False)


def nearest_int(x: float) -> int:
    """ckks_ctx.py:113-115."""
    return int(math.floor(x + 0.5)) if x >= 0 else -int(math.floor(-x + 0.5))


def slot_to_coeffs(y) -> List[float]:
    """ckks_ctx.py:117-126."""
    return [v.real for v in y] + [v.imag for v in y]


def fit_to_native_vector(vec, big_bound: int, modulus: int, ring_dim: int) -> List[int]:
    """ckks_ctx.py:128-153 (host helper on Python integers)."""
    dslots = len(vec)
    if dslots == 0:
        return [0] * ring_dim
    half, diff, gap = big_bound >> 1, big_bound - modulus, ring_dim // dslots
    native = [0] * ring_dim
    for i, val in enumerate(vec):
        n = int(val)
        native[gap * i] = (n - diff) % modulus if n > half else n % modulus
    return native


# ---------------------------------------------------------------------------
# negacyclic transforms per tower (util.py:763-827 with the reference's
# bit-reversed evaluation order)
# ---------------------------------------------------------------------------

class _Negacyclic:
    """Towers q_t of degree N: forward = psi^i twist, BAT NTT, full
    reduction (bit_reverse_array(ntt_negacyclic_bit_reverse(.)));
    inverse = BAT INTT, psi^-i twist, full reduction
    (intt_negacyclic_bit_reverse(bit_reverse_array(.))).  Limb-major (M, N)."""

    def __init__(self, moduli, degree: int):
        from . import ntt_mm
        t = _tensor.torch()
        self.moduli, self.N = list(moduli), degree
        r, c = util.default_rc(degree)
        self.ntt = ntt_mm.NTTCiphertextBarrettContext(self.moduli, {"r": r, "c": c})
        self.ff = ff_context.BarrettContext(self.moduli)
        psi = [util.root_of_unity(2 * degree, q) for q in self.moduli]
        fw = np.stack([util.powers(p, degree, q) for p, q in zip(psi, self.moduli)]).astype(U32)
        iv = np.stack([util.powers(pow(p, -1, q), degree, q) for p, q in zip(psi, self.moduli)]).astype(U32)
        self.psi = t.from_numpy(np.ascontiguousarray(fw)).to(_tensor.device())
        self.inv_psi = t.from_numpy(np.ascontiguousarray(iv)).to(_tensor.device())
        self._ws = None

    def _run_ntt(self, x, inverse):
        lib = _lib.lib()
        ws = _tensor.workspace(lib.cross_ntt_workspace_size(self.ntt.plan(), 1, _lib.LAYOUT_LIMB_MAJOR))
        out = _tensor.empty_u32(x.shape)
        _tensor.call("cross_ntt", self.ntt.plan(), int(inverse), x.data_ptr(), out.data_ptr(), 1,
                     _lib.LAYOUT_LIMB_MAJOR, ws.data_ptr(), ws.numel(), _lib.cuda_stream())
        return out

    def _mul(self, x, tab):
        out = _tensor.empty_u32(x.shape)
        _tensor.call("cross_mul_reduce_lm", self.ff.handle(), x.data_ptr(), tab.data_ptr() if tab is not None else None,
                     out.data_ptr(), self.N, _lib.cuda_stream())
        return out

    def forward(self, coefs):
        """(M, N) coefficients (any uint32) -> (M, N) evaluations in [0, q)."""
        x = _tensor.to_u32(coefs).reshape(len(self.moduli), self.N).contiguous()
        return self._mul(self._run_ntt(self._mul(x, self.psi), False), None)

    def inverse(self, evals):
        """(M, N) evaluations -> (M, N) coefficients in [0, q)."""
        x = _tensor.to_u32(evals).reshape(len(self.moduli), self.N).contiguous()
        return self._mul(self._run_ntt(x, True), self.inv_psi)


def _negacyclic(moduli, degree):
    t = _tensor.torch()
    key = (tuple(int(q) for q in moduli), degree, t.cuda.current_device())
    if key not in _NEGACYCLIC:
        _NEGACYCLIC[key] = _Negacyclic(moduli, degree)
    return _NEGACYCLIC[key]


_FF = {}


def _negacyclic_ff(moduli):
    key = tuple(int(q) for q in moduli)
    if key not in _FF:
        _FF[key] = ff_context.BarrettContext(list(key))
    return _FF[key]


def _rows(x, n_moduli=None):
    """A (rows, cols) uint32 CUDA tensor from nested lists / arrays / tensors."""
    t = _tensor.torch()
    if isinstance(x, t.Tensor):
        return _tensor.to_u32(x).contiguous()
    if isinstance(x, (list, tuple)):
        return _tensor.to_u32(np.array([np.asarray(r, dtype=object).astype(np.uint64) for r in x], np.uint64))
    return _tensor.to_u32(np.asarray(x).astype(np.uint64))


# ---------------------------------------------------------------------------
# encode / encrypt / decrypt / decode
# ---------------------------------------------------------------------------

def ckks_encode(slots, cycl_order: int, q_towers, p_towers, scale: float, noise_scale_degree: int = 1,
                max_bits_in_word: int = 61):
    """ckks_ctx.py:331-404: (degree, moduli) evaluations, bit-reversed per tower."""
    nh = len(slots)
    n, m = 2 * nh, cycl_order
    assert m == 4 * nh, "cycl_order must be 4*Nh for CKKS special FFT size"
    t = _tensor.torch()
    y = _fft_dev(_to_complex_dev(slots).reshape(1, nh), m, True)
    mx = t.zeros(1, dtype=t.float64, device=_tensor.device())
    _tensor.call("cross_ckks_max_abs_scaled", y.data_ptr(), 2 * nh, float(scale), mx.data_ptr(), _lib.cuda_stream())
    maxabs = float(mx.item())
    # ceil(log2 |v|) is non-decreasing in |v|: the largest value gives the reference's maximum
    logc = int(math.ceil(math.log2(maxabs))) if maxabs != 0.0 else 0
    if logc < 0:
        raise ValueError("Scaling factor too small")
    log_valid = logc if logc <= max_bits_in_word else max_bits_in_word
    log_approx = logc - log_valid
    factor = None
    if noise_scale_degree > 1:
        p = int(round(scale))
        if p != 1:
            power = pow(p, noise_scale_degree - 1)
            factor = t.from_numpy(np.array([power % q for q in q_towers], U32)).to(_tensor.device())
    neg = _negacyclic(q_towers, n)
    coefs = _tensor.empty_u32((len(q_towers), n))
    _tensor.call("cross_ckks_quantize", neg.ff.handle(), y.data_ptr(), nh, float(scale), log_approx,
                 factor.data_ptr() if factor is not None else None, coefs.data_ptr(), _lib.cuda_stream())
    return neg.forward(coefs).t().contiguous()


def _sample_coeffs(degree: int, kind: str, sigma_: float = sigma):
    """Coefficient samples: ternary {0, 1} (key_gen.py:18-21) or rounded
    Gaussian (key_gen.py:32-50), from a generator seeded by the OS's CSPRNG."""
    rng = np.random.Generator(np.random.PCG64(secrets.randbits(128)))
    if kind == "ternary":
        return rng.integers(0, 2, size=degree).astype(np.int64)
    return np.rint(rng.normal(0.0, sigma_, size=degree)).astype(np.int64)


def _rns_of(coeffs, moduli):
    """gen_rns_polynomial: integer coefficients reduced into every modulus,
    (M, N) on the device."""
    t = _tensor.torch()
    c = t.from_numpy(np.ascontiguousarray(np.asarray(coeffs, np.int64))).to(_tensor.device())
    out = _tensor.empty_u32((len(moduli), c.numel()))
    _tensor.call("cross_rns_from_signed", _negacyclic_ff(moduli).handle(), c.data_ptr(), c.numel(), out.data_ptr(),
                 _lib.cuda_stream())
    return out


def ckks_encrypt(plaintext, public_key, q_towers, noise_scale_degree: int = 1, sigma=sigma, v=None, e=None,
                 ba=None, e_ref=None, v_ref=None):
    """ckks_ctx.py:156-235: [c0, c1], each (degree, moduli).  v / e (given or
    sampled) are (moduli, degree) evaluations."""
    pt = _rows(plaintext)
    degree, nt = pt.shape[0], len(q_towers)
    neg = _negacyclic(q_towers, degree)
    if v is None:
        v = neg.forward(_rns_of(_sample_coeffs(degree, "ternary"), q_towers))
        if v_ref is not None:
            np.testing.assert_array_equal(_tensor.to_numpy(v), np.asarray(v_ref))
    if e is None:
        e0 = neg.forward(_rns_of(_sample_coeffs(degree, "gauss", sigma), q_towers))
        e1 = neg.forward(_rns_of(_sample_coeffs(degree, "gauss", sigma), q_towers))
        if e_ref is not None:
            np.testing.assert_array_equal(_tensor.to_numpy(e0), np.asarray(e_ref[0]))
            np.testing.assert_array_equal(_tensor.to_numpy(e1), np.asarray(e_ref[1]))
    else:
        e0, e1 = e[0], e[1]
    if isinstance(public_key, list) and pt.shape[1] < len(public_key[0]):
        # ckks_ctx.py:196-199 trims the caller's key lists in place
        diff = len(public_key[0]) - pt.shape[1]
        public_key[0] = public_key[0][:-diff]
        public_key[1] = public_key[1][:-diff]
    pk0 = _rows(public_key[0])[:nt].contiguous()
    pk1 = _rows(public_key[1])[:nt].contiguous()
    v, e0, e1 = (_rows(a)[:nt].contiguous() for a in (v, e0, e1))
    if pt.shape != (degree, nt) or any(tuple(a.shape) != (nt, degree) for a in (pk0, pk1, v, e0, e1)):
        raise ValueError(f"ckks_encrypt: plaintext must be (degree, {nt}) and keys / noise ({nt}, degree)")
    c0, c1 = _tensor.empty_u32((degree, nt)), _tensor.empty_u32((degree, nt))
    _tensor.call("cross_ckks_encrypt", neg.ff.handle(), pt.data_ptr(), v.data_ptr(), e0.data_ptr(), e1.data_ptr(),
                 pk0.data_ptr(), pk1.data_ptr(), int(noise_scale_degree), c0.data_ptr(), c1.data_ptr(), degree,
                 _lib.cuda_stream())
    if ba is not None:
        q = np.array(q_towers, np.int64)
        c0h, pth = _tensor.to_numpy(c0).astype(np.int64), _tensor.to_numpy(pt).astype(np.int64)
        np.testing.assert_array_equal(((c0h - pth) % q).T, np.asarray(ba[0]))
        np.testing.assert_array_equal(_tensor.to_numpy(c1).T, np.asarray(ba[1]))
    return [c0, c1]


def ckks_decrypt(ciphertext, private_key, q_towers):
    """ckks_ctx.py:238-328: (degree, moduli) coefficients."""
    t = _tensor.torch()
    if isinstance(ciphertext, t.Tensor):
        c = _tensor.to_u32(ciphertext).contiguous()
    else:
        c = t.stack([_rows(el) for el in ciphertext]).contiguous()
    if c.dim() != 3:
        raise ValueError("ckks_decrypt: ciphertext must be (elements, degree, moduli)")
    elements, degree, nt = c.shape
    s = _rows(private_key)[:nt].contiguous()
    if tuple(s.shape) != (nt, degree) or nt > len(q_towers):
        raise ValueError(f"ckks_decrypt: the secret key must cover the {nt} towers of degree {degree}")
    neg = _negacyclic(list(q_towers)[:nt], degree)
    acc = _tensor.empty_u32((nt, degree))
    _tensor.call("cross_ckks_decrypt_sum", neg.ff.handle(), c.data_ptr(), elements, s.data_ptr(), acc.data_ptr(),
                 degree, _lib.cuda_stream())
    return neg.inverse(acc).t().contiguous()


def _int_words(q: int) -> int:
    return max(1, (q.bit_length() + 31) // 32)


def _to_words(values, words: int) -> np.ndarray:
    buf = b"".join(int(v).to_bytes(4 * words, "little") for v in values)
    return np.frombuffer(buf, U32).reshape(len(values), words)


def _crt_tables(moduli):
    M = 1
    for q in moduli:
        M *= q
    W = _int_words(M)
    mi = [M // q for q in moduli]
    inv = np.array([pow(a, -1, q) for a, q in zip(mi, moduli)], U32)
    t = _tensor.torch()
    dev = _tensor.device()
    return (M, W, t.from_numpy(inv).to(dev), t.from_numpy(_to_words(mi, W).copy()).to(dev),
            t.from_numpy(_to_words([M], W)[0].copy()).to(dev))


def _crt_words(rns, moduli):
    """(degree, words) CUDA tensor of the CRT values of rns (degree, moduli)."""
    x = _rows(rns)
    if x.dim() != 2 or x.shape[1] != len(moduli):
        raise ValueError(f"CRT: residues must be (degree, {len(moduli)})")
    M, W, inv, mi, qw = _crt_tables(list(moduli))
    out = _tensor.empty_u32((x.shape[0], W))
    _tensor.call("cross_crt_combine", _negacyclic_ff(moduli).handle(), x.data_ptr(), x.shape[0], inv.data_ptr(),
                 mi.data_ptr(), qw.data_ptr(), W, out.data_ptr(), _lib.cuda_stream())
    return out, M, W


def _crt_combine_rns_plaintext(rns_plaintext, moduli) -> List[int]:
    """ckks_ctx.py:517-545 on the GPU: a list of Python integers."""
    words, _, _ = _crt_words(rns_plaintext, moduli)
    h = _tensor.to_numpy(words)
    return [int.from_bytes(row.tobytes(), "little") for row in h]


def _decode_words(x, W: int, q: int, scalingFactor: float, slots: int, p: int, degree: int,
                  CKKS_M_FACTOR: int = 1, ADD_NOISE: bool = False, as_array: bool = False):
    t = _tensor.torch()
    dev = _tensor.device()
    nh = degree // 2
    pow_p_pos, pow_p = pow(2, p), pow(2, -p)
    sf_pre = (1.0 / scalingFactor) * pow_p_pos
    qw = t.from_numpy(_to_words([q], W)[0].copy()).to(dev)
    hw = t.from_numpy(_to_words([q >> 1], W)[0].copy()).to(dev)
    cur = t.empty((slots, 2), dtype=t.float64, device=dev)
    flag = t.zeros(1, dtype=t.int32, device=dev)
    _tensor.call("cross_ckks_decode_scale", x.data_ptr(), W, qw.data_ptr(), hw.data_ptr(), sf_pre, slots, nh,
                 cur.data_ptr(), flag.data_ptr(), _lib.cuda_stream())
    sd_t = t.empty(1, dtype=t.float64, device=dev)
    _tensor.call("cross_ckks_decode_stddev", cur.data_ptr(), slots, sd_t.data_ptr(), _lib.cuda_stream())
    if int(flag.item()):
        raise OverflowError("int too large to convert to float")
    sd = float(sd_t.cpu()[0])
    logstd = math.log2(sd) if sd > 0 else float("-inf")
    if sd < 0.125 * math.sqrt(degree):
        sd = 0.125 * math.sqrt(degree)
    if logstd > p - 5.0:
        raise Exception("The decryption failed because the approximation error is too high. Check the parameters. ")
    scale = 0.5 * pow_p
    out = t.empty((slots, 2), dtype=t.float64, device=dev)
    _tensor.call("cross_ckks_decode_combine", cur.data_ptr(), out.data_ptr(), slots, scale, _lib.cuda_stream())
    if ADD_NOISE:
        # ckks_ctx.py:489-504: Gaussian noise of deviation sqrt(M + 1) * sd, times 2^-p
        rng = np.random.Generator(np.random.PCG64(secrets.randbits(128)))
        std = math.sqrt(CKKS_M_FACTOR + 1) * sd
        out += t.from_numpy(pow_p * rng.normal(0.0, std, size=(slots, 2))).to(dev)
    y = t.view_as_complex(out).reshape(1, slots)
    _fft_dev(y, degree * 2, False)
    if as_array:
        return y[0].real.cpu().numpy().astype(np.complex128)
    return [complex(float(v), 0.0) for v in y[0].real.cpu().numpy()]


def ckks_decode(plaintext, scalingFactor: float, slots: int, q: int, p: int, CKKS_M_FACTOR: int = 1,
                ADD_NOISE: bool = False):
    """ckks_ctx.py:407-514: plaintext = the CRT-combined coefficients (Python
    integers); returns the slots' complex values (real parts)."""
    degree = len(plaintext)
    if not 0 < slots <= degree // 2:
        raise ValueError(f"ckks_decode: slots={slots} must be in (0, degree/2]")
    W = _int_words(q)
    t = _tensor.torch()
    x = t.from_numpy(_to_words(plaintext, W).copy()).to(_tensor.device())
    return _decode_words(x, W, q, scalingFactor, slots, p, degree, CKKS_M_FACTOR, ADD_NOISE)


class CKKSContext:
    """ckks_ctx.py:551-716."""

    def __init__(self, parameters: dict):
        self.parameters = parameters
        self.degree = parameters["degree"]
        self.num_slots = parameters.get("num_slots", self.degree // 2)
        self.scalingFactor = parameters.get("scalingFactor", 0.0)
        self.output_scale = parameters.get("output_scale", 0.0)
        self.q_towers = parameters["q_towers"]
        self.p_towers = parameters.get("p_towers", [])
        self.p = parameters.get("p", 0)
        self.CKKS_M_FACTOR = parameters.get("CKKS_M_FACTOR", 1)
        self.moduli = self.q_towers
        self.public_key = parameters.get("public_key", None)
        self.secret_key = parameters.get("secret_key", None)
        self.rotation_key = parameters.get("rotation_key", None)
        self.evaluation_key = parameters.get("evaluation_key", None)

    def _wrap(self, elements, moduli):
        shapes = {"batch": 1, "num_elements": len(elements), "num_moduli": len(moduli), "degree": self.degree,
                  "precision": 32}
        res = ct.Ciphertext(shapes, parameters={"moduli": list(moduli)})
        res.set_batch_ciphertext(_tensor.torch().stack([_tensor.to_u32(e) for e in elements])[None].contiguous())
        return res

    def encrypt(self, plaintext: ct.Ciphertext, v=None, e=None, ba=None, e_ref=None, v_ref=None) -> ct.Ciphertext:
        """ckks_ctx.py:569-607."""
        if self.public_key is None:
            raise ValueError("Public key is not set in the context.")
        element = plaintext.get_element(0)[0]
        c0, c1 = ckks_encrypt(element, self.public_key, self.q_towers,
                              noise_scale_degree=self.parameters.get("noise_scale_degree", 1),
                              sigma=self.parameters.get("sigma", sigma), v=v, e=e, ba=ba, e_ref=e_ref, v_ref=v_ref)
        return self._wrap([c0, c1], self.q_towers)

    def decrypt(self, ciphertext: ct.Ciphertext) -> ct.Ciphertext:
        """ckks_ctx.py:609-640."""
        if self.secret_key is None:
            raise ValueError("Secret key is not set in the context.")
        towers = self.q_towers[:ciphertext.num_moduli]
        res = ckks_decrypt(ciphertext.ciphertext[0], self.secret_key, towers)
        return self._wrap([res], towers)

    def encode(self, slots, shift: int = 0) -> ct.Ciphertext:
        """ckks_ctx.py:642-666."""
        enc = ckks_encode(slots, self.degree * 2, self.q_towers, self.p_towers, self.scalingFactor,
                          max_bits_in_word=self.parameters.get("max_bits_in_word", 61))
        return self._wrap([enc], self.q_towers)

    def decode(self, encoded_plaintext: ct.Ciphertext, is_ntt: bool = False):
        """ckks_ctx.py:668-701."""
        rns = _tensor.to_u32(encoded_plaintext.ciphertext[0, 0])
        towers = list(self.q_towers[:len(encoded_plaintext.moduli)])
        if is_ntt:
            rns = _negacyclic(towers, self.degree).inverse(rns.t().contiguous()).t().contiguous()
        words, big_q, W = _crt_words(rns, towers)
        # the reference returns jnp.array of the complex list: the same values as an array
        return _decode_words(words, W, big_q, self.output_scale, self.num_slots, self.p, self.degree,
                             self.CKKS_M_FACTOR, as_array=True)

    def multiply(self, ciphertext1, ciphertext2):
        raise NotImplementedError("Mul function not implemented")

    def rotate(self, ciphertext, shift: int):
        raise NotImplementedError("Rotate function not implemented")

    def rescale(self, ciphertext):
        raise NotImplementedError("Rescale function not implemented")

    def add(self, ciphertext1, ciphertext2):
        raise NotImplementedError("Add function not implemented")

    def sub(self, ciphertext1, ciphertext2):
        raise NotImplementedError("Sub function not implemented")
