"""Pure-Python restatement of jaxite_word's CKKS client side (the oracle for
the GPU encode / encrypt / decrypt / decode and key generation).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Python ints and CPython complex / float arithmetic, in the reference's
operation order, so every integer and every double matches the reference:

  ckks_ctx.py:23-110   _roots, _rot_group, _bitrev_inplace, FFTSpecialInv, FFTSpecial
  ckks_ctx.py:113-153  nearest_int, slot_to_coeffs, fit_to_native_vector
  ckks_ctx.py:156-235  ckks_encrypt (with given v, e)
  ckks_ctx.py:331-404  ckks_encode
  ckks_ctx.py:407-514  ckks_decode (without the optional noise)
  ckks_ctx.py:517-545  _crt_combine_rns_plaintext
  util.py:707-798      ntt_bit_reverse, ntt_negacyclic_bit_reverse
  key_gen.py:299-347   gen_pke_pair (with given s, a, e coefficients)
  key_gen.py:77-297    modulus_switch, gen_evaluation_key, key_switch_gen,
                       precompute_rotation_key_map, gen_rotation_key (given a, e)
The decrypt side (ckks_ctx.py:238-328) is ``cross_oracle.ckks_decrypt``.
"""

from __future__ import annotations

import cmath
import math
from typing import List

from .cross_oracle import bit_reverse_array, intt_negacyclic, root_of_unity

MAX_INT_64 = 9223372036854775295          # ckks_ctx.py:14


def _roots(m: int) -> List[complex]:
    """ckks_ctx.py:23-24."""
    return [cmath.exp(1j * 2 * math.pi * k / m) for k in range(m)]


def _rot_group(m: int, nh: int, g: int = 5) -> List[int]:
    """ckks_ctx.py:27-32."""
    r = [1]
    for _ in range(1, nh):
        r.append((r[-1] * g) % m)
    return r


def _bitrev_inplace(a: list) -> None:
    """ckks_ctx.py:35-45."""
    n = len(a)
    j = 0
    for i in range(1, n):
        bit = n >> 1
        while j & bit:
            j ^= bit
            bit >>= 1
        j ^= bit
        if i < j:
            a[i], a[j] = a[j], a[i]


def fft_special_inv(vals: list, m: int) -> None:
    """ckks_ctx.py:48-80, in place."""
    nh = len(vals)
    roots = _roots(m)
    rg = _rot_group(m, nh)
    length = nh
    while length >= 1:
        half = length >> 1
        lenq = length << 2
        step = m // lenq
        for i in range(0, nh, length):
            for j in range(half):
                idx = ((lenq - (rg[j] % lenq)) % lenq) * step
                u = vals[i + j]
                t = vals[i + j + half]
                vals[i + j] = u + t
                vals[i + j + half] = (u - t) * roots[idx]
        length >>= 1
    inv = 1.0 / nh
    for k in range(nh):
        vals[k] *= inv
    _bitrev_inplace(vals)


def fft_special(vals: list, m: int) -> None:
    """ckks_ctx.py:83-110, in place."""
    nh = len(vals)
    roots = _roots(m)
    rg = _rot_group(m, nh)
    _bitrev_inplace(vals)
    length = 2
    while length <= nh:
        half = length >> 1
        lenq = length << 2
        step = m // lenq
        for i in range(0, nh, length):
            for j in range(half):
                idx = (rg[j] % lenq) * step
                u = vals[i + j]
                v = vals[i + j + half] * roots[idx]
                vals[i + j] = u + v
                vals[i + j + half] = u - v
        length <<= 1


def nearest_int(x: float) -> int:
    """ckks_ctx.py:113-115."""
    return int(math.floor(x + 0.5)) if x >= 0 else -int(math.floor(-x + 0.5))


def fit_to_native_vector(vec, big_bound: int, modulus: int, ring_dim: int) -> List[int]:
    """ckks_ctx.py:128-153."""
    dslots = len(vec)
    if dslots == 0:
        return [0] * ring_dim
    half = big_bound >> 1
    diff = big_bound - modulus
    gap = ring_dim // dslots
    native = [0] * ring_dim
    for i, val in enumerate(vec):
        n = int(val)
        native[gap * i] = (n - diff) % modulus if n > half else n % modulus
    return native


def ntt_negacyclic(a, q: int, psi: int) -> List[int]:
    """util.py:707-798 (ntt_bit_reverse after the psi^i twist): natural-order
    evaluations of the negacyclic transform."""
    n = len(a)
    a = [(int(a[i]) * pow(psi, i, q)) % q for i in range(n)]
    omega = pow(psi, 2, q)
    bits = n.bit_length() - 1
    for i in range(n):
        j = int(format(i, f"0{bits}b")[::-1], 2) if bits else 0
        if i < j:
            a[i], a[j] = a[j], a[i]
    length = 2
    while length <= n:
        w_m = pow(omega, n // length, q)
        half = length // 2
        for i in range(0, n, length):
            w = 1
            for j in range(i, i + half):
                u = a[j]
                v = a[j + half] * w % q
                a[j] = (u + v) % q
                a[j + half] = (u - v) % q
                w = w * w_m % q
        length *= 2
    return a


def ckks_encode(slots, cycl_order: int, q_towers, scale: float, noise_scale_degree: int = 1,
                max_bits_in_word: int = 61):
    """ckks_ctx.py:331-404: (degree, moduli) evaluations, bit-reversed per tower."""
    nh = len(slots)
    n = 2 * nh
    m = cycl_order
    assert m == 4 * nh, "cycl_order must be 4*Nh for CKKS special FFT size"
    y = list(slots)
    fft_special_inv(y, m)
    coeffs = [v.real for v in y] + [v.imag for v in y]
    scaled = [scale * v for v in coeffs]
    logc = -10 ** 9
    for v in scaled:
        absv = abs(v)
        if absv != 0.0:
            logci = int(math.ceil(math.log2(absv)))
            if logc < logci:
                logc = logci
    if logc == -10 ** 9:
        logc = 0
    if logc < 0:
        raise ValueError("Scaling factor too small")
    log_valid = logc if logc <= max_bits_in_word else max_bits_in_word
    log_approx = logc - log_valid
    approx_factor = 2.0 ** log_approx
    ints_base = [nearest_int(v / approx_factor) for v in scaled]
    ints_base = [x + MAX_INT_64 if x < 0 else x for x in ints_base]
    elements = [fit_to_native_vector(ints_base, MAX_INT_64, q, n) for q in q_towers]
    if log_approx > 0:
        step = 1 << log_approx
        ints = [[x * step % q_towers[i] for x in elements[i]] for i in range(len(q_towers))]
    else:
        ints = elements
    if noise_scale_degree > 1:
        p = int(round(scale))
        if p != 1:
            power = pow(p, noise_scale_degree - 1)
            ints = [[x * power % q_towers[i] for x in ints[i]] for i in range(len(q_towers))]
    res = [bit_reverse_array(ntt_negacyclic(ints[i], q, root_of_unity(m, q))) for i, q in enumerate(q_towers)]
    return [[res[t][d] for t in range(len(q_towers))] for d in range(n)]


def ckks_encrypt(plaintext, public_key, q_towers, v, e, noise_scale_degree: int = 1):
    """ckks_ctx.py:156-235 with given v (moduli, degree) and e = (e0, e1)
    (moduli, degree), all in evaluation form.  plaintext (degree, moduli)."""
    degree = len(plaintext)
    nt = len(q_towers)
    e0, e1 = e
    ns = noise_scale_degree
    pk0 = public_key[0][:nt]
    pk1 = public_key[1][:nt]
    c0 = [[0] * nt for _ in range(degree)]
    c1 = [[0] * nt for _ in range(degree)]
    for i in range(degree):
        for j in range(nt):
            q = q_towers[j]
            val0 = (v[j][i] * pk0[j][i] + ns * e0[j][i]) % q
            c0[i][j] = (val0 + plaintext[i][j]) % q
            c1[i][j] = (v[j][i] * pk1[j][i] + ns * e1[j][i]) % q
    return [c0, c1]


def crt_combine(rns, moduli) -> List[int]:
    """ckks_ctx.py:517-545."""
    M = 1
    for q in moduli:
        M *= q
    Mi = [M // q for q in moduli]
    inv = [pow(a, -1, q) for a, q in zip(Mi, moduli)]
    out = []
    for row in rns:
        X = 0
        for i, q in enumerate(moduli):
            X += (int(row[i]) % int(q)) * int(Mi[i]) * int(inv[i])
        out.append(X % M)
    return out


def decode_stddev(cur: list) -> float:
    """ckks_ctx.py:448-481: the approximation-error estimate of ckks_decode."""
    n = len(cur)
    conj = [None] * n
    for idx in range(1, n):
        z = cur[n - idx]
        conj[idx] = complex(-z.imag, -z.real)
    conj[0] = complex(cur[0].real, -cur[0].imag)
    s = n
    if s == 1:
        sd = cur[0].imag
    else:
        dslots = s * 2
        cv = [cur[i] - conj[i] for i in range(s // 2 + 1)]
        mean = 2 * sum((c.real + c.imag) for c in cv[1:(s // 2)])
        mean += cv[0].imag
        mean += 2 * cv[s // 2].real
        mean /= (dslots - 1.0)
        var = 2 * sum(((c.real - mean) ** 2 + (c.imag - mean) ** 2) for c in cv[1:(s // 2)])
        var += (cv[0].imag - mean) ** 2
        var += 2 * (cv[s // 2].real - mean) ** 2
        var /= (dslots - 2.0)
        sd = 0.5 * math.sqrt(var)
    return sd


def decode_stddev_check(cur: list, degree: int, p: int) -> None:
    """ckks_ctx.py:482-486: the approximation-error check of ckks_decode."""
    sd = decode_stddev(cur)
    logstd = math.log2(sd) if sd > 0 else float("-inf")
    if logstd > p - 5.0:
        raise Exception("The decryption failed because the approximation error is too high. Check the parameters. ")


def ckks_decode(plaintext, scaling_factor: float, slots: int, q: int, p: int):
    """ckks_ctx.py:407-514 (no added noise): complex slot values."""
    degree = len(plaintext)
    q_half = q >> 1
    nh = degree // 2
    pow_p_pos = pow(2, p)
    pow_p = pow(2, -p)
    sf_pre = (1.0 / scaling_factor) * pow_p_pos
    re_l, im_l = [], []
    for i in range(slots):
        rv = plaintext[i]
        re_l.append(int(-((q - rv) * sf_pre) if rv > q_half else rv * sf_pre))
        iv = plaintext[i + nh]
        im_l.append(int(-((q - iv) * sf_pre) if iv > q_half else iv * sf_pre))
    cur = [complex(re_l[i], im_l[i]) for i in range(slots)]
    decode_stddev_check(cur, degree, p)
    n = len(cur)
    conj = [None] * n
    for idx in range(1, n):
        z = cur[n - idx]
        conj[idx] = complex(-z.imag, -z.real)
    conj[0] = complex(cur[0].real, -cur[0].imag)
    scale = 0.5 * pow_p
    cur = [complex(re_l[i] * scale + conj[i].real * scale, im_l[i] * scale + conj[i].imag * scale)
           for i in range(slots)]
    fft_special(cur, degree * 2)
    return [complex(cur[i].real, 0.0) for i in range(slots)]


def decode_rns(rns, q_towers, scaling_factor, slots, p, is_ntt=False):
    """CKKSContext.decode (ckks_ctx.py:668-701): rns (degree, moduli)."""
    degree = len(rns)
    nt = len(rns[0])
    q_towers = list(q_towers)[:nt]
    if is_ntt:
        cols = []
        for t in range(nt):
            col = bit_reverse_array([rns[d][t] for d in range(degree)])
            cols.append(intt_negacyclic(col, q_towers[t], root_of_unity(2 * degree, q_towers[t])))
        rns = [[cols[t][d] for t in range(nt)] for d in range(degree)]
    big_q = 1
    for q in q_towers:
        big_q *= q
    return ckks_decode(crt_combine(rns, q_towers), scaling_factor, slots, big_q, p)


def gen_pke_pair(q_towers, p_towers, degree, s_coeffs, a_coeffs, e_coeffs, noise_scale: int = 1):
    """key_gen.py:299-347 with given coefficient vectors: s and e as integers
    (one vector), a per modulus.  Evaluations are bit-reversed per tower."""
    moduli = list(q_towers) + list(p_towers)

    def ev(coefs, q):
        return bit_reverse_array(ntt_negacyclic([c % q for c in coefs], q, root_of_unity(2 * degree, q)))

    s = [ev(s_coeffs, q) for q in moduli]
    a = [ev(a_coeffs[i], q) for i, q in enumerate(moduli)]
    e = [ev(e_coeffs, q) for q in moduli]
    b = [[((e[i][j] * noise_scale) % q - (a[i][j] * s[i][j]) % q) % q for j in range(degree)]
         for i, q in enumerate(moduli)]
    return {"public_key": [b, a], "secret_key": s[:len(q_towers)]}


# ---------------------------------------------------------------------------
# key_gen.py:77-297: key-switching keys with given a, e
# ---------------------------------------------------------------------------

def modulus_switch(values, cur: int, target: int) -> List[int]:
    """key_gen.py:77-105 (list form): centred lift from Z_cur to Z_target."""
    thr = (cur + 1) // 2
    return [v if v < thr else target + v - cur for v in (int(x) for x in values)]


def key_switch_gen(s_old, s_new, q_list, p_list, a, e, noise_scale: int = 1, dnum: int = 3):
    """key_gen.py:147-254 with the a and e samples given (parts x (Q+P) x N,
    evaluation form).  s_old (Q x N) and s_new (Q x N) in evaluation form."""
    degree = len(s_new[0])
    q_list, p_list = list(q_list), list(p_list)
    s_out = [intt_negacyclic(bit_reverse_array(list(limb)), q, root_of_unity(2 * degree, q))
             for limb, q in zip(s_new, q_list)]
    s_qp = [list(r) for r in s_out] + [modulus_switch(s_out[0], q_list[0], p) for p in p_list]
    s_eva = [bit_reverse_array(ntt_negacyclic(limb, q, root_of_unity(2 * degree, q)))
             for limb, q in zip(s_qp, q_list + p_list)]
    P = 1
    for p in p_list:
        P *= p
    pmq = [P % q for q in q_list]
    size_q, size_qp = len(q_list), len(q_list) + len(p_list)
    per = (size_q + dnum - 1) // dnum
    parts = math.ceil(size_q / per)
    moduli = q_list + p_list
    b_parts = []
    for part in range(parts):
        start, end = per * part, min(size_q, per * part + per)
        rows = []
        for i in range(size_qp):
            q = moduli[i]
            ar, er, sr = a[part][i], e[part][i], s_eva[i]
            if start <= i < end:
                rows.append([((-ar[j] * sr[j]) % q + (pmq[i] * s_old[i][j]) % q + (noise_scale * er[j]) % q) % q
                             for j in range(degree)])
            else:
                rows.append([((-ar[j] * sr[j]) % q + (noise_scale * er[j]) % q) % q for j in range(degree)])
        b_parts.append(rows)
    return {"a": a, "b": b_parts, "modulus": {"Q": q_list, "P": p_list}, "P": p_list,
            "shape": (parts, size_qp, degree)}


def gen_evaluation_key(private_key, q_list, p_list, a, e, noise_scale: int = 1, dnum: int = 3):
    """key_gen.py:108-144: s_old = s^2 (evaluation form)."""
    s_old = [[(x * x) % q for x in row] for row, q in zip(private_key, q_list)]
    return key_switch_gen(s_old, private_key, q_list, p_list, a, e, noise_scale, dnum)


def precompute_rotation_key_map(n: int, k: int) -> List[int]:
    """key_gen.py:273-285."""
    logm = (2 * n).bit_length() - 1
    logn = n.bit_length() - 1
    out = [0] * n
    for j in range(n):
        mul = ((j << 1) + 1) * k
        idx = (mul - ((mul >> logm) << logm)) >> 1
        jrev = int(format(j, f"0{logn}b")[::-1], 2) if logn else 0
        out[jrev] = int(format(idx, f"0{logn}b")[::-1], 2) if logn else 0
    return out


def gen_rotation_key(sk, q_list, p_list, rot_index: int, a, e, noise_scale: int = 1, dnum: int = 3):
    """key_gen.py:288-296: key from s to s permuted by the rotation's map."""
    from .cross_oracle import find_automorphism_index_2n_complex
    n = len(sk[0])
    k = find_automorphism_index_2n_complex(rot_index, 2 * n)
    order = precompute_rotation_key_map(n, pow(k, -1, 2 * n))
    sk_rot = [[row[order[j]] for j in range(n)] for row in sk]
    return key_switch_gen(sk, sk_rot, q_list, p_list, a, e, noise_scale, dnum)
