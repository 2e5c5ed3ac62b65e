"""Numpy restatement of the jaxite_word CKKS hot path (the oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Every routine below restates one function of EfficientPPML/CROSS
``jaxite_word`` (cited as ``file.py:line``) with the same integer
semantics: uint32 / uint64 arithmetic with wrap-around, the same lazy
Barrett representatives, the same operand orders.  The only liberty taken is
how the exact u8 x u8 contractions of the Basis-Aligned Transformation are
evaluated: the reference's ``jnp.einsum(..., preferred_element_type=u32)``
sums are exact integers (at most 255*255*4*R < 2^32), so they are computed
here with float64 BLAS, which is exact below 2^53, and converted back.

Layouts follow the reference: ciphertexts are (batch, elements, r, c, limbs),
limb-innermost, uint32.
"""

from __future__ import annotations

import functools
import math
from typing import List, Sequence

import numpy as np

U32 = np.uint32
U64 = np.uint64


# ---------------------------------------------------------------------------
# util.py: number theory and parameter generation
# ---------------------------------------------------------------------------

def prime_factors(n: int) -> set:
    """util.py:174-190."""
    factors = set()
    while n % 2 == 0:
        factors.add(2)
        n //= 2
    p = 3
    while p * p <= n:
        while n % p == 0:
            factors.add(p)
            n //= p
        p += 2
    if n > 1:
        factors.add(n)
    return factors


@functools.lru_cache(maxsize=None)
def find_generator(q: int) -> int:
    """util.py:193-213: smallest generator of GF(q)^*."""
    phi = q - 1
    factors = prime_factors(phi)
    for g in range(2, q):
        if all(pow(g, phi // p, q) != 1 for p in factors):
            return g
    raise ValueError("No generator found, check that q is prime.")


@functools.lru_cache(maxsize=None)
def root_of_unity(m: int, q: int) -> int:
    """util.py:219-249: minimal primitive m-th root of unity mod q."""
    assert (q - 1) % m == 0, "q-1 must be divisible by m"
    g = find_generator(q)
    r = pow(g, (q - 1) // m, q)
    half = m // 2
    best = None
    for k in range(1, m):
        if math.gcd(k, m) != 1:
            continue
        psi = pow(r, k, q)
        if pow(psi, half, q) == q - 1 and pow(psi, m, q) == 1:
            if best is None or psi < best:
                best = psi
    assert best is not None, "No primitive m-th root found"
    return best


def is_prime_deterministic(n: int) -> bool:
    """util.py:385-428: trial division + deterministic Miller-Rabin."""
    if n < 2:
        return False
    if n in (2, 3):
        return True
    if n % 2 == 0:
        return False
    for p in (3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37, 41, 43, 47, 53):
        if n == p:
            return True
        if n % p == 0:
            return False
    d, s = n - 1, 0
    while d % 2 == 0:
        d //= 2
        s += 1
    for a in (2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37):
        if a >= n:
            break
        x = pow(a, d, n)
        if x in (1, n - 1):
            continue
        for _ in range(s - 1):
            x = pow(x, 2, n)
            if x == n - 1:
                break
        else:
            return False
    return True


def find_moduli_ntt(total_number: int, precision: int, ntt_length: int) -> List[int]:
    """util.py:431-458: largest primes k*ntt_length+1 below 2^precision."""
    out = []
    k = (2 ** precision - 1) // ntt_length
    while len(out) < total_number and k > 0:
        cand = k * ntt_length + 1
        if is_prime_deterministic(cand):
            out.append(cand)
        k -= 1
    return out


def compute_qhat(original_moduli: Sequence[int], target_moduli: Sequence[int]):
    """util.py:311-353 (non perf_test branch): QHatInvModq, QHatModp."""
    Q = 1
    for qi in original_moduli:
        Q *= qi
    qhat_inv, qhat = [], []
    for qi in original_moduli:
        h = Q // qi
        qhat.append(h)
        qhat_inv.append(pow(h, -1, qi))
    qhat_modp = [[qhat[i] % p for p in target_moduli] for i in range(len(original_moduli))]
    return qhat_inv, qhat_modp


def gamma_beta(moduli_list: Sequence[int]):
    """util.py:461-492 (non perf_test branch)."""
    Q = 1
    for m in moduli_list[:-1]:
        Q *= m
    q_l = moduli_list[-1]
    q_inv = pow(Q, -1, q_l)
    gamma_common = (Q * q_inv - 1) // q_l
    gammas = [gamma_common % moduli_list[i] for i in range(len(moduli_list) - 1)]
    betas = [pow(q_l, -1, moduli_list[i]) for i in range(len(moduli_list) - 1)]
    return np.array(gammas, U64), np.array(betas, U64)


def bit_reverse(x: int, bits: int) -> int:
    """util.py:614-620."""
    r = 0
    for i in range(bits):
        if (x >> i) & 1:
            r |= 1 << (bits - 1 - i)
    return r


def bit_reverse_perm(n: int) -> List[int]:
    """ntt_mm.py:261-274 (get_bit_reverse_perm inside memory_aligned_transformation)."""
    bits = n.bit_length() - 1
    return [bit_reverse(i, bits) for i in range(n)]


def bit_reverse_array(a):
    """util.py:623-630."""
    x = list(a)
    bits = len(x).bit_length() - 1
    for i in range(len(x)):
        j = bit_reverse(i, bits)
        if i < j:
            x[i], x[j] = x[j], x[i]
    return x


def precompute_auto_map(n: int, k: int) -> List[int]:
    """util.py:652-668 (OpenFHE PrecomputeAutoMap)."""
    m = n << 1
    logm = int(round(math.log2(m)))
    logn = int(round(math.log2(n)))
    pre = [0] * n
    for j in range(n):
        t = ((j << 1) + 1) * k
        idx = (t - ((t >> logm) << logm)) >> 1
        pre[bit_reverse(j, logn)] = bit_reverse(idx, logn)
    return pre


def find_automorphism_index_2n_complex(i: int, m: int) -> int:
    """util.py:671-693."""
    if i == 0:
        return 1
    if i == m - 1:
        return int(i)
    if m <= 0 or (m & (m - 1)) != 0:
        raise ValueError("m should be a power of two.")
    g0 = pow(5, -1, m) if i < 0 else 5
    g = g0
    for _ in range(1, abs(i)):
        g = (g * g0) & (m - 1)
    return int(g)


def parse_ciphertext_string(input_str: str):
    """util.py:545-608: OpenFHE 'Element k: i: EVAL: [...] modulus: q' text."""
    import re
    data, modulus = [], []
    cur = None
    pat = re.compile(r'^(\d+):\s*EVAL:\s*\[(.*?)\]\s*modulus:\s*(\d+)')
    for line in input_str.strip().splitlines():
        line = line.strip()
        rem = None
        if line.startswith("Element"):
            cur = []
            data.append(cur)
            hm = re.match(r'^Element\s+\d+:\s*(.*)', line)
            rem = hm.group(1).strip() if hm else ""
            if not rem:
                continue
        else:
            rem = line
        em = pat.match(rem)
        if em:
            cur.append([int(v) for v in em.group(2).split()])
            if len(data) == 1:
                modulus.append(int(em.group(3)))
    return data, modulus


def powers_mod(base: int, count: int, q: int) -> np.ndarray:
    """[base^i mod q for i < count] (the list comprehensions of
    ciphertext.py:231-248, hemul.py:48-95, herot.py:83-92), vectorised as
    base^(a*B+b) = (base^B)^a * base^b."""
    blk = 1
    while blk * blk < count:
        blk *= 2
    lo = np.array([pow(base, b, q) for b in range(blk)], U64)
    step = pow(base, blk, q)
    nhi = (count + blk - 1) // blk
    hi = np.array([pow(step, a, q) for a in range(nhi)], U64)
    return ((hi[:, None] * lo[None, :]) % U64(q)).reshape(-1)[:count]


def twiddle_matrix(rows: int, cols: int, q: int, omega: int) -> np.ndarray:
    """ntt_mm.py:75-98: T[r, c] = omega^(r*c) mod q (as int64)."""
    wr = np.array([pow(omega, r, q) for r in range(rows)], U64)
    out = np.empty((rows, cols), U64)
    col = np.ones(rows, U64)
    for c in range(cols):
        out[:, c] = col
        col = (col * wr) % U64(q)
    return out.astype(np.int64)


# ---------------------------------------------------------------------------
# finite_field.py: Barrett reduction
# ---------------------------------------------------------------------------

class Barrett:
    """finite_field.py:170-272 (BarrettContext)."""

    def __init__(self, moduli):
        if isinstance(moduli, int):
            moduli = [moduli]
        self.moduli = list(moduli)
        s = [2 * math.ceil(math.log2(m)) for m in self.moduli]          # :177
        w = [min(x, 32) for x in s]                                      # :178
        sw = [a - b for a, b in zip(s, w)]                               # :179
        mm = [math.floor(2 ** a / q) for a, q in zip(s, self.moduli)]   # :180
        self.barrett_s, self.barrett_w, self.barrett_s_w, self.barrett_m = s, w, sw, mm
        self.m = np.array(mm, U64)
        self.q = np.array(self.moduli, U64)
        self.w = np.array(w, U64)
        self.s_w = np.array(sw, U64)

    def reduce(self, z) -> np.ndarray:
        """finite_field.py:219-230: z (..., M) uint64 -> uint32 (lazy, one
        conditional subtraction)."""
        z = np.asarray(z).astype(U64)
        z1 = z & U64(0xFFFFFFFF)
        z2 = z >> self.w
        t = ((z1 * self.m) >> self.w) + (z2 * self.m)
        t = t >> self.s_w
        z = z - t * self.q
        return np.where(z >= self.q, z - self.q, z).astype(U32)

    def reduce_limb(self, z, i: int) -> np.ndarray:
        """Same arithmetic as reduce() with the constants of limb i
        (finite_field.py:233-262 gives identical values)."""
        z = np.asarray(z).astype(U64)
        m, q, w, sw = self.m[i], self.q[i], self.w[i], self.s_w[i]
        z1 = z & U64(0xFFFFFFFF)
        t = ((z1 * m) >> w) + ((z >> w) * m)
        t = t >> sw
        z = z - t * q
        return np.where(z >= q, z - q, z).astype(U32)


# ---------------------------------------------------------------------------
# ntt_mm.py: BAT 3-step NTT
# ---------------------------------------------------------------------------

def _exact_u8_matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Exact integer product of two u8 matrices (sums < 2^53)."""
    assert 255 * 255 * a.shape[1] < 2 ** 53
    return (a.astype(np.float64) @ b.astype(np.float64)).astype(np.int64)


def _combine_bytes(p4: np.ndarray) -> np.ndarray:
    """ntt_mm.py:33-37: sum_p (acc_p << 8p) in uint64."""
    p4 = p4.astype(U64)
    return p4[..., 0] + (p4[..., 1] << U64(8)) + (p4[..., 2] << U64(16)) + (p4[..., 3] << U64(24))


def bat_col(x: np.ndarray, tbat: np.ndarray) -> np.ndarray:
    """einsum 'brcq,zqrp->bzcp' + byte recombination (ntt_mm.py:315,372,405).

    x: (B, R, C) uint32; tbat: (Z, 4, R, 4) uint8 -> (B, Z, C) uint64.
    """
    B, R, C = x.shape
    Z = tbat.shape[0]
    xb = np.ascontiguousarray(x.astype(U32)).view(np.uint8).reshape(B, R, C, 4)
    a = xb.transpose(0, 2, 1, 3).reshape(B * C, R * 4)
    t = tbat.transpose(2, 1, 0, 3).reshape(R * 4, Z * 4)
    p = _exact_u8_matmul(a, t).reshape(B, C, Z, 4)
    return _combine_bytes(p).transpose(0, 2, 1)


def bat_row(x: np.ndarray, tbat: np.ndarray) -> np.ndarray:
    """einsum 'brcq,cqnp->brnp' + byte recombination (ntt_mm.py:319,376,401).

    x: (B, R, C) uint32; tbat: (C, 4, Nn, 4) uint8 -> (B, R, Nn) uint64.
    """
    B, R, C = x.shape
    Nn = tbat.shape[2]
    xb = np.ascontiguousarray(x.astype(U32)).view(np.uint8).reshape(B * R, C * 4)
    t = tbat.reshape(C * 4, Nn * 4)
    p = _exact_u8_matmul(xb, t).reshape(B, R, Nn, 4)
    return _combine_bytes(p)


def basis_aligned_transformation(matrix: np.ndarray, moduli: Sequence[int]) -> np.ndarray:
    """ntt_mm.py:248-255: (rows, cols, M) u32 -> (rows, 4[q], cols, 4[p], M) u8
    with entry [x, q, y, p, m] = byte_p((T[x, y, m] << 8q) mod q_m)."""
    mu = matrix.astype(U64)
    shifted = np.array([mu << U64(8 * i) for i in range(4)], U64)     # (4, rows, cols, M)
    red = (shifted % np.array(moduli, U64)).astype(U32)
    u8 = np.ascontiguousarray(red).view(np.uint8).reshape(*red.shape, 4)  # (4, rows, cols, M, 4)
    return np.ascontiguousarray(u8.transpose(1, 0, 2, 4, 3))


class NTTBarrett:
    """ntt_mm.py:125-429 (NTTCiphertextContextBase + NTTCiphertextBarrettContext),
    non-perf_test constants."""

    def __init__(self, moduli, r: int, c: int):
        if isinstance(moduli, int):
            moduli = [moduli]
        self.moduli = list(moduli)
        self.r, self.c = r, c
        self.ff = Barrett(self.moduli)
        n = r * c
        self.psi_list = [root_of_unity(2 * n, q) for q in self.moduli]           # :148
        self.omega_list = [(p * p) % q for p, q in zip(self.psi_list, self.moduli)]  # :149
        perm_r, perm_c = bit_reverse_perm(r), bit_reverse_perm(c)                # :257-277
        t1, t2, t3, it1, it2, it3 = [], [], [], [], [], []
        for i, q in enumerate(self.moduli):                                      # :186-209
            om = self.omega_list[i]
            om_col, om_row = pow(om, c, q), pow(om, r, q)
            t1.append(twiddle_matrix(r, r, q, om_col)[perm_r, :])
            t2.append(twiddle_matrix(r, c, q, om)[perm_r, :])
            t3.append(twiddle_matrix(c, c, q, om_row)[:, perm_c])
            inv_col, inv_row = pow(om_col, -1, q), pow(om_row, -1, q)            # :211-240
            a = twiddle_matrix(c, c, q, inv_row)[perm_c, :]
            b = twiddle_matrix(r, c, q, pow(om, -1, q))[perm_r, :]  # gen_twiddle_matrix_inv
            d = twiddle_matrix(r, r, q, inv_col)[:, perm_r]
            b = (b * pow(c, -1, q)) % q
            d = (d * pow(r, -1, q)) % q
            it1.append(a)
            it2.append(b)
            it3.append(d)
        st = lambda lst: np.stack(lst, axis=-1).astype(U32)  # noqa: E731 -- moduli last
        self.ntt_tf_step1, self.ntt_tf_step2, self.ntt_tf_step3 = st(t1), st(t2), st(t3)
        self.intt_tf_step1, self.intt_tf_step2, self.intt_tf_step3 = st(it1), st(it2), st(it3)
        self.ntt_bat_tf_step1 = basis_aligned_transformation(self.ntt_tf_step1, self.moduli)
        self.ntt_bat_tf_step3 = basis_aligned_transformation(self.ntt_tf_step3, self.moduli)
        self.intt_bat_tf_step1 = basis_aligned_transformation(self.intt_tf_step1, self.moduli)
        self.intt_bat_tf_step3 = basis_aligned_transformation(self.intt_tf_step3, self.moduli)

    def ntt(self, v: np.ndarray) -> np.ndarray:
        """ntt_mm.py:351-378 (per limb, as ntt_limb 295-321)."""
        v = np.asarray(v).astype(U32)
        B = v.shape[0]
        out = np.empty((B, self.r, self.c, len(self.moduli)), U32)
        for m in range(len(self.moduli)):
            s1 = bat_col(v[..., m], self.ntt_bat_tf_step1[..., m])
            r1 = self.ff.reduce_limb(s1, m)
            r2 = self.ff.reduce_limb(r1.astype(U64) * self.ntt_tf_step2[..., m].astype(U64), m)
            s3 = bat_row(r2, self.ntt_bat_tf_step3[..., m])
            out[..., m] = self.ff.reduce_limb(s3, m)
        return out

    def intt(self, v: np.ndarray) -> np.ndarray:
        """ntt_mm.py:380-407 (per limb, as intt_limb 323-349)."""
        v = np.asarray(v).astype(U32)
        B = v.shape[0]
        out = np.empty((B, self.r, self.c, len(self.moduli)), U32)
        for m in range(len(self.moduli)):
            s1 = bat_row(v[..., m], self.intt_bat_tf_step1[..., m])
            r1 = self.ff.reduce_limb(s1, m)
            r2 = self.ff.reduce_limb(r1.astype(U64) * self.intt_tf_step2[..., m].astype(U64), m)
            s3 = bat_col(r2, self.intt_bat_tf_step3[..., m])
            out[..., m] = self.ff.reduce_limb(s3, m)
        return out


# ---------------------------------------------------------------------------
# bconv.py: basis conversion
# ---------------------------------------------------------------------------

class BConvBarrett:
    """bconv.py:40-258 (BConv + BConvBarrett), non-perf_test constants."""

    def __init__(self, overall_moduli):
        self.overall_moduli = list(overall_moduli)
        self.controls = []

    def control_gen(self, control_indices_list):
        """bconv.py:101-155."""
        self.controls = []
        for src_idx, dst_idx in control_indices_list:
            src = [self.overall_moduli[i] for i in src_idx]
            dst = [self.overall_moduli[i] for i in dst_idx]
            qhat_inv, qhat_modp = compute_qhat(src, dst)                          # :73
            qhat_modp = np.array(qhat_modp, U64).reshape(len(src), len(dst))
            shifted = np.array([qhat_modp << U64(8 * a) for a in range(4)], U64)  # :163-167
            red = (shifted % np.array(dst, U64)).astype(U32)
            u8 = np.ascontiguousarray(red).view(np.uint8).reshape(4, len(src), len(dst), 4)
            bat = np.ascontiguousarray(u8.transpose(1, 0, 2, 3).reshape(-1, len(dst), 4))  # :97
            self.controls.append(dict(src=src, dst=dst, ff_src=Barrett(src), ff_dst=Barrett(dst),
                                      qhat_inv=np.array(qhat_inv, U64), qhat_modp=qhat_modp, bat=bat))

    def basis_change_bat(self, x, control_index: int = 0) -> np.ndarray:
        """bconv.py:215-252: (..., sizeQ) -> (..., sizeP) uint32."""
        ctl = self.controls[control_index]
        x = np.asarray(x).astype(U64)
        cval = ctl["ff_src"].reduce(x * ctl["qhat_inv"])                         # :241-244
        lead = cval.shape[:-1]
        sq, sp = len(ctl["src"]), len(ctl["dst"])
        a = np.ascontiguousarray(cval).view(np.uint8).reshape(-1, 4 * sq)        # lhs.view(u8) :31
        p = _exact_u8_matmul(a, ctl["bat"].reshape(4 * sq, sp * 4)).reshape(*lead, sp, 4)
        return ctl["ff_dst"].reduce(_combine_bytes(p))                          # :247-250

    def basis_change(self, x, control_index: int = 0) -> np.ndarray:
        """bconv.py:173-212 (u64 MAC path)."""
        ctl = self.controls[control_index]
        x = np.asarray(x).astype(U64)
        cval = ctl["ff_src"].reduce(x * ctl["qhat_inv"]).astype(U64)
        acc = np.zeros(cval.shape[:-1] + (len(ctl["dst"]),), U64)
        for i in range(len(ctl["src"])):
            acc = acc + cval[..., i:i + 1] * ctl["qhat_modp"][i][None, :]
        return ctl["ff_dst"].reduce(acc)


# ---------------------------------------------------------------------------
# ciphertext.py: rescale, tensor product, key switch
# ---------------------------------------------------------------------------

def default_rc(degree: int):
    """ciphertext.py:63,69-70: r = 2^(floor(log2 N / 2)), c = N / r."""
    log_degree = int(math.log2(degree))
    r = 1 << (log_degree // 2)
    return r, degree // r


def _ntt_flat(ctx: NTTBarrett, x: np.ndarray, inverse: bool) -> np.ndarray:
    """ciphertext.py:154-164: reshape to (-1, r, c, M), transform, reshape back."""
    shape = x.shape
    y = x.reshape(-1, ctx.r, ctx.c, len(ctx.moduli))
    y = ctx.intt(y) if inverse else ctx.ntt(y)
    return y.reshape(shape)


def _modmul(ff: Barrett, x, table) -> np.ndarray:
    """ciphertext.py:189-193."""
    return ff.reduce(np.asarray(x).astype(U64) * np.asarray(table).astype(U64)).astype(U32)


class RescalePlan:
    """ciphertext.py:223-303 (modulus_switch_control_gen + rescale)."""

    def __init__(self, moduli, r: int, c: int):
        self.moduli = list(moduli)
        self.r, self.c = r, c
        n = r * c
        L = len(self.moduli)
        psis = [root_of_unity(2 * n, q) for q in self.moduli]
        pw = [powers_mod(psis[i], n, q) for i, q in enumerate(self.moduli)]
        gammas, betas = gamma_beta(self.moduli)
        gps = np.stack([(gammas[i] * pw[i]) % U64(self.moduli[i]) for i in range(L - 1)], 0)  # :240-243
        self.gammas_power_of_psi_no_last = gps.T.reshape(r, c, L - 1)
        inv_last = pow(psis[-1], -1, self.moduli[-1])
        self.power_of_last_tower_inv_psi = powers_mod(inv_last, n, self.moduli[-1]).reshape(r, c, 1)
        self.betas = betas
        self.threshold = np.uint32((self.moduli[-1] + 1) // 2)                  # :260
        self.drop_last = np.array(self.moduli[:-1], U64)
        self.q_last = self.moduli[-1]
        self.ntt_last = NTTBarrett([self.q_last], r, c)                          # :251 ct_last_limb
        self.ntt_rest = NTTBarrett(self.moduli[:-1], r, c)                       # after drop_last_modulus
        self.ff_last = Barrett([self.q_last])
        self.ff_rest = Barrett(self.moduli[:-1])

    def rescale(self, x: np.ndarray) -> np.ndarray:
        """ciphertext.py:267-303. x: (B, E, r, c, L) -> (B, E, r, c, L-1)."""
        x = np.asarray(x).astype(U32)
        last = _ntt_flat(self.ntt_last, x[..., -1:].astype(U32), inverse=True)   # :279-281
        last = _modmul(self.ff_last, last, self.power_of_last_tower_inv_psi)     # :282
        cond = last < self.threshold                                             # :285
        ge = self.drop_last - U64(self.q_last) + last.astype(U64)                # :287 (u64 wrap)
        coef = np.where(cond, last.astype(U64), ge)
        tw = coef.astype(U64) * self.gammas_power_of_psi_no_last.astype(U64)     # :291-293
        red = self.ff_rest.reduce(tw)                                            # :295
        nt = _ntt_flat(self.ntt_rest, red, inverse=False)                        # :296
        acc = x[..., :-1].astype(U64) * self.betas + nt.astype(U64)              # :299-301
        return self.ff_rest.reduce(acc)                                          # :302


def ciphertext_mult(ct: np.ndarray, ff: Barrett):
    """ciphertext.py:309-324: (B, 4, ...) -> ((B, 2, ...), (B, 1, ...))."""
    a0, a1, b0, b1 = (ct[:, i].astype(U64) for i in range(4))
    mul0 = ff.reduce(a0 * b0)
    mul2 = ff.reduce(a1 * b1)
    mul1 = ff.reduce(a0 * b1 + a1 * b0)
    return np.concatenate([mul0[:, None], mul1[:, None]], axis=1), mul2[:, None]


def digit_partition(size_q: int, dnum: int):
    """ciphertext.py:353-379 / herot.py:113-150: digits, complements, restore maps."""
    alpha = (size_q + dnum - 1) // dnum
    num_parts = (size_q + alpha - 1) // alpha
    groups = []
    for i in range(size_q):
        if i % alpha == 0:
            groups.append([i])
        else:
            groups[-1].append(i)
    return alpha, num_parts, groups


def _restore(sel, non_sel):
    order = list(sel) + list(non_sel)
    rest = [0] * len(order)
    for pos, val in enumerate(order):
        rest[val] = pos
    return rest


class KeySwitchPlan:
    """ciphertext.py:329-519 (key_switch_control_gen + key_switch) for a ciphertext
    with moduli `current` extended by `extend` with `dnum` digits."""

    def __init__(self, current, extend, dnum, evk_a, evk_b, r, c):
        self.current, self.extend = list(current), list(extend)
        dle = self.current + self.extend
        self.dle = dle
        self.r, self.c = r, c
        n = r * c
        Lc, K = len(self.current), len(self.extend)
        psis = [root_of_unity(2 * n, q) for q in dle]
        self.dl_power_of_psi = np.stack([powers_mod(psis[i], n, q) for i, q in enumerate(dle)], -1).reshape(r, c, len(dle))
        self.alpha, self.num_parts, groups = digit_partition(Lc, dnum)
        self.sel = groups[:self.num_parts]
        self.non_sel = [[i for i in range(len(dle)) if i not in g] for g in self.sel]
        self.rest = [_restore(s, ns) for s, ns in zip(self.sel, self.non_sel)]
        inv = [pow(psis[i], -1, q) for i, q in enumerate(self.current)]
        self.inv_psi = np.stack([powers_mod(inv[i], n, q) for i, q in enumerate(self.current)], -1).reshape(r, c, Lc)
        self.bconv = BConvBarrett(dle)
        self.bconv.control_gen([(s, ns) for s, ns in zip(self.sel, self.non_sel)])
        self.ntt_cur = NTTBarrett(self.current, r, c)
        self.ff_cur = Barrett(self.current)
        self.part_ntt = [NTTBarrett([dle[i] for i in ns], r, c) for ns in self.non_sel]
        self.part_ff = [Barrett([dle[i] for i in ns]) for ns in self.non_sel]
        self.ff_dle = Barrett(dle)
        ea, eb = np.asarray(evk_a), np.asarray(evk_b)                             # :450-451
        self.evk_a = np.concatenate([ea[..., :Lc], ea[..., ea.shape[-1] - K:]], -1).reshape(-1, r, c, len(dle)).astype(U64)
        self.evk_b = np.concatenate([eb[..., :Lc], eb[..., eb.shape[-1] - K:]], -1).reshape(-1, r, c, len(dle)).astype(U64)

    def key_switch(self, x: np.ndarray) -> np.ndarray:
        """ciphertext.py:455-519. x: (B, 1, r, c, Lc) NTT form -> (B, 2, r, c, Lc+K)."""
        input_ntt = np.asarray(x).astype(U32)
        coef = _ntt_flat(self.ntt_cur, input_ntt, inverse=True)                 # :480
        coef = _modmul(self.ff_cur, coef, self.inv_psi)                           # :481
        res0 = res1 = None
        for part in range(self.num_parts):
            sel, ns = self.sel[part], self.non_sel[part]
            tw = self.dl_power_of_psi[..., ns]                                   # :489
            ev = self.bconv.basis_change_bat(coef[..., sel], part)               # :490-493
            ev = _modmul(self.part_ff[part], ev, tw)                              # :496
            ev = _ntt_flat(self.part_ntt[part], ev, inverse=False)               # :499
            ext = np.concatenate([input_ntt[..., sel], ev], -1)[..., self.rest[part]]  # :502-506
            t0 = ext.astype(U64) * self.evk_b[part][None, None]
            t1 = ext.astype(U64) * self.evk_a[part][None, None]
            res0 = t0 if res0 is None else res0 + t0                             # :508-513
            res1 = t1 if res1 is None else res1 + t1
        return self.ff_dle.reduce(np.concatenate([res0, res1], axis=1))          # :515-518


# ---------------------------------------------------------------------------
# hemul.py: HE-Mult with relinearisation
# ---------------------------------------------------------------------------

class HEMul:
    """hemul.py:11-217 (num_eval_mult = 1 as in every reference caller)."""

    def __init__(self, batch, r, c, dnum, num_eval_mult, original_moduli, extend_moduli):
        assert num_eval_mult == 1
        self.batch, self.r, self.c, self.dnum = batch, r, c, dnum
        self.Q = list(original_moduli)
        self.P = list(extend_moduli)
        self.Qd = self.Q[:-1]
        n = r * c
        L1, K = len(self.Qd), len(self.P)
        self.rescale_plan = RescalePlan(self.Q, r, c)                            # :57-59
        self.ff_obj = Barrett(self.Qd)
        self.ntt_obj = NTTBarrett(self.Qd, r, c)
        rd, cd = default_rc(n)                                                   # :76-77 ct_extend
        self.ntt_ext = NTTBarrett(self.P, rd, cd)
        self.ff_ext = Barrett(self.P)
        dle = self.Qd + self.P
        psis = [root_of_unity(2 * n, q) for q in dle]                            # :86-95
        self.power_of_psi = np.stack([powers_mod(psis[i], n, dle[i]) for i in range(L1)], -1).reshape(r, c, L1)
        inv = [pow(psis[i], -1, dle[i]) for i in range(len(dle))]
        self.power_of_inv_psi_approx_down = np.stack(
            [powers_mod(inv[i], n, dle[i]) for i in range(L1, L1 + K)], -1).reshape(r, c, K)
        self.bconv = BConvBarrett(dle)                                           # :98-103
        self.bconv.control_gen([(list(range(L1, L1 + K)), list(range(L1)))])
        Pprod = 1
        for p in self.P:
            Pprod *= p
        self.PInvModq = np.array([pow(Pprod, -1, q) for q in self.Qd if q not in self.P], U32)  # :105-111
        self.q_corr = np.array(self.Qd, U32)

    def setup_relinearization(self, evk_a, evk_b):
        """hemul.py:134-151."""
        self.ks = KeySwitchPlan(self.Qd, self.P, self.dnum, evk_a, evk_b, self.r, self.c)

    def mul(self, ct: np.ndarray) -> np.ndarray:
        """hemul.py:153-217: (B, 4, r, c, L) -> (B, 2, r, c, L-1)."""
        L1 = len(self.Qd)
        K = len(self.P)
        x = self.rescale_plan.rescale(np.asarray(ct).astype(U32))                # :162-164
        post, d2 = ciphertext_mult(x, self.ff_obj)                               # :167
        ks = self.ks.key_switch(d2)                                              # :170-172
        ext = _ntt_flat(self.ntt_ext, ks[..., L1:L1 + K], inverse=True)          # :179-180
        ext = _modmul(self.ff_ext, ext, self.power_of_inv_psi_approx_down)      # :181
        nb = self.bconv.basis_change_bat(ext, 0)                                 # :183-186
        outs = []
        q = np.array(self.Qd, U32)
        for e in range(nb.shape[1]):                                             # :188-209
            t = _modmul(self.ff_obj, nb[:, e:e + 1], self.power_of_psi)
            t = _ntt_flat(self.ntt_obj, t, inverse=False)
            a = ks[:, e:e + 1, ..., :L1]
            sub = np.where(a < t, a + q - t, a - t)                              # u32 wrap
            outs.append(_modmul(self.ff_obj, sub, self.PInvModq))
        down = np.concatenate(outs, axis=1)
        res = post + down                                                        # :214 (u32 wrap)
        return np.where(res >= self.q_corr, res - self.q_corr, res)


# ---------------------------------------------------------------------------
# herot.py: HE-Rotate
# ---------------------------------------------------------------------------

class HERot:
    """herot.py:55-302.  Every internal Ciphertext is built without a
    finite_field_context (herot.py:160-175), so all transforms use the default
    (r, c) factorisation of ciphertext.py:69-70."""

    def __init__(self, r, c, dnum, q_moduli, p_moduli):
        self.r, self.c, self.dnum = r, c, dnum
        self.Q, self.P = list(q_moduli), list(p_moduli)
        self.overall = self.Q + self.P

    def control_gen(self, batch=1):
        """herot.py:66-175."""
        n = self.r * self.c
        L, K = len(self.Q), len(self.P)
        ov = self.overall
        psis = [root_of_unity(2 * n, q) for q in ov]
        self.power_of_psi = np.stack([powers_mod(psis[i], n, ov[i]) for i in range(len(ov))], -1)   # (N, L+K)
        inv = [pow(psis[i], -1, ov[i]) for i in range(len(ov))]
        pinv = np.stack([powers_mod(inv[i], n, ov[i]) for i in range(len(ov))], -1)
        self.power_of_inv_psi = pinv[:, :L]
        self.power_of_inv_psi_approx_down = pinv[:, L:L + K]
        Pprod = 1
        for p in self.P:
            Pprod *= p
        self.PInvModq = np.array([pow(Pprod, -1, q) for q in ov if q not in self.P], U32)
        self.alpha, self.num_parts, groups = digit_partition(L, self.dnum)
        self.sel = groups[:self.num_parts]
        self.non_sel = [[i for i in range(len(ov)) if i not in g] for g in self.sel]
        self.rest = [_restore(s, ns) for s, ns in zip(self.sel, self.non_sel)]
        ctl = [(s, ns) for s, ns in zip(self.sel, self.non_sel)]
        ctl.append((list(range(L, L + K)), list(range(L))))
        self.bconv = BConvBarrett(ov)
        self.bconv.control_gen(ctl)
        rd, cd = default_rc(n)
        self.ntt_in = NTTBarrett(self.Q, rd, cd)
        self.ff_in = Barrett(self.Q)
        self.part_ntt = [NTTBarrett([ov[i] for i in ns], rd, cd) for ns in self.non_sel]
        self.part_ff = [Barrett([ov[i] for i in ns]) for ns in self.non_sel]
        self.ff_full = Barrett(ov)
        self.ntt_approx = NTTBarrett(self.P, rd, cd)
        self.ff_approx = Barrett(self.P)

    def setup_rotate(self, evk_a, evk_b, coef_map):
        """herot.py:178-181."""
        self.evk_a = np.asarray(evk_a).astype(U64)
        self.evk_b = np.asarray(evk_b).astype(U64)
        self.coef_map = np.asarray(coef_map, np.int64)

    def rotate(self, ct: np.ndarray) -> np.ndarray:
        """herot.py:183-302: (B, 2, r, c, L) -> (B, 2, N, L)."""
        ct = np.asarray(ct).astype(U32)
        B = ct.shape[0]
        n = self.r * self.c
        L, K = len(self.Q), len(self.P)
        lead = ct.shape[2:-1]
        pip = self.power_of_psi.reshape(*lead, L + K)
        in_tower = ct[:, -1:, ..., :L]                                            # :201
        coef = _ntt_flat(self.ntt_in, in_tower, inverse=True)                    # :206
        coef = _modmul(self.ff_in, coef, self.power_of_inv_psi.reshape(*lead, L))  # :207
        res0 = res1 = None
        for part in range(self.dnum):                                            # :212
            sel, ns = self.sel[part], self.non_sel[part]
            ev = self.bconv.basis_change_bat(coef[..., sel], part)
            ev = _modmul(self.part_ff[part], ev, pip[..., ns])
            ev = _ntt_flat(self.part_ntt[part], ev, inverse=False)
            ext = np.concatenate([in_tower[..., sel], ev], -1)[..., self.rest[part]]
            t0 = ext.astype(U64) * self.evk_b[part][None, None]
            t1 = ext.astype(U64) * self.evk_a[part][None, None]
            res0 = t0 if res0 is None else res0 + t0
            res1 = t1 if res1 is None else res1 + t1
        ks = self.ff_full.reduce(np.concatenate([res0, res1], axis=1))          # :244-247
        q = np.array(self.Q, U32)
        outs = []
        for e in range(ks.shape[1]):                                             # :255-287
            sl = ks[:, e:e + 1, ..., L:L + K]
            t = _ntt_flat(self.ntt_approx, sl, inverse=True)
            t = _modmul(self.ff_approx, t, self.power_of_inv_psi_approx_down.reshape(*lead, K))
            t = self.bconv.basis_change_bat(t, self.dnum)
            t = _modmul(self.ff_in, t, pip[..., :L])
            t = _ntt_flat(self.ntt_in, t, inverse=False)
            a = ks[:, e:e + 1, ..., :L]
            sub = np.where(a < t, a + q - t, a - t)
            outs.append(_modmul(self.ff_in, sub, self.PInvModq))
        down = np.concatenate(outs, axis=1)
        base0 = ct[:, 0:1] + down[:, 0:1]                                        # :292-296
        base0 = np.where(base0 >= q, base0 - q, base0)
        res = down.copy()
        res[:, 0:1] = base0
        return np.take(res.reshape(-1, 2, n, L), self.coef_map, axis=2)          # :300


# ---------------------------------------------------------------------------
# add.py
# ---------------------------------------------------------------------------

def jax_add(a, b, moduli) -> np.ndarray:
    """add.py:7-27: (E, L, N) + (E, L, N), subtract q where result > q."""
    a = np.asarray(a)
    b = np.asarray(b)
    q = np.asarray(moduli).astype(a.dtype)[None, :, None]
    res = a + b
    return np.where(res > q, res - q, res)


# ---------------------------------------------------------------------------
# ckks_ctx.py: decrypt / decode (host side of the end-to-end check)
# ---------------------------------------------------------------------------

def intt_negacyclic(a, q, psi):
    """util.py:729-760 + 801-827 (intt_bit_reverse, intt_negacyclic_bit_reverse)."""
    n = len(a)
    a = list(a)
    omega = pow(psi, 2, q)
    inv_root = pow(omega, -1, q)
    length = n
    while length >= 2:
        w_m = pow(inv_root, n // length, q)
        half = length // 2
        for i in range(0, n, length):
            w = 1
            for j in range(i, i + half):
                u, v = a[j], a[j + half]
                a[j] = (u + v) % q
                a[j + half] = ((u - v) % q) * w % q
                w = w * w_m % q
        length //= 2
    a = bit_reverse_array(a)
    inv_n = pow(n, -1, q)
    a = [x * inv_n % q for x in a]
    psi_inv = pow(psi, -1, q)
    return [(a[i] * pow(psi_inv, i, q)) % q for i in range(n)]


def ckks_decrypt(ciphertext, secret_key, q_towers):
    """ckks_ctx.py:238-328.  ciphertext: list of elements (degree, moduli);
    secret_key (moduli, degree) in evaluation form."""
    num_el = len(ciphertext)
    degree = len(ciphertext[0])
    nt = len(ciphertext[0][0])
    s = secret_key[:nt] if nt < len(secret_key) else secret_key
    res = [[ciphertext[0][d][m] for m in range(nt)] for d in range(degree)]
    cur = [list(row) for row in s]
    for i in range(1, num_el):
        ci = ciphertext[i]
        for d in range(degree):
            for m in range(nt):
                res[d][m] = (res[d][m] + (ci[d][m] * cur[m][d]) % q_towers[m]) % q_towers[m]
        if i < num_el - 1:
            cur = [[(cur[m][d] * s[m][d]) % q_towers[m] for d in range(degree)] for m in range(nt)]
    out = [[0] * nt for _ in range(degree)]
    for m in range(nt):
        col = bit_reverse_array([res[d][m] for d in range(degree)])
        coef = intt_negacyclic(col, q_towers[m], root_of_unity(2 * degree, q_towers[m]))
        for d in range(degree):
            out[d][m] = coef[d]
    return out


def _fft_special(vals, m):
    """ckks_ctx.py:83-110 (FFTSpecial)."""
    import cmath
    nh = len(vals)
    roots = [cmath.exp(1j * 2 * math.pi * k / m) for k in range(m)]
    rg = [1]
    for _ in range(1, nh):
        rg.append((rg[-1] * 5) % m)
    vals = list(vals)
    n = nh
    j = 0
    for i in range(1, n):                                                        # _bitrev_inplace
        bit = n >> 1
        while j & bit:
            j ^= bit
            bit >>= 1
        j ^= bit
        if i < j:
            vals[i], vals[j] = vals[j], vals[i]
    length = 2
    while length <= nh:
        half = length >> 1
        lenq = length << 2
        step = m // lenq
        for i in range(0, nh, length):
            for jj in range(half):
                idx = (rg[jj] % lenq) * step
                u = vals[i + jj]
                v = vals[i + jj + half] * roots[idx]
                vals[i + jj] = u + v
                vals[i + jj + half] = u - v
        length <<= 1
    return vals


def ckks_decode(rns_poly, q_towers, scaling_factor, slots, p, ckks_m_factor=1):
    """ckks_ctx.py:668-701 (decode, is_ntt=False) -> 517-545 (CRT) -> 407-514
    (ckks_decode without the optional noise)."""
    degree = len(rns_poly)
    nt = len(rns_poly[0])
    q_towers = list(q_towers)[:nt]
    M = 1
    for q in q_towers:
        M *= q
    Mi = [M // q for q in q_towers]
    inv = [pow(a, -1, q) for a, q in zip(Mi, q_towers)]
    plain = []
    for d in range(degree):
        X = 0
        for i in range(nt):
            X += (int(rns_poly[d][i]) % q_towers[i]) * Mi[i] * inv[i]
        plain.append(X % M)
    q = M
    q_half = q >> 1
    nh = degree // 2
    sf_pre = (1.0 / scaling_factor) * pow(2, p)
    re_l, im_l = [], []
    for i in range(slots):
        rv = plain[i]
        re_l.append(int(-((q - rv) * sf_pre) if rv > q_half else rv * sf_pre))
        iv = plain[i + nh]
        im_l.append(int(-((q - iv) * sf_pre) if iv > q_half else iv * sf_pre))
    cur = [complex(re_l[i], im_l[i]) for i in range(slots)]
    n = len(cur)
    conj = [None] * n
    for idx in range(1, n):
        z = cur[n - idx]
        conj[idx] = complex(-z.imag, -z.real)
    conj[0] = complex(cur[0].real, -cur[0].imag)
    scale = 0.5 * pow(2, -p)
    cur = [complex(re_l[i] * scale + conj[i].real * scale, im_l[i] * scale + conj[i].imag * scale)
           for i in range(slots)]
    cur = _fft_special(cur, degree * 2)
    return np.array([complex(cur[i].real, 0.0) for i in range(slots)])
