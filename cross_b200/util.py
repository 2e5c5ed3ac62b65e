"""Host parameter math of the CKKS hot path (jaxite_word util.py).

Same results as the reference functions cited below, computed with
vectorised numpy where the reference loops in Python (the N = 2^16 tables
take seconds here instead of minutes).
"""
from __future__ import annotations

import math
from typing import List, Sequence

import numpy as np

U32, U64 = np.uint32, np.uint64


def is_power_of_two(x: int) -> bool:
    return x > 0 and (x & (x - 1)) == 0


def modinv(x: int, q: int) -> int:
    """util.py:169-171."""
    return int(pow(x, -1, q))


def prime_factors(n: int) -> set:
    """util.py:174-190."""
    f, p = set(), 3
    while n % 2 == 0:
        f.add(2)
        n //= 2
    while p * p <= n:
        while n % p == 0:
            f.add(p)
            n //= p
        p += 2
    if n > 1:
        f.add(n)
    return f


def find_generator(q: int) -> int:
    """util.py:193-213: the smallest generator of GF(q)^*."""
    phi = q - 1
    fs = prime_factors(phi)
    for g in range(2, q):
        if all(pow(g, phi // p, q) != 1 for p in fs):
            return g
    raise ValueError("No generator found, check that q is prime.")


def powers(base: int, count: int, q: int) -> np.ndarray:
    """[base^i mod q for i in range(count)] as uint64, via base^(aB+b) = (base^B)^a base^b."""
    if count <= 0:
        return np.zeros(0, U64)
    blk = 1 << max(0, (int(math.ceil(math.log2(count))) + 1) // 2)
    lo = np.empty(blk, U64)
    acc = 1
    for b in range(blk):
        lo[b] = acc
        acc = acc * base % q
    step = acc
    nhi = (count + blk - 1) // blk
    hi = np.empty(nhi, U64)
    acc = 1
    for a in range(nhi):
        hi[a] = acc
        acc = acc * step % q
    return ((hi[:, None] * lo[None, :]) % U64(q)).reshape(-1)[:count]


def root_of_unity(m: int, q: int) -> int:
    """util.py:219-249: the minimal primitive m-th root of unity mod q.

    For m a power of two, r = g^((q-1)/m) has order exactly m, so the
    candidates r^k with gcd(k, m) = 1 are exactly the odd powers, all of
    which pass the reference's order test; the result is their minimum.
    """
    assert (q - 1) % m == 0, "q-1 must be divisible by m"
    g = find_generator(q)
    r = pow(g, (q - 1) // m, q)
    if is_power_of_two(m) and m >= 2:
        return int(powers(r, m, q)[1::2].min())
    half, best = m // 2, None
    for k in range(1, m):
        if math.gcd(k, m) != 1:
            continue
        psi = pow(r, k, q)
        if pow(psi, half, q) == q - 1 and pow(psi, m, q) == 1 and (best is None or psi < best):
            best = psi
    assert best is not None, "No primitive m-th root found"
    return best


def is_prime_deterministic(n: int) -> bool:
    """util.py:385-428."""
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
    """util.py:431-458."""
    out, k = [], (2 ** precision - 1) // ntt_length
    while len(out) < total_number and k > 0:
        cand = k * ntt_length + 1
        if is_prime_deterministic(cand):
            out.append(cand)
        k -= 1
    return out


def compute_QHatInvModq_QHatModp(original_moduli: Sequence[int], target_moduli: Sequence[int]):
    """util.py:311-353."""
    Q = 1
    for q in original_moduli:
        Q *= q
    qhat = [Q // q for q in original_moduli]
    inv = [modinv(h, q) for h, q in zip(qhat, original_moduli)]
    return inv, [[h % p for p in target_moduli] for h in qhat]


def gamma_beta_calculation(moduli_list: Sequence[int]):
    """util.py:461-492."""
    Q = 1
    for m in moduli_list[:-1]:
        Q *= m
    ql = moduli_list[-1]
    gc = (Q * modinv(Q, ql) - 1) // ql
    gammas = [gc % m for m in moduli_list[:-1]]
    betas = [modinv(ql, m) for m in moduli_list[:-1]]
    return np.array(gammas, U64), np.array(betas, U64)


def bit_reverse(x: int, bits: int) -> int:
    """util.py:614-620."""
    r = 0
    for i in range(bits):
        if (x >> i) & 1:
            r |= 1 << (bits - 1 - i)
    return r


def bit_reverse_indices(n: int) -> np.ndarray:
    """util.py:633-645."""
    bits = int(math.log2(n))
    idx = np.arange(n, dtype=np.int64)
    rev = np.zeros(n, np.int64)
    for i in range(bits):
        rev |= ((idx >> i) & 1) << (bits - 1 - i)
    return rev


def precompute_auto_map(n: int, k: int) -> List[int]:
    """util.py:652-668 (OpenFHE PrecomputeAutoMap), vectorised."""
    m = n << 1
    j = np.arange(n, dtype=np.int64)
    t = ((j << 1) + 1) * k
    idx = (t % m) >> 1
    out = np.zeros(n, np.int64)
    rev = bit_reverse_indices(n)
    out[rev[j]] = rev[idx]
    return out.tolist()


def find_automorphism_index_2n_complex(i: int, m: int) -> int:
    """util.py:671-693."""
    if i == 0:
        return 1
    if i == m - 1:
        return int(i)
    if not is_power_of_two(m):
        raise ValueError("m should be a power of two.")
    g0 = pow(5, -1, m) if i < 0 else 5
    g = g0
    for _ in range(1, abs(i)):
        g = (g * g0) & (m - 1)
    return int(g)


def twiddle_matrix(rows: int, cols: int, q: int, omega: int) -> np.ndarray:
    """ntt_mm.py:75-98: T[r, c] = omega^(r*c) mod q."""
    wr = powers(omega, rows, q)
    out = np.empty((rows, cols), U64)
    col = np.ones(rows, U64)
    for c in range(cols):
        out[:, c] = col
        col = (col * wr) % U64(q)
    return out


def default_rc(degree: int):
    """ciphertext.py:63,69-70."""
    r = 1 << (int(math.log2(degree)) // 2)
    return r, degree // r


def barrett_constants(moduli: Sequence[int]):
    """finite_field.py:177-180, with the same float expressions."""
    s = [2 * math.ceil(math.log2(m)) for m in moduli]
    w = [min(x, 32) for x in s]
    sw = [a - b for a, b in zip(s, w)]
    m = [math.floor(2 ** a / q) for a, q in zip(s, moduli)]
    return s, w, sw, m


def random_parameters(shape, modulus_list, seed: int = 0, dtype=np.uint32):
    """Seeded stand-in of util.py:533-539: uniform in [0, min(moduli) - 1)."""
    rng = np.random.default_rng(seed)
    hi = min(modulus_list) - 1
    return rng.integers(0, hi, size=shape, dtype=np.uint64).astype(dtype)


def parse_ciphertext_string(input_str: str):
    """util.py:545-608: OpenFHE text format -> (data, moduli)."""
    import re
    data, modulus, cur = [], [], None
    pat = re.compile(r'^(\d+):\s*EVAL:\s*\[(.*?)\]\s*modulus:\s*(\d+)')
    for line in input_str.strip().splitlines():
        line = line.strip()
        if line.startswith("Element"):
            cur = []
            data.append(cur)
            hm = re.match(r'^Element\s+\d+:\s*(.*)', line)
            line = hm.group(1).strip() if hm else ""
            if not line:
                continue
        em = pat.match(line)
        if em:
            cur.append([int(v) for v in em.group(2).split()])
            idx = len(cur) - 1
            if len(data) == 1:
                modulus.append(int(em.group(3)))
            elif idx < len(modulus) and modulus[idx] != int(em.group(3)):
                raise ValueError(f"Inconsistent modulus at evaluation index {idx}")
    return data, modulus
