"""Host parameter math of the CKKS hot path (jaxite_word util.py).

Same results as the reference functions cited below, computed with
vectorised numpy where the reference loops in Python (the N = 2^16 tables
take seconds here instead of minutes).
"""
from __future__ import annotations

import copy
import functools
import math
from typing import List, Sequence

import numpy as np

U32, U64 = np.uint32, np.uint64


def num_bits(x: int) -> int:
    """util.py:61-63: x.bit_length() - 1."""
    return x.bit_length() - 1


def is_power_of_two(x: int) -> bool:
    return x > 0 and (x & (x - 1)) == 0


def to_tuple(a):
    """util.py:71-76: nested tuples of an array or nested sequence."""
    try:
        return tuple(to_tuple(i) for i in a)
    except TypeError:
        return a


def slice_first_k_along_axis0(arrays, k):
    """util.py:79-89: (obj[:k] for every obj)."""
    return tuple(arr[:k] for arr in arrays)


def slice_k_to_end_along_axis0(arrays, k):
    """util.py:92-102: (obj[k:] for every obj)."""
    return tuple(arr[k:] for arr in arrays)


def slice_kth_along_axis0(arrays, k):
    """util.py:105-115: (obj[k] for every obj)."""
    return tuple(arr[k] for arr in arrays)


def slice_0_to_k0_to_k1_along_axis0(arrays, k0, k1):
    """util.py:118-134: every object without its entries k0 .. k1-1.  Arrays
    (numpy or torch) are concatenated, as the reference does for jax arrays;
    sequences in a tuple or list are joined with ``+``."""
    first = arrays[0]
    if isinstance(first, np.ndarray):
        return tuple(np.concatenate([x[:k0], x[k1:]]) for x in arrays)
    if hasattr(first, "data_ptr"):
        import torch
        return tuple(torch.cat([x[:k0], x[k1:]]) for x in arrays)
    if isinstance(arrays, tuple):
        return tuple([arr[:k0] + arr[k1:] for arr in arrays])
    if isinstance(arrays, list):
        return [arr[:k0] + arr[k1:] for arr in arrays]
    raise ValueError(f"Unsupported type: {type(arrays)}")


def slice_k0_to_k1_axis0(arrays, k0, k1):
    """util.py:137-146: (obj[k0:k1] for every obj)."""
    return tuple(arr[k0:k1] for arr in arrays)


def extended_gcd(a, b):
    """util.py:151-157: (g, x, y) with a x + b y = g = gcd(a, b)."""
    if b == 0:
        return (a, 1, 0)
    g, x, y = extended_gcd(b, a % b)
    return (g, y, x - (a // b) * y)


def modinv_manual(x, q):
    """util.py:160-166: the inverse of x mod q by the extended Euclid."""
    g, inv, _ = extended_gcd(x, q)
    if g != 1:
        raise Exception(f'Modular inverse does not exist for {x} modulo {q}')
    return inv % q


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


def compute_QHatInvModq_QHatModp(original_moduli: Sequence[int], target_moduli: Sequence[int],
                                 perf_test: bool = False):
    """util.py:311-353 (perf_test builds the real constants too: same cost,
    checkable results)."""
    Q = 1
    for q in original_moduli:
        Q *= q
    qhat = [Q // q for q in original_moduli]
    inv = [modinv(h, q) for h, q in zip(qhat, original_moduli)]
    return inv, [[h % p for p in target_moduli] for h in qhat]


def gamma_beta_calculation(moduli_list: Sequence[int], perf_test: bool = False):
    """util.py:461-492 (perf_test builds the real constants too)."""
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


def bit_reverse_array(in_tower):
    """util.py:623-630: a copy of the sequence in bit-reversed index order
    (lists stay lists, arrays stay arrays)."""
    x = copy.deepcopy(in_tower)
    n = len(x)
    rev = bit_reverse_indices(n) if n > 1 else np.zeros(n, np.int64)
    if isinstance(x, np.ndarray):
        return x[rev]
    if hasattr(x, "data_ptr"):
        import torch
        return x[torch.as_tensor(rev, device=x.device)]
    if isinstance(x, tuple):
        return tuple(x[int(j)] for j in rev)
    return [x[int(j)] for j in rev]


@functools.lru_cache(maxsize=64)
def bit_reverse_indices(n: int) -> np.ndarray:
    """util.py:633-645.  Computed once per n and returned read-only (like the
    reference's jax array): every ciphertext object of degree n holds it."""
    bits = int(math.log2(n))
    idx = np.arange(n, dtype=np.int64)
    rev = np.zeros(n, np.int64)
    for i in range(bits):
        rev |= ((idx >> i) & 1) << (bits - 1 - i)
    rev.flags.writeable = False
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


def random_parameters(shape, modulus_list, dtype=np.int32, seed: int = 0):
    """Seeded stand-in of util.py:533-539: uniform in [0, min(moduli) - 1).
    numpy draws the values (the reference's come from jax.random, whose bits
    are not reproduced)."""
    rng = np.random.default_rng(seed)
    hi = min(modulus_list) - 1
    return rng.integers(0, hi, size=shape, dtype=np.uint64).astype(dtype)


def random_batched_ciphertext(shape, modulus_list, dtype=np.int32, seed: int = 0):
    """Seeded stand-in of util.py:497-512: shape (B, r, c, M), limb m uniform
    in [0, modulus_list[m])."""
    assert len(modulus_list) == shape[-1]
    rng = np.random.default_rng(seed)
    q = np.array(modulus_list, np.uint64)
    return (rng.integers(0, 2 ** 62, size=tuple(shape), dtype=np.uint64) % q).astype(dtype)


def random_ciphertext(shape, modulus_list, dtype=np.int32, seed: int = 0):
    """Seeded stand-in of util.py:515-530: shape (B, N, M), limb m uniform in
    [0, modulus_list[m])."""
    assert len(modulus_list) == shape[-1]
    rng = np.random.default_rng(seed)
    q = np.array(modulus_list, np.uint64)
    return (rng.integers(0, 2 ** 62, size=tuple(shape), dtype=np.uint64) % q).astype(dtype)


def any_primitive_root_of_unity(n: int, q: int) -> int:
    """util.py:252-288: g^((q-1)/n) for the generator g of find_generator,
    checked to have order exactly n."""
    if (q - 1) % n != 0:
        raise ValueError("n must divide q-1 for a primitive n-th root of unity to exist.")
    omega = pow(find_generator(q), (q - 1) // n, q)
    if pow(omega, n, q) != 1:
        raise ValueError("Something went wrong: omega^n != 1")
    for d in range(1, n):
        if n % d == 0 and pow(omega, d, q) == 1:
            raise ValueError("Found an exponent d < n with omega^d == 1, so omega is not primitive.")
    return omega


def compute_barrett_mu(modulus: int):
    """util.py:291-308: (mu, k) with b = 2^(floor(ln m) + 1), k the digits of m
    in base b, mu = floor(b^(2k) / m)."""
    b = 2 ** (math.floor(math.log(modulus)) + 1)
    k_val = math.floor(math.log(modulus, b)) + 1
    return (b ** (2 * k_val)) // modulus, k_val


def approx_mod_down_control_generation(current_moduli, target_moduli, perf_test: bool = False):
    """util.py:356-367: (P^-1 mod q for the target moduli, the index where the
    target moduli start and where the current ones start in current +
    target, QHatInvModq, QHatModp of current -> target)."""
    P = 1
    for m in current_moduli:
        P *= m
    p_inv = [modinv(P, q) for q in target_moduli]
    overall = list(current_moduli) + list(target_moduli)
    inv, qm = compute_QHatInvModq_QHatModp(current_moduli, target_moduli)
    return p_inv, len(overall) - len(target_moduli), len(overall) - len(current_moduli), inv, qm


def compute_powers_of_psi(ring_dim: int, moduli: Sequence[int], perf_test: bool = False) -> np.ndarray:
    """util.py:370-382: psi_q^i for i < ring_dim, psi_q = root_of_unity(2
    ring_dim, q), one row per modulus, uint64."""
    return np.stack([powers(root_of_unity(2 * ring_dim, q), ring_dim, q) for q in moduli]).astype(U64)


def chunk_decomposition(x: int, chunkwidth: int = 8) -> np.ndarray:
    """util.py:833-861: the chunkwidth-bit digits of x, least significant
    first (uint16 / uint32 for widths 16 / 32, else uint8)."""
    dtype = {16: np.uint16, 32: np.uint32}.get(chunkwidth, np.uint8)
    mask = (1 << chunkwidth) - 1
    out = []
    while x > 0:
        out.append(x & mask)
        x >>= chunkwidth
    return np.array(out, dtype=dtype)


def format_ciphertext_string(data, modulus) -> str:
    """The inverse of parse_ciphertext_string (util.py:545-608): OpenFHE's
    text form of a ciphertext, one ``Element k:`` group per element and one
    ``i: EVAL: [...] modulus: q_i`` line per tower.  data: (elements,
    towers, N) integers; modulus: one value per tower.  No counterpart in the
    reference, which only reads the format."""
    lines = []
    for k, element in enumerate(data):
        if len(element) != len(modulus):
            raise ValueError(f"element {k} has {len(element)} towers for {len(modulus)} moduli")
        for i, (tower, q) in enumerate(zip(element, modulus)):
            body = f"{i}: EVAL: [{' '.join(str(int(v)) for v in tower)}] modulus: {int(q)}"
            lines.append(f"Element {k}: {body}" if i == 0 else body)
    return "\n".join(lines) + "\n"


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
