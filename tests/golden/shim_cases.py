"""Cases recorded by make_golden_shim.py: the reference's own operators run on
seeded inputs at sizes its tests do not cover, stored as digests of their
outputs.  Shared by the generator and tests/test_oracle_shim.py, which
rebuilds the same inputs and holds the oracle to the digests."""
import hashlib

import numpy as np

U32 = np.uint32

# (name, kind, parameters); N = r * c
CASES = [
    ("ntt_barrett_64x64_m8", "ntt", dict(reduction="barrett", r=64, c=64, limbs=8, batch=2)),
    ("ntt_barrett_32x128_m4", "ntt", dict(reduction="barrett", r=32, c=128, limbs=4, batch=2)),
    ("ntt_montgomery_64x64_m4", "ntt", dict(reduction="montgomery", r=64, c=64, limbs=4, batch=2)),
    ("ntt_bat_lazy_64x64_m4", "ntt", dict(reduction="bat_lazy", r=64, c=64, limbs=4, batch=2)),
    ("ntt_barrett_256x256_m1", "ntt", dict(reduction="barrett", r=256, c=256, limbs=1, batch=1)),
    ("bconv_bat_n4096_8to23", "bconv", dict(bat=True, n=4096, sq=8, sp=23, batch=2)),
    ("bconv_plain_n4096_8to23", "bconv", dict(bat=False, n=4096, sq=8, sp=23, batch=2)),
    ("rescale_64x64_l6", "rescale", dict(r=64, c=64, limbs=6, batch=2)),
    ("hemul_64x64_l6_k2_dnum3", "hemul", dict(r=64, c=64, limbs=6, special=2, dnum=3, batch=1)),
    ("herot_64x64_l6_k2_dnum3", "herot", dict(r=64, c=64, limbs=6, special=2, dnum=3, batch=1, rotation=3)),
    # the benchmark point: N = 2^16, L = 24, K = 8, dnum = 3, one ciphertext
    ("bconv_bat_n65536_24to25", "bconv", dict(bat=True, n=65536, sq=24, sp=25, batch=1)),
    ("hemul_256x256_l24_k8_dnum3", "hemul", dict(r=256, c=256, limbs=24, special=8, dnum=3, batch=1)),
    ("herot_256x256_l24_k8_dnum3", "herot", dict(r=256, c=256, limbs=24, special=8, dnum=3, batch=1, rotation=5)),
    # the CKKS client (ckks_ctx.py) at N = 2^12 with six 28-bit towers
    ("ckks_encode_n4096_l6", "ckks_encode", dict(degree=4096, towers=6, scale=2.0 ** 40)),
    ("ckks_encrypt_n4096_l6", "ckks_encrypt", dict(degree=4096, towers=6, scale=2.0 ** 40)),
    ("ckks_decode_n4096_l6", "ckks_decode", dict(degree=4096, towers=6, scale=2.0 ** 40, p=40)),
    # the relinearisation key with given a and e (key_gen.py:108-254)
    ("evk_n4096_l6_k2_dnum3", "evk", dict(degree=4096, limbs=6, special=2, dnum=3)),
    # the variants at N = 2^16 (the BAT-lazy step-2 product wraps in uint64 there)
    ("ntt_montgomery_256x256_m1", "ntt", dict(reduction="montgomery", r=256, c=256, limbs=1, batch=1)),
    ("ntt_bat_lazy_256x256_m1", "ntt", dict(reduction="bat_lazy", r=256, c=256, limbs=1, batch=1)),
    # the BConv reduction variants (bconv.py:261-390); BConvMontgomery's plain
    # path needs size_q == size_p (bconv.py:280 broadcasts the one basis
    # against the other)
    ("bconv_montgomery_bat_n4096_8to23", "bconv", dict(bat=True, n=4096, sq=8, sp=23, batch=2, reduction="montgomery")),
    ("bconv_montgomery_plain_n4096_8to8", "bconv", dict(bat=False, n=4096, sq=8, sp=8, batch=2, reduction="montgomery")),
    ("bconv_bat_lazy_bat_n4096_8to23", "bconv", dict(bat=True, n=4096, sq=8, sp=23, batch=2, reduction="bat_lazy")),
    ("bconv_bat_lazy_plain_n4096_8to23", "bconv", dict(bat=False, n=4096, sq=8, sp=23, batch=2, reduction="bat_lazy")),
    ("bconv_shoup_plain_n4096_8to23", "bconv", dict(bat=False, n=4096, sq=8, sp=23, batch=2, reduction="shoup")),
    # the Shoup transform (byte convolutions, ntt_mm.py:443-587)
    ("ntt_shoup_64x64_m4", "ntt", dict(reduction="shoup", r=64, c=64, limbs=4, batch=2)),
    # the single-modulus contexts (ntt_sm.py:330-494); Shoup takes one matrix
    ("ntt_sm_barrett_64x64", "ntt_sm", dict(reduction="barrett", r=64, c=64, batch=2)),
    ("ntt_sm_montgomery_64x64", "ntt_sm", dict(reduction="montgomery", r=64, c=64, batch=2)),
    ("ntt_sm_bat_lazy_64x64", "ntt_sm", dict(reduction="bat_lazy", r=64, c=64, batch=2)),
    ("ntt_sm_shoup_64x64", "ntt_sm", dict(reduction="shoup", r=64, c=64, batch=0)),
    # the four finite_field.py reductions on products of residues
    # (moduli on the last axis; Shoup with its companion product)
    ("ff_barrett_4096x6", "ff", dict(reduction="barrett", rows=4096, limbs=6)),
    ("ff_montgomery_4096x6", "ff", dict(reduction="montgomery", rows=4096, limbs=6)),
    ("ff_shoup_4096x6", "ff", dict(reduction="shoup", rows=4096, limbs=6)),
    ("ff_bat_lazy_4096x6", "ff", dict(reduction="bat_lazy", rows=4096, limbs=6)),
    # the eight-GPU configuration: L = 35, K = 7, five key-switch digits
    ("hemul_256x256_l35_k7_dnum5", "hemul", dict(r=256, c=256, limbs=35, special=7, dnum=5, batch=1)),
    ("rescale_256x256_l24", "rescale", dict(r=256, c=256, limbs=24, batch=1)),
    ("herot_256x256_l35_k7_dnum5", "herot", dict(r=256, c=256, limbs=35, special=7, dnum=5, batch=1, rotation=7)),
]


def digest(a) -> str:
    a = np.ascontiguousarray(np.asarray(a))
    return hashlib.sha256(str(a.dtype).encode() + str(a.shape).encode() + a.tobytes()).hexdigest()


def residues(seed: int, shape, moduli) -> np.ndarray:
    """Uniform residues, limb m (the last axis) below moduli[m]."""
    rng = np.random.default_rng(seed)
    q = np.array(moduli, np.uint64)
    return (rng.integers(0, 2 ** 62, size=tuple(shape), dtype=np.uint64) % q).astype(U32)


def ckks_slots(name: str, p: dict):
    """N/2 complex slot values, real and imaginary parts uniform in [-1, 1)."""
    rng = np.random.default_rng(sum(map(ord, name)))
    v = rng.uniform(-1.0, 1.0, size=(p["degree"] // 2, 2))
    return [complex(a, b) for a, b in v]


def ckks_encrypt_operands(name: str, p: dict, moduli):
    """Public key (2, towers, N), v (towers, N) and e = (e0, e1) as Python
    integer lists of residues."""
    n, t = p["degree"], len(moduli)
    pk = residues(sum(map(ord, name)) + 1, (2, n, t), moduli).transpose(0, 2, 1)
    v = residues(sum(map(ord, name)) + 2, (n, t), moduli).T
    e = residues(sum(map(ord, name)) + 3, (2, n, t), moduli).transpose(0, 2, 1)
    as_lists = lambda a: [[[int(x) for x in row] for row in el] for el in a] if a.ndim == 3 else \
        [[int(x) for x in row] for row in a]  # noqa: E731
    return as_lists(pk), as_lists(v), as_lists(e)


def evk_operands(name: str, p: dict, moduli):
    """private key (Q x N), a and e (parts x (Q + P) x N) as integer lists of
    residues, evaluation form."""
    n, L, d = p["degree"], p["limbs"], p["dnum"]
    per = (L + d - 1) // d
    parts = -(-L // per)
    seed = sum(map(ord, name))
    sk = residues(seed, (n, L), moduli[:L]).T
    a = residues(seed + 1, (parts, n, len(moduli)), moduli).transpose(0, 2, 1)
    e = residues(seed + 2, (parts, n, len(moduli)), moduli).transpose(0, 2, 1)
    return sk.tolist(), a.tolist(), e.tolist()


def inputs(name: str, kind: str, p: dict, moduli):
    """The seeded operands of one case, in the reference's layouts."""
    seed = sum(map(ord, name))
    if kind == "ntt":
        return {"x": residues(seed, (p["batch"], p["r"], p["c"], p["limbs"]), moduli)}
    if kind == "ff":
        shape = (p["rows"], p["limbs"])
        a = residues(seed, shape, moduli).astype(np.uint64)
        t = residues(seed + 1, shape, moduli).astype(np.uint64)
        out = {"z": a * t}
        if p["reduction"] == "shoup":
            # z_s = a * floor(t 2^32 / q) (finite_field.py:295-302)
            ts = np.array([[(int(v) << 32) // q for v, q in zip(row, moduli)] for row in t.tolist()], np.uint64)
            out["z_s"] = a * ts
        return out
    if kind == "ntt_sm":
        shape = (p["batch"], p["r"], p["c"]) if p["batch"] else (p["r"], p["c"])
        return {"x": residues(seed, shape + (1,), moduli)[..., 0]}
    if kind == "bconv":
        return {"x": residues(seed, (p["batch"], p["n"], p["sq"]), moduli[:p["sq"]])}
    if kind == "rescale":
        return {"x": residues(seed, (p["batch"], 2, p["r"], p["c"], p["limbs"]), moduli)}
    L, K, d, r, c = p["limbs"], p["special"], p["dnum"], p["r"], p["c"]
    elems = 4 if kind == "hemul" else 2
    out = {"x": residues(seed, (p["batch"], elems, r, c, L), moduli[:L])}
    kshape = (d, r * c, L + K) if kind == "hemul" else (d, r, c, L + K)
    out["evk_a"] = residues(seed + 1, kshape, moduli)
    out["evk_b"] = residues(seed + 2, kshape, moduli)
    return out
