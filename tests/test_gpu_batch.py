"""GPU parity at the benchmarked batch sizes.

The benchmark runs HEMul.mul / HERot.rotate on 64 ciphertexts per call at
N = 2^16 (hemul.py:153-217, herot.py:183-302).  At that size the inputs are
larger than 2^31 bytes (L = 35) and every batch-dependent index path of the
kernels is exercised: the two-SM contraction's pair / row-block walk, the
key-switch inner product's item walk, the BConv tile walk and the 64-bit
offsets of every buffer.  Each test runs the full batch in one call, then

* compares ciphertexts 0, 31 and 63 bit for bit with the oracle, and
* compares every ciphertext with a one-ciphertext call of the same operator
  (the one-ciphertext path is itself held to the reference's own outputs by
  the N = 2^16 digests of tests/test_gpu_shim.py).

Inputs are seeded uniform residues drawn on the device (the values only need
to be residues below their limb's modulus)."""
import numpy as np
import pytest

from oracle import cross_oracle as O
from tests.conftest import rng_residues

pytestmark = pytest.mark.gpu
N, R, C = 65536, 256, 256
SAMPLES = (0, 31, 63)


def _device_residues(torch, shape, moduli, seed):
    """Seeded residues below moduli[l] along the last axis, made on cuda:0."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.randint(0, 2 ** 62, shape, generator=g, device="cuda", dtype=torch.int64)
    q = torch.tensor(moduli, dtype=torch.int64, device="cuda")
    return (x % q).to(torch.int32).view(torch.uint32)


def _keys(L, K, dnum, seed):
    ov = O.find_moduli_ntt(L + K, 28, 2 * N)
    rng = np.random.default_rng(seed)
    return ov[:L], ov[L:], rng_residues(rng, (dnum, N, L + K), ov), rng_residues(rng, (dnum, N, L + K), ov)


def _check_batch(torch, op, x, got, oracle_fn):
    """got = op(x) for the whole batch; check samples against the oracle and
    every ciphertext against a one-ciphertext call."""
    B = x.shape[0]
    for i in SAMPLES:
        want = oracle_fn(x[i:i + 1].cpu().numpy())
        np.testing.assert_array_equal(got[i:i + 1].cpu().numpy(), want, err_msg=f"ciphertext {i} vs oracle")
    one = torch.empty_like(got[:1])
    for i in range(B):
        op(x[i:i + 1], one)
        # integer operator: the tolerance is exact equality
        assert torch.equal(one.view(torch.int32), got[i:i + 1].view(torch.int32)), f"ciphertext {i} vs batch 1"


@pytest.mark.parametrize("L,K,dnum,batch", [(24, 8, 3, 64), (35, 7, 5, 64)])
def test_hemul_benchmarked_batch(L, K, dnum, batch):
    import torch
    from cross_b200 import hemul
    Q, P, ea, eb = _keys(L, K, dnum, seed=L)
    he = hemul.HEMul(batch, R, C, dnum, 1, Q, P)
    he.control_gen(degree_layout=(R, C))
    he.setup_relinearization(ea, eb)
    x = _device_residues(torch, (batch, 4, R, C, L), Q, seed=100 + L)
    got = he.mul(x)
    torch.cuda.synchronize()
    he.check_device()
    ref = O.HEMul(1, R, C, dnum, 1, Q, P)
    ref.setup_relinearization(ea, eb)
    _check_batch(torch, lambda a, o: he.mul(a, out=o), x, got, ref.mul)
    he.check_device()
    del x, got
    torch.cuda.empty_cache()


def test_herot_benchmarked_batch():
    import torch
    from cross_b200 import herot, util
    L, K, dnum, batch = 24, 8, 3, 64
    Q, P, ea, eb = _keys(L, K, dnum, seed=7)
    k = int(np.random.default_rng(0).integers(1, N // 2))
    cm = util.precompute_auto_map(N, util.find_automorphism_index_2n_complex(k, 2 * N))
    h = herot.HERot(R, C, dnum, Q, P)
    h.control_gen(batch=batch, degree_layout=(R, C))
    h.setup_rotate(ea, eb, cm)
    x = _device_residues(torch, (batch, 2, R, C, L), Q, seed=300)
    got = h.rotate(x)
    torch.cuda.synchronize()
    h.check_device()
    ref = O.HERot(R, C, dnum, Q, P)
    ref.control_gen(1)
    ref.setup_rotate(ea.reshape(dnum, R, C, -1), eb.reshape(dnum, R, C, -1), cm)
    _check_batch(torch, lambda a, o: h.rotate(a, out=o), x, got, ref.rotate)
    h.check_device()
    del x, got
    torch.cuda.empty_cache()
