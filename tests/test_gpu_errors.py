"""The reference's error behaviour on the device-backed objects: the checks
of ciphertext.py:203-227,455-461 raise the reference's exception types
before any device work.  And the failure path of the bounded device waits:
a wait that runs out reports a timeout and leaves the GPU usable."""
import pytest

pytestmark = pytest.mark.gpu


def _ct(num_moduli):
    from cross_b200 import ciphertext
    return ciphertext.Ciphertext({"batch": 1, "num_elements": 2, "num_moduli": num_moduli, "degree": 16,
                                  "precision": 32, "degree_layout": (4, 4)})


def test_single_limb_ciphertext_errors():
    c = _ct(1)
    with pytest.raises(ValueError, match="single-limb"):
        c.drop_last_modulus()
    with pytest.raises(ValueError, match="fewer than two moduli"):
        c.modulus_switch_control_gen()


def test_key_switch_before_control_gen():
    with pytest.raises(RuntimeError, match="key_switch_control_gen"):
        _ct(3).key_switch()


@pytest.mark.parametrize("bound_us", [50, 2000])
def test_bounded_wait_expires_and_the_context_stays_usable(bound_us):
    """A bounded device wait on a barrier that nothing arrives on gives up
    after its bound, records its code and lets the kernel return
    (cross_wait_selftest runs the wait helper every tensor-core kernel uses);
    the call reports CROSS_ERR_TIMEOUT, and the GPU then still computes an NTT
    bit-exactly."""
    import time
    import numpy as np
    import torch
    from cross_b200 import _lib, ntt_mm
    from oracle import cross_oracle as O
    from tests.conftest import rng_residues
    lib = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    rc = lib.cross_wait_selftest(bound_us * 1000, st)
    dt = time.perf_counter() - t0
    assert rc == -5, lib.cross_last_error()                       # CROSS_ERR_TIMEOUT
    assert b"expired" in lib.cross_last_error()
    assert dt >= bound_us * 1e-6
    with pytest.raises(TimeoutError):
        _lib.check(lib.cross_wait_selftest(bound_us * 1000, st), "cross_wait_selftest")
    q = O.find_moduli_ntt(3, 28, 2 * 65536)
    x = rng_residues(np.random.default_rng(bound_us), (2, 256, 256, 3), q)
    ctx = ntt_mm.NTTCiphertextBarrettContext(q, {"r": 256, "c": 256})
    np.testing.assert_array_equal(ctx.ntt(x).cpu().numpy(), O.NTTBarrett(q, 256, 256).ntt(x))
    ctx.check_device()
