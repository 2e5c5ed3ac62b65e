"""The reference's error behaviour on the device-backed objects: the checks
of ciphertext.py:203-227,455-461 raise the reference's exception types
before any device work."""
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
