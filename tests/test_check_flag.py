"""FLYAI_MOE_CHECK: the error-word check the Python surfaces run after a call.
Host logic only: the bits are fed in as a kernel would leave them."""
import pytest

from flyai_b200 import _lib


def test_set_bits_raise_and_clear_bits_pass():
    _lib.raise_on_error_bits(0, "x")
    with pytest.raises(_lib.FlyaiDeviceError, match="bounded wait"):
        _lib.raise_on_error_bits(1, "Mxfp4MoE.forward")


def test_check_is_off_unless_requested(monkeypatch):
    monkeypatch.setattr(_lib, "CHECK", False)
    assert not _lib.checking()
    monkeypatch.setattr(_lib, "CHECK", True)
    assert _lib.checking()          # no CUDA stream is capturing here
