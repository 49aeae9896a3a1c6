"""The C-ABI library loads and exports every declared entry point (CPU only).

No call here launches a kernel: only argument validation, which returns before
touching the device, and pure host arithmetic are exercised.
"""

import ctypes
import subprocess

import pytest

from helios_b200 import _native


@pytest.fixture(scope="module")
def lib():
    from helios_b200 import build

    build.build()  # no-op when the library is current
    return _native.load()


def test_every_declared_symbol_is_exported(lib):
    declared = _native.header_symbols()
    assert len(declared) >= 13
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(declared) <= exported
    assert set(declared) == set(_native.SIGNATURES)  # the binding covers exactly the header


def test_version_and_workspace_arithmetic(lib):
    assert lib.hb_version() == 1
    assert lib.hb_attention_workspace_bytes(0, 32, 128) == 256
    assert lib.hb_attention_workspace_bytes(10, 32, 128) == 256 + 10 * 32 * 129 * 4


def test_invalid_arguments_are_rejected_before_any_launch(lib):
    rc = lib.hb_rmsnorm(None, 0, None, None, ctypes.c_float(1e-6), None, 4, 7, None)
    assert rc == _native.HB_ERR_UNSUPPORTED and "multiple of 8" in _native.last_error()
    rc = lib.hb_paged_attention(None, None, None, 1, 256, None, 1, None, None, 1, None, None, 0, None, 0, None, 0, None,
                                0, 256, 1, 32, 8, 64, ctypes.c_float(1.0), None, 0, None, None)
    assert rc == _native.HB_ERR_UNSUPPORTED and "head_dim 128" in _native.last_error()
    rc = lib.hb_paged_attention(None, None, None, 1, 256, None, 1, None, None, 1, None, None, 0, None, 0, None, 0, None,
                                0, 256, 1, 32, 5, 128, ctypes.c_float(1.0), None, 0, None, None)
    assert rc == _native.HB_ERR_INVALID
    rc = lib.hb_tick_pack(None, 0, None, 0, None, 1, 1, 256, 1, 1, 16, 256, 32, 256, 0, None, None, None, None, None,
                          None, None, None, 0, None, 0, None, 0, None, 0, None, None, None)
    assert rc == _native.HB_ERR_INVALID
    with pytest.raises(ValueError, match="hb_swiglu"):
        _native.check(lib.hb_swiglu(None, None, 4, 7, None), "hb_swiglu")
    # Zero-sized work is a successful no-op that never reaches the device.
    assert lib.hb_sample(None, 1, 0, 1, None, None, None, None, None) == 0
    assert lib.hb_page_copy(None, 16, 1, 16, 1, None, None, 0, None) == 0
