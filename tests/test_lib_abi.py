"""CPU checks of the C ABI: the library loads, exports every declared symbol, and validates
arguments on the host (no kernel runs here)."""

import ctypes

import numpy as np
import pytest

from gemmagemini4hackathon2026_10_2425_b200 import _lib
from oracle import ops as oracle_ops


def test_every_declared_symbol_is_exported():
    declared = _lib.declared_symbols()
    assert len(declared) >= 29
    lib = _lib.lib()
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    assert set(declared) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_status_strings():
    lib = _lib.lib()
    assert lib.b2d_status_string(0) == b"ok"
    for st in range(1, 10):
        assert lib.b2d_status_string(st) not in (b"ok", b"unknown status")
    assert lib.b2d_version() >= 1


@pytest.mark.parametrize("hd,theta", [(64, 500000.0), (128, 10000.0), (16, 500000.0)])
def test_inv_freq_matches_oracle(hd, theta):
    out = (ctypes.c_float * (hd // 2))()
    assert _lib.lib().b2d_inv_freq(hd, theta, ctypes.addressof(out)) == 0
    np.testing.assert_array_equal(np.array(out, dtype=np.float32), oracle_ops.inv_freq(hd, theta))


def test_host_side_validation_errors():
    lib = _lib.lib()
    # NULL pointers are rejected before any CUDA call
    assert lib.b2d_gemv_f32(None, None, None, 4, 4, None) == _lib.ERR_NULL
    assert lib.b2d_rmsnorm(None, None, None, 1, 4, 1e-6, None) == _lib.ERR_NULL
    assert (
        lib.b2d_paged_decode_attn(
            None, 0, 0, None, None, None, 1, 1, None, None, 1, 1, 64, 1, 16, 0.0, 0, 1, None, 0, 64, None, 0, None
        )
        == _lib.ERR_NULL
    )
    assert lib.b2d_decoder_step(None, None, None, None, 1, None, None, 0, None) == _lib.ERR_NULL
    with pytest.raises(ValueError):
        _lib.call("b2d_gemv_f32", None, None, None, 4, 4, None)


def test_workspace_queries_are_positive():
    lib = _lib.lib()
    assert lib.b2d_paged_attn_workspace_bytes(64, 32, 8, 128, 8193) > 64 * 8 * 4
    assert lib.b2d_lm_head_argmax_workspace_bytes(128256, 32) > 0
