"""Known-answer tests for the 32-block quantized formats (the layout include/b200dec.h defines).

The reference has no quantized weights (roadmap only: ios_kernels/PLAN.md:175,256), so these
vectors pin the format itself: nibble order, sign decoding and exact fp32 dequantization.
"""

import numpy as np

from oracle import ops


def test_q4_nibble_order_and_sign():
    # byte 0x8F: low nibble 0xF -> -1 (element 0), high nibble 0x8 -> -8 (element 1)
    # byte 0x70: low nibble 0x0 ->  0 (element 2), high nibble 0x7 -> +7 (element 3)
    packed = np.array([[0x8F, 0x70]], dtype=np.uint8)
    np.testing.assert_array_equal(ops.unpack_q4(packed), [[-1, -8, 0, 7]])


def test_q4_pack_roundtrip_all_values():
    q = np.array([np.arange(-8, 8), np.arange(7, -9, -1)], dtype=np.int8)  # 16 values per row
    q = np.concatenate([q, q], axis=1)  # K = 32
    p = ops.pack_q4(q)
    assert p.shape == (2, 16)
    assert p[0, 0] == ((-8) & 0xF) | (((-7) & 0xF) << 4)
    np.testing.assert_array_equal(ops.unpack_q4(p), q)


def test_dequant_is_exact_in_fp32():
    rng = np.random.default_rng(3)
    M, K = 8, 96
    q8 = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    sc = np.abs(rng.standard_normal((M, K // 32)) * 0.01).astype(np.float16)
    w = ops.dequant_q8_32(q8, sc)
    assert w.dtype == np.float32
    exact = np.repeat(sc.astype(np.float64), 32, axis=1) * q8.astype(np.float64)
    np.testing.assert_array_equal(w.astype(np.float64), exact)  # fp32 holds s*q exactly
    q4 = rng.integers(-8, 8, size=(M, K), dtype=np.int8)
    w4 = ops.dequant_q4_32(ops.pack_q4(q4), sc)
    np.testing.assert_array_equal(
        w4.astype(np.float64), np.repeat(sc.astype(np.float64), 32, axis=1) * q4
    )


def test_quant_gemv_matches_dense():
    rng = np.random.default_rng(4)
    M, K = 16, 64
    q8 = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    sc = np.abs(rng.standard_normal((M, K // 32)) * 0.01).astype(np.float16)
    x = rng.standard_normal((3, K)).astype(np.float16)
    ref = x.astype(np.float64) @ (np.repeat(sc.astype(np.float64), 32, 1) * q8).T
    np.testing.assert_allclose(ops.gemv_q8_32(q8, sc, x), ref, rtol=1e-12)
