"""The arithmetic of the RMSNorm folded into the tcgen05 GEMM pair, restated in NumPy (CPU).

The producer GEMM (O / down projection, residual-add epilogue) writes the new residual x, the
hi / lo fp16 planes of x * gamma * e[t] and per-16-row-slice sums of x^2; the consumer GEMM
multiplies W by the planes and scales each token's product by r[t] / e[t] with
r[t] = rsqrt(mean(x[t]^2) + eps).  e[t] is the power of two at or below the token's previous
norm factor.  This file checks, against the float64 oracle's W @ (rmsnorm(x) * gamma):
  * the folded form is fp32-class accurate for residuals from 1e-3 to 1e5 in magnitude;
  * e is what makes that true: without it, large residuals overflow fp16 and small ones lose
    digits to fp16's subnormal floor in the lo plane.
The device kernels are checked against the oracle end to end in test_norm_fold_gpu.py and
test_bench_config_gpu.py; this is the numerical argument behind them.
"""

import numpy as np
import pytest

from oracle import ops as O


def pow2_floor(v: np.ndarray) -> np.ndarray:
    """Power of two at or below each positive value (1 for zero, inf, nan)."""
    out = np.ones_like(v, dtype=np.float32)
    ok = np.isfinite(v) & (v > 0)
    out[ok] = np.exp2(np.floor(np.log2(v[ok].astype(np.float64)))).astype(np.float32)
    return out


def folded(W, x, gamma, eps, r_prev):
    """W @ (rmsnorm(x) * gamma) the way the folded GEMM pair computes it (float64 products stand
    in for the tensor cores' fp32 accumulation of exact fp16 x fp16 products)."""
    x = x.astype(np.float32)
    e = pow2_floor(r_prev) if r_prev is not None else np.ones(x.shape[0], np.float32)
    v = (x * gamma[None, :]).astype(np.float32) * e[:, None]
    with np.errstate(over="ignore", invalid="ignore"):
        hi = v.astype(np.float16)
        lo = (v - hi.astype(np.float32)).astype(np.float16)
    # producer: sums of x^2 over 16-row slices, each in row order (fp32)
    D = x.shape[1]
    sq = (x * x).astype(np.float32).reshape(x.shape[0], D // 16, 16)
    slices = np.zeros(sq.shape[:2], np.float32)
    for i in range(16):
        slices += sq[:, :, i]
    # consumer: two halves of the slices, each as four interleaved fp32 sums, then combined
    S = D // 16
    halves = []
    for h in range(2):
        part = slices[:, h * S // 2 : (h + 1) * S // 2].reshape(x.shape[0], -1, 4)
        acc = np.zeros((x.shape[0], 4), np.float32)
        for j in range(part.shape[1]):
            acc += part[:, j, :]
        halves.append((acc[:, 0] + acc[:, 1]) + (acc[:, 2] + acc[:, 3]))
    ssum = halves[0] + halves[1]
    r = (1.0 / np.sqrt(ssum.astype(np.float64) / D + eps)).astype(np.float32)
    prod = (hi.astype(np.float64) + lo.astype(np.float64)) @ W.astype(np.float64).T
    return prod * (r / e)[:, None]


def _case(scale, seed=0, D=2048, M=256, B=8):
    r = np.random.default_rng(seed)
    x = (r.standard_normal((B, D)) * scale).astype(np.float32)
    x[:, 7] *= 40.0  # an outlier feature, as real residual streams have
    gamma = (r.random(D) + 0.5).astype(np.float32)
    W = (r.standard_normal((M, D)) * 0.02).astype(np.float16)
    return W, x, gamma


@pytest.mark.parametrize("scale", [1e-3, 1.0, 1e3, 1e5])
def test_folded_norm_matches_oracle(scale):
    W, x, gamma = _case(scale)
    eps = 1e-5
    ref = O.gemv(W, O.rmsnorm(x, gamma, eps))
    # the previous norm factor: the same token one sublayer earlier (here: 0.7 x this residual)
    r_prev = 1.0 / np.sqrt(np.mean((0.7 * x.astype(np.float64)) ** 2, axis=1) + eps)
    got = folded(W, x, gamma, eps, r_prev.astype(np.float32))
    err = np.max(np.abs(got - ref)) / np.max(np.abs(ref))
    assert err < 2e-6, f"scale {scale}: {err:.2e}"


def test_power_of_two_prescale_is_needed():
    eps = 1e-5
    W, x, gamma = _case(1e5)
    with np.errstate(over="ignore", invalid="ignore"):
        unscaled = folded(W, x, gamma, eps, None)
    assert not np.all(np.isfinite(unscaled)), "x * gamma fits fp16 without the prescale"
    W, x, gamma = _case(1e-3)
    ref = O.gemv(W, O.rmsnorm(x, gamma, eps))
    small = folded(W, x, gamma, eps, None)
    r_prev = (1.0 / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1) + eps)).astype(np.float32)
    scaled = folded(W, x, gamma, eps, r_prev)
    e_small = np.max(np.abs(small - ref)) / np.max(np.abs(ref))
    e_scaled = np.max(np.abs(scaled - ref)) / np.max(np.abs(ref))
    assert e_scaled < e_small / 10, f"prescale {e_scaled:.2e} vs none {e_small:.2e}"


def test_pow2_floor_is_exact_scaling():
    v = np.array([1.0, 1.5, 0.75, 3e-20, 7e30, 0.0, np.inf, np.nan], np.float32)
    p = pow2_floor(v)
    np.testing.assert_array_equal(p[:5], np.array([1.0, 1.0, 0.5, 2.0 ** -65, 2.0 ** 102], np.float32))
    np.testing.assert_array_equal(p[5:], np.ones(3, np.float32))
    x = np.float32(1.2345678)
    assert (x * p[3]) / p[3] == x  # scaling by a power of two and back is exact
