"""fp32-precision activations on the tensor cores: the B2D_F16X2 hi + lo fp16 planes.

The reference multiplies fp16 weights by fp32 activations (ios_kernels/kernels/
unsloth__Llama-3.2-1B-Instruct/kernel_metal_f16_20261024-1620/kernels.metal:106-131).  The
batched decode path carries each fp32 activation as hi = fp16(x) and lo = fp16(x - hi), and the
tcgen05 GEMM multiplies both planes in one MMA of twice the N.  These tests feed fp32 inputs
(not fp16-representable) and compare with the float64 oracle on the fp32 values:
elementwise 2e-3 with a floor (the fp16-path bound of BASELINE) and max-normalized 2e-5, an
order of magnitude inside what the same product reaches with plain fp16 operands.
"""

import numpy as np
import pytest
import torch

from gemmagemini4hackathon2026_10_2425_b200 import ops
from oracle import ops as O
from tests._tol import assert_norm_close, assert_rel_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
NORM_TOL = 2e-5


def d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def case(M, K, b, seed, xscale=1.0):
    r = np.random.default_rng(seed)
    W = (r.standard_normal((M, K)) * 0.02).astype(np.float16)
    X = (r.standard_normal((b, K)) * xscale).astype(np.float32)
    return W, X


def x2(X):
    return ops.to_f16x2(d(X))


def test_split_planes_bit_exact():
    """to_f16x2 / the kernels' split: hi = fp16(x), lo = fp16(x - hi), both round-to-nearest."""
    X = np.random.default_rng(0).standard_normal((4, 1000)).astype(np.float32) * 3
    t = x2(X).cpu().numpy()
    hi = X.astype(np.float16)
    lo = (X - hi.astype(np.float32)).astype(np.float16)
    np.testing.assert_array_equal(t[0].view(np.uint16), hi.view(np.uint16))
    np.testing.assert_array_equal(t[1].view(np.uint16), lo.view(np.uint16))


@pytest.mark.parametrize("M,K", [(3072, 2048), (2048, 2048), (2048, 8192), (1000, 520), (200, 72)])
@pytest.mark.parametrize("b", [1, 9, 16, 17, 32])
def test_hilo_store(M, K, b):
    W, X = case(M, K, b, M + 7 * K + b)
    y = ops.gemm_tc(d(W), x2(X)).cpu().numpy()
    ref = O.gemv(W, X)
    assert_rel_close(y, ref, 2e-3, what=f"{M}x{K} b{b}")
    assert_norm_close(y, ref, NORM_TOL, what=f"{M}x{K} b{b}")


def test_hilo_beats_fp16_operands():
    """The same product with fp16-rounded activations is off by ~2^-12 relative; hi/lo removes it."""
    W, X = case(2048, 2048, 32, 3)
    ref = O.gemv(W, X)
    e16 = np.max(np.abs(ops.gemm_tc(d(W), d(X.astype(np.float16))).cpu().numpy() - ref)) / np.max(np.abs(ref))
    e32 = np.max(np.abs(ops.gemm_tc(d(W), x2(X)).cpu().numpy() - ref)) / np.max(np.abs(ref))
    print(f"max-normalized error: fp16 operands {e16:.2e}, hi/lo planes {e32:.2e}")
    assert e32 < e16 / 10


def test_hilo_small_magnitudes():
    """Activations far below 1 (lo plane in fp16's subnormal range) keep fp32-level accuracy
    relative to the row's magnitude."""
    W, X = case(2048, 2048, 20, 4, xscale=1e-3)
    y = ops.gemm_tc(d(W), x2(X)).cpu().numpy()
    assert_norm_close(y, O.gemv(W, X), NORM_TOL)


def test_hilo_add_and_determinism():
    W, X = case(2048, 8192, 32, 5)
    y0 = np.random.default_rng(6).standard_normal((32, 2048)).astype(np.float32)
    y = d(y0.copy())
    ops.gemm_tc(d(W), x2(X), epilogue="add", y=y)
    ref = y0 + O.gemv(W, X)
    assert_rel_close(y.cpu().numpy(), ref, 2e-3)
    assert_norm_close(y.cpu().numpy(), ref, NORM_TOL)
    a = ops.gemm_tc(d(W), x2(X)).cpu().numpy()
    b = ops.gemm_tc(d(W), x2(X)).cpu().numpy()
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("b", [12, 32])
def test_hilo_swiglu_planes_out(b):
    """gate/up SwiGLU with hi/lo input and hi/lo output (what feeds the down projection)."""
    Wg, X = case(8192, 2048, b, 7)
    Wu, _ = case(8192, 2048, b, 8)
    h = torch.empty(2, b, 8192, dtype=torch.float16, device=DEV)
    ops.gemm_tc(d(Wg), x2(X), epilogue="swiglu", W_up=d(Wu), y=h)
    got = ops.from_f16x2(h).cpu().numpy()
    ref = O.swiglu(O.gemv(Wg, X), O.gemv(Wu, X))
    assert_rel_close(got, ref, 2e-3)
    assert_norm_close(got, ref, NORM_TOL)
    hv = h.cpu().numpy()  # the planes are a split: lo = fp16(v - hi), |lo| <= ulp(hi) / 2
    assert np.all(np.abs(hv[1].astype(np.float32)) <= np.abs(hv[0].astype(np.float32)) * 2.0**-11 + 2.0**-24)


@pytest.mark.parametrize("V,b", [(128256, 32), (5000, 20), (300, 9)])
def test_hilo_argmax(V, b):
    W, X = case(V, 2048 if V > 1000 else 128, b, V + b)
    tok, logits = ops.gemm_tc(d(W), x2(X), epilogue="argmax", return_logits=True)
    ref = O.gemv(W, X)
    lg = logits.cpu().numpy()
    assert_rel_close(lg, ref, 2e-3)
    assert_norm_close(lg, ref, NORM_TOL)
    np.testing.assert_array_equal(tok.cpu().numpy(), O.argmax(lg))
    srt = np.sort(ref, axis=1)
    safe = (srt[:, -1] - srt[:, -2]) > 1e-5 * np.abs(srt[:, -1])
    np.testing.assert_array_equal(tok.cpu().numpy()[safe], O.argmax(ref)[safe])


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("b", [9, 32])
def test_hilo_quantized(fmt, b):
    """Quantized weights dequantized in shared memory (fp16(scale*q) is the MMA operand), hi/lo x."""
    r = np.random.default_rng(11 + b)
    M, K = 4096, 4096
    if fmt == "q8":
        q = r.integers(-127, 128, (M, K)).astype(np.int8)
        qd = q
    else:
        qi = r.integers(-8, 8, (M, K))
        q, qd = O.pack_q4(qi), qi
    sc = np.abs(r.standard_normal((M, K // 32)) * 0.01).astype(np.float16)
    X = r.standard_normal((b, K)).astype(np.float32)
    Wq = ops.QWeight(fmt, d(q), d(sc))
    y = ops.gemm_tc_q(Wq, x2(X)).cpu().numpy()
    # the operand is fp16(scale * q): round the dequantized weight the same way in the oracle
    w16 = (O.dequant_q8_32(qd.astype(np.int8), sc)).astype(np.float16)
    ref = O.gemv(w16, X)
    assert_rel_close(y, ref, 2e-3)
    assert_norm_close(y, ref, NORM_TOL)


@pytest.mark.parametrize("D", [2048, 4100])  # register path; scalar path
def test_add_rmsnorm_planes(D):
    r = np.random.default_rng(D)
    x = r.standard_normal((5, D)).astype(np.float32)
    p = r.standard_normal((5, D)).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(D)).astype(np.float32)
    xt = d(x.copy())
    out = ops.add_rmsnorm_f16(xt, d(g), 1e-5, p=d(p), x2=True)
    got = ops.from_f16x2(out).cpu().numpy()
    ref = O.rmsnorm(x + p, g, 1e-5)
    # fp32 arithmetic (~1e-6 relative) carried by the planes to ~2^-22 relative, down to fp16's
    # subnormal spacing: below |v| = 2^-3 the lo plane is subnormal, an absolute 2^-25 floor
    np.testing.assert_array_less(np.abs(got - ref), 2e-6 * np.abs(ref) + 2.0**-24)
    assert_norm_close(got, ref, 1e-6, what="hi + lo planes")


def test_attention_planes_out():
    """Paged attention writing its output as hi/lo planes equals its fp32 output."""
    r = np.random.default_rng(21)
    hq, hk, hd, B = 32, 8, 64, 12
    lens = r.integers(0, 900, size=B).astype(np.int32)
    max_ctx = int(lens.max()) + 1
    need = [-(-(int(n) + 1) // 16) for n in lens]
    nblk = sum(need) + 2
    perm = r.permutation(nblk)
    table = np.full((B, -(-max_ctx // 16)), -1, np.int32)
    o = 0
    for b, k in enumerate(need):
        table[b, :k] = perm[o : o + k]
        o += k
    kp = r.standard_normal((nblk, hk, 16, hd)).astype(np.float16)
    vp = r.standard_normal((nblk, hk, 16, hd)).astype(np.float16)
    qkv = r.standard_normal((B, (hq + 2 * hk) * hd)).astype(np.float32)
    invf = d(O.inv_freq(hd, 500000.0))
    outs = []
    for planes in (False, True):
        out = torch.empty((2, B, hq * hd) if planes else (B, hq * hd), dtype=torch.float16 if planes else torch.float32, device=DEV)
        ops.paged_decode_attn(d(qkv), d(kp.copy()), d(vp.copy()), d(table), d(lens), invf, hq, hk, hd, max_ctx, out=out)
        outs.append(ops.from_f16x2(out).cpu().numpy() if planes else out.cpu().numpy())
    f32, planes = outs
    # the planes hold the same fp32 values to ~2^-22 relative (plus fp16's subnormal floor)
    np.testing.assert_allclose(planes, f32, rtol=2.0**-21, atol=2.0**-24)
