"""Parity of the GEMV family (CUDA, through the C ABI) with the float64 CPU oracle.

Tolerances: 1e-5 relative for the fp32 path (max-normalized: fp32
accumulation error scales with the terms, not with each result), 2e-3 for fp16 / quantized
paths (elementwise with a floor of 1e-3 * max|ref|); dequantized weights bit-exact.
"""

import numpy as np
import pytest
import torch

from gemmagemini4hackathon2026_10_2425_b200 import ops
from oracle import ops as O
from tests._tol import assert_norm_close, assert_rel_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rng(seed):
    return np.random.default_rng(seed)


def t(a, dtype=None):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV) if dtype is None else torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def test_gemv_f32_config1():
    """Config 1: W [2048, 2048] ~ N(0, 0.02), x ~ N(0, 1), fp32, 1e-5."""
    r = rng(1)
    W = (r.standard_normal((2048, 2048)) * 0.02).astype(np.float32)
    x = r.standard_normal(2048).astype(np.float32)
    y = ops.gemv_f32(t(W), t(x)).cpu().numpy()
    assert_norm_close(y, O.gemv(W, x), 1e-5, what="gemv_f32")


@pytest.mark.parametrize("M,K", [(2048, 4), (37, 36), (5, 4096), (3000, 2048)])
def test_gemv_f32_odd_shapes(M, K):
    r = rng(M + K)
    W = r.standard_normal((M, K)).astype(np.float32)
    x = r.standard_normal(K).astype(np.float32)
    assert_norm_close(ops.gemv_f32(t(W), t(x)).cpu().numpy(), O.gemv(W, x), 1e-5)


def _f16_case(M, K, b, seed):
    r = rng(seed)
    W = (r.standard_normal((M, K)) * 0.02).astype(np.float16)
    x = r.standard_normal((b, K)).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(K)).astype(np.float32)
    return W, x, g


@pytest.mark.parametrize(
    "M,K", [(2048, 2048), (16384, 2048), (2048, 16384), (256000, 2048), (40, 24), (100, 520)]
)
def test_rmsnorm_gemv_f16_config2(M, K):
    """Config 2 shapes (fused RMSNorm, eps 1e-6, gamma ~ 1 + N(0, 0.1)) plus ragged ones."""
    W, x, g = _f16_case(M, K, 1, M + 3 * K)
    y = ops.gemv(t(W), t(x), gamma=t(g), eps=1e-6).cpu().numpy()
    assert_rel_close(y, O.gemv_fused(W, x, g, 1e-6), 2e-3, what=f"{M}x{K}")


@pytest.mark.parametrize("b", [1, 2, 3, 4, 5, 8, 13, 16, 32])
def test_gemv_f16_batches(b):
    W, x, g = _f16_case(520, 1024, b, 11 + b)
    y = ops.gemv(t(W), t(x), gamma=t(g), eps=1e-5).cpu().numpy()
    assert_rel_close(y, O.gemv_fused(W, x, g, 1e-5), 2e-3)


@pytest.mark.parametrize("epi", ["store", "add", "gelu_mul", "swiglu"])
@pytest.mark.parametrize("b", [1, 4])
def test_gemv_epilogues(epi, b):
    r = rng(7)
    M, K = 1000, 512
    W, x, g = _f16_case(M, K, b, 21)
    Wu = (r.standard_normal((M, K)) * 0.02).astype(np.float16)
    y0 = r.standard_normal((b, M)).astype(np.float32)
    aux = r.standard_normal((b, M)).astype(np.float32)
    y = t(y0.copy())
    out = ops.gemv(
        t(W),
        t(x),
        gamma=t(g),
        eps=1e-6,
        epilogue=epi,
        W_up=t(Wu) if epi == "swiglu" else None,
        aux=t(aux) if epi == "gelu_mul" else None,
        y=y,
    )
    code = {"store": O.EPI_STORE, "add": O.EPI_ADD, "gelu_mul": O.EPI_GELU_MUL, "swiglu": O.EPI_SWIGLU}[epi]
    ref = O.gemv_fused(W, x, g, 1e-6, code, y_prev=y0, aux=aux, W_up=Wu)
    assert_rel_close(out.cpu().numpy(), ref, 2e-3, what=epi)


def test_gemv_fp16_activations_and_output():
    r = rng(5)
    M, K, b = 777, 640, 3
    W = (r.standard_normal((M, K)) * 0.02).astype(np.float16)
    x = r.standard_normal((b, K)).astype(np.float16)
    y = ops.gemv(t(W), t(x), out_dtype=torch.float16)
    assert y.dtype == torch.float16
    assert_rel_close(y.float().cpu().numpy(), O.gemv(W, x), 2e-3)


def _quant(M, K, fmt, seed):
    r = rng(seed)
    sc = np.abs(r.standard_normal((M, K // 32)) * 0.01).astype(np.float16)
    if fmt == "q8":
        q = r.integers(-127, 128, size=(M, K), dtype=np.int8)
        return q, q, sc
    qv = r.integers(-8, 8, size=(M, K), dtype=np.int8)
    return qv, O.pack_q4(qv), sc


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("M,K", [(4096, 4096), (14336, 4096), (96, 64)])
@pytest.mark.parametrize("b", [1, 16])
def test_quant_gemv_config3(fmt, M, K, b):
    qv, packed, sc = _quant(M, K, fmt, M + K + b)
    x = rng(9).standard_normal((b, K)).astype(np.float16)
    Wq = ops.QWeight(fmt, t(packed), t(sc))
    y = ops.gemv(Wq, t(x)).cpu().numpy()
    ref = O.gemv(O.dequant_q8_32(qv, sc), x)
    assert_rel_close(y, ref, 2e-3, what=f"{fmt} {M}x{K} b{b}")


@pytest.mark.parametrize("fmt", ["q8", "q4"])
def test_dequant_bit_exact(fmt):
    qv, packed, sc = _quant(300, 4096, fmt, 17)
    w = ops.dequant(ops.QWeight(fmt, t(packed), t(sc))).cpu().numpy()
    ref = O.dequant_q8_32(qv, sc) if fmt == "q8" else O.dequant_q4_32(packed, sc)
    assert w.dtype == np.float32
    np.testing.assert_array_equal(w.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("V,b", [(256000, 1), (128256, 4), (1000, 3), (50, 9)])
def test_lm_head_argmax(V, b):
    W, x, g = _f16_case(V, 2048 if V > 1000 else 64, b, V)
    tok, logits, mx = ops.lm_head_argmax(t(W), t(x), t(g), 1e-5, return_logits=True, return_max=True)
    ref_logits = O.gemv_fused(W, x, g, 1e-5)
    assert_rel_close(logits.cpu().numpy(), ref_logits, 2e-3)
    # the fused argmax must agree exactly with an argmax of the kernel's own logits
    np.testing.assert_array_equal(tok.cpu().numpy(), O.argmax(logits.cpu().numpy()))
    np.testing.assert_array_equal(mx.cpu().numpy(), logits.cpu().numpy().max(axis=1))
    # and with the oracle wherever the top-2 margin exceeds the tolerance
    srt = np.sort(ref_logits, axis=1)
    safe = (srt[:, -1] - srt[:, -2]) > 1e-3 * np.abs(srt[:, -1])
    np.testing.assert_array_equal(tok.cpu().numpy()[safe], O.argmax(ref_logits)[safe])


def test_argmax_ties_lowest_index():
    logits = np.zeros((3, 5000), np.float32)
    logits[0, [7, 4000]] = 3.0
    logits[1, :] = 1.0
    logits[2, [4999, 10, 11]] = [2.0, 2.0, 1.5]
    got = ops.argmax_f32(t(logits)).cpu().numpy()
    np.testing.assert_array_equal(got, [7, 0, 10])
    # the fused LM-head argmax: identical rows of W -> identical logits -> lowest index wins
    W = np.zeros((4096, 64), np.float16)
    W[[100, 3000, 4095]] = 0.5
    x = np.ones((2, 64), np.float32)
    tok = ops.lm_head_argmax(t(W), t(x)).cpu().numpy()
    np.testing.assert_array_equal(tok, [100, 100])


def test_argmax_combine_ties():
    vals = np.array([[1.0, 5.0], [2.0, 5.0], [2.0, 4.0]], np.float32)
    idx = np.array([[10, 900], [500, 20], [400, 1]], np.int32)
    got = ops.argmax_combine(t(vals), t(idx)).cpu().numpy()
    np.testing.assert_array_equal(got, [400, 20])


def test_small_ops():
    r = rng(12)
    x = r.standard_normal((3, 2048)).astype(np.float32)
    w = (1 + 0.1 * r.standard_normal(2048)).astype(np.float32)
    assert_rel_close(ops.rmsnorm(t(x), t(w), 1e-5).cpu().numpy(), O.rmsnorm(x, w, 1e-5), 1e-5)
    E = r.standard_normal((100, 64)).astype(np.float16)
    tok = np.array([3, 99, 0], np.int32)
    np.testing.assert_array_equal(ops.embed_f16(t(E), t(tok)).cpu().numpy(), O.embed(E, tok))


def test_bad_arguments_raise():
    W = torch.zeros(64, 64, dtype=torch.float16, device=DEV)
    x = torch.zeros(1, 64, dtype=torch.float32, device=DEV)
    with pytest.raises(ValueError):
        ops.gemv(W[:, 1:].contiguous(), x[:, 1:].contiguous())  # K=63: not a multiple of 8
    with pytest.raises(ValueError):  # misaligned base pointer
        base = torch.zeros(64 * 64 + 1, dtype=torch.float16, device=DEV)
        ops.gemv(base[1:].view(64, 64), x)
