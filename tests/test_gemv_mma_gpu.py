"""Parity of the tensor-core GEMV (exact integer fp16 weights on mma.sync, block scale in fp32)
with the float64 oracle, through the C ABI.

The path serves b2d_gemv for fp16 and 32-block quantized weights, so the cases cover what changes
inside it: fp16 activations used as they are vs hi + lo fp16 columns
(fp32 input or the fused RMSNorm), token groups (16 / 8 per pass over W), K slices per row tile
(small K: one slice, several row tiles per CTA), ragged row counts, every epilogue, activations
far from 1 in magnitude (the per-token power-of-two scale), and agreement with the CUDA-core path
on the same inputs.  Tolerance: 2e-3 elementwise with a floor of 1e-3 * max|ref| (the quantized /
fp16 bound of the decode path).
"""

import numpy as np
import pytest
import torch

from gemmagemini4hackathon2026_10_2425_b200 import ops
from oracle import ops as O
from tests._tol import assert_rel_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def quant(M, K, fmt, seed):
    r = np.random.default_rng(seed)
    sc = np.abs(r.standard_normal((M, K // 32)) * 0.01).astype(np.float16)
    if fmt == "q8":
        q = r.integers(-127, 128, size=(M, K), dtype=np.int8)
        return ops.QWeight("q8", t(q), t(sc)), O.dequant_q8_32(q, sc)
    qv = r.integers(-8, 8, size=(M, K), dtype=np.int8)
    packed = O.pack_q4(qv)
    return ops.QWeight("q4", t(packed), t(sc)), O.dequant_q4_32(packed, sc)


def weight(M, K, fmt, seed):
    if fmt == "f16":
        W = (np.random.default_rng(seed).standard_normal((M, K)) * 0.02).astype(np.float16)
        return t(W), W
    return quant(M, K, fmt, seed)


@pytest.fixture
def mma_formats():
    """Run the test with the given formats on the tensor-core path, then restore."""
    prev = ops.gemv_mma_formats()
    yield lambda fmts: ops.gemv_mma_formats(set(fmts))
    ops.gemv_mma_formats(prev)


@pytest.mark.parametrize("fmt", ["q8", "q4", "f16"])
@pytest.mark.parametrize("xkind", ["f16", "f16_norm", "f32", "f32_norm"])
@pytest.mark.parametrize("b", [1, 3, 8, 9, 16, 20])
def test_mma_gemv_activation_paths(fmt, xkind, b, mma_formats):
    mma_formats({fmt, "int8_b1"})  # a single token (b = 1, and the last of b = 9) takes the int8 path
    M, K = 1000, 1024
    Wd, Wref = weight(M, K, fmt, 100 + b)
    r = np.random.default_rng(7 * b + len(xkind))
    x = r.standard_normal((b, K)).astype(np.float16 if xkind.startswith("f16") else np.float32)
    g = (1 + 0.1 * r.standard_normal(K)).astype(np.float32) if xkind.endswith("norm") else None
    y = ops.gemv(Wd, t(x), gamma=None if g is None else t(g), eps=1e-5).cpu().numpy()
    ref = O.gemv_fused(Wref, x, g, 1e-5)
    assert_rel_close(y, ref, 2e-3, what=f"{fmt} {xkind} b{b}")


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("epi", ["store", "add", "gelu_mul", "swiglu"])
@pytest.mark.parametrize("b", [1, 5, 16])
@pytest.mark.parametrize("out", [torch.float32, torch.float16])
def test_mma_gemv_epilogues(fmt, epi, b, out):
    M, K = 700, 2048
    Wd, Wref = quant(M, K, fmt, 31)
    Ud, Uref = quant(M, K, fmt, 32)
    r = np.random.default_rng(33)
    x = r.standard_normal((b, K)).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(K)).astype(np.float32)
    y0 = r.standard_normal((b, M)).astype(np.float32)
    aux = r.standard_normal((b, M)).astype(np.float32)
    y = t(y0).to(out)
    res = ops.gemv(
        Wd, t(x), gamma=t(g), eps=1e-6, epilogue=epi, W_up=Ud if epi == "swiglu" else None,
        aux=t(aux) if epi == "gelu_mul" else None, y=y,
    )
    code = {"store": O.EPI_STORE, "add": O.EPI_ADD, "gelu_mul": O.EPI_GELU_MUL, "swiglu": O.EPI_SWIGLU}[epi]
    y_prev = y0.astype(np.float16).astype(np.float32) if out == torch.float16 else y0
    ref = O.gemv_fused(Wref, x, g, 1e-6, code, y_prev=y_prev, aux=aux, W_up=Uref)
    tol = 2e-3 if out == torch.float32 else 4e-3  # fp16 output adds one rounding (2^-11)
    assert_rel_close(res.float().cpu().numpy(), ref, tol, what=f"{fmt} {epi} b{b}")


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("M,K", [(16, 256), (33, 512), (4097, 256), (300, 14336), (5000, 4096)])
def test_mma_gemv_shapes(fmt, M, K):
    """K slices per row tile from 1 (K = 256: 4-bit rows are one 128-byte batch) to 16, row
    counts that are not multiples of 16, and K = 14336 normalized (2 tokens per pass)."""
    Wd, Wref = quant(M, K, fmt, M + K)
    r = np.random.default_rng(M)
    x = r.standard_normal((5, K)).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(K)).astype(np.float32)
    y = ops.gemv(Wd, t(x), gamma=t(g), eps=1e-6).cpu().numpy()
    assert_rel_close(y, O.gemv_fused(Wref, x, g, 1e-6), 2e-3, what=f"{fmt} {M}x{K}")


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("mag", [1e-6, 1e-2, 3e3, 1e5])
def test_mma_gemv_activation_magnitudes(fmt, mag):
    """fp32 activations far from 1 (1e5 overflows fp16; 1e-6 is below fp16's normal range): the
    per-token power-of-two scale keeps the hi/lo split exact to ~22 bits."""
    Wd, Wref = quant(512, 1024, fmt, 5)
    r = np.random.default_rng(6)
    x = (r.standard_normal((3, 1024)) * mag).astype(np.float32)
    x[1] *= 1e-3  # tokens with different magnitudes in one launch
    y = ops.gemv(Wd, t(x)).cpu().numpy()
    ref = O.gemv_fused(Wref, x)
    for b in range(3):  # each token against its own magnitude
        assert_rel_close(y[b], ref[b], 2e-3, what=f"{fmt} mag {mag} token {b}")


def test_mma_gemv_zero_token():
    Wd, Wref = quant(256, 512, "q8", 8)
    x = np.zeros((2, 512), np.float32)
    x[1] = np.random.default_rng(9).standard_normal(512)
    y = ops.gemv(Wd, t(x)).cpu().numpy()
    np.testing.assert_array_equal(y[0], 0.0)
    assert_rel_close(y[1], O.gemv_fused(Wref, x[1:])[0], 2e-3)


@pytest.mark.parametrize("fmt", ["q8", "q4"])
def test_mma_gemv_agrees_with_cuda_cores(fmt, mma_formats):
    """The same inputs through both paths (formats switched at run time)."""
    Wd, Wref = quant(2048, 4096, fmt, 77)
    r = np.random.default_rng(78)
    x = r.standard_normal((4, 4096)).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(4096)).astype(np.float32)
    mma_formats(set())
    y_cc = ops.gemv(Wd, t(x), gamma=t(g), eps=1e-6).cpu().numpy()
    mma_formats({fmt})
    y_tc = ops.gemv(Wd, t(x), gamma=t(g), eps=1e-6).cpu().numpy()
    ref = O.gemv_fused(Wref, x, g, 1e-6)
    assert_rel_close(y_cc, ref, 2e-3)
    assert_rel_close(y_tc, ref, 2e-3)
    # the tensor-core path is the more exact one: integer weights, ~22-bit activations
    e_tc = np.abs(y_tc - ref).max() / np.abs(ref).max()
    assert e_tc < 1e-5, e_tc


def test_mma_gemv_formats_switch(mma_formats):
    prev = mma_formats({"f16", "q4"})
    assert ops.gemv_mma_formats() == {"f16", "q4"}
    assert prev == {"f16", "q8", "q4"}  # the library default


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("xkind", ["f16", "f32_norm"])
@pytest.mark.parametrize("M,K", [(14336, 4096), (1000, 1024), (37, 256), (300, 14336)])
def test_int8_single_token_path(fmt, xkind, M, K, mma_formats):
    """One token on the integer tensor cores (3 int8 digits of a 21-bit fixed-point token, exact
    int32 block sums, 4-bit weights as q + 8 corrected by the blocks' digit sums) against the
    oracle and against the fp16-operand path on the same inputs."""
    Wd, Wref = quant(M, K, fmt, M + 3)
    r = np.random.default_rng(K)
    x = r.standard_normal((1, K)).astype(np.float16 if xkind == "f16" else np.float32)
    g = (1 + 0.1 * r.standard_normal(K)).astype(np.float32) if xkind.endswith("norm") else None
    gt = None if g is None else t(g)
    ref = O.gemv_fused(Wref, x, g, 1e-6)
    mma_formats({fmt, "int8_b1"})
    y8 = ops.gemv(Wd, t(x), gamma=gt, eps=1e-6).cpu().numpy()
    mma_formats({fmt})
    y16 = ops.gemv(Wd, t(x), gamma=gt, eps=1e-6).cpu().numpy()
    assert_rel_close(y8, ref, 2e-3, what=f"int8 {fmt} {M}x{K}")
    assert_rel_close(y16, ref, 2e-3, what=f"fp16 {fmt} {M}x{K}")
    # 21-bit token, exact integer block sums: max-normalized error ~1e-6
    e8 = np.abs(y8 - ref).max() / np.abs(ref).max()
    assert e8 < 2e-5, e8


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("mag", [1e-7, 1.0, 1e6])
def test_int8_single_token_magnitudes(fmt, mag, mma_formats):
    mma_formats({fmt, "int8_b1"})
    Wd, Wref = quant(256, 512, fmt, 15)
    x = (np.random.default_rng(16).standard_normal((1, 512)) * mag).astype(np.float32)
    y = ops.gemv(Wd, t(x)).cpu().numpy()
    assert_rel_close(y, O.gemv_fused(Wref, x), 2e-3, what=f"{fmt} mag {mag}")
    z = ops.gemv(Wd, t(np.zeros((1, 512), np.float32))).cpu().numpy()
    np.testing.assert_array_equal(z, 0.0)


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("epi", ["add", "gelu_mul", "swiglu"])
def test_int8_single_token_epilogues(fmt, epi, mma_formats):
    mma_formats({fmt, "int8_b1"})
    M, K = 600, 2048
    Wd, Wref = quant(M, K, fmt, 41)
    Ud, Uref = quant(M, K, fmt, 42)
    r = np.random.default_rng(43)
    x = r.standard_normal((1, K)).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(K)).astype(np.float32)
    y0 = r.standard_normal((1, M)).astype(np.float32)
    aux = r.standard_normal((1, M)).astype(np.float32)
    res = ops.gemv(
        Wd, t(x), gamma=t(g), eps=1e-6, epilogue=epi, W_up=Ud if epi == "swiglu" else None,
        aux=t(aux) if epi == "gelu_mul" else None, y=t(y0.copy()),
    )
    code = {"add": O.EPI_ADD, "gelu_mul": O.EPI_GELU_MUL, "swiglu": O.EPI_SWIGLU}[epi]
    ref = O.gemv_fused(Wref, x, g, 1e-6, code, y_prev=y0, aux=aux, W_up=Uref)
    assert_rel_close(res.cpu().numpy(), ref, 2e-3, what=f"{fmt} {epi}")


@pytest.mark.parametrize(
    "M,K,epi,norm",
    [(3072, 2048, "store", True), (2048, 2048, "add", False), (8192, 2048, "swiglu", True),
     (2048, 8192, "add", False)],
)
@pytest.mark.parametrize("b", [1, 5, 8])
def test_mma_gemv_f16_decoder_projections(M, K, epi, norm, b):
    """fp16 weights at the small-batch decode step's projections (QKV with the attention norm,
    O + residual, gate/up SwiGLU with the FFN norm, down + residual), fp32 activations."""
    r = np.random.default_rng(M + K + b)
    W = (r.standard_normal((M, K)) * 0.02).astype(np.float16)
    Wu = (r.standard_normal((M, K)) * 0.02).astype(np.float16)
    x = r.standard_normal((b, K)).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(K)).astype(np.float32) if norm else None
    y0 = r.standard_normal((b, M)).astype(np.float32)
    res = ops.gemv(
        t(W), t(x), gamma=None if g is None else t(g), eps=1e-5, epilogue=epi,
        W_up=t(Wu) if epi == "swiglu" else None, y=t(y0.copy()),
    )
    code = {"store": O.EPI_STORE, "add": O.EPI_ADD, "swiglu": O.EPI_SWIGLU}[epi]
    ref = O.gemv_fused(W, x, g, 1e-5, code, y_prev=y0, W_up=Wu)
    assert_rel_close(res.cpu().numpy(), ref, 2e-3, what=f"{M}x{K} {epi} b{b}")


@pytest.mark.parametrize("fmt", ["f16", "q8", "q4"])
@pytest.mark.parametrize("K", [2048, 8192])
def test_mma_gemv_accuracy_long_k(fmt, K, mma_formats):
    """Max-normalized error vs float64 stays at the fp32-accumulation level (< 1e-5) over long K,
    including rows whose terms cancel (a residual stream with a large mean)."""
    mma_formats({fmt})
    M = 1024
    Wd, Wref = weight(M, K, fmt, K + 1)
    r = np.random.default_rng(K + 2)
    x = (r.standard_normal((4, K)) + 3.0).astype(np.float32)  # large common mean: terms cancel
    y = ops.gemv(Wd, t(x)).cpu().numpy()
    ref = O.gemv_fused(Wref, x)
    e = np.abs(y - ref).max() / np.abs(ref).max()
    assert e < 1e-5, (fmt, K, e)
