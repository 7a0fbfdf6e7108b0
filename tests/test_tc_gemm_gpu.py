"""Tensor-core batched GEMV (tcgen05 / TMEM / TMA) against the float64 oracle.

fp16 weights and fp16 activations are exact inputs; the kernel accumulates in fp32 -> 2e-3
elementwise with a floor (the fp16-path tolerance); split-K sums are deterministic.
"""

import numpy as np
import pytest
import torch

from gemmagemini4hackathon2026_10_2425_b200 import ops
from oracle import ops as O
from tests._tol import assert_norm_close, assert_rel_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def case(M, K, b, seed, scale=0.02):
    r = np.random.default_rng(seed)
    W = (r.standard_normal((M, K)) * scale).astype(np.float16)
    X = r.standard_normal((b, K)).astype(np.float16)
    return W, X


def d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("M,K", [(3072, 2048), (2048, 2048), (2048, 8192), (4096, 4096), (14336, 4096), (1000, 520), (128, 64), (200, 72)])
@pytest.mark.parametrize("b", [1, 9, 16, 17, 32])
def test_tc_store(M, K, b):
    W, X = case(M, K, b, M + K + b)
    y = ops.gemm_tc(d(W), d(X)).cpu().numpy()
    assert_rel_close(y, O.gemv(W, X), 2e-3, what=f"{M}x{K} b{b}")


def test_tc_add_fp16_out_and_determinism():
    W, X = case(2048, 2048, 32, 5)
    y0 = np.random.default_rng(6).standard_normal((32, 2048)).astype(np.float32)
    y = d(y0.copy())
    ops.gemm_tc(d(W), d(X), epilogue="add", y=y)
    assert_rel_close(y.cpu().numpy(), y0 + O.gemv(W, X), 2e-3)
    a = ops.gemm_tc(d(W), d(X)).cpu().numpy()
    b = ops.gemm_tc(d(W), d(X)).cpu().numpy()
    np.testing.assert_array_equal(a, b)  # fixed-order split-K reduction
    h = ops.gemm_tc(d(W), d(X), out_dtype=torch.float16)
    assert h.dtype == torch.float16
    assert_rel_close(h.float().cpu().numpy(), O.gemv(W, X), 2e-3)


@pytest.mark.parametrize("b", [12, 32])
def test_tc_swiglu(b):
    Wg, X = case(8192, 2048, b, 7)
    Wu, _ = case(8192, 2048, b, 8)
    h = ops.gemm_tc(d(Wg), d(X), epilogue="swiglu", W_up=d(Wu), out_dtype=torch.float16)
    ref = O.swiglu(O.gemv(Wg, X), O.gemv(Wu, X))
    assert_rel_close(h.float().cpu().numpy(), ref, 2e-3)


def test_tc_gelu_mul():
    W, X = case(1024, 512, 20, 9)
    aux = np.random.default_rng(10).standard_normal((20, 1024)).astype(np.float32)
    y = ops.gemm_tc(d(W), d(X), epilogue="gelu_mul", aux=d(aux))
    assert_rel_close(y.cpu().numpy(), O.gelu_tanh(O.gemv(W, X)) * aux, 2e-3)


@pytest.mark.parametrize("V,b", [(128256, 32), (128256, 16), (5000, 20), (300, 9)])
def test_tc_argmax(V, b):
    W, X = case(V, 2048 if V > 1000 else 128, b, V + b)
    tok, logits = ops.gemm_tc(d(W), d(X), epilogue="argmax", return_logits=True)
    ref = O.gemv(W, X)
    lg = logits.cpu().numpy()
    assert_rel_close(lg, ref, 2e-3)
    np.testing.assert_array_equal(tok.cpu().numpy(), O.argmax(lg))
    srt = np.sort(ref, axis=1)
    safe = (srt[:, -1] - srt[:, -2]) > 1e-3 * np.abs(srt[:, -1])
    np.testing.assert_array_equal(tok.cpu().numpy()[safe], O.argmax(ref)[safe])


def test_tc_argmax_ties_and_offset():
    W = np.zeros((4096, 64), np.float16)
    W[[100, 3000, 4095]] = 0.5
    X = np.ones((10, 64), np.float16)
    tok = ops.gemm_tc(d(W), d(X), epilogue="argmax", index_offset=7).cpu().numpy()
    np.testing.assert_array_equal(tok, np.full(10, 107))


def test_tc_error_word_stays_zero():
    W, X = case(2048, 2048, 32, 11)
    ws = torch.zeros(ops.tc_workspace_bytes(2048, 2048, 32), dtype=torch.uint8, device=DEV)
    ops.gemm_tc(d(W), d(X), workspace=ws)
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 0


@pytest.mark.parametrize("D", [2048, 64, 4096, 4100, 2050])  # vector path; > 4096 or odd: scalar
@pytest.mark.parametrize("with_p", [True, False])
def test_add_rmsnorm_f16(D, with_p):
    r = np.random.default_rng(D)
    x = r.standard_normal((5, D)).astype(np.float32)
    p = r.standard_normal((5, D)).astype(np.float32) if with_p else np.zeros((5, D), np.float32)
    g = (1 + 0.1 * r.standard_normal(D)).astype(np.float32)
    xt = d(x.copy())
    out = ops.add_rmsnorm_f16(xt, d(g), 1e-5, p=d(p) if with_p else None)
    np.testing.assert_array_equal(xt.cpu().numpy(), x + p)  # fp32 add, bit-exact
    assert_rel_close(out.float().cpu().numpy(), O.rmsnorm(x + p, g, 1e-5), 2e-3)


def test_tc_workspace_shared_across_shapes():
    """One workspace reused by calls of different shapes (as the decoder does): each call's
    split-K partials must never land on another call's arrival counters."""
    nbytes = max(ops.tc_workspace_bytes(M, K, 32, e) for M, K, e in [(4096, 4096, "store"), (14336, 4096, "store"), (8192, 2048, "swiglu"), (128256, 2048, "argmax")])
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    for M, K in [(4096, 4096), (14336, 4096), (2048, 8192), (14336, 4096), (3072, 2048)]:
        W, X = case(M, K, 32, M * 3 + K)
        y = ops.gemm_tc(d(W), d(X), workspace=ws).cpu().numpy()
        assert_rel_close(y, O.gemv(W, X), 2e-3, what=f"shared ws {M}x{K}")


def qcase(M, K, fmt, seed):
    r = np.random.default_rng(seed)
    sc = np.abs(r.standard_normal((M, K // 32)) * 0.01).astype(np.float16)
    if fmt == "q8":
        q = r.integers(-127, 128, size=(M, K), dtype=np.int8)
        return q, q, sc
    qv = r.integers(-8, 8, size=(M, K), dtype=np.int8)
    return qv, O.pack_q4(qv), sc


# The quantized tensor-core operand is fp16(scale * q): one fp16 rounding per weight, so the
# check is max-normalized (2e-3 of max|y|), not elementwise.
@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("M,K", [(4096, 4096), (14336, 4096), (4096, 14336), (96, 64), (200, 96), (1000, 544)])
@pytest.mark.parametrize("b", [9, 16, 32])
def test_tc_quant_config3(fmt, M, K, b):
    qv, packed, sc = qcase(M, K, fmt, M + 7 * K + b)
    X = np.random.default_rng(b).standard_normal((b, K)).astype(np.float16)
    Wq = ops.QWeight(fmt, d(packed), d(sc))
    y = ops.gemm_tc_q(Wq, d(X)).cpu().numpy()
    assert_norm_close(y, O.gemv(O.dequant_q8_32(qv, sc), X), 2e-3, what=f"tc {fmt} {M}x{K} b{b}")


@pytest.mark.parametrize("fmt", ["q8", "q4"])
def test_tc_quant_add_gelu_fp16_out(fmt):
    M, K, b = 2048, 8192, 16
    qv, packed, sc = qcase(M, K, fmt, 31)
    W = O.dequant_q8_32(qv, sc)
    r = np.random.default_rng(32)
    X = r.standard_normal((b, K)).astype(np.float16)
    y0 = r.standard_normal((b, M)).astype(np.float32)
    aux = r.standard_normal((b, M)).astype(np.float32)
    Wq = ops.QWeight(fmt, d(packed), d(sc))
    y = d(y0.copy())
    ops.gemm_tc_q(Wq, d(X), epilogue="add", y=y)
    y2 = d(y0.copy())
    ops.gemm_tc_q(Wq, d(X), epilogue="add", y=y2)
    np.testing.assert_array_equal(y.cpu().numpy(), y2.cpu().numpy())  # deterministic split-K
    assert_norm_close(y.cpu().numpy(), y0 + O.gemv(W, X), 2e-3, what=f"{fmt} add")
    g = ops.gemm_tc_q(Wq, d(X), epilogue="gelu_mul", aux=d(aux), out_dtype=torch.float16)
    ref = O.gemv_fused(W, X.astype(np.float32), None, 0.0, O.EPI_GELU_MUL, aux=aux)
    assert_norm_close(g.float().cpu().numpy(), ref, 3e-3, what=f"{fmt} gelu_mul")


def test_tc_quant_bad_arguments_raise():
    qv, packed, sc = qcase(256, 96, "q8", 3)
    Wq = ops.QWeight("q8", d(packed), d(sc))
    with pytest.raises(ValueError):
        ops.gemm_tc_q(Wq, d(np.zeros((33, 96), np.float16)))  # batch > 32
    with pytest.raises(ValueError):
        ops.gemm_tc_q(Wq, d(np.zeros((4, 96), np.float16)), epilogue="swiglu")


def np_pack_tc(W):
    """NumPy restatement of the packed tile layout (b2d_tc_pack_f16)."""
    M, K = W.shape
    mt, kt = -(-M // 128), -(-K // 64)
    Wp = np.zeros((mt * 128, kt * 64), np.float16)
    Wp[:M, :K] = W
    out = np.zeros((mt, kt, 128, 64), np.float16)  # tile image: [row][8 chunks of 8]
    for r in range(128):
        perm = [(c ^ (r % 8)) for c in range(8)]  # chunk c of row r sits at slot c ^ (r % 8)
        src = Wp.reshape(mt, 128, kt, 64)[:, r].reshape(mt, kt, 8, 8)
        dst = np.zeros_like(src)
        dst[:, :, perm] = src
        out[:, :, r] = dst.reshape(mt, kt, 64)
    return out.reshape(-1).view(np.uint8)


@pytest.mark.parametrize("M,K", [(256, 128), (200, 72), (1000, 520)])
def test_tc_pack_layout_bit_exact(M, K):
    W = np.random.default_rng(M).standard_normal((M, K)).astype(np.float16)
    got = ops.pack_tc(d(W)).buf.cpu().numpy()
    np.testing.assert_array_equal(got, np_pack_tc(W))


@pytest.mark.parametrize("epi", ["store", "add", "swiglu", "argmax"])
@pytest.mark.parametrize("M,K,b", [(3072, 2048, 32), (2048, 8192, 32), (1000, 520, 16), (200, 72, 9)])
def test_tc_packed_equals_rowmajor(epi, M, K, b):
    """Same tiles reach the MMA either way: results are bit-identical."""
    W, X = case(M, K, b, 3 * M + K)
    Wu, _ = case(M, K, b, 5 * M + K)
    y0 = np.random.default_rng(8).standard_normal((b, M)).astype(np.float32)
    out = []
    for packed in (False, True):
        Wa = ops.pack_tc(d(W)) if packed else d(W)
        Wb = (ops.pack_tc(d(Wu)) if packed else d(Wu)) if epi == "swiglu" else None
        if epi == "argmax":
            tok, lg = ops.gemm_tc(Wa, d(X), epilogue="argmax", return_logits=True)
            out.append((tok.cpu().numpy(), lg.cpu().numpy()))
        else:
            y = d(y0.copy())
            r = ops.gemm_tc(Wa, d(X), epilogue=epi, W_up=Wb, y=y if epi in ("store", "add") else None)
            out.append((r.float().cpu().numpy(),))
    for a, c in zip(*out):
        np.testing.assert_array_equal(a, c)
    if epi == "store":
        assert_rel_close(out[1][0], O.gemv(W, X), 2e-3)

