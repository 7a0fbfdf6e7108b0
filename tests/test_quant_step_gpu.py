"""The decode step on 32-block quantized projections (b2d_decoder_set_layer_q), against the oracle.

The five projections of every layer stay in their stored format on the device (q8_32: 1.06 bytes
per weight, q4_32: 0.56) and the step streams them as stored.  What each path computes:
  * batch < 9, the tensor-core GEMV: integers exact in fp16, the block scale applied to each
    block's fp32 result -- the exactly dequantized weights w = float(scale) * q;
  * batch >= 9, the tcgen05 GEMM: its MMA operand is fp16(scale * q), one fp16 rounding of the
    dequantized weight; gate/up runs as an up GEMM and a gate GEMM with the SILU_MUL epilogue.
The oracle (oracle/step.py) is fed those same weights and evaluated over the cache the GPU
wrote (elementwise 2e-3 with a floor), and the tcgen05 path is also compared max-normalized with
the exact dequantization.  A quantized weights file (the reference's format with the 32-block
extension) also decodes end to end.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from gemmagemini4hackathon2026_10_2425_b200 import weights as W
from gemmagemini4hackathon2026_10_2425_b200.engine import DecodeEngine, make_block_table
from gemmagemini4hackathon2026_10_2425_b200.tp import ModelShape
from oracle import ops as O
from oracle import step as S
from tests._tol import assert_norm_close, assert_rel_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = Path(__file__).resolve().parent / "golden"
MATS = ("wqkv", "wo", "wgate", "wup", "wdown")


def quantized_model(cfg, fmt, seed):
    """Seeded weights with every projection quantized: (stored tensors, quant map, exactly
    dequantized weights, fp16(scale * q) weights)."""
    w = S.synth_weights(cfg, seed=seed)
    stored, quant, exact, rounded = dict(w), {}, dict(w), dict(w)
    for i in range(cfg.n_layers):
        for n in MATS:
            name = f"l{i}.{n}"
            q, sc = W.quantize(w[name], fmt)
            stored[name], stored[name + ".scales"] = q, sc
            quant[name] = fmt
            deq = W.dequantize(q, sc, fmt)
            exact[name], rounded[name] = deq, deq.astype(np.float16)
    return stored, quant, exact, rounded


@pytest.mark.parametrize("fmt", ["q8_32", "q4_32"])
@pytest.mark.parametrize("batch", [5, 24])
def test_quantized_step_matches_oracle(fmt, batch):
    cfg = S.ModelConfig(2048, 2, 32, 8, 64, 8192, 4096, 1e-5, 500000.0)
    stored, quant, exact, rounded = quantized_model(cfg, fmt, seed=31)
    r = np.random.default_rng(32 + batch)
    lens = r.integers(0, 1200, size=batch).tolist()
    max_ctx = 1216
    nblk = sum(-(-(n + 1) // 16) for n in lens) + 4
    table = make_block_table(lens, max_ctx // 16, nblk, seed=33).numpy()
    pshape = (nblk, cfg.n_kv_heads, 16, cfg.head_dim)
    kp = [r.standard_normal(pshape).astype(np.float16) for _ in range(cfg.n_layers)]
    vp = [r.standard_normal(pshape).astype(np.float16) for _ in range(cfg.n_layers)]
    tokens = r.integers(0, cfg.vocab, size=batch).tolist()
    shape = ModelShape(cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab, cfg.eps, cfg.theta)
    eng = DecodeEngine(shape, max_batch=batch, max_ctx=max_ctx, n_blocks=nblk)
    eng.alloc_kv()
    for i in range(cfg.n_layers):
        eng.k_pages[i].copy_(torch.from_numpy(kp[i]))
        eng.v_pages[i].copy_(torch.from_numpy(vp[i]))
    eng.load_weights({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in stored.items()}, quant)
    # the device holds the stored integers, not fp16 copies
    assert eng.layers[0]["wqkv"].dtype == (torch.int8 if fmt == "q8_32" else torch.uint8)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(DEV)
    tok, ln, tb = d(tokens), d(lens), d(table)
    nxt = torch.empty_like(tok)
    logits = torch.empty(batch, eng.lm_rows, dtype=torch.float32, device=DEV)
    eng.step(tok, ln, tb, nxt, logits, use_graph=True)
    eng.stream.synchronize()
    eng.check()
    got = logits.cpu().numpy()
    gk = [k.cpu().numpy() for k in eng.k_pages]
    gv = [v.cpu().numpy() for v in eng.v_pages]
    eng.close()
    what_path = exact if batch < 9 else rounded
    same_kv, _ = S.decode_step(what_path, cfg, tokens, lens, table, gk, gv, append=False)
    assert_rel_close(got, same_kv, 2e-3, what=f"{fmt} batch {batch} vs oracle over the GPU's KV")
    ref, ref_next = S.decode_step(exact, cfg, tokens, lens, table, kp, vp)
    assert_norm_close(got, ref, 2e-3, what=f"{fmt} batch {batch} vs exact dequantization")
    np.testing.assert_array_equal(nxt.cpu().numpy(), O.argmax(got))


@pytest.mark.parametrize("fmt", ["q8_32", "q4_32"])
@pytest.mark.parametrize("batch", [1, 9])
def test_quantized_weights_file_decodes(tmp_path, monkeypatch, fmt, batch):
    """The tiny reference-converter file, quantized with convert_weights' quantizer, loaded as
    stored: the prompt runs through decode steps and the last position's logits match the
    oracle fed the same (dequantized) weights."""
    src = GOLD / "tiny_llama_weights.bin"
    path = tmp_path / f"{fmt}.bin"
    W.quantize_file(src, path, fmt)
    wf = W.read_weights(path)
    shape = W.shape_from_config(wf.config)
    cfg = S.ModelConfig(shape.dim, shape.n_layers, shape.n_heads, shape.n_kv_heads, shape.head_dim, shape.ffn_dim, shape.vocab, shape.eps, shape.theta)
    ref = np.load(GOLD / "tiny_llama_ref.npz")
    prompt = ref["prompt"].tolist()
    max_ctx = 64
    nblk = batch * (max_ctx // 16) + 2
    dev = torch.device("cuda", 0)
    eng = DecodeEngine(shape, max_batch=batch, max_ctx=max_ctx, n_blocks=nblk, device=dev)
    eng.alloc_kv()
    eng.load_weights_file(path)
    assert eng.layers[0]["wo"].dtype in (torch.int8, torch.uint8)
    table = make_block_table([max_ctx - 1] * batch, max_ctx // 16, nblk, seed=3, headroom=0).to(dev)
    logits = torch.empty(batch, eng.lm_rows, dtype=torch.float32, device=dev)
    nxt = torch.empty(batch, dtype=torch.int32, device=dev)
    for pos, t in enumerate(prompt):
        eng.step(torch.full((batch,), t, dtype=torch.int32, device=dev), torch.full((batch,), pos, dtype=torch.int32, device=dev), table, nxt, logits, use_graph=False)
    eng.stream.synchronize()
    got = logits.cpu().numpy()
    eng.close()
    # the oracle on the same weights: exact dequantization (batch 1) or fp16(scale * q) (batch 9)
    t = {k: np.asarray(v) for k, v in W.tensors_for_engine(wf, keep_quant=True).items()}
    w = {k: v for k, v in t.items() if not k.endswith(".scales") and k != "lm_head"}
    for name, f in wf.quant.items():
        deq = W.dequantize(t[name], t[name + ".scales"], f)
        w[name] = deq if batch < 9 else deq.astype(np.float16)
    invf = W.inv_freq_from_config(wf.config)
    kp = [np.zeros((nblk, cfg.n_kv_heads, 16, cfg.head_dim), np.float16) for _ in range(cfg.n_layers)]
    vp = [np.zeros_like(k) for k in kp]
    tb = table.cpu().numpy()
    monkeypatch.setattr(O, "inv_freq", lambda hd, theta, rs=None: invf)  # the file's Llama-3 scaling
    for pos, t_ in enumerate(prompt):
        lg, _ = S.decode_step(w, cfg, [t_] * batch, [pos] * batch, tb, kp, vp)
    for b in range(batch):
        assert_norm_close(got[b], lg[b], 2e-3, what=f"{fmt} file, batch {batch}, row {b}")
