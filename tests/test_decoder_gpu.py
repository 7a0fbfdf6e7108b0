"""The whole decode step (b2d_decoder_step) against the CPU oracle and the HF golden vectors."""

import numpy as np
import pytest
import torch

from gemmagemini4hackathon2026_10_2425_b200.engine import DecodeEngine, make_block_table
from gemmagemini4hackathon2026_10_2425_b200.tp import ModelShape
from oracle import ops as O
from oracle import step as S
from tests._tol import assert_norm_close, assert_rel_close
from tests.test_oracle_golden import _tiny_cfg, _tiny_weights, build_paged_cache

pytestmark = pytest.mark.gpu
DEV = "cuda"


def to_shape(cfg: S.ModelConfig) -> ModelShape:
    return ModelShape(cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab, cfg.eps, cfg.theta)


def run_engine(cfg, w, tokens, lens, table, kp, vp, n_steps=1, use_graph=True):
    """Load weights + pages into a DecodeEngine, run n_steps steps on the same inputs."""
    max_ctx = table.shape[1] * 16
    eng = DecodeEngine(to_shape(cfg), max_batch=len(tokens), max_ctx=max_ctx, n_blocks=kp[0].shape[0])
    eng.alloc_kv()
    for i in range(cfg.n_layers):
        eng.k_pages[i].copy_(torch.from_numpy(kp[i]))
        eng.v_pages[i].copy_(torch.from_numpy(vp[i]))
    eng.load_weights({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in w.items()})
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(DEV)
    tok, ln, tb = d(tokens), d(lens), d(table)
    nxt = torch.empty_like(tok)
    logits = torch.empty(len(tokens), eng.lm_rows, dtype=torch.float32, device=DEV)
    for _ in range(n_steps):
        eng.step(tok, ln, tb, nxt, logits, use_graph=use_graph)
    eng.stream.synchronize()
    out = (logits.cpu().numpy(), nxt.cpu().numpy(), [k.cpu().numpy() for k in eng.k_pages], [v.cpu().numpy() for v in eng.v_pages])
    eng.close()
    return out


@pytest.mark.parametrize("use_graph", [False, True])
def test_decode_step_matches_hf_golden(golden, use_graph):
    """Tiny HF Llama (fixture): engine logits == HF last-position logits (fp16 cache)."""
    cfg = _tiny_cfg(golden)
    w = _tiny_weights(golden, cfg)
    lens, table, kp, vp = build_paged_cache(golden, cfg, np.float16)
    tokens = [int(golden[f"llm_s{b}_ids"][-1]) for b in range(len(lens))]
    # pad the block table to a full max_ctx row
    logits, nxt, gk, gv = run_engine(cfg, w, tokens, lens, table, kp, vp, n_steps=2, use_graph=use_graph)
    ref_logits, ref_next = S.decode_step(w, cfg, tokens, lens, table, [k.copy() for k in kp], [v.copy() for v in vp])
    assert_rel_close(logits, ref_logits, 2e-3, what="logits vs oracle")
    for b in range(len(lens)):
        # HF keeps K/V in fp32, the engine (like the reference) in fp16: compare max-normalized
        hf = golden[f"llm_s{b}_logits"]
        assert_norm_close(logits[b], hf, 1e-2, what="logits vs HF (fp16 KV cache)")
        assert int(np.argmax(logits[b])) == int(np.argmax(hf))
    np.testing.assert_array_equal(nxt, ref_next)


def test_decode_step_llama_shape_small_batch():
    """1B-layout layer widths with 2 layers and a small vocab, ragged contexts."""
    cfg = S.ModelConfig(2048, 2, 32, 8, 64, 8192, 4096, 1e-5, 500000.0)
    w = S.synth_weights(cfg, seed=5)
    r = np.random.default_rng(6)
    lens = [700, 33, 1500, 0, 257]
    max_ctx = 1600
    table = make_block_table(lens, -(-max_ctx // 16), 400, seed=7).numpy()
    shape = (400, cfg.n_kv_heads, 16, cfg.head_dim)
    kp = [r.standard_normal(shape).astype(np.float16) for _ in range(cfg.n_layers)]
    vp = [r.standard_normal(shape).astype(np.float16) for _ in range(cfg.n_layers)]
    tokens = r.integers(0, cfg.vocab, size=len(lens)).tolist()
    kp_orig_v = [v.copy() for v in vp]
    logits, nxt, gk, gv = run_engine(cfg, w, tokens, lens, table, kp, vp)
    ref_logits, ref_next = S.decode_step(w, cfg, tokens, lens, table, kp, vp)
    # The appended K/V are fp16 roundings of computed values, and the step's logits depend on
    # which way each one rounds: sequence 3 (no context) attends only to its own V, where one
    # fp16 ulp moves near-zero logits by 4e-3 - 9e-3 of the elementwise bound (max-normalized:
    # 1e-5).  Elementwise, the step is therefore checked against the oracle evaluated over the
    # cache the GPU wrote; the independent oracle is checked max-normalized.
    same_kv, _ = S.decode_step(
        w, cfg, tokens, lens, table, [k.copy() for k in gk], [v.copy() for v in gv], append=False
    )
    assert_rel_close(logits, same_kv, 2e-3, what="logits vs oracle over the GPU's KV")
    assert_norm_close(logits, ref_logits, 2e-3, what="logits vs oracle")
    srt = np.sort(ref_logits, axis=1)
    safe = (srt[:, -1] - srt[:, -2]) > 2e-3 * np.abs(srt[:, -1])
    np.testing.assert_array_equal(nxt[safe], ref_next[safe])
    # the appended token lands exactly in its page slot; its value comes from the fp32 QKV
    # GEMV, so it may differ from the float64 oracle by one fp16 rounding
    for a, b, orig in zip(gv, vp, kp_orig_v):
        changed_gpu = np.any(a.view(np.uint16) != orig.view(np.uint16), axis=-1)
        changed_ref = np.any(b.view(np.uint16) != orig.view(np.uint16), axis=-1)
        np.testing.assert_array_equal(changed_gpu, changed_ref)
        np.testing.assert_allclose(a.astype(np.float32), b.astype(np.float32), rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("use_graph", [False, True])
def test_decode_step_tensor_core_batch(use_graph):
    """Batch 24 takes the tcgen05 path (hi/lo fp16 activation planes, fused norms)."""
    cfg = S.ModelConfig(2048, 2, 32, 8, 64, 8192, 4096, 1e-5, 500000.0)
    w = S.synth_weights(cfg, seed=15)
    r = np.random.default_rng(16)
    lens = r.integers(0, 1200, size=24).tolist()
    max_ctx = 1300
    nblk = sum(-(-(n + 1) // 16) for n in lens) + 4
    table = make_block_table(lens, -(-max_ctx // 16), nblk, seed=17).numpy()
    shape = (nblk, cfg.n_kv_heads, 16, cfg.head_dim)
    kp = [r.standard_normal(shape).astype(np.float16) for _ in range(cfg.n_layers)]
    vp = [r.standard_normal(shape).astype(np.float16) for _ in range(cfg.n_layers)]
    tokens = r.integers(0, cfg.vocab, size=len(lens)).tolist()
    logits, nxt, gk, gv = run_engine(cfg, w, tokens, lens, table, kp, vp, use_graph=use_graph)
    ref_logits, ref_next = S.decode_step(w, cfg, tokens, lens, table, [k.copy() for k in kp], [v.copy() for v in vp])
    # every projection's activation operand carries fp32 precision (hi + lo fp16 planes), so the
    # step is checked elementwise, over the cache the GPU wrote (the appended K/V are fp16
    # roundings whose direction moves near-zero logits; see the batch-5 test), and
    # max-normalized against the independent oracle
    same_kv, _ = S.decode_step(
        w, cfg, tokens, lens, table, [k.copy() for k in gk], [v.copy() for v in gv], append=False
    )
    assert_rel_close(logits, same_kv, 2e-3, what="tensor-core step vs oracle over the GPU's KV")
    assert_norm_close(logits, ref_logits, 2e-3, what="tensor-core step logits")
    np.testing.assert_array_equal(nxt, O.argmax(logits))
    srt = np.sort(ref_logits, axis=1)
    safe = (srt[:, -1] - srt[:, -2]) > 2e-3 * np.abs(srt[:, -1])
    np.testing.assert_array_equal(nxt[safe], ref_next[safe])
