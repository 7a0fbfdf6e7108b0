"""RMSNorm folded into the tcgen05 GEMM pair of the single-GPU step (batch >= 9).

The O and down projections write x * gamma (times a power of two) and per-slice sums of x^2,
and the next GEMM scales its product by the norm factor; quantized layers keep a separate
add_rmsnorm launch after each residual add.  Checked here:
  * the folded step against the same step with the separate launches (B2D_NORM_FOLD=0, read
    once per process, so that step runs in a child process): the same arithmetic up to rounding
    order, 1e-4 max-normalized;
  * a model whose layers alternate fp16 and q8_32 weights -- every transition between a folded
    and an unfolded boundary -- against the oracle, elementwise over the cache the GPU wrote.
"""

import json
import os
import subprocess
import sys
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
ROOT = Path(__file__).resolve().parent.parent
CFG = S.ModelConfig(2048, 3, 32, 8, 64, 8192, 4096, 1e-5, 500000.0)
MATS = ("wqkv", "wo", "wgate", "wup", "wdown")


def _inputs(batch, seed):
    r = np.random.default_rng(seed)
    lens = r.integers(0, 1200, size=batch).tolist()
    max_ctx = 1216
    nblk = sum(-(-(n + 1) // 16) for n in lens) + 4
    table = make_block_table(lens, max_ctx // 16, nblk, seed=seed + 1).numpy()
    shape = (nblk, CFG.n_kv_heads, 16, CFG.head_dim)
    kp = [r.standard_normal(shape).astype(np.float16) for _ in range(CFG.n_layers)]
    vp = [r.standard_normal(shape).astype(np.float16) for _ in range(CFG.n_layers)]
    tokens = r.integers(0, CFG.vocab, size=batch).tolist()
    return lens, max_ctx, nblk, table, kp, vp, tokens


def _step(w, quant, batch, seed):
    """One graph-replayed step on cuda:0: (logits, next tokens, K pages, V pages)."""
    lens, max_ctx, nblk, table, kp, vp, tokens = _inputs(batch, seed)
    shape = ModelShape(CFG.dim, CFG.n_layers, CFG.n_heads, CFG.n_kv_heads, CFG.head_dim, CFG.ffn_dim, CFG.vocab, CFG.eps, CFG.theta)
    dev = torch.device("cuda", 0)
    eng = DecodeEngine(shape, max_batch=batch, max_ctx=max_ctx, n_blocks=nblk, device=dev)
    eng.alloc_kv()
    for i in range(CFG.n_layers):
        eng.k_pages[i].copy_(torch.from_numpy(kp[i]))
        eng.v_pages[i].copy_(torch.from_numpy(vp[i]))
    eng.load_weights({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in w.items()}, quant or None)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(dev)
    tok, ln, tb = d(tokens), d(lens), d(table)
    nxt = torch.empty_like(tok)
    logits = torch.empty(batch, eng.lm_rows, dtype=torch.float32, device=dev)
    eng.step(tok, ln, tb, nxt, logits, use_graph=True)
    eng.stream.synchronize()
    eng.check()
    out = (logits.cpu().numpy(), nxt.cpu().numpy(), [k.cpu().numpy() for k in eng.k_pages], [v.cpu().numpy() for v in eng.v_pages])
    eng.close()
    return out


def _child(out_path: str, batch: int, seed: int) -> None:
    """Entry point of the child process: the fp16 step with the environment it was given."""
    logits, nxt, _, _ = _step(S.synth_weights(CFG, seed=seed), None, batch, seed)
    np.savez(out_path, logits=logits, nxt=nxt)


def test_folded_step_matches_separate_norm_launches(tmp_path):
    batch, seed = 24, 41
    got, got_next, _, _ = _step(S.synth_weights(CFG, seed=seed), None, batch, seed)
    out = tmp_path / "nofold.npz"
    code = f"import sys; sys.path.insert(0, {json.dumps(str(ROOT))}); from tests.test_norm_fold_gpu import _child; _child({json.dumps(str(out))}, {batch}, {seed})"
    env = dict(os.environ, B2D_NORM_FOLD="0")
    r = subprocess.run([sys.executable, "-c", code], env=env, cwd=str(ROOT), capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    ref = np.load(out)
    assert_norm_close(got, ref["logits"], 1e-4, what="folded vs separate RMSNorm launches")
    srt = np.sort(ref["logits"], axis=1)
    safe = (srt[:, -1] - srt[:, -2]) > 1e-4 * np.abs(srt).max(axis=1)
    np.testing.assert_array_equal(got_next[safe], ref["nxt"][safe])


def test_mixed_fp16_and_quantized_layers_match_oracle():
    """Layers fp16, q8_32, fp16: the fp16 layer before a quantized one ends with a separate
    norm, the quantized layer norms separately, and the fp16 layer after it folds again
    starting from a normalized operand."""
    batch, seed = 24, 51
    w = S.synth_weights(CFG, seed=seed)
    stored, quant, rounded = dict(w), {}, dict(w)
    for n in MATS:
        name = f"l1.{n}"
        q, sc = W.quantize(w[name], "q8_32")
        stored[name], stored[name + ".scales"] = q, sc
        quant[name] = "q8_32"
        rounded[name] = W.dequantize(q, sc, "q8_32").astype(np.float16)  # the tcgen05 operand
    got, got_next, gk, gv = _step(stored, quant, batch, seed)
    lens, _, _, table, kp, vp, tokens = _inputs(batch, seed)
    same_kv, _ = S.decode_step(rounded, CFG, tokens, lens, table, gk, gv, append=False)
    assert_rel_close(got, same_kv, 2e-3, what="mixed-format step vs oracle over the GPU's KV")
    ref, _ = S.decode_step(rounded, CFG, tokens, lens, table, kp, vp)
    assert_norm_close(got, ref, 2e-3, what="mixed-format step vs independent oracle")
    np.testing.assert_array_equal(got_next, O.argmax(got))
