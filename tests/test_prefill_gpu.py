"""Chunked prefill (b2d_decoder_prefill) against the oracle run one token at a time, and against
HF transformers on the golden tiny Llama.

Prefill pushes up to max_batch consecutive positions of one sequence through one decode step:
the chunk's K/V are written first (rope_kv_append), then every row attends to the positions up
to its own.  Chunks of 9 or more rows take the tcgen05 projections with fp16 activation
operands, so the model-level checks are max-normalized (2e-3), like the batched decode step's;
the K/V written into the pages are compared slot by slot.
"""

import numpy as np
import pytest
import torch

from gemmagemini4hackathon2026_10_2425_b200 import weights as W
from gemmagemini4hackathon2026_10_2425_b200.engine import DecodeEngine
from gemmagemini4hackathon2026_10_2425_b200.tp import ModelShape
from oracle import step as S
from tests._tol import assert_norm_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = "tests/golden"
# Llama layout at a width the float64 oracle runs token by token in well under a second per step
SMALL = S.ModelConfig(512, 2, 8, 2, 64, 2048, 2048, 1e-5, 500000.0)


def _engine(cfg, w, max_ctx, n_blocks, max_batch=32):
    shape = ModelShape(cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab, cfg.eps, cfg.theta)
    eng = DecodeEngine(shape, max_batch=max_batch, max_ctx=max_ctx, n_blocks=n_blocks)
    eng.alloc_kv()
    eng.load_weights({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in w.items()})
    return eng


def _oracle_prefill(w, cfg, ids, table_row, kp, vp, start=0):
    """The oracle's decode step, one token at a time (batch 1): logits of the last position."""
    logits = None
    for i, t in enumerate(ids):
        logits, _ = S.decode_step(w, cfg, [t], [start + i], table_row[None, :], kp, vp)
    return logits[0]


@pytest.mark.parametrize("n", [1, 8, 33, 70])
def test_prefill_matches_tokenwise_oracle(n):
    cfg = SMALL
    w = S.synth_weights(cfg, seed=21)
    r = np.random.default_rng(22 + n)
    ids = r.integers(0, cfg.vocab, size=n).tolist()
    max_ctx, n_blocks = 128, 24
    table_row = r.permutation(n_blocks)[: max_ctx // 16].astype(np.int32)  # scattered pages
    eng = _engine(cfg, w, max_ctx, n_blocks)
    logits = torch.empty(eng.lm_rows, dtype=torch.float32, device=DEV)
    ids_d, tb = torch.tensor(ids, dtype=torch.int32, device=DEV), torch.from_numpy(table_row).to(DEV)
    torch.cuda.synchronize()  # inputs made on the current stream; the engine runs on its own
    nxt = eng.prefill(ids_d, tb, 0, logits=logits)
    eng.stream.synchronize()
    shape = (n_blocks, cfg.n_kv_heads, 16, cfg.head_dim)
    kp = [np.zeros(shape, np.float16) for _ in range(cfg.n_layers)]
    vp = [np.zeros(shape, np.float16) for _ in range(cfg.n_layers)]
    ref = _oracle_prefill(w, cfg, ids, table_row, kp, vp)
    got = logits.cpu().numpy()
    assert_norm_close(got, ref, 2e-3, what=f"prefill logits n={n}")
    assert int(nxt.item()) == int(np.argmax(got))
    # every prompt position's K/V landed in its page slot
    for li in range(cfg.n_layers):
        gk, gv = eng.k_pages[li].cpu().numpy(), eng.v_pages[li].cpu().numpy()
        for pos in range(n):
            blk, slot = table_row[pos // 16], pos % 16
            np.testing.assert_allclose(gk[blk, :, slot].astype(np.float32), kp[li][blk, :, slot].astype(np.float32), rtol=2e-2, atol=2e-2)
            np.testing.assert_allclose(gv[blk, :, slot].astype(np.float32), vp[li][blk, :, slot].astype(np.float32), rtol=2e-2, atol=2e-2)
        untouched = np.setdiff1d(np.arange(n_blocks), table_row[: -(-n // 16)])
        assert not gk[untouched].any() and not gv[untouched].any()  # no stray writes
    eng.close()


def test_prefill_continues_from_start_pos():
    """A second prefill at start_pos = 40 extends the same sequence: the final logits equal the
    oracle over the whole 70 tokens, and equal a single 70-token prefill (max-normalized)."""
    cfg = SMALL
    w = S.synth_weights(cfg, seed=31)
    r = np.random.default_rng(32)
    ids = r.integers(0, cfg.vocab, size=70).tolist()
    table_row = np.arange(8, dtype=np.int32)
    eng = _engine(cfg, w, 128, 8)
    d = lambda a: torch.tensor(a, dtype=torch.int32, device=DEV)
    tb = torch.from_numpy(table_row).to(DEV)
    lg1, lg2 = (torch.empty(eng.lm_rows, dtype=torch.float32, device=DEV) for _ in range(2))
    a, b, c = d(ids[:40]), d(ids[40:]), d(ids)
    torch.cuda.synchronize()
    eng.prefill(a, tb, 0)
    eng.prefill(b, tb, 40, logits=lg2)
    eng.prefill(c, tb, 0, logits=lg1)
    eng.stream.synchronize()
    shape = (8, cfg.n_kv_heads, 16, cfg.head_dim)
    kp = [np.zeros(shape, np.float16) for _ in range(2)]
    vp = [np.zeros(shape, np.float16) for _ in range(2)]
    ref = _oracle_prefill(w, cfg, ids, table_row, kp, vp)
    assert_norm_close(lg2.cpu().numpy(), ref, 2e-3, what="two-part prefill")
    assert_norm_close(lg1.cpu().numpy(), lg2.cpu().numpy(), 2e-3, what="one vs two prefills")
    eng.close()


def test_prefill_then_decode_matches_hf_greedy():
    """The golden tiny Llama from the reference's weights file: prefill the prompt, compare the
    last position's logits with HF's, then decode HF's greedy continuation."""
    ref = np.load(f"{GOLD}/tiny_llama_ref.npz")
    prompt, greedy = ref["prompt"].tolist(), ref["greedy"].tolist()
    wf = W.read_weights(f"{GOLD}/tiny_llama_weights.bin")
    shape = W.shape_from_config(wf.config)
    eng = DecodeEngine(shape, max_batch=32, max_ctx=64, n_blocks=4)
    eng.alloc_kv()
    eng.load_weights_file(f"{GOLD}/tiny_llama_weights.bin")
    table = torch.arange(4, dtype=torch.int32, device=DEV)
    logits = torch.empty(eng.lm_rows, dtype=torch.float32, device=DEV)
    ids_d = torch.tensor(prompt, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    with torch.cuda.stream(eng.stream):  # every op below is ordered on the engine's stream
        nxt = eng.prefill(ids_d, table, 0, logits=logits)
        eng.stream.synchronize()
        assert_norm_close(logits.cpu().numpy(), ref["last_logits"], 1e-2, what="prefill vs HF")
        toks = [int(nxt.item())]
        tok = nxt.clone()
        pos = torch.tensor([len(prompt)], dtype=torch.int32, device=DEV)
        out = torch.empty(1, dtype=torch.int32, device=DEV)
        for _ in range(len(greedy) - 1):
            eng.step(tok, pos, table.view(1, -1), out, use_graph=False)
            eng.stream.synchronize()
            toks.append(int(out.item()))
            tok.copy_(out)
            pos += 1
    assert toks == greedy
    eng.close()
