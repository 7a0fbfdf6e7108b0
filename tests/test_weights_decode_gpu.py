"""A weights file written by the reference's converter, loaded into the CUDA decode step: the
prompt runs through decode steps (one token per step fills the paged cache) and the last
position's logits and the greedy continuation match HF transformers on the same model
(tests/golden/make_weights_file.py).  Batch 1 takes the CUDA-core path, batch 9 the tensor-core
path (nine copies of the sequence)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from gemmagemini4hackathon2026_10_2425_b200 import weights as W
from gemmagemini4hackathon2026_10_2425_b200.engine import DecodeEngine, make_block_table
from tests._tol import assert_norm_close

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("batch", [1, 9])
def test_weights_file_decode_matches_hf(batch):
    ref = np.load(GOLD / "tiny_llama_ref.npz")
    prompt, greedy = ref["prompt"].tolist(), ref["greedy"].tolist()
    wf = W.read_weights(GOLD / "tiny_llama_weights.bin")
    shape = W.shape_from_config(wf.config)
    max_ctx = 64
    nblk = batch * (max_ctx // 16) + 2
    dev = torch.device("cuda", 0)
    eng = DecodeEngine(shape, max_batch=batch, max_ctx=max_ctx, n_blocks=nblk, device=dev)
    eng.alloc_kv()
    eng.load_weights_file(GOLD / "tiny_llama_weights.bin")
    table = make_block_table([max_ctx - 1] * batch, max_ctx // 16, nblk, seed=3, headroom=0).to(dev)
    logits = torch.empty(batch, eng.lm_rows, dtype=torch.float32, device=dev)
    nxt = torch.empty(batch, dtype=torch.int32, device=dev)
    seq = list(prompt)
    out = []
    for pos in range(len(prompt) + len(greedy) - 1):
        tok = torch.full((batch,), seq[pos], dtype=torch.int32, device=dev)
        ctx = torch.full((batch,), pos, dtype=torch.int32, device=dev)
        eng.step(tok, ctx, table, nxt, logits, use_graph=False)
        eng.stream.synchronize()
        if pos == len(prompt) - 1:
            for b in range(batch):
                assert_norm_close(logits[b].cpu().numpy(), ref["last_logits"], 2e-3, what=f"b{batch} seq {b}")
        if pos >= len(prompt) - 1:
            t = nxt.cpu().numpy()
            assert (t == t[0]).all()
            out.append(int(t[0]))
            seq.append(int(t[0]))
    assert out == greedy
    eng.close()


@pytest.mark.parametrize("batch", [1, 9])
def test_device_resident_generate_matches_hf(batch):
    """b2d_decoder_generate: after the prompt, the greedy continuation runs as back-to-back
    graph launches with the next token fed back on the device."""
    ref = np.load(GOLD / "tiny_llama_ref.npz")
    prompt, greedy = ref["prompt"].tolist(), ref["greedy"].tolist()
    wf = W.read_weights(GOLD / "tiny_llama_weights.bin")
    shape = W.shape_from_config(wf.config)
    max_ctx = 64
    nblk = batch * (max_ctx // 16) + 2
    dev = torch.device("cuda", 0)
    eng = DecodeEngine(shape, max_batch=batch, max_ctx=max_ctx, n_blocks=nblk, device=dev)
    eng.alloc_kv()
    eng.load_weights_file(GOLD / "tiny_llama_weights.bin")
    table = make_block_table([max_ctx - 1] * batch, max_ctx // 16, nblk, seed=4, headroom=0).to(dev)
    nxt = torch.empty(batch, dtype=torch.int32, device=dev)
    for pos, t in enumerate(prompt[:-1]):
        eng.step(torch.full((batch,), t, dtype=torch.int32, device=dev), torch.full((batch,), pos, dtype=torch.int32, device=dev), table, nxt, use_graph=False)
    tok = torch.full((batch,), prompt[-1], dtype=torch.int32, device=dev)
    ctx = torch.full((batch,), len(prompt) - 1, dtype=torch.int32, device=dev)
    ring = eng.generate(tok, ctx, table, len(greedy))
    eng.stream.synchronize()
    got = ring.cpu().numpy()
    for b in range(batch):
        assert got[:, b].tolist() == greedy
    assert (ctx.cpu().numpy() == len(prompt) - 1 + len(greedy)).all()
    assert (tok.cpu().numpy() == greedy[-1]).all()
    eng.close()
