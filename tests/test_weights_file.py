"""The reference's flat weights file (reader / writer / config), pinned to a file written by the
reference's own converter (tests/golden/make_weights_file.py) and to transformers' Llama-3 RoPE
frequencies."""

from pathlib import Path

import numpy as np
import pytest

from gemmagemini4hackathon2026_10_2425_b200 import weights as W

GOLD = Path(__file__).resolve().parent / "golden"
FILE = GOLD / "tiny_llama_weights.bin"


def test_reads_the_reference_converter_output():
    wf = W.read_weights(FILE)
    s = W.shape_from_config(wf.config)
    assert (s.dim, s.n_layers, s.n_heads, s.n_kv_heads, s.head_dim, s.ffn_dim, s.vocab) == (128, 2, 4, 2, 64, 128, 256)
    names = {"embed", "final_norm"} | {f"l{i}.{n}" for i in range(2) for n in ("attn_norm", "wqkv", "wo", "ffn_norm", "wgate", "wup", "wdown")}
    assert set(wf.tensors) == names  # tied embeddings: no lm_head
    assert wf.tensors["l0.wqkv"].shape == (s.qkv_dim, s.dim) and wf.tensors["l0.wqkv"].dtype == np.float16
    assert wf.tensors["l1.wo"].shape == (s.dim, s.n_heads * s.head_dim)
    assert wf.tensors["l0.wgate"].shape == (s.ffn_dim, s.dim) and wf.tensors["l0.wdown"].shape == (s.dim, s.ffn_dim)
    assert wf.tensors["l0.attn_norm"].dtype == np.float32 and wf.tensors["final_norm"].shape == (s.dim,)
    assert FILE.stat().st_size % W.PAGE == 0
    assert "lm_head" in W.tensors_for_engine(wf)


def test_write_read_round_trip(tmp_path):
    wf = W.read_weights(FILE)
    out = tmp_path / "copy.bin"
    size = W.write_weights(out, wf.config, {k: np.asarray(v) for k, v in wf.tensors.items()})
    assert size % W.PAGE == 0
    wf2 = W.read_weights(out)
    assert wf2.config == wf.config
    for k, v in wf.tensors.items():
        np.testing.assert_array_equal(wf2.tensors[k], v)
    # same layout rule as the reference converter: the bytes are identical
    assert out.read_bytes() == FILE.read_bytes()


def test_llama3_inv_freq_matches_transformers():
    wf = W.read_weights(FILE)
    ref = np.load(GOLD / "tiny_llama_ref.npz")["inv_freq"]  # HF's own rotary_emb.inv_freq
    np.testing.assert_allclose(W.inv_freq_from_config(wf.config), ref, rtol=2.5e-7, atol=0)
    plain = {k: v for k, v in wf.config.items() if k != "rope_parameters"}
    plain["rope_theta"] = 500000.0  # the top-level style of the Hub's config.json
    np.testing.assert_allclose(
        W.inv_freq_from_config(plain), 1.0 / 500000.0 ** (np.arange(0, 64, 2) / 64), rtol=1e-7
    )


def test_rejects_truncated_file(tmp_path):
    bad = tmp_path / "bad.bin"
    bad.write_bytes(FILE.read_bytes()[: 70000])
    with pytest.raises(ValueError):
        W.read_weights(bad)
