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


# ---- quantized projections (32-block q8 / q4, the formats of include/b200dec.h) --------------


@pytest.mark.parametrize("fmt", ["q8_32", "q4_32"])
def test_quantize_matches_the_format(fmt):
    """quantize() produces the header's layout: the oracle's independent dequantizer reads it back
    bit-exactly, every element is within half a step of the input, zero blocks stay zero."""
    from oracle import ops as O

    r = np.random.default_rng(3)
    w = (r.standard_normal((48, 256)) * 0.02).astype(np.float16)
    w[5, 64:96] = 0  # an all-zero block
    q, sc = W.quantize(w, fmt)
    assert sc.dtype == np.float16 and sc.shape == (48, 8)
    d = W.dequantize(q, sc, fmt)
    ref = O.dequant_q8_32(q, sc) if fmt == "q8_32" else O.dequant_q4_32(q, sc)
    np.testing.assert_array_equal(d.view(np.uint32), ref.view(np.uint32))
    step = np.repeat(sc.astype(np.float32), 32, axis=1)
    assert np.all(np.abs(d - w.astype(np.float32)) <= 0.5 * step * (1 + 2e-3) + 1e-12)
    assert not d[5, 64:96].any()
    if fmt == "q8_32":
        assert q.dtype == np.int8 and q.shape == (48, 256) and np.abs(q).max() <= 127
    else:
        assert q.dtype == np.uint8 and q.shape == (48, 128)
        np.testing.assert_array_equal(q, O.pack_q4(O.unpack_q4(q)))  # element 2j in the low nibble


@pytest.mark.parametrize("fmt", ["q8_32", "q4_32"])
def test_quantized_file_round_trip(tmp_path, fmt):
    out = tmp_path / f"{fmt}.bin"
    size = W.quantize_file(FILE, out, fmt)
    assert size % W.PAGE == 0 and size < FILE.stat().st_size
    src, wf = W.read_weights(FILE), W.read_weights(out)
    assert wf.config == src.config
    mats = {f"l{i}.{n}" for i in range(2) for n in W.QUANT_MATRICES}
    assert set(wf.quant) == mats and set(wf.quant.values()) == {fmt}
    for name in mats:
        q, sc = W.quantize(np.asarray(src.tensors[name]), fmt)
        np.testing.assert_array_equal(wf.tensors[name], q)
        np.testing.assert_array_equal(wf.tensors[name + ".scales"], sc)
    for name in ("embed", "final_norm", "l0.attn_norm"):  # untouched
        np.testing.assert_array_equal(wf.tensors[name], src.tensors[name])
    # the engine's view: fp16(scale * q) under the plain names, no .scales entries
    t = W.tensors_for_engine(wf)
    assert not any(k.endswith(".scales") for k in t)
    assert t["l0.wqkv"].dtype == np.float16 and t["l0.wqkv"].shape == src.tensors["l0.wqkv"].shape
    np.testing.assert_array_equal(
        t["l1.wdown"], W.dequantize(wf.tensors["l1.wdown"], wf.tensors["l1.wdown.scales"], fmt).astype(np.float16)
    )
    # a copy keeps the quantization marks
    W.write_weights(tmp_path / "copy.bin", wf.config, {k: np.asarray(v) for k, v in wf.tensors.items()}, wf.quant)
    assert W.read_weights(tmp_path / "copy.bin").quant == wf.quant


def test_quantized_file_errors(tmp_path):
    wf = W.read_weights(FILE)
    t = {k: np.asarray(v) for k, v in wf.tensors.items()}
    with pytest.raises(ValueError):
        W.quantize(np.zeros((4, 48), np.float16), "q8_32")  # K not a multiple of 32
    with pytest.raises(ValueError):
        W.quantize(np.zeros((4, 64), np.float16), "q5_32")
    W.write_weights(tmp_path / "bad.bin", wf.config, t, {"l0.wo": "q8_32"})  # no l0.wo.scales
    with pytest.raises(ValueError):
        W.read_weights(tmp_path / "bad.bin")


@pytest.mark.parametrize("fmt", ["q8_32", "q4_32"])
def test_quantize_torch_matches_numpy(fmt):
    """The device-side quantizer (synthetic weights) follows the same absmax rule bit for bit."""
    import torch

    r = np.random.default_rng(5)
    w = (r.standard_normal((64, 256)) * 0.02).astype(np.float16)
    w[3, :32] = 0  # an all-zero block: scale 0, q 0
    q, sc = W.quantize(w, fmt)
    qt, st = W.quantize_torch(torch.from_numpy(w), fmt)
    np.testing.assert_array_equal(q, qt.numpy())
    np.testing.assert_array_equal(sc.view(np.uint16), st.numpy().view(np.uint16))
