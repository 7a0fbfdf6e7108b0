"""Pin the CPU oracle against golden vectors made with HF transformers' Llama modules.

The fixtures come from tests/golden/make_golden.py (transformers' LlamaRMSNorm, rotary
embedding, LlamaMLP, eager GQA attention and a whole tiny LlamaForCausalLM).  HF computes in
fp32, the oracle in float64, so the tolerances here are fp32-level.
"""

import numpy as np

from oracle import ops, step


def rel_err(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30)


def test_rmsnorm_matches_hf(golden):
    y = ops.rmsnorm(golden["rms_x"], golden["rms_w"], float(golden["rms_eps"]))
    assert rel_err(y, golden["rms_y"]) < 1e-6


def test_inv_freq_matches_hf(golden):
    hd = golden["rope_q"].shape[-1]
    ours = ops.inv_freq(hd, float(golden["rope_theta"]))
    # HF builds inv_freq in fp32 arithmetic, the reference in double then casts: <= 1 ulp apart.
    np.testing.assert_allclose(ours, golden["rope_inv_freq"], rtol=2.5e-7, atol=0)


def test_rope_matches_hf(golden):
    pos = golden["rope_pos"]
    invf = golden["rope_inv_freq"]
    qr = ops.rope(golden["rope_q"], pos[None, :], invf)  # q: [Hq, P, HD]
    kr = ops.rope(golden["rope_k"], pos[None, :], invf)
    assert rel_err(qr, golden["rope_qr"]) < 2e-6
    assert rel_err(kr, golden["rope_kr"]) < 2e-6


def test_swiglu_mlp_matches_hf(golden):
    x = golden["mlp_x"]
    h = ops.swiglu(ops.gemv(golden["mlp_wg"], x), ops.gemv(golden["mlp_wu"], x))
    y = ops.gemv(golden["mlp_wd"], h)
    assert rel_err(y, golden["mlp_y"]) < 1e-5


def test_gqa_attention_matches_hf(golden):
    q, k, v = golden["attn_q"], golden["attn_k"], golden["attn_v"]
    out = ops.attention(q, k, v, scale=k.shape[-1] ** -0.5)
    assert rel_err(out, golden["attn_out"]) < 1e-5


def _tiny_cfg(golden):
    d, nl, hq, hk, hd, ffn, vocab = (int(v) for v in golden["llm_config"])
    eps, theta = (float(v) for v in golden["llm_eps_theta"])
    return step.ModelConfig(d, nl, hq, hk, hd, ffn, vocab, eps, theta)


def _tiny_weights(golden, cfg):
    w = {"embed": golden["llm_embed"], "final_norm": golden["llm_final_norm"]}
    for i in range(cfg.n_layers):
        for n in ("attn_norm", "wqkv", "wo", "ffn_norm", "wgate", "wup", "wdown"):
            w[f"l{i}.{n}"] = golden[f"llm_l{i}_{n}"]
    return w


def build_paged_cache(golden, cfg, kv_dtype, seed=0):
    """Scatter HF's per-sequence K/V caches into randomly permuted 16-token pages."""
    lens = [int(p) - 1 for p in golden["llm_prompt_lens"]]
    per_seq = [-(-(n + 1) // ops.PAGE_TOKENS) for n in lens]
    nblk = sum(per_seq) + 3
    rng = np.random.default_rng(seed)
    perm = rng.permutation(nblk)
    table = np.zeros((len(lens), max(per_seq)), np.int32)
    c = 0
    for b, k in enumerate(per_seq):
        table[b, :k] = perm[c : c + k]
        c += k
    shape = (nblk, cfg.n_kv_heads, ops.PAGE_TOKENS, cfg.head_dim)
    kp = [np.full(shape, 7.0, kv_dtype) for _ in range(cfg.n_layers)]
    vp = [np.full(shape, 7.0, kv_dtype) for _ in range(cfg.n_layers)]
    for b, n in enumerate(lens):
        for i in range(cfg.n_layers):
            K, V = golden[f"llm_s{b}_l{i}_k"], golden[f"llm_s{b}_l{i}_v"]
            for pos in range(n):
                blk, slot = ops.page_slot(table, b, pos)
                kp[i][blk, :, slot] = K[:, pos]
                vp[i][blk, :, slot] = V[:, pos]
    return lens, table, kp, vp


def test_decode_step_matches_hf_llama(golden):
    """One ragged batch decode step of the oracle equals HF's last-position logits."""
    cfg = _tiny_cfg(golden)
    w = _tiny_weights(golden, cfg)
    lens, table, kp, vp = build_paged_cache(golden, cfg, np.float64)
    tokens = [int(golden[f"llm_s{b}_ids"][-1]) for b in range(len(lens))]
    logits, nxt = step.decode_step(w, cfg, tokens, lens, table, kp, vp)
    for b in range(len(lens)):
        ref = golden[f"llm_s{b}_logits"]
        assert rel_err(logits[b], ref) < 2e-5, b
        assert nxt[b] == int(np.argmax(ref))


def test_decode_step_tp_equals_single(golden):
    """The simulated tensor-parallel step computes the same logits for tp = 1, 2."""
    cfg = _tiny_cfg(golden)
    w = _tiny_weights(golden, cfg)
    ref = None
    for tp in (1, 2):
        lens, table, kp, vp = build_paged_cache(golden, cfg, np.float16)
        tokens = [int(golden[f"llm_s{b}_ids"][-1]) for b in range(len(lens))]
        logits, nxt = step.decode_step_tp(w, cfg, tp, tokens, lens, table, kp, vp)
        if ref is None:
            ref = (logits, nxt, kp)
            l1, n1 = step.decode_step(w, cfg, tokens, lens, *build_paged_cache(golden, cfg, np.float16)[1:])
            assert rel_err(logits, l1) < 1e-12
        else:
            assert rel_err(logits, ref[0]) < 1e-12
            np.testing.assert_array_equal(nxt, ref[1])
            for a, b in zip(kp, ref[2]):
                np.testing.assert_array_equal(a, b)


def test_decode_step_over_written_cache(golden):
    """append=False (the mode the GPU tests use to evaluate the oracle over the cache a GPU step
    wrote): over pages that already hold the new tokens' K/V it reproduces the appending step
    exactly and writes nothing."""
    cfg = _tiny_cfg(golden)
    w = _tiny_weights(golden, cfg)
    lens, table, kp, vp = build_paged_cache(golden, cfg, np.float16)
    tokens = [int(golden[f"llm_s{b}_ids"][-1]) for b in range(len(lens))]
    l1, n1 = step.decode_step(w, cfg, tokens, lens, table, kp, vp)  # appends into kp / vp
    kp2, vp2 = [k.copy() for k in kp], [v.copy() for v in vp]
    l2, n2 = step.decode_step(w, cfg, tokens, lens, table, kp2, vp2, append=False)
    np.testing.assert_array_equal(l1, l2)
    np.testing.assert_array_equal(n1, n2)
    for a, b in zip(kp + vp, kp2 + vp2):
        np.testing.assert_array_equal(a, b)


def test_argmax_ties_lowest_index():
    x = np.array([[1.0, 3.0, 3.0, 2.0], [5.0, 5.0, 5.0, 5.0]])
    np.testing.assert_array_equal(ops.argmax(x), [1, 0])
