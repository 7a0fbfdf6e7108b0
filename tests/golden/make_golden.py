"""Generate the golden vectors that pin the CPU oracle (run once; outputs are committed).

    python tests/golden/make_golden.py        # writes tests/golden/hf_llama_ops.npz

The reference's kernels are Metal and cannot run here, and the reference holds no op-level
golden vectors.  Its own correctness harness compares against HF transformers' Llama in fp32
on CPU (ios_kernels/benchmarking/reference.py:64-70), so that is what pins the oracle: each
op (RMSNorm, RoPE, SwiGLU MLP, GQA attention) and one whole decode position of a tiny random
Llama are evaluated here with transformers' own modules and saved with their inputs.
transformers is the third-party dependency the reference pins at 5.20.2 (ios_kernels/uv.lock);
this container has 5.5.0, whose Llama modules compute the same math.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch
from transformers import LlamaConfig, LlamaForCausalLM
from transformers.models.llama import modeling_llama as ml

OUT = Path(__file__).resolve().parent / "hf_llama_ops.npz"

# Tiny Llama with the GQA ratio of the BASELINE configs (4 query heads per KV head).
CFG = dict(
    hidden_size=128,
    intermediate_size=256,
    num_hidden_layers=2,
    num_attention_heads=8,
    num_key_value_heads=2,
    head_dim=64,
    vocab_size=384,
    rms_norm_eps=1e-5,
    rope_theta=500000.0,
    tie_word_embeddings=True,
    attn_implementation="eager",
)
PROMPT_LENS = (5, 19, 33)  # ragged: three sequences, context crosses a 16-token page boundary


def main() -> None:
    torch.manual_seed(1234)
    g = {}
    cfg = LlamaConfig(**CFG)
    d, hq, hk, hd = cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim

    # RMSNorm
    norm = ml.LlamaRMSNorm(d, eps=cfg.rms_norm_eps)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(d))
    x = torch.randn(4, d)
    g["rms_x"], g["rms_w"], g["rms_eps"] = x.numpy(), norm.weight.detach().numpy(), np.float64(cfg.rms_norm_eps)
    g["rms_y"] = norm(x).detach().numpy()

    # RoPE (rotate_half convention) at a spread of positions
    rot = ml.LlamaRotaryEmbedding(cfg)
    pos = torch.tensor([[0, 1, 7, 16, 63, 500, 4095]])
    q = torch.randn(1, hq, pos.shape[1], hd)
    k = torch.randn(1, hk, pos.shape[1], hd)
    cos, sin = rot(q, pos)
    qr, kr = ml.apply_rotary_pos_emb(q, k, cos, sin)
    g["rope_inv_freq"] = rot.inv_freq.numpy()
    g["rope_theta"] = np.float64(cfg.rope_parameters["rope_theta"])
    g["rope_pos"], g["rope_q"], g["rope_k"] = pos[0].numpy(), q[0].numpy(), k[0].numpy()
    g["rope_qr"], g["rope_kr"] = qr[0].numpy(), kr[0].numpy()

    # SwiGLU MLP
    mlp = ml.LlamaMLP(cfg)
    for p in mlp.parameters():
        torch.nn.init.normal_(p, std=0.05)
    xm = torch.randn(3, d)
    g["mlp_x"] = xm.numpy()
    g["mlp_wg"] = mlp.gate_proj.weight.detach().numpy()
    g["mlp_wu"] = mlp.up_proj.weight.detach().numpy()
    g["mlp_wd"] = mlp.down_proj.weight.detach().numpy()
    g["mlp_y"] = mlp(xm).detach().numpy()

    # GQA single-query attention (eager path, no mask: the query is the last position)
    n = 37
    qa = torch.randn(1, hq, 1, hd)
    ka = torch.randn(1, hk, n, hd)
    va = torch.randn(1, hk, n, hd)
    mod = torch.nn.Module()
    mod.num_key_value_groups = hq // hk
    mod.training = False
    out, _ = ml.eager_attention_forward(mod, qa, ka, va, None, scaling=hd**-0.5)
    g["attn_q"], g["attn_k"], g["attn_v"] = qa[0, :, 0].numpy(), ka[0].numpy(), va[0].numpy()
    g["attn_out"] = out[0, 0].numpy()  # [Hq, HD]

    # Whole decode position of a tiny random Llama, weights rounded to fp16 values
    model = LlamaForCausalLM(cfg).eval()
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() == 2:
                p.copy_(p.half().float())
            else:  # norm weights: perturb around 1 so the test sees them
                p.copy_(1 + 0.1 * torch.randn_like(p))
    sd = model.state_dict()
    g["llm_embed"] = sd["model.embed_tokens.weight"].half().numpy()
    g["llm_final_norm"] = sd["model.norm.weight"].numpy()
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        g[f"llm_l{i}_attn_norm"] = sd[p + "input_layernorm.weight"].numpy()
        g[f"llm_l{i}_wqkv"] = torch.cat([sd[p + f"self_attn.{c}_proj.weight"] for c in "qkv"]).half().numpy()
        g[f"llm_l{i}_wo"] = sd[p + "self_attn.o_proj.weight"].half().numpy()
        g[f"llm_l{i}_ffn_norm"] = sd[p + "post_attention_layernorm.weight"].numpy()
        g[f"llm_l{i}_wgate"] = sd[p + "mlp.gate_proj.weight"].half().numpy()
        g[f"llm_l{i}_wup"] = sd[p + "mlp.up_proj.weight"].half().numpy()
        g[f"llm_l{i}_wdown"] = sd[p + "mlp.down_proj.weight"].half().numpy()
    gen = torch.Generator().manual_seed(99)
    for s, plen in enumerate(PROMPT_LENS):
        ids = torch.randint(0, cfg.vocab_size, (1, plen), generator=gen)
        with torch.no_grad():
            pre = model(ids[:, :-1], use_cache=True)
            full = model(ids)
        g[f"llm_s{s}_ids"] = ids[0].numpy().astype(np.int32)
        g[f"llm_s{s}_logits"] = full.logits[0, -1].numpy()
        for i in range(cfg.num_hidden_layers):
            layer = pre.past_key_values.layers[i]
            g[f"llm_s{s}_l{i}_k"] = layer.keys[0].numpy()  # [Hkv, plen-1, HD], rotated
            g[f"llm_s{s}_l{i}_v"] = layer.values[0].numpy()
    g["llm_config"] = np.array(
        [d, cfg.num_hidden_layers, hq, hk, hd, cfg.intermediate_size, cfg.vocab_size], dtype=np.int64
    )
    g["llm_eps_theta"] = np.array([cfg.rms_norm_eps, cfg.rope_parameters["rope_theta"]], dtype=np.float64)
    g["llm_prompt_lens"] = np.array(PROMPT_LENS, dtype=np.int64)
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1024:.0f} KiB, {len(g)} arrays)")


if __name__ == "__main__":
    main()
