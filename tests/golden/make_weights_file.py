"""Generate the weights-file fixtures with the reference's own converter (run once; committed).

    python tests/golden/make_weights_file.py --reference PATH_TO_REFERENCE_CHECKOUT

(or set REFERENCE_ROOT); PATH_TO_REFERENCE_CHECKOUT is the root of the reference project, the
directory that holds ios_kernels/.

1. A tiny random Llama (HF transformers, Llama-3 RoPE scaling on) is saved as a HF snapshot
   (config.json + model.safetensors) under a temporary HOME.
2. The reference's converter, ios_kernels/kernels/unsloth__Llama-3.2-1B-Instruct/
   kernel_metal_f16_20261024-1620/convert_weights.py, run unchanged from the reference tree,
   turns it into the reference's flat weights file -> tests/golden/tiny_llama_weights.bin.
3. HF evaluates the fp16-rounded model on a fixed prompt: the last position's logits and a
   greedy continuation -> tests/golden/tiny_llama_ref.npz.

The tests then load the converter's file with this repository's reader, run the prompt through
the CUDA decode step and compare with HF.  The reference tree is only needed here, not by the
tests.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch
from transformers import LlamaConfig, LlamaForCausalLM

HERE = Path(__file__).resolve().parent
# the reference's converter, relative to the reference project's root
REF_CONVERTER = Path("ios_kernels/kernels/unsloth__Llama-3.2-1B-Instruct/kernel_metal_f16_20261024-1620/convert_weights.py")
REPO = "tiny/llama-b200-fixture"
CFG = dict(
    hidden_size=128,
    intermediate_size=128,
    num_hidden_layers=2,
    num_attention_heads=4,
    num_key_value_heads=2,
    head_dim=64,
    vocab_size=256,
    rms_norm_eps=1e-5,
    rope_theta=500000.0,
    rope_scaling={
        "rope_type": "llama3",
        "factor": 32.0,
        "low_freq_factor": 1.0,
        "high_freq_factor": 4.0,
        "original_max_position_embeddings": 64,
    },
    max_position_embeddings=4096,
    tie_word_embeddings=True,
    attn_implementation="eager",
)
PROMPT = [1, 17, 200, 33, 5, 99, 128, 64, 7, 250, 3, 42, 11, 180, 2, 77, 19, 8, 140]  # 19 tokens: > one page
GEN = 6


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("REFERENCE_ROOT"), help="root of the reference project checkout")
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference PATH (or set REFERENCE_ROOT) to the reference project's root")
    converter = Path(args.reference) / REF_CONVERTER
    if not converter.exists():
        raise SystemExit(f"{converter} not found")
    torch.manual_seed(2027)
    model = LlamaForCausalLM(LlamaConfig(**CFG)).eval()
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() == 2:
                p.copy_(p.half().float())  # the file stores fp16: make HF use the same values
            else:
                p.copy_(1 + 0.1 * torch.randn_like(p))
    with tempfile.TemporaryDirectory() as home:
        snap = Path(home) / ".cache/huggingface/hub" / f"models--{REPO.replace('/', '--')}" / "snapshots" / "fixture"
        snap.mkdir(parents=True)
        model.save_pretrained(snap, safe_serialization=True)
        out = Path(home) / "weights.bin"
        env = dict(os.environ, HOME=home)
        subprocess.run([sys.executable, str(converter), "--repo", REPO, "--out", str(out)], check=True, env=env)
        shutil.copy(out, HERE / "tiny_llama_weights.bin")
    ids = torch.tensor([PROMPT])
    with torch.no_grad():
        logits = model(ids).logits[0, -1].numpy()
        gen = model.generate(ids, max_new_tokens=GEN, do_sample=False)[0, len(PROMPT) :].numpy()
    np.savez_compressed(
        HERE / "tiny_llama_ref.npz",
        prompt=np.array(PROMPT, np.int32),
        last_logits=logits.astype(np.float32),
        greedy=gen.astype(np.int32),
        inv_freq=model.model.rotary_emb.inv_freq.numpy().astype(np.float32),
    )
    print("wrote", HERE / "tiny_llama_weights.bin", (HERE / "tiny_llama_weights.bin").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
