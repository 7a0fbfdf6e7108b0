"""The kernel-folder binary end to end on the GPU: the kernel folder's `llm` loads the weights file
written by the reference's converter and, over the --serve protocol, returns HF transformers'
greedy continuation of the golden prompt (tests/golden/make_weights_file.py)."""

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from tests._tol import assert_norm_close

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
KERNEL_DIR = ROOT / "gemmagemini4hackathon2026_10_2425_b200" / "kernels" / "unsloth__Llama-3.2-1B-Instruct" / "kernel_b200_cuda_20261202-1200"
LLM = KERNEL_DIR / "llm"
GOLD = ROOT / "tests" / "golden"


@pytest.mark.timeout(300)
def test_serve_protocol_greedy_matches_hf():
    ref = np.load(GOLD / "tiny_llama_ref.npz")
    prompt, greedy = ref["prompt"].tolist(), ref["greedy"].tolist()
    p = subprocess.Popen(
        [sys.executable, str(LLM), "--weights", str(GOLD / "tiny_llama_weights.bin"), "--serve", "--max-ctx", "64"],
        stdin=subprocess.PIPE,
        stdout=subprocess.PIPE,
        text=True,
        bufsize=1,
    )

    def read():
        line = p.stdout.readline()
        assert line, f"llm exited ({p.poll()})"
        return json.loads(line)

    def send(obj):
        p.stdin.write((obj if isinstance(obj, str) else json.dumps(obj)) + "\n")
        p.stdin.flush()

    try:
        ready = read()
        assert ready["ready"] and ready["max_ctx"] == 64 and ready["vocab"] == 256
        send({"ids": prompt, "max_tokens": len(greedy), "stop_ids": []})
        toks = []
        while True:
            m = read()
            if "token" in m:
                toks.append(m["token"])
            else:
                break
        assert toks == greedy
        assert m["done"] and m["finish_reason"] == "length"
        assert m["prompt_tokens"] == len(prompt) and m["completion_tokens"] == len(greedy)
        send("this is not json")
        assert "error" in read()
        send({"ids": prompt, "max_tokens": 5, "stop_ids": [greedy[0]]})  # stops at once
        m = read()
        assert m["done"] and m["finish_reason"] == "stop" and m["completion_tokens"] == 0
        p.stdin.close()
        assert p.wait(timeout=60) == 0
    finally:
        if p.poll() is None:
            p.kill()


@pytest.mark.timeout(300)
def test_prompt_ids_mode_dumps_logits(tmp_path):
    ref = np.load(GOLD / "tiny_llama_ref.npz")
    prompt, greedy = ref["prompt"].tolist(), ref["greedy"].tolist()
    dump = tmp_path / "logits.bin"
    r = subprocess.run(
        [sys.executable, str(LLM), "--weights", str(GOLD / "tiny_llama_weights.bin"), "--max-ctx", "64",
         "--prompt-ids", ",".join(map(str, prompt)), "--gen", "3", "--dump-logits", str(dump)],
        capture_output=True, text=True, timeout=240,
    )
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["tokens"] == greedy[:3]
    assert_norm_close(np.fromfile(dump, "<f4"), ref["last_logits"], 2e-3, what="dumped logits")
