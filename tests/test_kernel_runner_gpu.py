"""The kernel folder driven by the reference's own, unchanged KernelRunner.

KernelRunner (ios_kernels/surfaces/runners/kernel_runner.py:20-96) reads kernel.json, starts the
manifest's binary with --weights/--serve/--max-ctx, waits for the ready line, and streams tokens
for chat messages, tokenizing with the HF tokenizer of the manifest's hf_repo.  The tokenizer
needs a downloaded HF snapshot, so this test swaps the module's ChatTokenizer for a stub that
turns the messages into the golden prompt's ids and each token id into its decimal text; the
runner's own code is untouched.  The weights file is the one the reference's converter wrote
(tests/golden/make_weights_file.py), and the streamed tokens must be HF's greedy continuation.

Needs a GPU and REFERENCE_ROOT pointing at a checkout of the reference project (skipped
otherwise).
"""

import os
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
GOLD = ROOT / "tests" / "golden"
KDIR = ROOT / "gemmagemini4hackathon2026_10_2425_b200" / "kernels" / "unsloth__Llama-3.2-1B-Instruct" / "kernel_b200_cuda_20261202-1200"


class _StubDecoder:
    def __init__(self):
        self.ids = []

    def add(self, tok: int) -> str:
        self.ids.append(int(tok))
        return f"{int(tok)} "

    def flush(self) -> str:
        return ""


def _stub_tokenizer(prompt):
    class StubChatTokenizer:
        def __init__(self, repo: str):
            self.repo = repo
            self.stop_ids = []

        def encode(self, messages):
            return list(prompt)

        def decoder(self):
            return _StubDecoder()

    return StubChatTokenizer


@pytest.mark.timeout(600)
def test_reference_kernel_runner_streams_hf_greedy(monkeypatch):
    root = os.environ.get("REFERENCE_ROOT")
    surfaces = Path(root or "") / "ios_kernels" / "surfaces" / "runners" / "kernel_runner.py"
    if not root or not surfaces.is_file():
        pytest.skip("REFERENCE_ROOT does not point at a checkout of the reference project")
    monkeypatch.syspath_prepend(str(Path(root) / "ios_kernels"))
    from surfaces.runners import kernel_runner as kr  # the reference's module, unchanged

    ref = np.load(GOLD / "tiny_llama_ref.npz")
    prompt, greedy = ref["prompt"].tolist(), ref["greedy"].tolist()
    monkeypatch.setattr(kr, "ChatTokenizer", _stub_tokenizer(prompt))
    monkeypatch.setenv("PATH", str(Path(sys.executable).parent) + os.pathsep + os.environ.get("PATH", ""))
    runner = kr.KernelRunner(kernel=str(KDIR), weights=str(GOLD / "tiny_llama_weights.bin"), max_ctx=64)
    try:
        chunks = list(runner.stream([{"role": "user", "content": "hi"}], max_tokens=len(greedy)))
    finally:
        runner.close()
    text = "".join(c.text for c in chunks)
    assert [int(t) for t in text.split()] == greedy
    last = chunks[-1]
    assert last.finish_reason == "length"
    assert (last.prompt_tokens, last.completion_tokens) == (len(prompt), len(greedy))
