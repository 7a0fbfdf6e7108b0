"""The package's kernel tree against the reference project's kernel-folder contract.

The reference drives kernels through folders named kernels/<model>/kernel_<name>_<YYYYMMDD-HHMM>/
(ios_kernels/utils/check_kernel_tree.py:16-18), each with a README.md that opens with a title and
a yaml lineage header of exactly the keys kernel, model, origin, parent, change (:38-66) and a
kernel.json with hf_repo, weights, build, binary, convert (:19, :69-84); KernelRunner runs the
manifest's `binary` directly (ios_kernels/surfaces/runners/kernel_runner.py:27-41).

The first tests restate those rules in this file and always run.  With REFERENCE_ROOT set to a
checkout of the reference project, the reference's own checker is also run, unchanged, on this
tree.  The last test links the folder into a reference-style tree and starts its binary through
the link (--help needs no GPU), the way a maintainer installs it.
"""

import importlib.util
import json
import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
KERNELS = ROOT / "gemmagemini4hackathon2026_10_2425_b200" / "kernels"
MODEL = "unsloth__Llama-3.2-1B-Instruct"
NAME_RE = re.compile(r"^kernel_[a-z0-9]+(?:_[a-z0-9]+)*_\d{8}-\d{4}$")


def kernel_dirs():
    return sorted(d for d in (KERNELS / MODEL).iterdir() if d.is_dir() and d.name.startswith("kernel_"))


def test_tree_layout():
    assert (KERNELS / "README.md").is_file()
    assert (KERNELS / MODEL / "README.md").is_file()
    dirs = kernel_dirs()
    assert dirs, "no kernel folder"
    for d in dirs:
        assert NAME_RE.match(d.name), d.name


@pytest.mark.parametrize("kdir", kernel_dirs(), ids=lambda d: d.name)
def test_readme_lineage_header(kdir):
    text = (kdir / "README.md").read_text()
    m = re.match(r"\A# (?P<title>.+)\n\n```yaml\n(?P<body>.*?)\n```\n", text, re.DOTALL)
    assert m, "README must open with '# <folder>', a blank line and a yaml block"
    assert m["title"] == kdir.name
    pairs = [line.split(":", 1) for line in m["body"].splitlines()]
    assert [k.strip() for k, _ in pairs] == ["kernel", "model", "origin", "parent", "change"]
    h = {k.strip(): v.strip() for k, v in pairs}
    assert h["kernel"] == kdir.name and h["model"] == MODEL
    assert (h["origin"], h["parent"]) == ("root", "none")
    assert h["change"]


@pytest.mark.parametrize("kdir", kernel_dirs(), ids=lambda d: d.name)
def test_manifest(kdir):
    man = json.loads((kdir / "kernel.json").read_text())
    for key in ("hf_repo", "weights", "build", "binary", "convert"):
        assert key in man, key
    assert man["hf_repo"].replace("/", "__") == MODEL
    for key in ("build", "convert", "binary"):
        assert (kdir / man[key]).is_file(), key
    binary = kdir / man["binary"]
    assert os.access(binary, os.X_OK) and binary.read_text().startswith("#!")


def _reference_checker():
    root = os.environ.get("REFERENCE_ROOT")
    if not root:
        return None
    path = Path(root) / "ios_kernels" / "utils" / "check_kernel_tree.py"
    if not path.is_file():
        return None
    spec = importlib.util.spec_from_file_location("reference_check_kernel_tree", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_checker_accepts_tree():
    mod = _reference_checker()
    if mod is None:
        pytest.skip("REFERENCE_ROOT does not point at a checkout of the reference project")
    files = [str(p.relative_to(KERNELS)) for p in KERNELS.rglob("*") if p.is_file() and "__pycache__" not in p.parts]
    assert mod.check(KERNELS, files) == []


def test_binary_runs_through_a_link(tmp_path):
    """Linked into another project's kernels/<model>/ directory, the scripts find this package."""
    kdir = kernel_dirs()[-1]
    model_dir = tmp_path / "ios_kernels" / "kernels" / MODEL
    model_dir.mkdir(parents=True)
    (model_dir / kdir.name).symlink_to(kdir, target_is_directory=True)
    env = {k: v for k, v in os.environ.items() if k != "B2D_REPO"}
    r = subprocess.run([str(model_dir / kdir.name / "llm"), "--help"], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "--serve" in r.stdout and "--bench-tg" in r.stdout
    r = subprocess.run([sys.executable, str(model_dir / kdir.name / "convert_weights.py"), "--check", str(ROOT / "tests" / "golden" / "tiny_llama_weights.bin")], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "wqkv" in r.stdout
