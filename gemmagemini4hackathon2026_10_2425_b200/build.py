"""Build libb200dec.so (the C-ABI CUDA library) in-tree for sm_100a with nvcc.

    python -m gemmagemini4hackathon2026_10_2425_b200.build [-v] [--force]

Objects go to gemmagemini4hackathon2026_10_2425_b200/_build/, the library next to this file.
Rebuilds only what changed (source or shared header newer than its object).  The CUDA runtime
is linked statically; NCCL is linked against the copy that ships with PyTorch, so the library
and torch.distributed share one libnccl.so.2 in a process.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libb200dec.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["capi.cu", "gemv.cu", "gemv_mma.cu", "ops.cu", "attention.cu", "decoder.cu", "noalloc.cu", "tc_gemm.cu", "tp_peer.cu"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set $NVCC)")


def nccl_dirs() -> tuple[Path, Path]:
    """(include dir, lib dir) of the NCCL that torch loads."""
    import importlib.util

    spec = importlib.util.find_spec("nvidia")
    if spec and spec.submodule_search_locations:
        for loc in spec.submodule_search_locations:
            base = Path(loc) / "nccl"
            if (base / "include" / "nccl.h").exists() and (base / "lib" / "libnccl.so.2").exists():
                return base / "include", base / "lib"
    if Path("/usr/include/nccl.h").exists():
        return Path("/usr/include"), Path("/usr/lib/x86_64-linux-gnu")
    raise RuntimeError("nccl.h not found")


def _needs(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def build(verbose: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    inc, libdir = nccl_dirs()
    headers = list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    flags = [
        *ARCH,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        "-I",
        str(ROOT / "include"),
        "-I",
        str(inc),
        "--expt-relaxed-constexpr",
    ]
    if verbose:
        flags += ["-Xptxas", "-v"]
    jobs = []
    for name in SOURCES:
        src, obj = CSRC / name, BUILD / (Path(name).stem + ".o")
        if force or _needs(obj, src, headers):
            jobs.append([nvcc(), *flags, "-c", str(src), "-o", str(obj)])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for cmd, r in ex.map(run, jobs):
            if verbose or r.returncode:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode:
                raise RuntimeError(f"nvcc failed: {' '.join(cmd[-3:])}")
    objs = [str(BUILD / (Path(n).stem + ".o")) for n in SOURCES]
    if force or jobs or not LIB.exists():
        link = [
            nvcc(),
            *ARCH,
            "-shared",
            "-cudart",
            "static",
            "-o",
            str(LIB),
            *objs,
            "-L",
            str(libdir),
            "-l:libnccl.so.2",
            "-Xlinker",
            f"-rpath,{libdir}",
        ]
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true", help="show nvcc output and -Xptxas -v")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))


if __name__ == "__main__":
    main()
