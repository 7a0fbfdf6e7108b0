#!/usr/bin/env python3
"""Build step of the kernel folder: compiles libb200dec.so (sm_100a) in-tree."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from gemmagemini4hackathon2026_10_2425_b200.build import build  # noqa: E402

print(build())
