#!/usr/bin/env python3
"""Build step of the kernel folder: compiles libb200dec.so (sm_100a) in-tree."""
from _repo import add_package_to_path

add_package_to_path()
from gemmagemini4hackathon2026_10_2425_b200.build import build  # noqa: E402

print(build())
