#!/usr/bin/env python3
"""Convert step of the kernel folder.  The weights file format is the reference's own (flat fp16
file with a JSON header, fused [q|k|v], fp32 norms), so its converter's output loads unchanged;
this script re-writes or validates such a file with gemmagemini4hackathon2026_10_2425_b200.weights:

    convert_weights.py --check PATH          print the config and tensor table
    convert_weights.py --copy SRC --out DST  rewrite SRC in canonical layout
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
import numpy as np  # noqa: E402

from gemmagemini4hackathon2026_10_2425_b200 import weights as W  # noqa: E402

ap = argparse.ArgumentParser()
ap.add_argument("--check")
ap.add_argument("--copy")
ap.add_argument("--out")
a = ap.parse_args()
if a.check:
    wf = W.read_weights(a.check)
    print(W.shape_from_config(wf.config))
    for k, v in wf.tensors.items():
        print(f"{k:20s} {str(v.dtype):8s} {tuple(v.shape)}")
elif a.copy and a.out:
    wf = W.read_weights(a.copy)
    print(W.write_weights(a.out, wf.config, {k: np.asarray(v) for k, v in wf.tensors.items()}), "bytes")
else:
    ap.error("--check PATH or --copy SRC --out DST")
