#!/usr/bin/env python3
"""Convert step of the kernel folder.  The weights file format is the reference's own (flat fp16
file with a JSON header, fused [q|k|v], fp32 norms), so its converter's output loads unchanged;
this script re-writes or validates such a file with gemmagemini4hackathon2026_10_2425_b200.weights:

    convert_weights.py --check PATH          print the config and tensor table
    convert_weights.py --copy SRC --out DST  rewrite SRC in canonical layout
    convert_weights.py --quantize q8|q4 SRC --out DST
                                             projections as 32-block int8 / 4-bit + fp16 scales
"""
import argparse

import numpy as np
from _repo import add_package_to_path

add_package_to_path()

from gemmagemini4hackathon2026_10_2425_b200 import weights as W  # noqa: E402

ap = argparse.ArgumentParser()
ap.add_argument("--check")
ap.add_argument("--copy")
ap.add_argument("--out")
ap.add_argument("--quantize", nargs=2, metavar=("FORMAT", "SRC"))
a = ap.parse_args()
if a.check:
    wf = W.read_weights(a.check)
    print(W.shape_from_config(wf.config))
    for k, v in wf.tensors.items():
        q = (wf.quant or {}).get(k, "")
        print(f"{k:20s} {str(v.dtype):8s} {tuple(v.shape)} {q}")
elif a.copy and a.out:
    wf = W.read_weights(a.copy)
    sz = W.write_weights(a.out, wf.config, {k: np.asarray(v) for k, v in wf.tensors.items()}, wf.quant)
    print(sz, "bytes")
elif a.quantize and a.out:
    fmt = {"q8": "q8_32", "q4": "q4_32"}.get(a.quantize[0])
    if fmt is None:
        ap.error("--quantize takes q8 or q4")
    print(W.quantize_file(a.quantize[1], a.out, fmt), "bytes")
else:
    ap.error("--check PATH, --copy SRC --out DST or --quantize q8|q4 SRC --out DST")
