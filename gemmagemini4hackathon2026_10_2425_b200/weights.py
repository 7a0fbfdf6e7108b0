"""The reference's flat weights file: reader, writer and model configuration.

Format (written by the reference's converter, LK/convert_weights.py:1-94; read by its engine,
LK/main.swift:113-148):

    [0:8)     little-endian u64 = header length H
    [8:8+H)   UTF-8 JSON header {"config": <HF config.json>, "tensors": {name: {"offset", "shape",
              "dtype"}}}
    ...       tensor data; every tensor starts on a 256-byte boundary (absolute offsets); the file
              is padded to a 16 KiB multiple

Tensor names: embed, l{i}.attn_norm, l{i}.wqkv (rows [q | k | v]), l{i}.wo, l{i}.ffn_norm,
l{i}.wgate, l{i}.wup, l{i}.wdown, final_norm, and lm_head when the embeddings are not tied; fp16
matrices, fp32 norms.  Files of this format load directly into DecodeEngine
(`DecodeEngine.load_weights_file`), sharded per tensor-parallel rank on the way.

Extension (no reference counterpart; the 32-block formats of include/b200dec.h): a projection
matrix may be stored quantized as its integer tensor under its own name -- int8 [M, K] ("q8_32")
or uint8 [M, K/2] with element 2j in the low nibble and value (n ^ 8) - 8 ("q4_32") -- plus
`<name>.scales` fp16 [M, K/32], and a "quant" key in the matrix's header entry.  The arrays are
exactly the operands b2d_gemv / b2d_gemm_tc_q take; readers that do not know the key (the
reference's JSON decoding ignores unknown keys) see plain integer tensors.
"""

from __future__ import annotations

import json
import math
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .tp import ModelShape

ALIGN = 256
PAGE = 16384
QUANT_FORMATS = ("q8_32", "q4_32")
QUANT_MATRICES = ("wqkv", "wo", "wgate", "wup", "wdown")  # per-layer projections
HEADER_RESERVE = 64 * 1024  # the reference converter's fixed header prefix


@dataclass
class WeightsFile:
    config: dict
    tensors: dict[str, np.ndarray]  # read-only views of the mapped file
    path: Path
    quant: dict[str, str] | None = None  # matrix name -> "q8_32" / "q4_32"


def read_weights(path: str | Path) -> WeightsFile:
    """Map a weights file; tensors are zero-copy views (np.memmap)."""
    path = Path(path)
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    if raw.size < 8:
        raise ValueError(f"{path}: too short for a weights file")
    hlen = int(np.frombuffer(raw[:8].tobytes(), "<u8")[0])
    if 8 + hlen > raw.size:
        raise ValueError(f"{path}: header length {hlen} exceeds the file")
    header = json.loads(raw[8 : 8 + hlen].tobytes().decode("utf-8"))
    tensors, quant = {}, {}
    for name, meta in header["tensors"].items():
        if "quant" in meta:
            if meta["quant"] not in QUANT_FORMATS:
                raise ValueError(f"{path}: tensor {name} has unknown quantization {meta['quant']!r}")
            quant[name] = meta["quant"]
        dt = np.dtype(meta["dtype"])
        shape = tuple(int(d) for d in meta["shape"])
        off = int(meta["offset"])
        n = int(np.prod(shape)) * dt.itemsize
        if off % ALIGN or off + n > raw.size:
            raise ValueError(f"{path}: tensor {name} at {off} (+{n} B) is misaligned or out of range")
        tensors[name] = raw[off : off + n].view(dt).reshape(shape)
    for name in quant:
        if name + ".scales" not in tensors:
            raise ValueError(f"{path}: quantized tensor {name} has no {name}.scales")
    return WeightsFile(header["config"], tensors, path, quant)


def write_weights(
    path: str | Path, config: dict, tensors: dict[str, np.ndarray], quant: dict[str, str] | None = None
) -> int:
    """Write tensors (in the given order) in the reference's layout; returns the file size.
    `quant` marks quantized matrices (their `<name>.scales` must be among the tensors)."""
    quant = quant or {}
    off = HEADER_RESERVE
    meta = {}
    for name, arr in tensors.items():
        off = -(-off // ALIGN) * ALIGN
        meta[name] = {"offset": off, "shape": list(arr.shape), "dtype": str(arr.dtype)}
        if name in quant:
            meta[name]["quant"] = quant[name]
        off += arr.nbytes
    total = -(-off // PAGE) * PAGE
    header = json.dumps({"config": config, "tensors": meta}).encode()
    if 8 + len(header) > HEADER_RESERVE:
        raise ValueError("header does not fit the reserved prefix")
    with open(path, "wb") as f:
        f.write(len(header).to_bytes(8, "little"))
        f.write(header)
        for name, arr in tensors.items():
            f.seek(meta[name]["offset"])
            f.write(np.ascontiguousarray(arr).tobytes())
        f.truncate(total)
    return total


def _rope(cfg: dict) -> tuple[float, dict]:
    """(rope_theta, scaling dict) from either config style: top-level rope_theta / rope_scaling
    (the Hub's Llama-3.2 config.json, as LK/main.swift:89-96 reads it) or the newer
    rope_parameters block that holds both."""
    rp = cfg.get("rope_parameters") or {}
    theta = cfg.get("rope_theta", rp.get("rope_theta"))
    if theta is None:
        raise KeyError("config has neither rope_theta nor rope_parameters.rope_theta")
    scaling = cfg.get("rope_scaling") or (rp if rp.get("rope_type", "default") != "default" else {})
    return float(theta), scaling or {}


def shape_from_config(cfg: dict) -> ModelShape:
    """HF config.json fields -> the decode step's shape (LK/main.swift:78-87)."""
    d = int(cfg["hidden_size"])
    nh = int(cfg["num_attention_heads"])
    return ModelShape(
        dim=d,
        n_layers=int(cfg["num_hidden_layers"]),
        n_heads=nh,
        n_kv_heads=int(cfg["num_key_value_heads"]),
        head_dim=int(cfg.get("head_dim") or d // nh),
        ffn_dim=int(cfg["intermediate_size"]),
        vocab=int(cfg["vocab_size"]),
        eps=float(cfg["rms_norm_eps"]),
        theta=_rope(cfg)[0],
    )


def inv_freq_from_config(cfg: dict) -> np.ndarray:
    """RoPE inverse frequencies in float64, then fp32, with Llama-3 scaling when the config asks
    for it (LK/main.swift:89-108; the published Llama-3 rule: wavelengths shorter than
    orig_ctx / high_freq_factor keep their frequency, longer than orig_ctx / low_freq_factor are
    divided by `factor`, and the band between is interpolated linearly in orig_ctx / wavelength)."""
    shape = shape_from_config(cfg)
    hd, theta = shape.head_dim, shape.theta
    inv = [1.0 / theta ** (2 * i / hd) for i in range(hd // 2)]
    rs = _rope(cfg)[1]
    if rs.get("rope_type", rs.get("type")) == "llama3":
        factor = float(rs["factor"])
        lo, hi = float(rs["low_freq_factor"]), float(rs["high_freq_factor"])
        old = float(rs["original_max_position_embeddings"])
        out = []
        for f in inv:
            wavelen = 2 * math.pi / f
            if wavelen < old / hi:
                out.append(f)
            elif wavelen > old / lo:
                out.append(f / factor)
            else:
                smooth = (old / wavelen - lo) / (hi - lo)
                out.append((1 - smooth) * f / factor + smooth * f)
        inv = out
    return np.asarray(inv, dtype=np.float64).astype(np.float32)


def tensors_for_engine(wf: WeightsFile, keep_quant: bool = False) -> dict[str, np.ndarray]:
    """The file's tensors under the names DecodeEngine.load_weights takes (lm_head falls back to
    the tied embedding).  With keep_quant, quantized matrices stay as stored (integers under the
    plain name, `<name>.scales` beside them; wf.quant names their format) for the decode step's
    quantized projections.  Without it they become fp16(scale * q), the fp16 operand the tcgen05
    quantized GEMM feeds its MMA."""
    t = dict(wf.tensors)
    if not keep_quant:
        for name, fmt in (wf.quant or {}).items():
            t[name] = dequantize(t[name], t.pop(name + ".scales"), fmt).astype(np.float16)
    if "lm_head" not in t:
        t["lm_head"] = t["embed"]
    return t


# ---- 32-block quantization (the formats of include/b200dec.h) -------------------------------


def quantize(w: np.ndarray, fmt: str) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric absmax quantization of a [M, K] matrix (K % 32 == 0) into 32-element blocks:
    scale = fp16(max|w| / qmax) (qmax 127 for q8, 7 for q4), q = clip(rint(w / scale)).
    Returns (q, scales): int8 [M, K] or packed uint8 [M, K/2]; fp16 [M, K/32]."""
    if fmt not in QUANT_FORMATS:
        raise ValueError(f"unknown format {fmt!r}")
    w = np.asarray(w, dtype=np.float32)
    m, k = w.shape
    if k % 32:
        raise ValueError("K must be a multiple of 32")
    qmax, qmin = (127, -127) if fmt == "q8_32" else (7, -8)
    blocks = w.reshape(m, k // 32, 32)
    scales = (np.abs(blocks).max(axis=2) / qmax).astype(np.float16)
    s32 = scales.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(s32 > 0, np.rint(blocks / s32), 0.0)
    q = np.clip(q, qmin, qmax).astype(np.int8).reshape(m, k)
    return (q if fmt == "q8_32" else pack_q4(q)), scales


def quantize_torch(w, fmt: str):
    """quantize() on a torch tensor (any device): the same absmax rule, so seeded synthetic
    weights can be quantized where they are generated.  Returns (q, scales) as torch tensors."""
    import torch

    if fmt not in QUANT_FORMATS:
        raise ValueError(f"unknown format {fmt!r}")
    m, k = w.shape
    if k % 32:
        raise ValueError("K must be a multiple of 32")
    qmax, qmin = (127, -127) if fmt == "q8_32" else (7, -8)
    blocks = w.float().reshape(m, k // 32, 32)
    scales = (blocks.abs().amax(dim=2) / qmax).half()
    s32 = scales.float().unsqueeze(-1)
    q = torch.where(s32 > 0, torch.round(blocks / torch.where(s32 > 0, s32, 1.0)), 0.0)
    q = q.clamp(qmin, qmax).to(torch.int8).reshape(m, k)
    if fmt == "q4_32":
        n = (q.to(torch.int16) & 0xF).to(torch.uint8)
        q = n[:, 0::2] | (n[:, 1::2] << 4)
    return q.contiguous(), scales.contiguous()


def pack_q4(q: np.ndarray) -> np.ndarray:
    """int8 values in [-8, 7], [M, K] -> uint8 [M, K/2]: element 2j in the low nibble."""
    n = (np.asarray(q, dtype=np.int16) & 0xF).astype(np.uint8)
    return (n[:, 0::2] | (n[:, 1::2] << 4)).astype(np.uint8)


def dequantize(q: np.ndarray, scales: np.ndarray, fmt: str) -> np.ndarray:
    """fp32 [M, K] = float(scale) * q, exact."""
    if fmt == "q8_32":
        v = np.asarray(q, dtype=np.int8).astype(np.float32)
    else:
        p = np.asarray(q, dtype=np.uint8)
        lo = ((p & 0xF) ^ 8).astype(np.float32) - 8.0
        hi = (((p >> 4) & 0xF) ^ 8).astype(np.float32) - 8.0
        v = np.empty((p.shape[0], p.shape[1] * 2), np.float32)
        v[:, 0::2], v[:, 1::2] = lo, hi
    m, k = v.shape
    return (v.reshape(m, k // 32, 32) * np.asarray(scales, np.float32)[..., None]).reshape(m, k)


def quantize_file(src: str | Path, dst: str | Path, fmt: str) -> int:
    """Rewrite a weights file with every per-layer projection (wqkv, wo, wgate, wup, wdown)
    quantized to `fmt`; embeddings, LM head and norms stay as they are.  Returns the size."""
    wf = read_weights(src)
    out, quant = {}, {}
    for name, t in wf.tensors.items():
        if name.split(".")[-1] in QUANT_MATRICES and t.ndim == 2 and name not in (wf.quant or {}):
            q, sc = quantize(np.asarray(t), fmt)
            out[name], out[name + ".scales"] = q, sc
            quant[name] = fmt
        else:
            out[name] = np.asarray(t)
    quant.update(wf.quant or {})
    return write_weights(dst, wf.config, out, quant)
