"""Tensor-parallel sharding of a Llama-style decoder's weights (host side, torch tensors).

The reference is single-GPU (one Metal device, LK/main.swift:152-215); this is the extension
BASELINE config 5 asks for.  Megatron pairing:
  * wqkv   [(Hq + 2 Hkv) HD, D]  column-parallel: rank r keeps its q heads, then its k heads,
                                 then its v heads, so its local qkv rows keep the reference's
                                 [q | k | v] order (LK/kernels.metal:176-177);
  * wo     [D, Hq HD]            row-parallel: columns of rank r's q heads;
  * wgate, wup [F, D]            column-parallel: rows [r F/tp, (r+1) F/tp);
  * wdown  [D, F]                row-parallel: the matching columns;
  * LM head (tied embedding) [V, D]  vocab-parallel: rows [r ceil(V/tp), ...);
  * norms and the embedding table are replicated.
Rank r's q heads read only rank r's KV heads because heads split contiguously and tp divides
Hkv.  The per-rank KV page pools hold Hkv/tp heads.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class ModelShape:
    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn_dim: int
    vocab: int
    eps: float
    theta: float

    @property
    def qkv_dim(self) -> int:
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim


LLAMA_1B = ModelShape(2048, 16, 32, 8, 64, 8192, 128256, 1e-5, 500000.0)


def check_tp(shape: ModelShape, tp: int) -> None:
    if tp < 1 or shape.n_kv_heads % tp or shape.ffn_dim % tp or shape.n_heads % shape.n_kv_heads:
        raise ValueError(f"tp={tp} must divide n_kv_heads={shape.n_kv_heads} and ffn_dim={shape.ffn_dim}")


def vocab_rows(shape: ModelShape, rank: int, tp: int) -> tuple[int, int]:
    """[start, stop) of rank's LM-head rows."""
    per = -(-shape.vocab // tp)
    return rank * per, min((rank + 1) * per, shape.vocab)


def qkv_rows(shape: ModelShape, rank: int, tp: int) -> torch.Tensor:
    """Row indices of wqkv owned by rank, in local [q | k | v] order."""
    hd = shape.head_dim
    hq, hk = shape.n_heads // tp, shape.n_kv_heads // tp
    q = torch.arange(rank * hq * hd, (rank + 1) * hq * hd)
    k = shape.n_heads * hd + torch.arange(rank * hk * hd, (rank + 1) * hk * hd)
    v = (shape.n_heads + shape.n_kv_heads) * hd + torch.arange(rank * hk * hd, (rank + 1) * hk * hd)
    return torch.cat([q, k, v])


def shard_layer(w: dict[str, torch.Tensor], shape: ModelShape, rank: int, tp: int) -> dict[str, torch.Tensor]:
    """One layer's weights (keys attn_norm, wqkv, wo, ffn_norm, wgate, wup, wdown) -> rank's shard."""
    check_tp(shape, tp)
    hd, hq, f = shape.head_dim, shape.n_heads // tp, shape.ffn_dim // tp
    rows = qkv_rows(shape, rank, tp).to(w["wqkv"].device)
    return {
        "attn_norm": w["attn_norm"].contiguous(),
        "wqkv": w["wqkv"].index_select(0, rows).contiguous(),
        "wo": w["wo"][:, rank * hq * hd : (rank + 1) * hq * hd].contiguous(),
        "ffn_norm": w["ffn_norm"].contiguous(),
        "wgate": w["wgate"][rank * f : (rank + 1) * f].contiguous(),
        "wup": w["wup"][rank * f : (rank + 1) * f].contiguous(),
        "wdown": w["wdown"][:, rank * f : (rank + 1) * f].contiguous(),
    }


def shard_layer_quant(
    w: dict[str, torch.Tensor], shape: ModelShape, rank: int, tp: int, fmt: str
) -> dict[str, torch.Tensor]:
    """shard_layer for a layer whose five projections are stored in the 32-block format `fmt`
    ("q8_32": int8 [M, K]; "q4_32": uint8 [M, K/2], two elements per byte), each with
    `<name>.scales` fp16 [M, K/32].  Column-parallel matrices split their rows (integers and
    scales alike); row-parallel ones split K, which must stay a multiple of 32 per rank."""
    check_tp(shape, tp)
    hd, hq, f = shape.head_dim, shape.n_heads // tp, shape.ffn_dim // tp
    per_byte = 2 if fmt == "q4_32" else 1
    rows = qkv_rows(shape, rank, tp).to(w["wqkv"].device)

    def cols(name: str, a: int, b: int) -> tuple[torch.Tensor, torch.Tensor]:
        if a % 32 or b % 32:
            raise ValueError(f"{name}: a rank's K range [{a}, {b}) must hold whole 32-element blocks")
        q, sc = w[name], w[name + ".scales"]
        return q[:, a // per_byte : b // per_byte].contiguous(), sc[:, a // 32 : b // 32].contiguous()

    out = {"attn_norm": w["attn_norm"].contiguous(), "ffn_norm": w["ffn_norm"].contiguous()}
    out["wqkv"] = w["wqkv"].index_select(0, rows).contiguous()
    out["wqkv.scales"] = w["wqkv.scales"].index_select(0, rows).contiguous()
    out["wo"], out["wo.scales"] = cols("wo", rank * hq * hd, (rank + 1) * hq * hd)
    for n in ("wgate", "wup"):
        out[n] = w[n][rank * f : (rank + 1) * f].contiguous()
        out[n + ".scales"] = w[n + ".scales"][rank * f : (rank + 1) * f].contiguous()
    out["wdown"], out["wdown.scales"] = cols("wdown", rank * f, (rank + 1) * f)
    return out


def shard_head(embed: torch.Tensor, shape: ModelShape, rank: int, tp: int) -> torch.Tensor:
    a, b = vocab_rows(shape, rank, tp)
    return embed[a:b].contiguous()
