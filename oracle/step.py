"""Whole decode step of a Llama-style model over a ragged paged batch (TEST INFRASTRUCTURE ONLY).

Restates Engine.encodeDecode (LK/main.swift:321-347) for a batch of B sequences that each
decode one token, with the KV cache paged (see oracle.ops).  Weight names follow the
reference's weights file (LK/convert_weights.py:60-72): embed, l{i}.attn_norm, l{i}.wqkv
(rows [q | k | v]), l{i}.wo, l{i}.ffn_norm, l{i}.wgate, l{i}.wup, l{i}.wdown, final_norm;
the LM head is tied to `embed` (LK/main.swift:306).

`decode_step_tp` restates the same step under tensor parallelism (Megatron column/row
pairing, vocab-parallel LM head), simulating the ranks and their all-reduce with sums.  It
defines what the sharded CUDA path must compute; it is not used by the product.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import ops


@dataclass(frozen=True)
class ModelConfig:
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


# random-init Llama-style 1B (eps 1e-5 as in Llama-3.2-1B's config).
LLAMA_1B = ModelConfig(2048, 16, 32, 8, 64, 8192, 128256, 1e-5, 500000.0)


def synth_weights(cfg: ModelConfig, seed: int, std: float = 0.02) -> dict[str, np.ndarray]:
    """Seeded random-init weights: fp16 matrices ~ N(0, std), fp32 norm weights = 1."""
    rng = np.random.default_rng(seed)

    def mat(m, k):
        return (rng.standard_normal((m, k), dtype=np.float32) * std).astype(np.float16)

    w = {"embed": mat(cfg.vocab, cfg.dim)}
    for i in range(cfg.n_layers):
        w[f"l{i}.attn_norm"] = np.ones(cfg.dim, np.float32)
        w[f"l{i}.wqkv"] = mat(cfg.qkv_dim, cfg.dim)
        w[f"l{i}.wo"] = mat(cfg.dim, cfg.n_heads * cfg.head_dim)
        w[f"l{i}.ffn_norm"] = np.ones(cfg.dim, np.float32)
        w[f"l{i}.wgate"] = mat(cfg.ffn_dim, cfg.dim)
        w[f"l{i}.wup"] = mat(cfg.ffn_dim, cfg.dim)
        w[f"l{i}.wdown"] = mat(cfg.dim, cfg.ffn_dim)
    w["final_norm"] = np.ones(cfg.dim, np.float32)
    return w


def _layer_attention(cfg, qkv, k_pages, v_pages, block_table, ctx_lens, invf, n_heads, n_kv, append=True):
    return ops.paged_decode_attention(
        qkv, k_pages, v_pages, block_table, ctx_lens, n_heads, n_kv, cfg.head_dim, invf, append=append
    )


def decode_step(w, cfg: ModelConfig, tokens, ctx_lens, block_table, k_pages, v_pages, append=True):
    """One decode step for B sequences.  Returns (logits [B, V] float64, next tokens [B]).

    tokens[b] is the token at position ctx_lens[b]; k_pages/v_pages are per-layer lists of
    [n_blocks, Hkv, 16, HD] arrays, updated in place with the new token's K/V.  With
    append=False the pages must already hold the new token's (rotated, fp16) K/V -- e.g. the
    pages a GPU step wrote -- and are only read, so the step is evaluated over exactly that cache.
      x = embed(tokens)                                          LK/main.swift:323-330
      per layer:                                                 LK/main.swift:332-341
        qkv = rmsnorm(x, attn_norm) @ wqkv^T
        att = attention(rope(q), paged K/V with rope(k), v appended)
        x  += att @ wo^T
        x  += (silu(xn @ wgate^T) * (xn @ wup^T)) @ wdown^T,  xn = rmsnorm(x, ffn_norm)
      logits = rmsnorm(x, final_norm) @ embed^T; next = argmax   LK/main.swift:342-345
    """
    invf = ops.inv_freq(cfg.head_dim, cfg.theta)
    x = ops.embed(w["embed"], tokens)
    for i in range(cfg.n_layers):
        qkv = ops.gemv(w[f"l{i}.wqkv"], ops.rmsnorm(x, w[f"l{i}.attn_norm"], cfg.eps))
        att = _layer_attention(
            cfg, qkv, k_pages[i], v_pages[i], block_table, ctx_lens, invf, cfg.n_heads, cfg.n_kv_heads, append
        )
        x = x + ops.gemv(w[f"l{i}.wo"], att)
        xn = ops.rmsnorm(x, w[f"l{i}.ffn_norm"], cfg.eps)
        h = ops.swiglu(ops.gemv(w[f"l{i}.wgate"], xn), ops.gemv(w[f"l{i}.wup"], xn))
        x = x + ops.gemv(w[f"l{i}.wdown"], h)
    logits = ops.gemv(w["embed"], ops.rmsnorm(x, w["final_norm"], cfg.eps))
    return logits, ops.argmax(logits)


# --------------------------------------------------------------------------------------------
# Tensor parallelism (extension; the reference is single-GPU)
# --------------------------------------------------------------------------------------------


def tp_slices(cfg: ModelConfig, rank: int, tp: int) -> dict[str, slice]:
    """Index ranges owned by `rank` out of `tp`: heads, KV heads, FFN rows and vocab rows.

    QKV and gate/up are column-parallel (output rows split), O and down are row-parallel
    (input columns split), the LM head is vocab-parallel.  Heads split contiguously, so rank r
    holds q heads [r*Hq/tp, (r+1)*Hq/tp) and the KV heads they read.
    """
    if cfg.n_kv_heads % tp or cfg.ffn_dim % tp:
        raise ValueError("tp must divide n_kv_heads and ffn_dim")
    hq, hk, f = cfg.n_heads // tp, cfg.n_kv_heads // tp, cfg.ffn_dim // tp
    v = -(-cfg.vocab // tp)
    return {
        "q_heads": slice(rank * hq, (rank + 1) * hq),
        "kv_heads": slice(rank * hk, (rank + 1) * hk),
        "ffn": slice(rank * f, (rank + 1) * f),
        "vocab": slice(rank * v, min((rank + 1) * v, cfg.vocab)),
    }


def decode_step_tp(w, cfg: ModelConfig, tp: int, tokens, ctx_lens, block_table, k_pages, v_pages):
    """decode_step with the weights sharded over `tp` simulated ranks.

    k_pages/v_pages hold all KV heads; rank r only touches its KV-head slice.  Partial outputs
    of the row-parallel GEMVs are summed (the all-reduce); the LM head's per-rank (max, index)
    pairs are combined with ties to the lowest global index.
    """
    hd = cfg.head_dim
    invf = ops.inv_freq(hd, cfg.theta)
    x = ops.embed(w["embed"], tokens)
    sl = [tp_slices(cfg, r, tp) for r in range(tp)]
    for i in range(cfg.n_layers):
        wqkv = w[f"l{i}.wqkv"]
        xn = ops.rmsnorm(x, w[f"l{i}.attn_norm"], cfg.eps)
        o_sum = np.zeros_like(x)
        for s in sl:
            qh, kh = s["q_heads"], s["kv_heads"]
            rows = np.concatenate(
                [
                    np.arange(qh.start * hd, qh.stop * hd),
                    cfg.n_heads * hd + np.arange(kh.start * hd, kh.stop * hd),
                    (cfg.n_heads + cfg.n_kv_heads) * hd + np.arange(kh.start * hd, kh.stop * hd),
                ]
            )
            qkv = ops.gemv(wqkv[rows], xn)
            kp, vp = k_pages[i][:, kh], v_pages[i][:, kh]
            att = ops.paged_decode_attention(
                qkv, kp, vp, block_table, ctx_lens, qh.stop - qh.start, kh.stop - kh.start, hd, invf
            )
            k_pages[i][:, kh], v_pages[i][:, kh] = kp, vp
            o_sum += ops.gemv(w[f"l{i}.wo"][:, qh.start * hd : qh.stop * hd], att)
        x = x + o_sum
        xn = ops.rmsnorm(x, w[f"l{i}.ffn_norm"], cfg.eps)
        d_sum = np.zeros_like(x)
        for s in sl:
            f = s["ffn"]
            h = ops.swiglu(ops.gemv(w[f"l{i}.wgate"][f], xn), ops.gemv(w[f"l{i}.wup"][f], xn))
            d_sum += ops.gemv(w[f"l{i}.wdown"][:, f], h)
        x = x + d_sum
    xn = ops.rmsnorm(x, w["final_norm"], cfg.eps)
    logits = np.concatenate([ops.gemv(w["embed"][s["vocab"]], xn) for s in sl], axis=-1)
    best = None
    for s in sl:  # per-rank (max, idx) then the global combine, ties -> lowest index
        part = ops.gemv(w["embed"][s["vocab"]], xn)
        v, idx = part.max(axis=-1), part.argmax(axis=-1) + s["vocab"].start
        if best is None:
            best = (v, idx)
        else:
            take = v > best[0]
            best = (np.where(take, v, best[0]), np.where(take, idx, best[1]))
    return logits, best[1].astype(np.int32)


# --------------------------------------------------------------------------------------------
# float32 NumPy port of the same step, for the timed CPU baseline (bench.py)
# --------------------------------------------------------------------------------------------


class CpuDecodeF32:
    """The decode step above in float32 with BLAS, pre-widened weights (widening is outside any
    timer).  Used only as the CPU baseline that bench.py times; parity uses decode_step."""

    def __init__(self, cfg: ModelConfig, w, k_pages, v_pages, block_table, ctx_lens, layers=None):
        self.cfg = cfg
        self.layers = list(range(cfg.n_layers)) if layers is None else list(layers)
        f = lambda a: np.ascontiguousarray(np.asarray(a, dtype=np.float32))
        self.w = {}
        for i in self.layers:
            for n in ("attn_norm", "wqkv", "wo", "ffn_norm", "wgate", "wup", "wdown"):
                self.w[f"l{i}.{n}"] = f(w[f"l{i}.{n}"])
        self.embed16 = np.asarray(w["embed"])
        self.head = f(w["embed"])
        self.final_norm = f(w["final_norm"])
        self.k_pages, self.v_pages = k_pages, v_pages
        self.table = np.asarray(block_table)
        self.lens = np.asarray(ctx_lens, dtype=np.int64)
        self.invf = ops.inv_freq(cfg.head_dim, cfg.theta)

    @staticmethod
    def _rms(x, g, eps):
        return x * (1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)).astype(np.float32) * g

    def _rope(self, v, pos):
        half = v.shape[-1] // 2
        ang = pos.astype(np.float32)[:, None, None] * self.invf[None, None, :]
        c, s = np.cos(ang), np.sin(ang)
        a, b = v[..., :half], v[..., half:]
        return np.concatenate([a * c - b * s, b * c + a * s], axis=-1)

    def layer(self, i: int, x: np.ndarray) -> np.ndarray:
        c, w = self.cfg, self.w
        hq, hk, hd = c.n_heads, c.n_kv_heads, c.head_dim
        bsz = x.shape[0]
        qkv = self._rms(x, w[f"l{i}.attn_norm"], c.eps) @ w[f"l{i}.wqkv"].T
        q = self._rope(qkv[:, : hq * hd].reshape(bsz, hq, hd), self.lens)
        k = self._rope(qkv[:, hq * hd : (hq + hk) * hd].reshape(bsz, hk, hd), self.lens)
        v = qkv[:, (hq + hk) * hd :].reshape(bsz, hk, hd)
        kp, vp = self.k_pages[i], self.v_pages[i]
        att = np.empty((bsz, hq, hd), np.float32)
        g = hq // hk
        scale = np.float32(1.0 / np.sqrt(hd))
        for b in range(bsz):
            pos = int(self.lens[b])
            blk, slot = int(self.table[b, pos // ops.PAGE_TOKENS]), pos % ops.PAGE_TOKENS
            kp[blk, :, slot], vp[blk, :, slot] = k[b], v[b]
            n = pos + 1
            nb = -(-n // ops.PAGE_TOKENS)
            ids = self.table[b, :nb]
            K = kp[ids].transpose(1, 0, 2, 3).reshape(hk, -1, hd)[:, :n].astype(np.float32)
            V = vp[ids].transpose(1, 0, 2, 3).reshape(hk, -1, hd)[:, :n].astype(np.float32)
            qs = (q[b] * scale).reshape(hk, g, hd)
            s = np.matmul(qs, K.transpose(0, 2, 1))  # [hk, g, n]
            s = np.exp(s - s.max(axis=-1, keepdims=True))
            att[b] = (np.matmul(s, V) / s.sum(axis=-1, keepdims=True)).reshape(hq, hd)
        x = x + att.reshape(bsz, -1) @ w[f"l{i}.wo"].T
        xn = self._rms(x, w[f"l{i}.ffn_norm"], c.eps)
        gt = xn @ w[f"l{i}.wgate"].T
        h = gt / (1.0 + np.exp(-gt)) * (xn @ w[f"l{i}.wup"].T)
        return x + h @ w[f"l{i}.wdown"].T

    def lm_head(self, x: np.ndarray) -> np.ndarray:
        logits = self._rms(x, self.final_norm, self.cfg.eps) @ self.head.T
        return np.argmax(logits, axis=-1).astype(np.int32)

    def embed(self, tokens) -> np.ndarray:
        return self.embed16[np.asarray(tokens)].astype(np.float32)
