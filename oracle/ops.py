"""NumPy float64 restatement of every decode-step op (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module; the
product path never does.  Each function cites the reference lines it restates.  Paths are
relative to the reference project; two aliases keep the citations short:

  LK = ios_kernels/kernels/unsloth__Llama-3.2-1B-Instruct/kernel_metal_f16_20261024-1620
  GK = ios_kernels/kernels/google__gemma-4-E2B-it/kernel_metal_f16_20261025-1225

Rules shared by every function here:
  * inputs are taken at their exact stored values (fp16 weights widened exactly), and all
    arithmetic is float64, so the oracle is the "infinitely precise" answer for the stored bytes;
  * where the reference rounds a value to storage (K/V written to the fp16 cache, the fp32
    RoPE angle), the oracle rounds at the same place;
  * extensions with no reference code (32-block int8/4-bit weights, paged KV, ragged batches)
    are defined here and in the C header include/b200dec.h, and pinned by known-answer tests.
"""

from __future__ import annotations

import numpy as np

PAGE_TOKENS = 16  # tokens per KV page (paged-cache extension)
QBLOCK = 32  # elements per quantization block

# GEMV epilogues.  Values match include/b200dec.h (B2D_EPI_*).  STORE/ADD/GELU_MUL mirror
# GK/kernels.metal:151-198 (EPI 0/1/2); SWIGLU mirrors LK/kernels.metal:139-173; ARGMAX fuses
# LK/kernels.metal:307-345 into the LM-head GEMV.
EPI_STORE, EPI_ADD, EPI_GELU_MUL, EPI_SWIGLU, EPI_ARGMAX = 0, 1, 2, 3, 4


def f64(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float64)


# --------------------------------------------------------------------------------------------
# Norms, activations, GEMV
# --------------------------------------------------------------------------------------------


def rmsnorm(x, w, eps: float) -> np.ndarray:
    """y = x * rsqrt(mean(x^2) + eps) * w over the last axis; w applied directly (no 1+w).

    LK/kernels.metal:71-89 (sum of squares, eps inside the rsqrt, weight after the scale).
    """
    x = f64(x)
    ss = np.sum(x * x, axis=-1, keepdims=True)
    return x * (1.0 / np.sqrt(ss / x.shape[-1] + eps)) * f64(w)


def gemv(W, x) -> np.ndarray:
    """y[..., r] = sum_k W[r, k] * x[..., k]  (LK/kernels.metal:106-131, fp32 accumulation there)."""
    return f64(x) @ f64(W).T


def silu(g) -> np.ndarray:
    g = f64(g)
    return g / (1.0 + np.exp(-g))


def swiglu(g, u) -> np.ndarray:
    """h = silu(g) * u  (LK/kernels.metal:171: g / (1 + exp(-g)) * u)."""
    return silu(g) * f64(u)


def gelu_tanh(x) -> np.ndarray:
    """GK/kernels.metal:26-28 (tanh approximation)."""
    x = f64(x)
    return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


def gemv_fused(
    W,
    x,
    gamma=None,
    eps: float = 1e-6,
    epilogue: int = EPI_STORE,
    y_prev=None,
    aux=None,
    W_up=None,
):
    """The fused decode GEMV: optional RMSNorm prologue, then one of the epilogues.

    x: [b, K] (or [K]).  Returns the new y (float64) for STORE/ADD/GELU_MUL/SWIGLU, and
    (logits, argmax per row) for ARGMAX.
      * prologue: x <- rmsnorm(x, gamma, eps)                     LK/main.swift:333-334 fused
      * STORE:    y = W x                                         LK/kernels.metal:130
      * ADD:      y = y_prev + W x                                LK/kernels.metal:135
      * GELU_MUL: y = gelu_tanh(W x) * aux                        GK/kernels.metal:186
      * SWIGLU:   y = silu(W x) * (W_up x)                        LK/kernels.metal:171
      * ARGMAX:   logits = W x, token = argmax (ties -> lowest)   LK/main.swift:305-315
    """
    x = f64(x)
    if gamma is not None:
        x = rmsnorm(x, gamma, eps)
    acc = gemv(W, x)
    if epilogue == EPI_STORE:
        return acc
    if epilogue == EPI_ADD:
        return f64(y_prev) + acc
    if epilogue == EPI_GELU_MUL:
        return gelu_tanh(acc) * f64(aux)
    if epilogue == EPI_SWIGLU:
        return swiglu(acc, gemv(W_up, x))
    if epilogue == EPI_ARGMAX:
        return acc, argmax(acc)
    raise ValueError(f"unknown epilogue {epilogue}")


def argmax(logits) -> np.ndarray:
    """Greedy token per row; ties go to the lowest index (LK/kernels.metal:326, like torch.argmax)."""
    return np.argmax(f64(logits), axis=-1).astype(np.int32)


def embed(E, tokens) -> np.ndarray:
    """x[t] = float(E[tokens[t]])  (LK/kernels.metal:31-39)."""
    return f64(np.asarray(E)[np.asarray(tokens, dtype=np.int64)])


# --------------------------------------------------------------------------------------------
# 32-block quantized weights (extension: BASELINE config 3; no reference code exists)
#
#   q8_32: qs int8 [M, K] row-major, values in [-127, 127]; scales fp16 [M, K/32].
#   q4_32: qs uint8 [M, K/2]; byte j of row r holds element 2j in its low nibble and 2j+1 in
#          its high nibble; a nibble n decodes to ((n ^ 8) - 8), i.e. 4-bit two's complement
#          in [-8, 7]; scales fp16 [M, K/32].
#   dequant: w[r, k] = float32(scale[r, k // 32]) * float32(q[r, k]).  The product of an
#          11-bit and an at-most-8-bit significand fits in fp32's 24 bits, so it is exact.
# --------------------------------------------------------------------------------------------


def pack_q4(q) -> np.ndarray:
    """int values in [-8, 7], shape [M, K] (K even) -> packed uint8 [M, K/2]."""
    q = np.asarray(q, dtype=np.int16)
    if q.min(initial=0) < -8 or q.max(initial=0) > 7:
        raise ValueError("q4 values must lie in [-8, 7]")
    lo = (q[..., 0::2] & 0xF).astype(np.uint8)
    hi = (q[..., 1::2] & 0xF).astype(np.uint8)
    return (lo | (hi << 4)).astype(np.uint8)


def unpack_q4(packed) -> np.ndarray:
    """packed uint8 [M, K/2] -> int8 [M, K] (low nibble first)."""
    p = np.asarray(packed, dtype=np.uint8)
    lo = ((p & 0xF).astype(np.int16) ^ 8) - 8
    hi = (((p >> 4) & 0xF).astype(np.int16) ^ 8) - 8
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.int8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


def dequant_q8_32(qs, scales) -> np.ndarray:
    """Exact fp32 dequantized weights [M, K]."""
    qs = np.asarray(qs, dtype=np.int8)
    s = np.asarray(scales, dtype=np.float16).astype(np.float32)
    return np.repeat(s, QBLOCK, axis=-1)[..., : qs.shape[-1]] * qs.astype(np.float32)


def dequant_q4_32(packed, scales) -> np.ndarray:
    """Exact fp32 dequantized weights [M, K]."""
    return dequant_q8_32(unpack_q4(packed), scales)


def gemv_q8_32(qs, scales, x) -> np.ndarray:
    return gemv(dequant_q8_32(qs, scales), x)


def gemv_q4_32(packed, scales, x) -> np.ndarray:
    return gemv(dequant_q4_32(packed, scales), x)


# --------------------------------------------------------------------------------------------
# RoPE, KV cache, attention
# --------------------------------------------------------------------------------------------


def inv_freq(head_dim: int, theta: float, rope_scaling: dict | None = None) -> np.ndarray:
    """RoPE inverse frequencies, computed in double and stored as fp32 (LK/main.swift:90-108).

    Optional Llama-3 frequency scaling follows the same lines (LK/main.swift:95-107).
    """
    i = np.arange(head_dim // 2, dtype=np.float64)
    inv = 1.0 / np.power(float(theta), 2.0 * i / head_dim)
    if rope_scaling and rope_scaling.get("rope_type") == "llama3":
        factor = float(rope_scaling["factor"])
        lo = float(rope_scaling["low_freq_factor"])
        hi = float(rope_scaling["high_freq_factor"])
        old = float(rope_scaling["original_max_position_embeddings"])
        wavelen = 2.0 * np.pi / inv
        smooth = (old / wavelen - lo) / (hi - lo)
        mid = (1.0 - smooth) * inv / factor + smooth * inv
        inv = np.where(wavelen < old / hi, inv, np.where(wavelen > old / lo, inv / factor, mid))
    return inv.astype(np.float32)


def rope(v, pos, invf) -> np.ndarray:
    """rotate_half RoPE on the last axis (LK/kernels.metal:195-212).

    Pairs are (i, i + HD/2).  The angle is the fp32 product float(pos) * inv_freq[i], as in the
    kernel (LK/kernels.metal:203); cos/sin of that fp32 angle are then taken exactly.
      ra = a*c - b*s,  rb = b*c + a*s
    v: [..., HD]; pos: scalar or array broadcastable to v.shape[:-1].
    """
    v = f64(v)
    half = v.shape[-1] // 2
    pos32 = np.asarray(pos, dtype=np.float32)[..., None]
    ang = (pos32 * np.asarray(invf, dtype=np.float32)).astype(np.float32).astype(np.float64)
    c, s = np.cos(ang), np.sin(ang)
    a, b = v[..., :half], v[..., half:]
    return np.concatenate([a * c - b * s, b * c + a * s], axis=-1)


def page_slot(block_table, seq: int, pos: int) -> tuple[int, int]:
    """Physical (block, slot) of token `pos` of sequence `seq` in the paged cache."""
    return int(block_table[seq][pos // PAGE_TOKENS]), pos % PAGE_TOKENS


def kv_append_paged(k_pages, v_pages, block_table, positions, k_new, v_new) -> None:
    """Write one token per sequence into the paged cache, rounding to fp16 like the reference.

    Pages are [n_blocks, Hkv, PAGE_TOKENS, HD] (the reference's contiguous [kv_head][max_ctx][HD]
    cache of LK/kernels.metal:10 and LK/kernels.metal:218-222, cut into 16-token pages).
    k_new/v_new: [B, Hkv, HD] (k already rotated).
    """
    for b, pos in enumerate(np.asarray(positions).tolist()):
        blk, slot = page_slot(block_table, b, pos)
        k_pages[blk, :, slot, :] = np.asarray(k_new[b]).astype(k_pages.dtype)
        v_pages[blk, :, slot, :] = np.asarray(v_new[b]).astype(v_pages.dtype)


def gather_kv(pages, block_table_row, n: int) -> np.ndarray:
    """Tokens [0, n) of one sequence as [Hkv, n, HD] (float64)."""
    nblk = (n + PAGE_TOKENS - 1) // PAGE_TOKENS
    blocks = np.asarray(block_table_row[:nblk], dtype=np.int64)
    g = f64(pages[blocks])  # [nblk, Hkv, 16, HD]
    g = g.transpose(1, 0, 2, 3).reshape(pages.shape[1], nblk * PAGE_TOKENS, pages.shape[3])
    return g[:, :n, :]


def attention(q, K, V, scale: float, window: int = 0) -> np.ndarray:
    """Single-query attention for one sequence (LK/kernels.metal:235-305, window GK:343).

    q: [Hq, HD]; K, V: [Hkv, n, HD], keys 0..n-1 where n-1 is the query's own position.
    The query is pre-multiplied by `scale` in fp32 (LK/kernels.metal:255), softmax subtracts the
    max, and the weighted sum is divided by the sum at the end (:300).  GQA: q head h reads KV
    head h // (Hq/Hkv) (:245).  window > 0 keeps keys [n - window, n) (GK/kernels.metal:343).
    """
    q = np.asarray(q)
    hq, n = q.shape[0], K.shape[1]
    group = hq // K.shape[0]
    qs = f64((np.asarray(q, dtype=np.float32) * np.float32(scale)).astype(np.float32))
    start = n - window if (window and n > window) else 0
    out = np.empty((hq, q.shape[1]), dtype=np.float64)
    for h in range(hq):
        kh = K[h // group, start:n]
        vh = V[h // group, start:n]
        s = kh @ qs[h]
        p = np.exp(s - s.max())
        out[h] = (p @ vh) / p.sum()
    return out


def paged_decode_attention(
    qkv,
    k_pages,
    v_pages,
    block_table,
    ctx_lens,
    n_heads: int,
    n_kv_heads: int,
    head_dim: int,
    invf,
    scale: float | None = None,
    window: int = 0,
    append: bool = True,
) -> np.ndarray:
    """Decode attention for a ragged batch over a paged cache, with RoPE and KV append.

    qkv: [B, (Hq + 2*Hkv) * HD], each row laid out [q | k | v] as in LK/kernels.metal:176-177.
    Sequence b holds ctx_lens[b] cached tokens; its new token sits at pos = ctx_lens[b]:
      1. q and k are rotated at pos (LK/kernels.metal:195-212);
      2. if `append`, rotated k and v are rounded to the cache dtype and written at pos
         (LK/kernels.metal:214-222, in pages);
      3. the query attends over keys [0, pos] (LK/kernels.metal:246, n = pos + 1).
    k_pages/v_pages are updated in place.  Returns out [B, Hq*HD] in float64.
    """
    qkv = np.asarray(qkv)
    bsz = qkv.shape[0]
    hq, hk, hd = n_heads, n_kv_heads, head_dim
    if scale is None:
        scale = 1.0 / np.sqrt(hd)  # LK/main.swift:293
    pos = np.asarray(ctx_lens, dtype=np.int64)
    q = f64(qkv[:, : hq * hd]).reshape(bsz, hq, hd)
    k = f64(qkv[:, hq * hd : (hq + hk) * hd]).reshape(bsz, hk, hd)
    v = f64(qkv[:, (hq + hk) * hd : (hq + 2 * hk) * hd]).reshape(bsz, hk, hd)
    # The reference rotates q in place in its fp32 qkv buffer, so the rotated q is fp32.
    qr = rope(q, pos[:, None], invf).astype(np.float32)
    kr = rope(k, pos[:, None], invf)
    if append:
        kv_append_paged(k_pages, v_pages, block_table, pos, kr, v)
    out = np.empty((bsz, hq * hd), dtype=np.float64)
    for b in range(bsz):
        n = int(pos[b]) + 1
        K = gather_kv(k_pages, block_table[b], n)
        V = gather_kv(v_pages, block_table[b], n)
        out[b] = attention(qr[b], K, V, scale, window).reshape(-1)
    return out
