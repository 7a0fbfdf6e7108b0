"""Torch-facing wrappers of the decode-step entry points (libb200dec.so via ctypes).

Every function takes CUDA tensors the caller owns, checks shapes/dtypes on the host, launches
on torch's current stream and returns the output tensor(s).  Bad arguments raise ValueError
(the library's B2D_ERR_* status), CUDA / NCCL failures raise B2DError.  There is no CPU path:
calling these without the CUDA library or a GPU raises.

Reference mapping (LK = ios_kernels/kernels/unsloth__Llama-3.2-1B-Instruct/
kernel_metal_f16_20261024-1620): gemv* <- matvec_f16 / matvec_gate_up_silu
(LK/kernels.metal:106-173), rmsnorm <- LK/kernels.metal:71-89, paged_decode_attn <-
attention + rope_kv (LK/kernels.metal:182-305), lm_head_argmax <- argmax (:307-345).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import call

_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16}
EPILOGUES = {
    "store": _lib.EPI_STORE,
    "add": _lib.EPI_ADD,
    "gelu_mul": _lib.EPI_GELU_MUL,
    "swiglu": _lib.EPI_SWIGLU,
}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("all tensors must be CUDA tensors (no CPU path exists)")
        if t is not None and not t.is_contiguous():
            raise ValueError("tensors must be contiguous")


@dataclass
class QWeight:
    """32-block quantized matrix: fmt 'q8' (q int8 [M, K]) or 'q4' (q uint8 [M, K/2]),
    scales fp16 [M, K/32].  See include/b200dec.h for the exact bit layout."""

    fmt: str
    q: torch.Tensor
    scales: torch.Tensor

    @property
    def shape(self) -> tuple[int, int]:
        m = self.q.shape[0]
        k = self.q.shape[1] * (2 if self.fmt == "q4" else 1)
        return m, k

    @property
    def dtype_code(self) -> int:
        return _lib.Q8_32 if self.fmt == "q8" else _lib.Q4_32


class Workspace:
    """Zero-filled device scratch, grown on demand and reused (kernels leave it re-zeroed)."""

    def __init__(self):
        self._buf: dict[int, torch.Tensor] = {}

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        b = self._buf.get(idx)
        if b is None or b.numel() < nbytes:
            b = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            self._buf[idx] = b
        return b


_WS_ATTN = Workspace()
_WS_ARGMAX = Workspace()


def gemv(
    W,
    x: torch.Tensor,
    *,
    gamma: torch.Tensor | None = None,
    eps: float = 1e-6,
    epilogue: str = "store",
    W_up=None,
    aux: torch.Tensor | None = None,
    y: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.float32,
) -> torch.Tensor:
    """y[b] = epilogue(W @ rmsnorm?(x[b])) for x [batch, K] (or [K]); W is a fp32/fp16 tensor
    [M, K] or a QWeight.  For 'add', y is read and updated in place."""
    squeeze = x.dim() == 1
    x2 = x.unsqueeze(0) if squeeze else x
    if isinstance(W, QWeight):
        wq, ws, wcode = W.q, W.scales, W.dtype_code
        M, K = W.shape
    else:
        if W.dtype not in _DT:
            raise ValueError(f"unsupported weight dtype {W.dtype}")
        wq, ws, wcode = W, None, _DT[W.dtype]
        M, K = W.shape
    if x2.dtype not in _DT or x2.shape[-1] != K:
        raise ValueError(f"x must be fp32/fp16 [batch, {K}]")
    up_q = up_s = None
    if W_up is not None:
        if isinstance(W_up, QWeight):
            up_q, up_s = W_up.q, W_up.scales
        else:
            up_q = W_up
    batch = x2.shape[0]
    if y is None:
        if epilogue == "add":
            raise ValueError("epilogue 'add' needs y")
        y = torch.empty(batch, M, dtype=out_dtype, device=x.device)
    y2 = y.unsqueeze(0) if y.dim() == 1 else y
    _need_cuda(wq, ws, up_q, up_s, x2, gamma, aux, y2)
    if y2.dtype not in _DT or tuple(y2.shape) != (batch, M):
        raise ValueError(f"y must be fp32/fp16 [{batch}, {M}]")
    call(
        "b2d_gemv",
        wcode,
        _ptr(wq),
        _ptr(ws),
        _ptr(up_q),
        _ptr(up_s),
        _DT[x2.dtype],
        _ptr(x2),
        K,
        _ptr(gamma),
        float(eps),
        EPILOGUES[epilogue],
        _DT[y2.dtype],
        _ptr(y2),
        M,
        _ptr(aux),
        M,
        K,
        batch,
        _stream(),
    )
    return y2[0] if squeeze and y.dim() == 1 else y


_MMA_FMT = {"f16": _lib.F16, "q8": _lib.Q8_32, "q4": _lib.Q4_32, "int8_b1": 4}


def gemv_mma_formats(formats: set[str] | None = None) -> set[str]:
    """Weight formats ('f16', 'q8', 'q4') that gemv() runs on the tensor-core GEMV, plus
    'int8_b1' (a quantized single token on the integer tensor cores); `formats` replaces the set
    (process-wide).  Returns the previous set."""
    mask = -1 if formats is None else sum(1 << _MMA_FMT[f] for f in formats)
    prev = _lib.lib().b2d_gemv_mma_formats(mask)
    return {f for f, d in _MMA_FMT.items() if (prev >> d) & 1}


def gemv_f32(W: torch.Tensor, x: torch.Tensor, y: torch.Tensor | None = None) -> torch.Tensor:
    """Config 1: fp32 y = W @ x (x [K])."""
    M, K = W.shape
    if W.dtype != torch.float32 or x.dtype != torch.float32 or x.shape != (K,):
        raise ValueError("gemv_f32 needs fp32 W [M, K] and x [K]")
    y = torch.empty(M, dtype=torch.float32, device=x.device) if y is None else y
    _need_cuda(W, x, y)
    call("b2d_gemv_f32", W.data_ptr(), x.data_ptr(), y.data_ptr(), M, K, _stream())
    return y


def dequant(Wq: QWeight) -> torch.Tensor:
    """Exact fp32 dequantized weights [M, K]."""
    M, K = Wq.shape
    w = torch.empty(M, K, dtype=torch.float32, device=Wq.q.device)
    _need_cuda(Wq.q, Wq.scales)
    name = "b2d_dequant_q8_32" if Wq.fmt == "q8" else "b2d_dequant_q4_32"
    call(name, Wq.q.data_ptr(), Wq.scales.data_ptr(), w.data_ptr(), M, K, _stream())
    return w


def lm_head_argmax(
    W: torch.Tensor,
    x: torch.Tensor,
    gamma: torch.Tensor | None = None,
    eps: float = 1e-6,
    *,
    index_offset: int = 0,
    return_logits: bool = False,
    return_max: bool = False,
):
    """tokens[b] = argmax(W @ rmsnorm?(x[b])) + index_offset (fp16 W [V, K], fp32 x [B, K])."""
    V, K = W.shape
    x2 = x.unsqueeze(0) if x.dim() == 1 else x
    B = x2.shape[0]
    if W.dtype != torch.float16 or x2.dtype != torch.float32 or x2.shape[1] != K:
        raise ValueError("lm_head_argmax needs fp16 W [V, K] and fp32 x [B, K]")
    tokens = torch.empty(B, dtype=torch.int32, device=x.device)
    logits = torch.empty(B, V, dtype=torch.float32, device=x.device) if return_logits else None
    mx = torch.empty(B, dtype=torch.float32, device=x.device) if return_max else None
    _need_cuda(W, x2, gamma)
    nbytes = _lib.lib().b2d_lm_head_argmax_workspace_bytes(V, B)
    ws = _WS_ARGMAX.get(nbytes, x.device)
    call(
        "b2d_lm_head_argmax",
        W.data_ptr(),
        x2.data_ptr(),
        K,
        _ptr(gamma),
        float(eps),
        V,
        K,
        B,
        int(index_offset),
        _ptr(logits),
        tokens.data_ptr(),
        _ptr(mx),
        ws.data_ptr(),
        ws.numel(),
        _stream(),
    )
    out = [tokens]
    if return_logits:
        out.append(logits)
    if return_max:
        out.append(mx)
    return out[0] if len(out) == 1 else tuple(out)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x2 = x.unsqueeze(0) if x.dim() == 1 else x
    y = torch.empty_like(x2)
    _need_cuda(x2, w)
    call("b2d_rmsnorm", x2.data_ptr(), w.data_ptr(), y.data_ptr(), x2.shape[0], x2.shape[1], float(eps), _stream())
    return y.view_as(x)


def embed_f16(E: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
    V, Dm = E.shape
    x = torch.empty(tokens.numel(), Dm, dtype=torch.float32, device=E.device)
    _need_cuda(E, tokens)
    call("b2d_embed_f16", E.data_ptr(), tokens.data_ptr(), x.data_ptr(), Dm, tokens.numel(), _stream())
    return x


def argmax_f32(logits: torch.Tensor, index_offset: int = 0) -> torch.Tensor:
    l2 = logits.unsqueeze(0) if logits.dim() == 1 else logits
    out = torch.empty(l2.shape[0], dtype=torch.int32, device=logits.device)
    _need_cuda(l2)
    call("b2d_argmax_f32", l2.data_ptr(), l2.shape[1], l2.shape[0], out.data_ptr(), int(index_offset), _stream())
    return out


def argmax_combine(vals: torch.Tensor, idxs: torch.Tensor) -> torch.Tensor:
    """vals/idxs [n_parts, batch] -> tokens [batch] (ties -> lowest index)."""
    out = torch.empty(vals.shape[1], dtype=torch.int32, device=vals.device)
    _need_cuda(vals, idxs)
    call("b2d_argmax_combine", vals.data_ptr(), idxs.data_ptr(), vals.shape[0], vals.shape[1], out.data_ptr(), _stream())
    return out


def inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """RoPE inverse frequencies (host double -> fp32), as a CPU tensor."""
    out = (ctypes.c_float * (head_dim // 2))()
    call("b2d_inv_freq", head_dim, float(theta), ctypes.addressof(out))
    return torch.tensor(list(out), dtype=torch.float32)


def rope_kv_append(qkv, k_pages, v_pages, block_table, ctx_lens, inv_freq_dev, n_heads, n_kv_heads, head_dim):
    """Rotate q in place in qkv and write rotated k / v at pos = ctx_lens[b] (paged)."""
    _need_cuda(qkv, k_pages, v_pages, block_table, ctx_lens, inv_freq_dev)
    call(
        "b2d_rope_kv_append",
        qkv.data_ptr(),
        _DT[qkv.dtype],
        qkv.shape[1],
        k_pages.data_ptr(),
        v_pages.data_ptr(),
        block_table.data_ptr(),
        block_table.shape[1],
        k_pages.shape[0],
        ctx_lens.data_ptr(),
        inv_freq_dev.data_ptr(),
        n_heads,
        n_kv_heads,
        head_dim,
        qkv.shape[0],
        _stream(),
    )


def to_f16x2(x: torch.Tensor) -> torch.Tensor:
    """fp32 [B, K] -> the B2D_F16X2 form fp16 [2, B, K]: hi = fp16(x), lo = fp16(x - hi)."""
    hi = x.to(torch.float16)
    return torch.stack([hi, (x - hi.float()).to(torch.float16)])


def from_f16x2(t: torch.Tensor) -> torch.Tensor:
    """fp16 [2, B, K] hi + lo planes -> fp32 [B, K]."""
    return t[0].float() + t[1].float()


def _is_x2(t: torch.Tensor | None) -> bool:
    return t is not None and t.dim() == 3 and t.shape[0] == 2 and t.dtype == torch.float16


def attn_workspace_bytes(batch, n_heads, n_kv_heads, head_dim, max_ctx) -> int:
    return int(_lib.lib().b2d_paged_attn_workspace_bytes(batch, n_heads, n_kv_heads, head_dim, max_ctx))


def paged_decode_attn(
    qkv: torch.Tensor,
    k_pages: torch.Tensor,
    v_pages: torch.Tensor,
    block_table: torch.Tensor,
    ctx_lens: torch.Tensor,
    inv_freq_dev: torch.Tensor | None,
    n_heads: int,
    n_kv_heads: int,
    head_dim: int,
    max_ctx: int,
    *,
    scale: float = 0.0,
    window: int = 0,
    append: bool = True,
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.float32,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    """Ragged paged decode attention; see include/b200dec.h b2d_paged_decode_attn.  `out` may be
    fp16 [2, B, Hq*HD]: the output as B2D_F16X2 hi + lo planes."""
    B = qkv.shape[0]
    if out is None:
        out = torch.empty(B, n_heads * head_dim, dtype=out_dtype, device=qkv.device)
    out_dt = _lib.F16X2 if _is_x2(out) else _DT[out.dtype]
    nbytes = attn_workspace_bytes(B, n_heads, n_kv_heads, head_dim, max_ctx)
    ws = workspace if workspace is not None else _WS_ATTN.get(nbytes, qkv.device)
    _need_cuda(qkv, k_pages, v_pages, block_table, ctx_lens, inv_freq_dev, out, ws)
    if block_table.dtype != torch.int32 or ctx_lens.dtype != torch.int32:
        raise ValueError("block_table and ctx_lens must be int32")
    call(
        "b2d_paged_decode_attn",
        qkv.data_ptr(),
        _DT[qkv.dtype],
        qkv.shape[1],
        k_pages.data_ptr(),
        v_pages.data_ptr(),
        block_table.data_ptr(),
        block_table.shape[1],
        k_pages.shape[0],
        ctx_lens.data_ptr(),
        _ptr(inv_freq_dev),
        n_heads,
        n_kv_heads,
        head_dim,
        B,
        max_ctx,
        float(scale),
        int(window),
        1 if append else 0,
        out.data_ptr(),
        out_dt,
        out.shape[-1],
        ws.data_ptr(),
        ws.numel(),
        _stream(),
    )
    return out


_WS_TC = Workspace()
_TC_EPI = {"store": _lib.EPI_STORE, "add": _lib.EPI_ADD, "gelu_mul": _lib.EPI_GELU_MUL, "swiglu": _lib.EPI_SWIGLU, "argmax": _lib.EPI_ARGMAX, "silu_mul": _lib.EPI_SILU_MUL}


@dataclass
class TcPacked:
    """fp16 weights [M, K] in the tensor-core tile layout (b2d_tc_pack_f16): 16 KB tiles of 128
    rows x 64 columns, already in the MMA's swizzled shared-memory image."""

    buf: torch.Tensor  # uint8 [b2d_tc_packed_bytes(M, K)]
    M: int
    K: int

    @property
    def shape(self) -> tuple[int, int]:
        return self.M, self.K


def pack_tc(W: torch.Tensor) -> TcPacked:
    """Repack fp16 W [M, K] (row-major) into the tensor-core tile layout."""
    if W.dtype != torch.float16 or W.dim() != 2 or W.stride(1) != 1:
        raise ValueError("pack_tc needs fp16 W [M, K] with unit column stride")
    M, K = W.shape
    buf = torch.empty(_lib.lib().b2d_tc_packed_bytes(M, K), dtype=torch.uint8, device=W.device)
    _need_cuda(W, buf)
    call("b2d_tc_pack_f16", W.data_ptr(), W.stride(0), M, K, buf.data_ptr(), _stream())
    return TcPacked(buf, M, K)


def tc_workspace_bytes(M: int, K: int, batch: int, epilogue: str = "store") -> int:
    return int(_lib.lib().b2d_gemm_tc_workspace_bytes(M, K, batch, _TC_EPI[epilogue]))


def gemm_tc(
    W: torch.Tensor | TcPacked,
    X: torch.Tensor,
    *,
    epilogue: str = "store",
    W_up: torch.Tensor | TcPacked | None = None,
    aux: torch.Tensor | None = None,
    y: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.float32,
    index_offset: int = 0,
    return_logits: bool = False,
    workspace: torch.Tensor | None = None,
):
    """Tensor-core batched GEMV (tcgen05): y[b] = epilogue(W @ X[b]) for fp16 W [M, K] and fp16
    X [batch <= 32, K], or X fp16 [2, batch, K]: fp32-precision activations as B2D_F16X2 hi + lo
    planes (to_f16x2).  y may be fp16 [2, batch, M] (B2D_F16X2 output) as well.  For 'argmax'
    returns tokens (and logits if asked).  W (and W_up) may be row-major or packed by pack_tc."""
    M, K = W.shape
    x2 = _is_x2(X)
    B = X.shape[-2]
    packed = isinstance(W, TcPacked)
    if packed != (W_up is None or isinstance(W_up, TcPacked)) and W_up is not None:
        raise ValueError("W and W_up must both be packed or both row-major")
    if (not packed and W.dtype != torch.float16) or X.dtype != torch.float16 or X.shape[-1] != K:
        raise ValueError("gemm_tc needs fp16 W [M, K] and fp16 X [batch, K] (or [2, batch, K])")
    if packed and x2:
        raise ValueError("hi/lo activations run on row-major weights")
    Wt = W.buf if packed else W
    Wu = (W_up.buf if packed else W_up) if W_up is not None else None
    ws = workspace if workspace is not None else _WS_TC.get(tc_workspace_bytes(M, K, B, epilogue), X.device)
    tokens = logits = None
    if epilogue == "argmax":
        tokens = torch.empty(B, dtype=torch.int32, device=X.device)
        logits = torch.empty(B, M, dtype=torch.float32, device=X.device) if return_logits else None
        ydt = _lib.F32
    else:
        if y is None:
            if epilogue == "add":
                raise ValueError("epilogue 'add' needs y")
            y = torch.empty(B, M, dtype=out_dtype, device=X.device)
        if _is_x2(y) and tuple(y.shape) == (2, B, M):
            ydt = _lib.F16X2
        elif y.dtype in _DT and tuple(y.shape) == (B, M):
            ydt = _DT[y.dtype]
        else:
            raise ValueError(f"y must be fp32/fp16 [{B}, {M}] or fp16 [2, {B}, {M}]")
    _need_cuda(Wt, X, Wu, aux, y, ws, tokens, logits)
    head = () if packed else (_lib.F16X2 if x2 else _lib.F16,)
    call(
        "b2d_gemm_tc_packed" if packed else "b2d_gemm_tc_ex",
        *head,
        Wt.data_ptr(),
        _ptr(Wu),
        X.data_ptr(),
        K,
        _TC_EPI[epilogue],
        ydt,
        _ptr(y),
        M,
        _ptr(aux),
        M,
        K,
        B,
        _ptr(logits),
        _ptr(tokens),
        None,
        int(index_offset),
        ws.data_ptr(),
        ws.numel(),
        _stream(),
    )
    if epilogue == "argmax":
        return (tokens, logits) if return_logits else tokens
    return y


def gemm_tc_q(
    Wq: QWeight,
    X: torch.Tensor,
    *,
    epilogue: str = "store",
    aux: torch.Tensor | None = None,
    y: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.float32,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    """Tensor-core batched GEMV over 32-block quantized weights: y[b] = epilogue(W @ X[b]) with
    W = scale * q dequantized in shared memory to fp16 (the MMA operand), fp16 X [batch <= 32, K]
    or hi + lo planes fp16 [2, batch, K].  Epilogues 'store', 'add', 'gelu_mul'."""
    M, K = Wq.shape
    x2 = _is_x2(X)
    B = X.shape[-2]
    if X.dtype != torch.float16 or X.shape[-1] != K:
        raise ValueError("gemm_tc_q needs fp16 X [batch, K] (or [2, batch, K])")
    if epilogue not in ("store", "add", "gelu_mul", "silu_mul"):
        raise ValueError(f"gemm_tc_q: unsupported epilogue {epilogue!r}")
    ws = workspace if workspace is not None else _WS_TC.get(tc_workspace_bytes(M, K, B, epilogue), X.device)
    if y is None:
        if epilogue == "add":
            raise ValueError("epilogue 'add' needs y")
        y = torch.empty(B, M, dtype=out_dtype, device=X.device)
    if y.dtype not in _DT or tuple(y.shape) != (B, M):
        raise ValueError(f"y must be fp32/fp16 [{B}, {M}]")
    _need_cuda(Wq.q, Wq.scales, X, aux, y, ws)
    call(
        "b2d_gemm_tc_q_ex",
        _lib.F16X2 if x2 else _lib.F16,
        Wq.dtype_code,
        Wq.q.data_ptr(),
        Wq.scales.data_ptr(),
        X.data_ptr(),
        K,
        _TC_EPI[epilogue],
        _DT[y.dtype],
        y.data_ptr(),
        M,
        _ptr(aux),
        M,
        K,
        B,
        ws.data_ptr(),
        ws.numel(),
        _stream(),
    )
    return y


def _ptr_array(ts) -> ctypes.Array:
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def tp_allreduce_add_rmsnorm(
    parts: list[torch.Tensor],
    sigs: list[torch.Tensor],
    epochs: torch.Tensor,
    rank: int,
    x: torch.Tensor,
    err: torch.Tensor,
    gamma: torch.Tensor | None = None,
    eps: float = 1e-5,
    out16: torch.Tensor | None = None,
    slot0: int = 0,
    timeout_ns: int = 10_000_000_000,
) -> torch.Tensor | None:
    """x += parts[0] + ... + parts[tp-1] (rank order) after a per-row barrier on the ranks'
    signal arrays; returns fp16 rmsnorm(x) * gamma if gamma is given.  parts: the ranks'
    partials [rows, D] fp32 as mapped in this process; sigs: the ranks' uint32 signal arrays;
    epochs: this rank's uint32 epoch counters; err: device int32 error word (a barrier that
    times out writes B2D_ERR_TIMEOUT there and leaves its row unchanged)."""
    rows, D = x.shape
    if gamma is not None and out16 is None:
        out16 = torch.empty(rows, D, dtype=torch.float16, device=x.device)
    _need_cuda(x, err, epochs, gamma, out16, *parts, *sigs)
    call(
        "b2d_tp_allreduce_add_rmsnorm",
        ctypes.cast(_ptr_array(parts), ctypes.c_void_p),
        ctypes.cast(_ptr_array(sigs), ctypes.c_void_p),
        epochs.data_ptr(),
        rank,
        len(parts),
        slot0,
        x.data_ptr(),
        _ptr(gamma),
        float(eps),
        _ptr(out16),
        D,
        rows,
        int(timeout_ns),
        err.data_ptr(),
        _stream(),
    )
    return out16


def tp_argmax_gather(
    vals: list[torch.Tensor],
    idxs: list[torch.Tensor],
    sigs: list[torch.Tensor],
    epochs: torch.Tensor,
    rank: int,
    slot: int,
    err: torch.Tensor,
    timeout_ns: int = 10_000_000_000,
) -> torch.Tensor:
    """Best (value, index) over the ranks' LM-head candidates per token (ties -> lower index)."""
    B = vals[0].numel()
    tokens = torch.empty(B, dtype=torch.int32, device=vals[0].device)
    _need_cuda(tokens, epochs, err, *vals, *idxs, *sigs)
    call(
        "b2d_tp_argmax_gather",
        ctypes.cast(_ptr_array(vals), ctypes.c_void_p),
        ctypes.cast(_ptr_array(idxs), ctypes.c_void_p),
        ctypes.cast(_ptr_array(sigs), ctypes.c_void_p),
        epochs.data_ptr(),
        rank,
        len(vals),
        slot,
        B,
        tokens.data_ptr(),
        int(timeout_ns),
        err.data_ptr(),
        _stream(),
    )
    return tokens


def add_rmsnorm_f16(x: torch.Tensor, gamma: torch.Tensor, eps: float, p: torch.Tensor | None = None, x2: bool = False) -> torch.Tensor:
    """x += p (if given, in place); returns fp16 rmsnorm(x) * gamma, or with x2 the B2D_F16X2
    hi + lo planes fp16 [2, rows, D]."""
    out = torch.empty(((2,) if x2 else ()) + tuple(x.shape), dtype=torch.float16, device=x.device)
    _need_cuda(x, gamma, p)
    call(
        "b2d_add_rmsnorm", x.data_ptr(), _ptr(p), gamma.data_ptr(), float(eps), _lib.F16X2 if x2 else _lib.F16,
        out.data_ptr(), x.shape[0], x.shape[1], _stream(),
    )
    return out
