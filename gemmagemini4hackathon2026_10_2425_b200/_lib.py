"""ctypes binding of libb200dec.so (the C ABI declared in include/b200dec.h).

Loading fails loudly: there is no CPU fallback.  If the library has not been built, call
gemmagemini4hackathon2026_10_2425_b200.build.build() (or `python -m ...build`).
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb200dec.so"
HEADER = Path(__file__).resolve().parents[1] / "include" / "b200dec.h"

OK, ERR_NULL, ERR_SHAPE, ERR_ALIGN, ERR_UNSUPPORTED, ERR_WORKSPACE = 0, 1, 2, 3, 4, 5
ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_STATE = 6, 7, 8, 9
F32, F16, Q8_32, Q4_32, F16X2 = 0, 1, 2, 3, 4
EPI_STORE, EPI_ADD, EPI_GELU_MUL, EPI_SWIGLU, EPI_ARGMAX, EPI_SILU_MUL = 0, 1, 2, 3, 4, 5

P = C.c_void_p
I = C.c_int
Z = C.c_size_t
Fl = C.c_float
D = C.c_double


class ModelConfig(C.Structure):
    """b2d_model_config."""

    _fields_ = [
        ("dim", I),
        ("n_layers", I),
        ("n_heads", I),
        ("n_kv_heads", I),
        ("head_dim", I),
        ("ffn_dim", I),
        ("vocab", I),
        ("eps", Fl),
        ("rope_theta", D),
        ("max_batch", I),
        ("max_ctx", I),
        ("max_blocks", I),
        ("n_blocks", I),
    ]


# name -> (restype, argtypes)
SIGNATURES = {
    "b2d_status_string": (C.c_char_p, [I]),
    "b2d_last_cuda_error": (I, []),
    "b2d_version": (I, []),
    "b2d_launch_counter": (C.c_longlong, []),
    "b2d_gemv_f32": (I, [P, P, P, I, I, P]),
    "b2d_gemv": (I, [I, P, P, P, P, I, P, I, P, Fl, I, I, P, I, P, I, I, I, P]),
    "b2d_gemv_mma_formats": (I, [I]),
    "b2d_rmsnorm_gemv_f16": (I, [P, P, P, Fl, P, I, I, I, I, P, P, P]),
    "b2d_gemv_q8_32": (I, [P, P, P, P, I, I, I, P]),
    "b2d_gemv_q4_32": (I, [P, P, P, P, I, I, I, P]),
    "b2d_dequant_q8_32": (I, [P, P, P, I, I, P]),
    "b2d_dequant_q4_32": (I, [P, P, P, I, I, P]),
    "b2d_lm_head_argmax_workspace_bytes": (Z, [I, I]),
    "b2d_lm_head_argmax": (I, [P, P, I, P, Fl, I, I, I, I, P, P, P, P, Z, P]),
    "b2d_rmsnorm": (I, [P, P, P, I, I, Fl, P]),
    "b2d_add_rmsnorm_f16": (I, [P, P, P, Fl, P, I, I, P]),
    "b2d_embed_rmsnorm_f16": (I, [P, P, P, P, Fl, P, I, I, P]),
    "b2d_gemm_tc_workspace_bytes": (Z, [I, I, I, I]),
    "b2d_gemm_tc": (I, [P, P, P, I, I, I, P, I, P, I, I, I, P, P, P, I, P, Z, P]),
    "b2d_gemm_tc_q": (I, [I, P, P, P, I, I, I, P, I, P, I, I, I, P, Z, P]),
    "b2d_gemm_tc_ex": (I, [I, P, P, P, I, I, I, P, I, P, I, I, I, P, P, P, I, P, Z, P]),
    "b2d_gemm_tc_q_ex": (I, [I, I, P, P, P, I, I, I, P, I, P, I, I, I, P, Z, P]),
    "b2d_add_rmsnorm": (I, [P, P, P, Fl, I, P, I, I, P]),
    "b2d_tc_packed_bytes": (Z, [I, I]),
    "b2d_tc_pack_f16": (I, [P, I, I, I, P, P]),
    "b2d_gemm_tc_packed": (I, [P, P, P, I, I, I, P, I, P, I, I, I, P, P, P, I, P, Z, P]),
    "b2d_embed_f16": (I, [P, P, P, I, I, P]),
    "b2d_argmax_f32": (I, [P, I, I, P, I, P]),
    "b2d_argmax_combine": (I, [P, P, I, I, P, P]),
    "b2d_add_f32": (I, [P, P, Z, P]),
    "b2d_inv_freq": (I, [I, D, P]),
    "b2d_rope_kv_append": (I, [P, I, I, P, P, P, I, I, P, P, I, I, I, I, P]),
    "b2d_attn_chunk_tokens": (I, [I, I, I]),
    "b2d_paged_attn_workspace_bytes": (Z, [I, I, I, I, I]),
    "b2d_paged_decode_attn": (
        I,
        [P, I, I, P, P, P, I, I, P, P, I, I, I, I, I, Fl, I, I, P, I, I, P, Z, P],
    ),
    "b2d_paged_decode_attn_noalloc_max_scratch_bytes": (Z, []),
    "b2d_paged_decode_attn_noalloc_error": (I, []),
    "b2d_paged_decode_attn_noalloc": (
        I,
        [P, I, I, P, P, P, I, I, P, P, I, I, I, I, I, Fl, I, I, P, I, I, P],
    ),
    "b2d_nccl_unique_id_bytes": (I, []),
    "b2d_nccl_get_unique_id": (I, [P]),
    "b2d_decoder_create": (I, [C.POINTER(ModelConfig), I, I, P, C.POINTER(P)]),
    "b2d_decoder_destroy": (I, [P]),
    "b2d_decoder_set_layer": (I, [P, I, P, P, P, P, P, P, P, P, P]),
    "b2d_decoder_set_layer_q": (I, [P, I, I, P, P, P, P, P, P, P, P, P, P, P, P, P, P]),
    "b2d_decoder_set_head": (I, [P, P, P, I, P]),
    "b2d_decoder_step": (I, [P, P, P, P, I, P, P, I, P]),
    "b2d_decoder_peer_collectives": (I, [P]),
    "b2d_decoder_generate": (I, [P, P, P, P, I, I, P, I, P, P]),
    "b2d_decoder_prefill": (I, [P, P, I, P, I, P, P, P]),
    "b2d_decoder_set_inv_freq": (I, [P, P, I]),
    "b2d_decoder_error": (I, [P]),
    "b2d_tp_allreduce_add_rmsnorm": (I, [P, P, P, I, I, I, P, P, Fl, P, I, I, C.c_longlong, P, P]),
    "b2d_tp_argmax_gather": (I, [P, P, P, P, I, I, I, I, P, C.c_longlong, P, P]),
}

_lib = None
_lock = threading.Lock()


class B2DError(RuntimeError):
    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn}: {msg} (status {status})")
        self.status = status


def lib() -> C.CDLL:
    """Load the library once; raise if it is missing (no fallback path exists)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run "
                    "`python -m gemmagemini4hackathon2026_10_2425_b200.build`"
                )
            h = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                f = getattr(h, name)
                f.restype = res
                f.argtypes = args
            _lib = h
        return _lib


def call(name: str, *args) -> int:
    """Call an entry point; translate a non-zero status into ValueError / RuntimeError."""
    st = getattr(lib(), name)(*args)
    if st != OK:
        msg = lib().b2d_status_string(st).decode()
        if st == ERR_CUDA:
            msg += f" (cudaError {lib().b2d_last_cuda_error()})"
        if st in (ERR_NULL, ERR_SHAPE, ERR_ALIGN, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_STATE):
            raise ValueError(f"{name}: {msg} (status {st})")
        raise B2DError(name, st, msg)
    return st


def declared_symbols() -> list[str]:
    """Every function name declared in include/b200dec.h."""
    import re

    text = HEADER.read_text()
    return sorted(set(re.findall(r"^B2D_API [^(]*?\b(b2d_\w+)\(", text, flags=re.M)))
