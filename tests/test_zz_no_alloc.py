"""The allocation-free attention entry point against the workspace one, through the C ABI.

b2d_paged_decode_attn_noalloc exists for callers that cannot allocate device memory (code
inside another framework's memory pool, plugins whose host forbids cudaMalloc after start-up):
it keeps its split-K scratch in a fixed device array inside the library.  This test calls it
twice in a row, on different ragged batches, and checks each result against
b2d_paged_decode_attn with a caller-provided workspace on identical copies of the inputs.  The
allocation-free calls run on a side stream of their own (PyTorch creates non-blocking streams,
which do not wait for the legacy default stream), and after each one the error query reports
that no device-side wait gave up.  The file is named so that pytest collects it last; it also
passes alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from gemmagemini4hackathon2026_10_2425_b200 import _lib
from oracle import ops as O
from tests._tol import assert_rel_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(lens, hq, hk, hd, seed):
    r = np.random.default_rng(seed)
    B = len(lens)
    max_ctx = max(lens) + 1
    max_blocks = -(-max_ctx // 16)
    need = [-(-(n + 1) // 16) for n in lens]
    nblk = sum(need) + 3
    perm = r.permutation(nblk)
    table = np.full((B, max_blocks), -1, np.int32)
    o = 0
    for b, k in enumerate(need):
        table[b, :k] = perm[o : o + k]
        o += k
    kp = r.standard_normal((nblk, hk, 16, hd)).astype(np.float16)
    vp = r.standard_normal((nblk, hk, 16, hd)).astype(np.float16)
    qkv = r.standard_normal((B, (hq + 2 * hk) * hd)).astype(np.float32)
    return dict(kp=kp, vp=vp, qkv=qkv, table=table, lens=np.array(lens, np.int32), max_ctx=max_ctx)


def _call(c, hq, hk, hd, theta, noalloc: bool, stream=None):
    """One call through the C ABI on fresh device copies; returns (out, k_pages, v_pages)."""
    lib = _lib.lib()
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    qkv, kp, vp, table, lens = d(c["qkv"]), d(c["kp"]), d(c["vp"]), d(c["table"]), d(c["lens"])
    invf = d(O.inv_freq(hd, theta))
    B = qkv.shape[0]
    out = torch.full((B, hq * hd), float("nan"), dtype=torch.float32, device=DEV)
    torch.cuda.synchronize()  # inputs copied before a call on another stream reads them
    stream = (stream or torch.cuda.current_stream()).cuda_stream
    common = (
        qkv.data_ptr(), _lib.F32, qkv.shape[1], kp.data_ptr(), vp.data_ptr(), table.data_ptr(),
        table.shape[1], kp.shape[0], lens.data_ptr(), invf.data_ptr(), hq, hk, hd, B,
        c["max_ctx"], 0.0, 0, 1, out.data_ptr(), _lib.F32, out.shape[1],
    )
    if noalloc:
        st = lib.b2d_paged_decode_attn_noalloc(*common, stream)
        assert st == _lib.OK, lib.b2d_status_string(st)
        st = lib.b2d_paged_decode_attn_noalloc_error()
    else:
        nbytes = lib.b2d_paged_attn_workspace_bytes(B, hq, hk, hd, c["max_ctx"])
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
        st = lib.b2d_paged_decode_attn(*common, ws.data_ptr(), ctypes.c_size_t(nbytes), stream)
    assert st == _lib.OK, lib.b2d_status_string(st)
    torch.cuda.synchronize()
    return out.cpu().numpy(), kp.cpu().numpy(), vp.cpu().numpy()


def test_noalloc_matches_workspace_entry_twice():
    hq, hk, hd, theta = 32, 8, 128, 10000.0
    cases = [
        _case([1500, 17, 4095, 300, 0], hq, hk, hd, seed=1),  # several split-K chunks
        _case([40, 2000, 999], hq, hk, hd, seed=2),  # a second, different call
    ]
    side = torch.cuda.Stream()
    for c in cases:
        a, ka, va = _call(c, hq, hk, hd, theta, noalloc=True, stream=side)
        b, kb, vb = _call(c, hq, hk, hd, theta, noalloc=False)
        assert np.all(np.isfinite(a))
        assert_rel_close(a, b, 2e-3, what="noalloc vs workspace entry point")
        np.testing.assert_array_equal(ka.view(np.uint16), kb.view(np.uint16))
        np.testing.assert_array_equal(va.view(np.uint16), vb.view(np.uint16))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.lib()
    cap = lib.b2d_paged_decode_attn_noalloc_max_scratch_bytes()
    assert cap == 16 << 20
    # 256 sequences x 32 KV heads x 64k context needs far more than the fixed scratch
    assert lib.b2d_paged_attn_workspace_bytes(256, 32, 32, 128, 65536) > cap
    dummy = torch.zeros(16, dtype=torch.float32, device=DEV)
    p = dummy.data_ptr()
    st = lib.b2d_paged_decode_attn_noalloc(
        p, _lib.F32, 12288, p, p, p, 4096, 1, p, p, 32, 32, 128, 256, 65536, 0.0, 0, 1, p,
        _lib.F32, 4096, torch.cuda.current_stream().cuda_stream,
    )
    assert st == _lib.ERR_WORKSPACE
