"""Parity of paged decode attention (RoPE + KV append + split-K GQA) with the CPU oracle.

fp16 path tolerance 2e-3 (elementwise with floor); KV page placement bit-exact for V, K within
one fp16 ulp (RoPE's cos/sin differ from the float64 oracle by ~1 fp32 ulp, which can flip a
rounding), untouched slots bit-identical to their sentinel.
"""

import numpy as np
import pytest
import torch

from gemmagemini4hackathon2026_10_2425_b200 import ops
from oracle import ops as O
from tests._tol import assert_rel_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
SENTINEL = np.float16(-3.25)


def make_case(lens, hq, hk, hd, seed, qkv_dtype=np.float32, extra_blocks=5):
    r = np.random.default_rng(seed)
    B = len(lens)
    max_ctx = max(lens) + 1
    max_blocks = -(-max_ctx // 16)
    need = [-(-(n + 1) // 16) for n in lens]
    nblk = sum(need) + extra_blocks
    perm = r.permutation(nblk)
    table = np.full((B, max_blocks), -1, np.int32)
    o = 0
    for b, k in enumerate(need):
        table[b, :k] = perm[o : o + k]
        o += k
    kp = np.full((nblk, hk, 16, hd), SENTINEL, np.float16)
    vp = np.full((nblk, hk, 16, hd), SENTINEL, np.float16)
    for b, n in enumerate(lens):  # cached tokens 0..n-1 get random values
        for pos in range(n):
            blk, slot = O.page_slot(table, b, pos)
            kp[blk, :, slot] = r.standard_normal((hk, hd)).astype(np.float16)
            vp[blk, :, slot] = r.standard_normal((hk, hd)).astype(np.float16)
    qkv = r.standard_normal((B, (hq + 2 * hk) * hd)).astype(np.float16).astype(qkv_dtype)
    return dict(table=table, kp=kp, vp=vp, qkv=qkv, lens=np.array(lens, np.int32), max_ctx=max_ctx)


def run_gpu(c, hq, hk, hd, theta, window=0, append=True, out_dtype=torch.float32, max_ctx=None):
    invf = O.inv_freq(hd, theta)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    kp, vp = dev(c["kp"]), dev(c["vp"])
    out = ops.paged_decode_attn(
        dev(c["qkv"]),
        kp,
        vp,
        dev(c["table"]),
        dev(c["lens"]),
        dev(invf),
        hq,
        hk,
        hd,
        max_ctx or c["max_ctx"],
        window=window,
        append=append,
        out_dtype=out_dtype,
    )
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), kp.cpu().numpy(), vp.cpu().numpy()


def run_oracle(c, hq, hk, hd, theta, window=0, append=True):
    kp, vp = c["kp"].copy(), c["vp"].copy()
    out = O.paged_decode_attention(
        c["qkv"], kp, vp, c["table"], c["lens"], hq, hk, hd, O.inv_freq(hd, theta), window=window, append=append
    )
    return out, kp, vp


def check_pages(gk, gv, rk, rv):
    np.testing.assert_array_equal(gv.view(np.uint16), rv.view(np.uint16))  # placement + values
    diff = np.abs(gk.view(np.uint16).astype(np.int32) - rk.view(np.uint16).astype(np.int32))
    assert diff.max() <= 1, "K differs by more than one fp16 ulp"
    assert (diff > 0).mean() < 0.01


@pytest.mark.parametrize(
    "lens",
    [
        [0],  # empty cache: attend to the appended token only
        [15, 16, 17, 1],  # page boundaries
        [31, 500, 1023, 64],
        [4095, 100, 2048],  # several split-K chunks
    ],
)
@pytest.mark.parametrize("hd,hq,hk", [(128, 32, 8), (64, 32, 8), (64, 8, 8), (128, 8, 1), (256, 8, 1)])
def test_paged_attention_matches_oracle(lens, hd, hq, hk):
    theta = 10000.0 if hd == 128 else 500000.0
    c = make_case(lens, hq, hk, hd, seed=sum(lens) + hd + hq)
    go, gk, gv = run_gpu(c, hq, hk, hd, theta)
    ro, rk, rv = run_oracle(c, hq, hk, hd, theta)
    assert_rel_close(go, ro, 2e-3, what=f"out {lens}")
    check_pages(gk, gv, rk, rv)


def test_config4_like_ragged_batch():
    """BASELINE config 4 shape (32/8 heads, HD 128, theta 1e4, 16-token pages, random block
    table) with a smaller batch so the float64 oracle stays fast."""
    r = np.random.default_rng(44)
    lens = r.integers(128, 8193, size=6).tolist()
    c = make_case(lens, 32, 8, 128, seed=45)
    go, gk, gv = run_gpu(c, 32, 8, 128, 10000.0)
    ro, rk, rv = run_oracle(c, 32, 8, 128, 10000.0)
    assert_rel_close(go, ro, 2e-3)
    check_pages(gk, gv, rk, rv)


@pytest.mark.parametrize("window", [1, 16, 100, 5000])
def test_sliding_window(window):
    c = make_case([300, 2000, 50], 8, 2, 128, seed=window)
    go, _, _ = run_gpu(c, 8, 2, 128, 10000.0, window=window)
    ro, _, _ = run_oracle(c, 8, 2, 128, 10000.0, window=window)
    assert_rel_close(go, ro, 2e-3)


def test_fp16_qkv_and_fp16_out():
    c = make_case([200, 33], 16, 4, 64, seed=3, qkv_dtype=np.float16)
    go, gk, gv = run_gpu(c, 16, 4, 64, 500000.0, out_dtype=torch.float16)
    ro, rk, rv = run_oracle(c, 16, 4, 64, 500000.0)
    assert_rel_close(go, ro, 2e-3)
    check_pages(gk, gv, rk, rv)


def test_no_append_then_rope_kv_append():
    """append=0 reads a cache the standalone rope_kv_append kernel filled: same result."""
    hq, hk, hd, theta = 8, 2, 64, 500000.0
    c = make_case([40, 77, 0], hq, hk, hd, seed=8)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    qkv, kp, vp = dev(c["qkv"]), dev(c["kp"]), dev(c["vp"])
    table, lens, invf = dev(c["table"]), dev(c["lens"]), dev(O.inv_freq(hd, theta))
    ops.rope_kv_append(qkv, kp, vp, table, lens, invf, hq, hk, hd)
    out = ops.paged_decode_attn(qkv, kp, vp, table, lens, None, hq, hk, hd, c["max_ctx"], append=False)
    ro, rk, rv = run_oracle(c, hq, hk, hd, theta)
    assert_rel_close(out.cpu().numpy(), ro, 2e-3)
    check_pages(kp.cpu().numpy(), vp.cpu().numpy(), rk, rv)
    # q was rotated in place, as the reference's rope_kv does (LK/kernels.metal:214-216)
    q = c["qkv"][:, : hq * hd].reshape(3, hq, hd)
    rq = O.rope(q, c["lens"][:, None], O.inv_freq(hd, theta)).reshape(3, -1)
    assert_rel_close(qkv[:, : hq * hd].cpu().numpy(), rq, 1e-5)


def test_workspace_is_reusable_across_calls():
    """The arrival counters return to zero: back-to-back calls give identical results."""
    c = make_case([1500, 900, 3000], 32, 8, 128, seed=12)
    a, _, _ = run_gpu(c, 32, 8, 128, 10000.0)
    b, _, _ = run_gpu(c, 32, 8, 128, 10000.0)
    np.testing.assert_array_equal(a, b)


def test_out_of_pool_block_ids_are_skipped():
    """Block-table entries outside [0, n_blocks) are never dereferenced."""
    c = make_case([40], 8, 2, 64, seed=2)
    c["table"][0, 1] = 10**6  # second page: tokens 16..31 become invisible
    go, _, _ = run_gpu(c, 8, 2, 64, 500000.0)
    assert np.all(np.isfinite(go))


def test_workspace_shared_across_batch_shapes():
    """Calls with different (batch, KV heads) share one workspace: counters and partials live
    in fixed, separate regions."""
    ws = torch.zeros(ops.attn_workspace_bytes(40, 32, 8, 128, 4100), dtype=torch.uint8, device=DEV)
    for lens, hq, hk in [([300, 4000], 32, 8), ([3000] * 40, 32, 8), ([50, 2100, 900], 8, 2)]:
        c = make_case(lens, hq, hk, 128, seed=len(lens) * 7 + hk)
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
        out = ops.paged_decode_attn(
            dev(c["qkv"]), dev(c["kp"]), dev(c["vp"]), dev(c["table"]), dev(c["lens"]),
            dev(O.inv_freq(128, 10000.0)), hq, hk, 128, c["max_ctx"], workspace=ws,
        )
        ro, _, _ = run_oracle(c, hq, hk, 128, 10000.0)
        assert_rel_close(out.cpu().numpy(), ro, 2e-3)


def test_large_batch_many_short_sequences():
    """300 short sequences (one chunk each, most CTAs of the grid idle): same results."""
    r = np.random.default_rng(300)
    lens = r.integers(0, 40, size=300).tolist()
    c = make_case(lens, 32, 8, 64, seed=301, extra_blocks=2)
    go, gk, gv = run_gpu(c, 32, 8, 64, 500000.0)
    ro, rk, rv = run_oracle(c, 32, 8, 64, 500000.0)
    assert_rel_close(go, ro, 2e-3)
    check_pages(gk, gv, rk, rv)


def test_long_chunks_of_1024_keys():
    """40 sequences of 2000-3500 tokens: the chunk heuristic picks 1024-key chunks (the largest),
    so each CTA's page list is the longest the kernel supports."""
    from gemmagemini4hackathon2026_10_2425_b200 import _lib

    r = np.random.default_rng(1024)
    lens = r.integers(2000, 3500, size=40).tolist()
    assert _lib.lib().b2d_attn_chunk_tokens(40, 8, max(lens) + 1) == 1024
    c = make_case(lens, 32, 8, 64, seed=1025, extra_blocks=3)
    go, gk, gv = run_gpu(c, 32, 8, 64, 500000.0)
    ro, rk, rv = run_oracle(c, 32, 8, 64, 500000.0)
    assert_rel_close(go, ro, 2e-3)
    check_pages(gk, gv, rk, rv)
