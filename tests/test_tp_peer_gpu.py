"""Peer-memory tensor-parallel collectives on one GPU.

The ranks' buffers are all local here, and every other rank's barrier arrival is written into
the signal array by the host before the launch (as if the peers had already announced their
partials), so no kernel ever waits on another kernel.  The timeout test leaves one arrival
unset: the bounded wait must give up, report B2D_ERR_TIMEOUT through the error word, leave the
row unchanged and keep the context usable.  The 2-GPU decode-step test covers the real
cross-process path.
"""

import numpy as np
import pytest
import torch

from gemmagemini4hackathon2026_10_2425_b200 import _lib, ops
from oracle import ops as O
from tests._tol import assert_rel_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
SIG_STRIDE = 8  # signal words per slot (one per source rank)


def _arrive(sig, slot0, rows, ranks, epoch):
    """Host-side stand-in for the peers' announcements of `epoch` on rows [slot0, slot0+rows)."""
    s = sig.view(-1, SIG_STRIDE)
    for r in ranks:
        s[slot0 : slot0 + rows, r] = epoch


@pytest.mark.parametrize("tp,rank", [(2, 0), (3, 2), (8, 5)])
def test_allreduce_add_rmsnorm_sums_in_rank_order(tp, rank):
    rows, D, slot0 = 5, 2048, 3
    r = np.random.default_rng(tp * 10 + rank)
    parts_np = [r.standard_normal((rows, D)).astype(np.float32) for _ in range(tp)]
    x_np = r.standard_normal((rows, D)).astype(np.float32)
    g_np = (1 + 0.1 * r.standard_normal(D)).astype(np.float32)
    parts = [torch.from_numpy(p).to(DEV) for p in parts_np]
    sig = torch.zeros((slot0 + rows) * SIG_STRIDE, dtype=torch.int32, device=DEV)
    epochs = torch.zeros(slot0 + rows, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    x = torch.from_numpy(x_np.copy()).to(DEV)
    g = torch.from_numpy(g_np).to(DEV)
    others = [q for q in range(tp) if q != rank]
    for it in (1, 2):  # two uses: the epochs advance per slot
        _arrive(sig, slot0, rows, others, it)
        out = ops.tp_allreduce_add_rmsnorm(parts, [sig] * tp, epochs, rank, x, err, gamma=g, eps=1e-5, slot0=slot0)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        s = parts_np[0].copy()
        for p in parts_np[1:]:
            s += p
        x_np = x_np + s  # float32, same order as the kernel -> bit-identical
        np.testing.assert_array_equal(x.cpu().numpy(), x_np)
        assert_rel_close(out.float().cpu().numpy(), O.rmsnorm(x_np, g_np, 1e-5), 2e-3)
        sv = sig.view(-1, SIG_STRIDE).cpu().numpy()
        assert (sv[slot0 : slot0 + rows, rank] == it).all()  # this rank announced its rows
        assert (epochs.cpu().numpy()[slot0:] == it).all()


def test_allreduce_without_norm_only_adds():
    tp, rank, rows, D = 2, 1, 3, 64
    parts = [torch.randn(rows, D, device=DEV) for _ in range(tp)]
    sig = torch.zeros(rows * SIG_STRIDE, dtype=torch.int32, device=DEV)
    epochs = torch.zeros(rows, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    x = torch.randn(rows, D, device=DEV)
    want = x + (parts[0] + parts[1])
    _arrive(sig, 0, rows, [0], 1)
    assert ops.tp_allreduce_add_rmsnorm(parts, [sig, sig], epochs, rank, x, err) is None
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    torch.testing.assert_close(x, want, rtol=0, atol=0)


def test_barrier_timeout_reports_error_and_context_survives():
    """A peer that never arrives: the bounded wait ends with B2D_ERR_TIMEOUT, x is untouched."""
    tp, rank, rows, D = 2, 0, 4, 256
    parts = [torch.randn(rows, D, device=DEV) for _ in range(tp)]
    sig = torch.zeros(rows * SIG_STRIDE, dtype=torch.int32, device=DEV)
    epochs = torch.zeros(rows, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    x = torch.randn(rows, D, device=DEV)
    x0 = x.clone()
    _arrive(sig, 0, rows - 1, [1], 1)  # the peer announced rows 0..rows-2 only
    ops.tp_allreduce_add_rmsnorm(parts, [sig, sig], epochs, rank, x, err, timeout_ns=20_000_000)
    torch.cuda.synchronize()
    assert int(err.item()) == _lib.ERR_TIMEOUT
    torch.testing.assert_close(x[rows - 1], x0[rows - 1], rtol=0, atol=0)  # the row that timed out
    torch.testing.assert_close(x[: rows - 1], x0[: rows - 1] + parts[0][: rows - 1] + parts[1][: rows - 1])
    # the context is still usable
    y = ops.gemm_tc(torch.ones(128, 64, dtype=torch.float16, device=DEV), torch.ones(16, 64, dtype=torch.float16, device=DEV))
    assert float(y[0, 0]) == 64.0


def test_argmax_gather_ties_lowest_index():
    tp, rank, B, slot = 4, 2, 37, 40
    r = np.random.default_rng(4)
    vals = r.standard_normal((tp, B)).astype(np.float32)
    idxs = (np.arange(tp)[:, None] * 1000 + r.integers(0, 1000, size=(tp, B))).astype(np.int32)
    vals[:, 0] = 10.0  # all ranks tie on token 0: lowest index wins
    idxs[:, 0] = [3500, 2100, 1700, 900]
    sig = torch.zeros((slot + 1) * SIG_STRIDE, dtype=torch.int32, device=DEV)
    epochs = torch.zeros(slot + 1, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    _arrive(sig, slot, 1, [q for q in range(tp) if q != rank], 1)
    tv = [torch.from_numpy(v).to(DEV) for v in vals]
    ti = [torch.from_numpy(i).to(DEV) for i in idxs]
    tok = ops.tp_argmax_gather(tv, ti, [sig] * tp, epochs, rank, slot, err).cpu().numpy()
    assert int(err.item()) == 0
    best = np.argmax(vals, axis=0)
    want = idxs[best, np.arange(B)]
    want[0] = 900
    np.testing.assert_array_equal(tok, want)


def test_bad_arguments_raise():
    x = torch.zeros(2, 6, device=DEV)  # D % 4 != 0
    z = torch.zeros(16, dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError):
        ops.tp_allreduce_add_rmsnorm([x, x], [z, z], z, 0, x, z)
    x = torch.zeros(2, 8, device=DEV)
    with pytest.raises(ValueError):  # tp > 8
        ops.tp_allreduce_add_rmsnorm([x] * 9, [z] * 9, z, 0, x, z)
