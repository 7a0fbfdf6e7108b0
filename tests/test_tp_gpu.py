"""Tensor-parallel decode step on 2, 4 and 8 GPUs against the single-GPU oracle.

Each world size runs only where that many GPUs are visible; each rank is a spawned process that builds its
DecodeEngine shard, runs one step (CUDA-core path at batch 5, tensor-core path at batch 24),
with the peer-memory collectives and with NCCL (B2D_TP_COLLECTIVE=nccl),
and sends its vocab-shard logits and the combined next tokens back to the test.  A q8_32 case
shards quantized projections (rows of the column-parallel ones, 32-element K blocks of the
row-parallel ones) and checks them against the oracle fed the weights the tcgen05 path
multiplies, fp16(scale * q).
"""

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _rendezvous() -> str:
    """A file rendezvous for the spawned ranks (no TCP port to race for between tests)."""
    import tempfile

    fd, path = tempfile.mkstemp(prefix="b2d_tp_rdzv_")
    os.close(fd)
    os.unlink(path)  # the store creates it
    return "file://" + path


def _case(batch):
    from gemmagemini4hackathon2026_10_2425_b200.engine import make_block_table
    from oracle import step as S

    cfg = S.ModelConfig(2048, 2, 32, 8, 64, 8192, 4096, 1e-5, 500000.0)
    w = S.synth_weights(cfg, seed=21)
    r = np.random.default_rng(22 + batch)
    lens = r.integers(0, 900, size=batch).tolist()
    max_ctx = 1024
    nblk = sum(-(-(n + 1) // 16) for n in lens) + 4
    table = make_block_table(lens, max_ctx // 16, nblk, seed=23).numpy()
    shape = (nblk, cfg.n_kv_heads, 16, cfg.head_dim)
    kp = [r.standard_normal(shape).astype(np.float16) for _ in range(cfg.n_layers)]
    vp = [r.standard_normal(shape).astype(np.float16) for _ in range(cfg.n_layers)]
    tokens = r.integers(0, cfg.vocab, size=batch).tolist()
    return cfg, w, lens, max_ctx, nblk, table, kp, vp, tokens


def _quantized(w, cfg, fmt):
    """(stored tensors, quant map, fp16(scale * q) weights) with every projection quantized."""
    from gemmagemini4hackathon2026_10_2425_b200 import weights as W

    stored, quant, rounded = dict(w), {}, dict(w)
    for i in range(cfg.n_layers):
        for n in ("wqkv", "wo", "wgate", "wup", "wdown"):
            name = f"l{i}.{n}"
            qv, sc = W.quantize(w[name], fmt)
            stored[name], stored[name + ".scales"], quant[name] = qv, sc, fmt
            rounded[name] = W.dequantize(qv, sc, fmt).astype(np.float16)
    return stored, quant, rounded


def _rank(rank, world, rdzv, batch, collective, q, fmt=None):
    import torch.distributed as dist
    from datetime import timedelta

    from gemmagemini4hackathon2026_10_2425_b200.engine import DecodeEngine, share_nccl_id
    from gemmagemini4hackathon2026_10_2425_b200.tp import ModelShape

    os.environ.update(B2D_TP_COLLECTIVE=collective)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=rdzv, rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    try:
        cfg, w, lens, max_ctx, nblk, table, kp, vp, tokens = _case(batch)
        shape = ModelShape(cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab, cfg.eps, cfg.theta)
        eng = DecodeEngine(shape, max_batch=batch, max_ctx=max_ctx, n_blocks=nblk, tp_rank=rank, tp_size=world, nccl_id=share_nccl_id(rank), device=dev)
        eng.alloc_kv()
        hk = cfg.n_kv_heads // world
        for i in range(cfg.n_layers):  # this rank's KV heads
            eng.k_pages[i].copy_(torch.from_numpy(np.ascontiguousarray(kp[i][:, rank * hk : (rank + 1) * hk])))
            eng.v_pages[i].copy_(torch.from_numpy(np.ascontiguousarray(vp[i][:, rank * hk : (rank + 1) * hk])))
        if fmt:
            stored, quant, _ = _quantized(w, cfg, fmt)
            eng.load_weights({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in stored.items()}, quant)
        else:
            eng.load_weights({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in w.items()})
        i32 = lambda a: torch.tensor(np.asarray(a, np.int32), device=dev)
        tok, ln, tb = i32(tokens), i32(lens), torch.from_numpy(table).to(dev)
        nxt = torch.empty_like(tok)
        logits = torch.empty(batch, eng.lm_rows, dtype=torch.float32, device=dev)
        eng.step(tok, ln, tb, nxt, logits, use_graph=True)
        eng.step(tok, ln, tb, nxt, logits, use_graph=True)  # replay
        eng.stream.synchronize()
        eng.check()  # no peer barrier timed out
        q.put((rank, logits.cpu().numpy(), nxt.cpu().numpy(), eng.peer_collectives()))
        eng.close()
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize(
    "world",
    [pytest.param(w, marks=pytest.mark.skipif(torch.cuda.device_count() < w, reason=f"needs {w} GPUs")) for w in (2, 4, 8)],
)
@pytest.mark.parametrize(
    "collective,batch,fmt",
    [("peer", 5, None), ("peer", 24, None), ("nccl", 5, None), ("nccl", 24, None), ("peer", 24, "q8_32")],
)
@pytest.mark.timeout(600)
def test_tp_decode_step_matches_oracle(batch, collective, fmt, world):
    from oracle import step as S
    from tests._tol import assert_norm_close

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rdzv = _rendezvous()
    procs = [ctx.Process(target=_rank, args=(r, world, rdzv, batch, collective, q, fmt)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        rank, lg, nx, peer = q.get(timeout=500)
        got[rank] = (lg, nx)
        assert peer == (collective == "peer")  # the path asked for is the path that ran
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    cfg, w, lens, max_ctx, nblk, table, kp, vp, tokens = _case(batch)
    if fmt:
        w = _quantized(w, cfg, fmt)[2]
    ref_logits, ref_next = S.decode_step(w, cfg, tokens, lens, table, kp, vp)
    logits = np.concatenate([got[r][0] for r in range(world)], axis=1)
    assert_norm_close(logits, ref_logits, 2e-3, what=f"tp{world} logits b{batch}")
    for r in range(1, world):
        np.testing.assert_array_equal(got[0][1], got[r][1])  # every rank agrees on the tokens
    np.testing.assert_array_equal(got[0][1], np.argmax(logits, axis=1))


def _prefill_rank(rank, world, rdzv, q):
    """One rank of a tensor-parallel prefill: 40 prompt tokens (a 32-row tensor-core chunk and an
    8-row CUDA-core chunk), then the last position's logits shard."""
    import torch.distributed as dist
    from datetime import timedelta

    from gemmagemini4hackathon2026_10_2425_b200.engine import DecodeEngine, share_nccl_id
    from gemmagemini4hackathon2026_10_2425_b200.tp import ModelShape

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=rdzv, rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    try:
        cfg, w, ids, table_row = _prefill_case()
        shape = ModelShape(cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab, cfg.eps, cfg.theta)
        eng = DecodeEngine(shape, max_batch=32, max_ctx=128, n_blocks=8, tp_rank=rank, tp_size=world, nccl_id=share_nccl_id(rank), device=dev)
        eng.alloc_kv()
        eng.load_weights({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in w.items()})
        ids_d = torch.tensor(np.asarray(ids, np.int32), device=dev)
        tb = torch.from_numpy(table_row).to(dev)
        logits = torch.empty(eng.lm_rows, dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        nxt = eng.prefill(ids_d, tb, 0, logits=logits)
        eng.stream.synchronize()
        eng.check()
        q.put((rank, logits.cpu().numpy(), int(nxt.item())))
        eng.close()
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


def _prefill_case():
    from oracle import step as S

    # 16 / 8 heads: at TP8 each rank holds 2 query heads and 1 KV head (256 QKV rows)
    cfg = S.ModelConfig(512, 2, 16, 8, 64, 2048, 2048, 1e-5, 500000.0)
    w = S.synth_weights(cfg, seed=41)
    ids = np.random.default_rng(42).integers(0, cfg.vocab, size=40).tolist()
    return cfg, w, ids, np.arange(8, dtype=np.int32)


@pytest.mark.parametrize(
    "world",
    [pytest.param(w, marks=pytest.mark.skipif(torch.cuda.device_count() < w, reason=f"needs {w} GPUs")) for w in (2, 8)],
)
@pytest.mark.timeout(600)
def test_tp_prefill_matches_oracle(world):
    """b2d_decoder_prefill is collective: every rank prefills its heads' K/V and shard of the
    model; the concatenated last-position logits match the oracle run token by token."""
    from oracle import step as S
    from tests._tol import assert_norm_close

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rdzv = _rendezvous()
    procs = [ctx.Process(target=_prefill_rank, args=(r, world, rdzv, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        rank, lg, nx = q.get(timeout=500)
        got[rank] = (lg, nx)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    cfg, w, ids, table_row = _prefill_case()
    shape = (8, cfg.n_kv_heads, 16, cfg.head_dim)
    kp = [np.zeros(shape, np.float16) for _ in range(cfg.n_layers)]
    vp = [np.zeros(shape, np.float16) for _ in range(cfg.n_layers)]
    ref = None
    for i, t in enumerate(ids):
        ref, _ = S.decode_step(w, cfg, [t], [i], table_row[None, :], kp, vp)
    logits = np.concatenate([got[r][0] for r in range(world)])
    assert_norm_close(logits, ref[0], 2e-3, what=f"tp{world} prefill logits")
    for r in range(1, world):
        assert got[r][1] == got[0][1]  # every rank agrees on the next token
    assert got[0][1] == int(np.argmax(logits))
