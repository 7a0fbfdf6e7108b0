"""Tensor-parallel host logic on CPU: 2 gloo ranks shard the tiny golden Llama with the
product's sharding (gemmagemini4hackathon2026_10_2425_b200.tp), run the step's math on their
shards, exchange partial sums exactly where the CUDA path does (all-reduce after O and down,
all-gather of the LM head's (max, index) pairs) and must reproduce the unsharded oracle."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gemmagemini4hackathon2026_10_2425_b200 import tp as T
from oracle import ops as O
from oracle import step as S


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, golden_path, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tests.test_oracle_golden import _tiny_cfg, _tiny_weights, build_paged_cache

        g = dict(np.load(golden_path))
        cfg = _tiny_cfg(g)
        w = _tiny_weights(g, cfg)
        shape = T.ModelShape(cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab, cfg.eps, cfg.theta)
        lens, table, kp, vp = build_paged_cache(g, cfg, np.float16)
        tokens = [int(g[f"llm_s{b}_ids"][-1]) for b in range(len(lens))]
        hq, hk, hd = cfg.n_heads // world, cfg.n_kv_heads // world, cfg.head_dim
        invf = O.inv_freq(hd, cfg.theta)
        x = O.embed(w["embed"], tokens)
        for i in range(cfg.n_layers):
            full = {n: torch.from_numpy(np.asarray(w[f"l{i}.{n}"])) for n in ("attn_norm", "wqkv", "wo", "ffn_norm", "wgate", "wup", "wdown")}
            sh = {k: v.numpy() for k, v in T.shard_layer(full, shape, rank, world).items()}
            qkv = O.gemv(sh["wqkv"], O.rmsnorm(x, sh["attn_norm"], cfg.eps))
            kl = np.ascontiguousarray(kp[i][:, rank * hk : (rank + 1) * hk])
            vl = np.ascontiguousarray(vp[i][:, rank * hk : (rank + 1) * hk])
            att = O.paged_decode_attention(qkv, kl, vl, table, lens, hq, hk, hd, invf)
            part = torch.from_numpy(O.gemv(sh["wo"], att))
            dist.all_reduce(part)  # the all-reduce after the row-parallel O projection
            x = x + part.numpy()
            xn = O.rmsnorm(x, sh["ffn_norm"], cfg.eps)
            h = O.swiglu(O.gemv(sh["wgate"], xn), O.gemv(sh["wup"], xn))
            part = torch.from_numpy(O.gemv(sh["wdown"], h))
            dist.all_reduce(part)  # after the row-parallel down projection
            x = x + part.numpy()
        head = T.shard_head(torch.from_numpy(np.asarray(w["embed"])), shape, rank, world).numpy()
        a, _ = T.vocab_rows(shape, rank, world)
        logits = O.gemv(head, O.rmsnorm(x, w["final_norm"], cfg.eps))
        cand = torch.tensor(np.stack([logits.max(axis=1), logits.argmax(axis=1) + a], axis=1))
        allc = [torch.zeros_like(cand) for _ in range(world)]
        dist.all_gather(allc, cand)  # the (max, index) all-gather
        best_v, best_i = allc[0][:, 0].numpy(), allc[0][:, 1].numpy()
        for c in allc[1:]:
            v, idx = c[:, 0].numpy(), c[:, 1].numpy()
            take = (v > best_v) | ((v == best_v) & (idx < best_i))
            best_v, best_i = np.where(take, v, best_v), np.where(take, idx, best_i)
        if rank == 0:
            ref_logits, ref_next = S.decode_step(w, cfg, tokens, lens, table, *build_paged_cache(g, cfg, np.float16)[2:])
            q.put((best_i.astype(np.int64).tolist(), ref_next.astype(np.int64).tolist(), float(np.max(np.abs(best_v - ref_logits.max(axis=1))))))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_tp2_gloo_matches_single_rank_oracle():
    from tests.conftest import GOLDEN

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(GOLDEN / "hf_llama_ops.npz"), q)) for r in range(2)]
    for p in procs:
        p.start()
    got, ref, dv = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == ref
    assert dv < 1e-9


def test_shard_layout_matches_oracle_slices():
    """Product sharding == oracle's definition of rank-owned heads / FFN rows / vocab rows."""
    cfg = S.ModelConfig(256, 1, 8, 4, 32, 96, 1001, 1e-5, 1e4)
    shape = T.ModelShape(cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab, cfg.eps, cfg.theta)
    for tp in (1, 2, 4):
        for r in range(tp):
            sl = S.tp_slices(cfg, r, tp)
            a, b = T.vocab_rows(shape, r, tp)
            assert (a, b) == (sl["vocab"].start, sl["vocab"].stop)
            rows = T.qkv_rows(shape, r, tp).numpy()
            hd = cfg.head_dim
            q = np.arange(sl["q_heads"].start * hd, sl["q_heads"].stop * hd)
            assert np.array_equal(rows[: len(q)], q)
            assert len(rows) == (cfg.n_heads + 2 * cfg.n_kv_heads) // tp * hd
    with pytest.raises(ValueError):
        T.check_tp(shape, 3)


@pytest.mark.parametrize("fmt", ["q8_32", "q4_32"])
@pytest.mark.parametrize("tp", [2, 8])
def test_quantized_shards_dequantize_to_the_fp16_shards(fmt, tp):
    """shard_layer_quant cuts the stored integers and their scales so that every rank's shard
    dequantizes to exactly the same slice of the dequantized matrix that shard_layer gives the
    fp16 path (rows of the column-parallel projections, 32-element K blocks of the row-parallel
    ones), and the shards put back together are the whole matrix."""
    from gemmagemini4hackathon2026_10_2425_b200 import weights as W

    cfg = S.ModelConfig(512, 1, 16, 8, 64, 2048, 1000, 1e-5, 1e4)
    shape = T.ModelShape(cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab, cfg.eps, cfg.theta)
    w = S.synth_weights(cfg, seed=3)
    full_q, full_deq = {}, {}
    for n in ("wqkv", "wo", "wgate", "wup", "wdown"):
        q, sc = W.quantize(w[f"l0.{n}"], fmt)
        full_q[n], full_q[n + ".scales"] = torch.from_numpy(q), torch.from_numpy(sc)
        full_deq[n] = torch.from_numpy(W.dequantize(q, sc, fmt))
    full_q["attn_norm"] = full_q["ffn_norm"] = torch.ones(cfg.dim)
    full_deq["attn_norm"] = full_deq["ffn_norm"] = torch.ones(cfg.dim)
    for r in range(tp):
        qs = T.shard_layer_quant(full_q, shape, r, tp, fmt)
        fs = T.shard_layer(full_deq, shape, r, tp)
        for n in ("wqkv", "wo", "wgate", "wup", "wdown"):
            deq = W.dequantize(qs[n].numpy(), qs[n + ".scales"].numpy(), fmt)
            np.testing.assert_array_equal(deq, fs[n].numpy())
