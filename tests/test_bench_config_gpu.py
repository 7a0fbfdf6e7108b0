"""Parity of the exact benchmarked workload: BASELINE config 5 as bench.py builds it.

16 layers, d_model 2048, 32/8 heads, head_dim 64, SwiGLU 8192, vocab 128256, batch 32 ragged
contexts U[512, 4096] over a randomly permuted page table, random-init weights (bench.py's
seeds).  One decode step through the tensor-core path (the headline measurement's path) is
compared with the float64 oracle (oracle/step.py), evaluated on the host layer by layer from
the GPU's own weights:

  * elementwise against the oracle run over the KV cache the GPU wrote (the appended K/V are
    fp16 roundings; see test_decoder_gpu.py for why that is the elementwise reference):
    2e-3 with a floor of 1e-2 of the largest logit; and, at a floor of 1e-3, no worse than twice
    the error of plain fp32 arithmetic -- the NumPy float32 port of the same step
    (oracle/step.py CpuDecodeF32, round-to-nearest BLAS) evaluated the same way.  The reference
    computes in fp32 (LK/kernels.metal:106-131); sixteen layers of fp32 accumulation put its own
    near-zero logits about 4e-3 off at the 1e-3 floor (max-normalized ~5e-6), so that floor
    measures fp32 itself, and the GPU is held to fp32's own figure there;
  * max-normalized at 2e-3 against the independent oracle that appends its own K/V;
  * every appended K/V slot against the independent oracle's, within 2e-3 (fp16 rounding);
  * next tokens: the argmax of the GPU's logits, and the oracle's wherever the top two logits
    are not within the tolerance of each other.

The oracle needs ~16 GB of host memory and a few minutes of host time.
"""

import numpy as np
import pytest
import torch

from oracle import ops as O
from oracle import step as S
from tests._tol import assert_norm_close, assert_rel_close

pytestmark = pytest.mark.gpu


def test_config5_step_matches_oracle():
    import bench

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    eng, table, lens, tokens0 = bench.config5_engine(dev, steps_total=1)
    cfg = S.LLAMA_1B
    assert (eng.shape.dim, eng.shape.n_layers, eng.shape.vocab) == (cfg.dim, cfg.n_layers, cfg.vocab)
    try:
        B = len(lens)
        tok = torch.from_numpy(tokens0).to(dev)
        ctx = torch.from_numpy(lens.copy()).to(dev)
        nxt = torch.empty_like(tok)
        logits = torch.empty(B, eng.lm_rows, dtype=torch.float32, device=dev)
        kp0 = [k.cpu().numpy() for k in eng.k_pages]  # the cache before the step
        vp0 = [v.cpu().numpy() for v in eng.v_pages]
        eng.step(tok, ctx, table, nxt, logits, use_graph=True)
        eng.stream.synchronize()
        eng.check()
        got, got_next = logits.cpu().numpy(), nxt.cpu().numpy()
        gk = [k.cpu().numpy() for k in eng.k_pages]
        gv = [v.cpu().numpy() for v in eng.v_pages]
        w = {"embed": eng.embed.cpu().numpy(), "final_norm": eng.final_norm.cpu().numpy()}
        for i, L in enumerate(eng.layers):
            for n, t in L.items():
                w[f"l{i}.{n}"] = t.cpu().numpy()
        tb = table.cpu().numpy()
    finally:
        eng.close()
        del eng
        torch.cuda.empty_cache()

    same_kv, _ = S.decode_step(w, cfg, tokens0, lens, tb, gk, gv, append=False)
    assert_rel_close(got, same_kv, 2e-3, floor_frac=1e-2, what="config-5 logits vs oracle over the GPU's KV")
    # fp32 arithmetic on the same step: the NumPy port appends its own K/V into copies of the
    # cache, then the float64 oracle is evaluated over that cache
    k32, v32 = [k.copy() for k in kp0], [v.copy() for v in vp0]
    port = S.CpuDecodeF32(cfg, w, k32, v32, tb, lens)
    x = port.embed(tokens0)
    for i in range(cfg.n_layers):
        x = port.layer(i, x)
    lg32 = port._rms(x, port.final_norm, cfg.eps) @ port.head.T
    del port, x
    ref32, _ = S.decode_step(w, cfg, tokens0, lens, tb, k32, v32, append=False)
    del k32, v32

    def scaled(a, r, floor):
        return float(np.max(np.abs(a - r) / np.maximum(np.abs(r), floor * np.max(np.abs(r)))))

    e_gpu, e_f32 = scaled(got, same_kv, 1e-3), scaled(lg32, ref32, 1e-3)
    print(f"elementwise error at a 1e-3 floor: GPU {e_gpu:.2e}, fp32 port {e_f32:.2e}")
    assert e_gpu <= 2 * e_f32, f"GPU {e_gpu:.2e} vs fp32 arithmetic {e_f32:.2e}"
    ref, ref_next = S.decode_step(w, cfg, tokens0, lens, tb, kp0, vp0)
    assert_norm_close(got, ref, 2e-3, what="config-5 logits vs independent oracle")
    np.testing.assert_array_equal(got_next, O.argmax(got))
    srt = np.sort(ref, axis=1)
    safe = (srt[:, -1] - srt[:, -2]) > 2e-3 * np.abs(srt[:, -1])
    assert safe.sum() >= B // 2
    np.testing.assert_array_equal(got_next[safe], ref_next[safe])
    # the appended token of every sequence, in every layer, landed in its page slot with the
    # oracle's value up to one fp16 rounding (kp0 / vp0 now hold the independent oracle's
    # appends); no other slot differs
    blk = tb[np.arange(B), lens // 16]
    slot = lens % 16
    for layer in range(cfg.n_layers):
        for name, gpu, mine in (("K", gk[layer], kp0[layer]), ("V", gv[layer], vp0[layer])):
            np.testing.assert_allclose(
                gpu[blk, :, slot].astype(np.float32), mine[blk, :, slot].astype(np.float32), rtol=2e-3, atol=2e-3
            )
            changed = np.any(gpu.view(np.uint16) != mine.view(np.uint16), axis=-1)
            changed[blk, :, slot] = False
            assert not changed.any(), f"layer {layer}: {name} pages differ outside the appended slots"
