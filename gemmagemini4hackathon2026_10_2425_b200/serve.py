"""The kernel-folder binary of the reference, on the B200 decode path.

The reference's Python side drives a model through a kernel folder (kernel.json + a `binary`) that
speaks a JSON-lines protocol on stdin/stdout (IK/surfaces/DESIGN_AND_LIMITATIONS.md:70-88;
implemented by LK/main.swift:494-622, driven by IK/surfaces/runners/kernel_runner.py:20-96).
This module is that binary for the CUDA path; the `llm` of the package's kernel folder
(kernels/unsloth__Llama-3.2-1B-Instruct/kernel_b200_cuda_20261202-1200/) runs its main().  Same flags:

    --weights PATH --max-ctx N --serve
    --prompt-ids a,b,c --gen N [--dump-logits PATH]
    --bench-pp N --bench-tg N [--reps R]
    (--kernels / --define / --no-gemm are accepted for compatibility and ignored)

--serve protocol (one JSON object per line):
    -> {"ready": true, "max_ctx": N, "vocab": V, "device": "..."}          once, after warm-up
    <- {"ids": [...], "max_tokens": n, "stop_ids": [...]}
    -> {"token": t} per generated token (a stop token is not sent)
    -> {"done": true, "finish_reason": "stop"|"length", "prompt_tokens", "completion_tokens",
        "prefill_s", "decode_s"}
    -> {"error": "..."} for a bad request (the process keeps serving); EOF on stdin ends it.

One sequence at a time (batch 1), greedy, every request from an empty cache.  The prompt is
prefilled in chunks of 32 consecutive positions per step (b2d_decoder_prefill: tcgen05
projections, each chunk's K/V written before its rows attend); --no-gemm prefills one token per
decode step, as the reference's --no-gemm does.

Generation never waits for the host between steps: each step is one launch of the device-
resident loop (b2d_decoder_generate: step + next token fed back + position advanced, all on the
GPU), up to WINDOW steps are in flight, and the host reads each token from pinned memory once its
step's event has completed -- the reference's window of command buffers in flight
(LK/main.swift:473-491).  A stop token seen on the host ends the request; the steps already in
flight past it only write cache positions the next request overwrites.  --bench-tg times n steps
launched back to back with one synchronization at the end (LK/main.swift:374-381, 605-618).
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys
import time

BOS = 128000


def parse_args(argv=None) -> argparse.Namespace:
    ap = argparse.ArgumentParser(prog="llm", description=__doc__.split("\n\n")[0])
    ap.add_argument("--weights", required=True)
    ap.add_argument("--max-ctx", type=int, default=4096)
    ap.add_argument("--serve", action="store_true")
    ap.add_argument("--prompt-ids", default="")
    ap.add_argument("--gen", type=int, default=0)
    ap.add_argument("--dump-logits", default=None)
    ap.add_argument("--bench-pp", type=int, default=0)
    ap.add_argument("--bench-tg", type=int, default=0)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--kernels", default=None, help="ignored (Metal source path in the reference)")
    ap.add_argument("--define", action="append", default=[], help="ignored (Metal defines in the reference)")
    ap.add_argument("--no-gemm", action="store_true", help="prefill one token per decode step instead of 32-position chunks")
    return ap.parse_args(argv)


def parse_request(line: str, vocab: int, max_ctx: int) -> tuple[list[int], int, set[int]]:
    """One --serve request -> (ids, max_tokens, stop_ids); ValueError with the reference's
    messages for a bad one (LK/main.swift:513-524)."""
    try:
        req = json.loads(line)
        ids = [int(t) for t in req["ids"]]
        if not ids:
            raise ValueError
    except (ValueError, KeyError, TypeError):
        raise ValueError('expected {"ids": [int, ...], "max_tokens": int}') from None
    bad = next((t for t in ids if t < 0 or t >= vocab), None)
    if bad is not None:
        raise ValueError(f"token id {bad} out of range")
    if len(ids) >= max_ctx:
        raise ValueError(f"prompt has {len(ids)} tokens, max_ctx is {max_ctx}")
    max_tokens = min(int(req.get("max_tokens", 256)), max_ctx - len(ids))
    stop = {int(t) for t in req.get("stop_ids", [])}
    return ids, max_tokens, stop


PREFILL_CHUNK = 32  # positions per prefill step (the tcgen05 projections take up to 32 rows)
WINDOW = 3  # decode steps in flight while streaming (the reference keeps 3 command buffers queued)


class Session:
    """One sequence on one GPU: the weights file in a DecodeEngine, a contiguous block table,
    and a captured decode step fed through pinned host buffers."""

    def __init__(self, weights: str, max_ctx: int, chunked_prefill: bool = True):
        import torch

        from . import weights as W
        from .engine import DecodeEngine

        self.torch = torch
        wf = W.read_weights(weights)
        self.shape = W.shape_from_config(wf.config)
        self.max_ctx = max_ctx
        blocks = -(-max_ctx // 16)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.chunked = chunked_prefill
        batch = PREFILL_CHUNK if chunked_prefill else 1
        self.eng = DecodeEngine(self.shape, max_batch=batch, max_ctx=max_ctx, n_blocks=blocks, device=dev)
        self.eng.alloc_kv()
        self.eng.load_weights_file(weights)
        self.table = torch.arange(blocks, dtype=torch.int32, device=dev).view(1, blocks)
        i32 = dict(dtype=torch.int32, device=dev)
        self.tok, self.pos, self.nxt = torch.zeros(1, **i32), torch.zeros(1, **i32), torch.zeros(1, **i32)
        self.logits = torch.empty(1, self.eng.lm_rows, dtype=torch.float32, device=dev)
        self.h_in = torch.zeros(2, dtype=torch.int32).pin_memory()
        self.h_out = torch.zeros(1, dtype=torch.int32).pin_memory()
        # device-resident loop: a ring of generated tokens, copied to pinned host slots
        self.ring_len = 4 * WINDOW
        self.ring = torch.zeros(self.ring_len, 1, **i32)
        self.ring_count = torch.zeros(1, **i32)
        self.h_ring = torch.zeros(self.ring_len, dtype=torch.int32).pin_memory()
        self.events = [torch.cuda.Event() for _ in range(self.ring_len)]
        self.device_name = torch.cuda.get_device_name(dev)

    @property
    def vocab(self) -> int:
        return self.shape.vocab

    def step(self, token: int, pos: int) -> int:
        """Decode `token` at position `pos`; returns the greedy next token."""
        s = self.eng.stream
        self.h_in[0], self.h_in[1] = token, pos
        with self.torch.cuda.stream(s):
            self.tok.copy_(self.h_in[0:1], non_blocking=True)
            self.pos.copy_(self.h_in[1:2], non_blocking=True)
            self.eng.step(self.tok, self.pos, self.table, self.nxt, self.logits, use_graph=True)
            self.h_out.copy_(self.nxt, non_blocking=True)
        s.synchronize()
        return int(self.h_out[0])

    def prefill(self, ids: list[int], want_logits: bool = False) -> int:
        """Run the prompt (positions 0..n-1) and return the first generated token; with
        want_logits, last_logits() then holds the last position's logits."""
        if not self.chunked:
            nxt = 0
            for p, t in enumerate(ids):
                nxt = self.step(t, p)
            return nxt
        torch = self.torch
        s = self.eng.stream
        ids_h = torch.tensor(ids, dtype=torch.int32).pin_memory()
        with torch.cuda.stream(s):
            ids_d = ids_h.to(self.tok.device, non_blocking=True)
            self.eng.prefill(ids_d, self.table[0], 0, next_token=self.nxt,
                             logits=self.logits[0] if want_logits else None)
            self.h_out.copy_(self.nxt, non_blocking=True)
        s.synchronize()
        return int(self.h_out[0])

    def last_logits(self):
        return self.logits[0].float().cpu().numpy()

    def _start(self, token_dev_or_host, pos: int) -> None:
        """Set the loop's input token (a host int, or None: the prefill's next token already on
        the device) and position; resets the ring count."""
        s = self.eng.stream
        with self.torch.cuda.stream(s):
            if token_dev_or_host is None:
                self.tok.copy_(self.nxt)
            else:
                self.h_in[0] = int(token_dev_or_host)
                self.tok.copy_(self.h_in[0:1], non_blocking=True)
            self.h_in[1] = pos
            self.pos.copy_(self.h_in[1:2], non_blocking=True)
            self.ring_count.zero_()

    def _launch(self, k: int) -> None:
        """Enqueue loop step k (the k-th since _start): one step + advance, then the token's copy
        into pinned host slot k % ring_len and an event that marks it readable."""
        s = self.eng.stream
        slot = k % self.ring_len
        with self.torch.cuda.stream(s):
            self.eng.generate(self.tok, self.pos, self.table, 1, self.ring, self.ring_count)
            self.h_ring[slot : slot + 1].copy_(self.ring[slot], non_blocking=True)
            self.events[slot].record(s)

    def _token(self, k: int) -> int:
        slot = k % self.ring_len
        self.events[slot].synchronize()
        return int(self.h_ring[slot])

    def generate(self, first: int | None, pos: int, n: int):
        """Yield up to n tokens following `first` (host int, or None after prefill: the device's
        next token) at position pos, with up to WINDOW steps in flight.  The caller may stop
        early; steps already enqueued then just finish."""
        self._start(first, pos)
        launched = 0
        for k in range(n):
            while launched < min(k + WINDOW, n):
                self._launch(launched)
                launched += 1
            yield self._token(k)

    def run_steps(self, first: int, pos: int, n: int) -> None:
        """n loop steps back to back from token `first` at `pos`, one synchronization at the end."""
        self._start(first, pos)
        s = self.eng.stream
        with self.torch.cuda.stream(s):
            self.eng.generate(self.tok, self.pos, self.table, n, self.ring, self.ring_count)
        s.synchronize()


def _emit(obj: dict, out) -> None:
    out.write(json.dumps(obj) + "\n")
    out.flush()


def serve(sess: Session, inp=sys.stdin, out=sys.stdout) -> None:
    sess.prefill([BOS % sess.vocab] * 2)  # warm-up: graph capture, first launches
    sess.step(0, 2)
    list(sess.generate(None, 3, 2))
    _emit({"ready": True, "max_ctx": sess.max_ctx, "vocab": sess.vocab, "device": sess.device_name}, out)
    for line in inp:
        if not line.strip():
            continue
        try:
            ids, max_tokens, stop = parse_request(line, sess.vocab, sess.max_ctx)
        except ValueError as e:
            _emit({"error": str(e)}, out)
            continue
        t0 = time.perf_counter()
        tok = sess.prefill(ids)
        t_prefill = time.perf_counter() - t0
        t1 = time.perf_counter()
        produced, finish = 0, "length"
        following = sess.generate(None, len(ids), max_tokens - 1)
        while produced < max_tokens:
            if tok in stop:
                finish = "stop"
                break
            _emit({"token": tok}, out)
            produced += 1
            if produced >= max_tokens:
                break
            tok = next(following)
        following.close()
        _emit(
            {
                "done": True,
                "finish_reason": finish,
                "prompt_tokens": len(ids),
                "completion_tokens": produced,
                "prefill_s": t_prefill,
                "decode_s": time.perf_counter() - t1,
            },
            out,
        )


def _stats(xs: list[float]) -> tuple[float, float]:
    return statistics.fmean(xs), (statistics.stdev(xs) if len(xs) > 1 else 0.0)


def main(argv=None) -> int:
    a = parse_args(argv)
    sess = Session(a.weights, a.max_ctx, chunked_prefill=not a.no_gemm)
    s = sess.shape
    print(f"device: {sess.device_name}, dim {s.dim}, layers {s.n_layers}, vocab {s.vocab}, gemm {str(sess.chunked).lower()}", file=sys.stderr)
    if a.prompt_ids:
        ids = [int(t) for t in a.prompt_ids.split(",")]
        if len(ids) + a.gen > a.max_ctx:
            raise SystemExit("prompt + gen exceeds --max-ctx")
        t0 = time.perf_counter()
        tok = sess.prefill(ids, want_logits=bool(a.dump_logits))
        t_prefill = time.perf_counter() - t0
        if a.dump_logits:
            sess.last_logits().astype("<f4").tofile(a.dump_logits)
        toks = [tok]
        t1 = time.perf_counter()
        toks += list(sess.generate(None, len(ids), max(a.gen - 1, 0)))
        t_dec = time.perf_counter() - t1
        print(json.dumps({
            "tokens": toks[: a.gen],
            "prefill_s": t_prefill,
            "decode_s": t_dec,
            "decode_tok_s": (a.gen - 1) / t_dec if a.gen > 1 and t_dec > 0 else 0,
        }))
    if a.bench_pp > 0 or a.bench_tg > 0:
        report = {"tunables": {"prefill": f"chunks of {PREFILL_CHUNK}" if sess.chunked else "decode steps", "batch": 1, "graph": True}}
        if a.bench_pp > 0:
            n = min(a.bench_pp, a.max_ctx - 1)
            ids = [(i * 7919 % 100000 + 1000) % s.vocab for i in range(n)]
            sess.prefill(ids)
            rates = []
            for _ in range(a.reps):
                t0 = time.perf_counter()
                sess.prefill(ids)
                rates.append(n / (time.perf_counter() - t0))
            m, sd = _stats(rates)
            report["pp"] = {"n": n, "tok_s": m, "std": sd}
            print(f"pp{n}: {m:.1f} ± {sd:.1f} tok/s", file=sys.stderr)
        if a.bench_tg > 0:
            n = min(a.bench_tg, a.max_ctx - 1)
            bos = BOS % s.vocab

            def run():
                sess.run_steps(bos, 0, n)

            run()
            rates = []
            for _ in range(a.reps):
                t0 = time.perf_counter()
                run()
                rates.append(n / (time.perf_counter() - t0))
            m, sd = _stats(rates)
            report["tg"] = {"n": n, "tok_s": m, "std": sd}
            print(f"tg{n}: {m:.1f} ± {sd:.1f} tok/s", file=sys.stderr)
        print(json.dumps(report))
    if a.serve:
        serve(sess)
    sess.eng.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
