"""DecodeEngine: host side of the decode step (the reference's Swift Engine, LK/main.swift:152-391).

Owns, per rank: the sharded fp16 weights, the paged KV pools, and a b2d_decoder handle from
libb200dec.so that runs the whole step (optionally captured in a CUDA graph).  Tensor
parallelism uses one process per GPU; the NCCL unique id travels over torch.distributed.

Weights are named like the reference's weights file (LK/convert_weights.py:60-72): embed,
l{i}.attn_norm, l{i}.wqkv, l{i}.wo, l{i}.ffn_norm, l{i}.wgate, l{i}.wup, l{i}.wdown, final_norm;
the LM head is tied to embed (LK/main.swift:306).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib, tp as tpmod
from ._lib import call
from .tp import ModelShape

PAGE = 16


def nccl_unique_id() -> bytes:
    n = _lib.lib().b2d_nccl_unique_id_bytes()
    buf = ctypes.create_string_buffer(n)
    call("b2d_nccl_get_unique_id", ctypes.addressof(buf))
    return buf.raw


def share_nccl_id(rank: int) -> bytes:
    """Rank 0 makes the id; every rank of the default torch.distributed group receives it."""
    import torch.distributed as dist

    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


class DecodeEngine:
    """A Llama-style decoder for one rank of `tp_size` (tp_size 1 = single GPU)."""

    def __init__(
        self,
        shape: ModelShape,
        *,
        max_batch: int,
        max_ctx: int,
        n_blocks: int,
        tp_rank: int = 0,
        tp_size: int = 1,
        nccl_id: bytes | None = None,
        device: torch.device | None = None,
    ):
        tpmod.check_tp(shape, tp_size)
        self.shape, self.rank, self.tp = shape, tp_rank, tp_size
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.max_batch, self.max_ctx, self.n_blocks = max_batch, max_ctx, n_blocks
        self.max_blocks = -(-max_ctx // PAGE)
        self.hq, self.hk = shape.n_heads // tp_size, shape.n_kv_heads // tp_size
        cfg = _lib.ModelConfig(
            shape.dim,
            shape.n_layers,
            shape.n_heads,
            shape.n_kv_heads,
            shape.head_dim,
            shape.ffn_dim,
            shape.vocab,
            shape.eps,
            shape.theta,
            max_batch,
            max_ctx,
            self.max_blocks,
            n_blocks,
        )
        self._h = ctypes.c_void_p()
        idbuf = None
        if tp_size > 1:
            if nccl_id is None:
                raise ValueError("tp_size > 1 needs the NCCL unique id from rank 0")
            idbuf = ctypes.create_string_buffer(nccl_id, len(nccl_id))
        with torch.cuda.device(self.device):
            call(
                "b2d_decoder_create",
                ctypes.byref(cfg),
                tp_rank,
                tp_size,
                ctypes.addressof(idbuf) if idbuf is not None else None,
                ctypes.byref(self._h),
            )
        self.lm_rows = tpmod.vocab_rows(shape, tp_rank, tp_size)[1] - tpmod.vocab_rows(shape, tp_rank, tp_size)[0]
        self.layers: list[dict[str, torch.Tensor]] = []
        self.k_pages: list[torch.Tensor] = []
        self.v_pages: list[torch.Tensor] = []
        self.stream = torch.cuda.Stream(device=self.device)

    # -- setup ------------------------------------------------------------------------------

    def alloc_kv(self, fill_seed: int | None = None) -> None:
        """Allocate this rank's page pools: per layer K and V [n_blocks, Hkv/tp, 16, HD] fp16.
        With fill_seed, fill them with seeded N(0, 1) values (synthetic cache contents)."""
        s = self.shape
        shp = (self.n_blocks, self.hk, PAGE, s.head_dim)
        g = torch.Generator(device=self.device)
        if fill_seed is not None:
            g.manual_seed(fill_seed + 7919 * self.rank)
        self.k_pages, self.v_pages = [], []
        for _ in range(s.n_layers):
            if fill_seed is None:
                k = torch.zeros(shp, dtype=torch.float16, device=self.device)
                v = torch.zeros(shp, dtype=torch.float16, device=self.device)
            else:
                k = torch.randn(shp, generator=g, dtype=torch.float16, device=self.device)
                v = torch.randn(shp, generator=g, dtype=torch.float16, device=self.device)
            self.k_pages.append(k)
            self.v_pages.append(v)

    def load_weights(self, w: dict[str, torch.Tensor], quant: dict[str, str] | None = None) -> None:
        """Full (unsharded) weights -> this rank's shards on the device, registered with the
        library.  Needs alloc_kv() first.  `quant` maps matrix names to "q8_32" / "q4_32" for
        projections stored quantized (w[name] the integers, w[name + ".scales"] the fp16 block
        scales); a layer's five projections then share one format and stay quantized on the
        device (b2d_decoder_set_layer_q)."""
        if not self.k_pages:
            raise RuntimeError("alloc_kv() before load_weights()")
        s, dev = self.shape, self.device
        quant = quant or {}
        self.layers = []
        names = ("attn_norm", "wqkv", "wo", "ffn_norm", "wgate", "wup", "wdown")
        mats = ("wqkv", "wo", "wgate", "wup", "wdown")
        for i in range(s.n_layers):
            fmts = {quant.get(f"l{i}.{n}") for n in mats}
            if len(fmts) != 1:
                raise ValueError(f"layer {i}: all five projections must share one weight format, got {sorted(map(str, fmts))}")
            fmt = fmts.pop()
            full = {n: w[f"l{i}.{n}"] for n in names}
            if fmt is None:
                sh = {k: v.to(dev) for k, v in tpmod.shard_layer(full, s, self.rank, self.tp).items()}
                for k in mats:
                    sh[k] = sh[k].half().contiguous()
            else:
                full.update({f"{n}.scales": w[f"l{i}.{n}.scales"] for n in mats})
                sh = {k: v.to(dev) for k, v in tpmod.shard_layer_quant(full, s, self.rank, self.tp, fmt).items()}
                for k in mats:
                    sh[k + ".scales"] = sh[k + ".scales"].half().contiguous()
            sh["attn_norm"] = sh["attn_norm"].float().contiguous()
            sh["ffn_norm"] = sh["ffn_norm"].float().contiguous()
            self.layers.append(sh)
            code = {None: _lib.F16, "q8_32": _lib.Q8_32, "q4_32": _lib.Q4_32}[fmt]
            sc = (lambda k: None) if fmt is None else (lambda k: sh[k + ".scales"].data_ptr())
            call(
                "b2d_decoder_set_layer_q",
                self._h,
                i,
                code,
                sh["attn_norm"].data_ptr(),
                sh["wqkv"].data_ptr(),
                sc("wqkv"),
                sh["wo"].data_ptr(),
                sc("wo"),
                sh["ffn_norm"].data_ptr(),
                sh["wgate"].data_ptr(),
                sc("wgate"),
                sh["wup"].data_ptr(),
                sc("wup"),
                sh["wdown"].data_ptr(),
                sc("wdown"),
                self.k_pages[i].data_ptr(),
                self.v_pages[i].data_ptr(),
            )
        self.embed = w["embed"].to(dev).half().contiguous()
        head = w["lm_head"].to(dev).half().contiguous() if "lm_head" in w else self.embed
        self.lm_head = tpmod.shard_head(head, s, self.rank, self.tp)
        self.final_norm = w["final_norm"].to(dev).float().contiguous()
        call(
            "b2d_decoder_set_head",
            self._h,
            self.embed.data_ptr(),
            self.lm_head.data_ptr(),
            self.lm_rows,
            self.final_norm.data_ptr(),
        )

    def set_inv_freq(self, inv_freq) -> None:
        """RoPE inverse frequencies (head_dim / 2 floats), e.g. weights.inv_freq_from_config()."""
        import numpy as np

        a = np.ascontiguousarray(np.asarray(inv_freq, dtype=np.float32))
        call("b2d_decoder_set_inv_freq", self._h, a.ctypes.data, a.size)

    def load_weights_file(self, path, dequantize: bool = False) -> dict:
        """Load a weights file in the reference's format (weights.py) into this rank's shards
        and apply its RoPE settings; returns the file's config.  Needs alloc_kv() first.
        Projections stored quantized stay quantized on the device (the decode step streams
        them as stored); dequantize=True expands them to fp16(scale * q) instead."""
        from . import weights as W

        wf = W.read_weights(path)
        shape = W.shape_from_config(wf.config)
        if shape != self.shape:
            raise ValueError(f"{path}: model shape {shape} does not match this engine's {self.shape}")
        import numpy as np

        # the mapped file is read-only: each tensor is copied once on its way to the device
        t = W.tensors_for_engine(wf, keep_quant=not dequantize)
        self.load_weights({k: torch.from_numpy(np.array(v)) for k, v in t.items()}, None if dequantize else wf.quant)
        self.set_inv_freq(W.inv_freq_from_config(wf.config))
        return wf.config

    def random_weights(self, seed: int, std: float = 0.02, quant: str | None = None) -> None:
        """Seeded random-init weights generated on the device (fp16 ~ N(0, std), norms = 1).
        Every rank draws the same full matrices and keeps its shard.  quant ("q8_32" /
        "q4_32") stores the five projections of every layer in that 32-block format instead,
        quantized from the same fp16 draws (weights.quantize_torch)."""
        from . import weights as W

        s, dev = self.shape, self.device
        g = torch.Generator(device=dev)
        g.manual_seed(seed)

        def mat(m, k):
            return (torch.randn(m, k, generator=g, device=dev, dtype=torch.float32) * std).half()

        w = {"embed": mat(s.vocab, s.dim), "final_norm": torch.ones(s.dim, device=dev)}
        qmap = {}
        for i in range(s.n_layers):
            w[f"l{i}.attn_norm"] = torch.ones(s.dim, device=dev)
            w[f"l{i}.wqkv"] = mat(s.qkv_dim, s.dim)
            w[f"l{i}.wo"] = mat(s.dim, s.n_heads * s.head_dim)
            w[f"l{i}.ffn_norm"] = torch.ones(s.dim, device=dev)
            w[f"l{i}.wgate"] = mat(s.ffn_dim, s.dim)
            w[f"l{i}.wup"] = mat(s.ffn_dim, s.dim)
            w[f"l{i}.wdown"] = mat(s.dim, s.ffn_dim)
            if quant:
                for n in ("wqkv", "wo", "wgate", "wup", "wdown"):
                    name = f"l{i}.{n}"
                    w[name], w[name + ".scales"] = W.quantize_torch(w[name], quant)
                    qmap[name] = quant
        self.load_weights(w, qmap or None)
        del w
        torch.cuda.empty_cache()

    def weight_bytes(self) -> int:
        n = sum(t.numel() * t.element_size() for L in self.layers for t in L.values())
        return n + self.lm_head.numel() * 2 + self.final_norm.numel() * 4

    # -- step -------------------------------------------------------------------------------

    def step(
        self,
        tokens: torch.Tensor,
        ctx_lens: torch.Tensor,
        block_table: torch.Tensor,
        next_tokens: torch.Tensor,
        logits: torch.Tensor | None = None,
        use_graph: bool = True,
    ) -> torch.Tensor:
        """Enqueue one decode step on self.stream (no host sync).  tokens/ctx_lens/next_tokens
        int32 [B]; block_table int32 [B, max_blocks]; logits (optional) fp32 [B, lm_rows]."""
        B = tokens.numel()
        for t in (tokens, ctx_lens, block_table, next_tokens):
            if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous():
                raise ValueError("tokens, ctx_lens, block_table, next_tokens: contiguous CUDA int32")
        if block_table.shape != (B, self.max_blocks):
            raise ValueError(f"block_table must be [{B}, {self.max_blocks}]")
        call(
            "b2d_decoder_step",
            self._h,
            tokens.data_ptr(),
            ctx_lens.data_ptr(),
            block_table.data_ptr(),
            B,
            next_tokens.data_ptr(),
            None if logits is None else logits.data_ptr(),
            1 if use_graph else 0,
            self.stream.cuda_stream,
        )
        return next_tokens

    def generate(
        self,
        tokens: torch.Tensor,
        ctx_lens: torch.Tensor,
        block_table: torch.Tensor,
        n_steps: int,
        ring: torch.Tensor | None = None,
        ring_count: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Enqueue n_steps greedy decode steps that feed each other on the device (no host sync).
        tokens / ctx_lens (int32 [B], device) advance in place; returns the ring [n_steps, B] the
        generated tokens land in (pass ring / ring_count to keep appending to your own)."""
        B = tokens.numel()
        for t in (tokens, ctx_lens, block_table):
            if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous():
                raise ValueError("tokens, ctx_lens, block_table: contiguous CUDA int32")
        if ring is None:
            ring = torch.zeros(max(n_steps, 1), B, dtype=torch.int32, device=tokens.device)
        if ring_count is None:
            ring_count = torch.zeros(1, dtype=torch.int32, device=tokens.device)
        call(
            "b2d_decoder_generate",
            self._h,
            tokens.data_ptr(),
            ctx_lens.data_ptr(),
            block_table.data_ptr(),
            B,
            n_steps,
            ring.data_ptr(),
            ring.shape[0],
            ring_count.data_ptr(),
            self.stream.cuda_stream,
        )
        return ring

    def prefill(
        self,
        tokens: torch.Tensor,
        seq_table: torch.Tensor,
        start_pos: int = 0,
        next_token: torch.Tensor | None = None,
        logits: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Enqueue the prefill of one sequence (no host sync): tokens int32 [n] (device) at
        positions start_pos .. start_pos + n - 1, K/V written into the pages of seq_table
        (int32 [max_blocks], device), in chunks of max_batch positions per step.  Returns
        next_token (int32 [1]): the greedy token after the last one; logits (fp32 [lm_rows])
        receives the last position's logits if given."""
        n = tokens.numel()
        for t in (tokens, seq_table):
            if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous():
                raise ValueError("tokens, seq_table: contiguous CUDA int32")
        if seq_table.numel() != self.max_blocks:
            raise ValueError(f"seq_table must hold {self.max_blocks} block ids")
        if next_token is None:
            next_token = torch.empty(1, dtype=torch.int32, device=tokens.device)
        if logits is not None and (logits.dtype != torch.float32 or logits.numel() < self.lm_rows):
            raise ValueError(f"logits must be fp32 with >= {self.lm_rows} elements")
        call(
            "b2d_decoder_prefill",
            self._h,
            tokens.data_ptr(),
            n,
            seq_table.data_ptr(),
            start_pos,
            next_token.data_ptr(),
            None if logits is None else logits.data_ptr(),
            self.stream.cuda_stream,
        )
        return next_token

    def peer_collectives(self) -> bool:
        """True if the tensor-parallel sums run over NVLink peer memory (False: NCCL or tp 1)."""
        return bool(_lib.lib().b2d_decoder_peer_collectives(self._h))

    def check(self) -> None:
        """Synchronize and raise if a device-side peer barrier timed out since the last check."""
        st = _lib.lib().b2d_decoder_error(self._h)
        if st:
            raise _lib.B2DError("b2d_decoder_error", st, _lib.lib().b2d_status_string(st).decode())

    def close(self) -> None:
        """Free the handle.  With tp > 1 this is collective: every rank calls it."""
        if self._h:
            _lib.lib().b2d_decoder_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover
        # tensor-parallel handles are freed collectively by close(), never by the collector
        try:
            if self.tp == 1:
                self.close()
        except Exception:
            pass


def make_block_table(ctx_lens, max_blocks: int, n_blocks: int, seed: int, headroom: int = 1):
    """Seeded random page assignment: sequence b gets ceil((ctx_b + headroom)/16) distinct
    physical pages from a random permutation of [0, n_blocks).  Returns int32 [B, max_blocks]
    (unused entries -1) on the CPU."""
    import numpy as np

    need = [-(-(int(c) + headroom) // PAGE) for c in ctx_lens]
    if sum(need) > n_blocks:
        raise ValueError("page pool too small")
    perm = np.random.default_rng(seed).permutation(n_blocks)
    table = np.full((len(need), max_blocks), -1, dtype=np.int32)
    o = 0
    for b, k in enumerate(need):
        table[b, :k] = perm[o : o + k]
        o += k
    return torch.from_numpy(table)
