"""Llama-shaped target / draft models for the verify forward (random init).

The reference has no model (ModelRunner::step emits `last + 1`,
csrc/src/engine/model_runner.cpp:106-173); its speculative engine takes any
runner with `.forward(input_ids, kv_cache_handles) -> logits[B, S, V]`
(cudaforge/speculative.py:30-55).  This module provides that runner, built
from this library's kernels only: per layer RMSNorm -> QKV (W4A16 or dense) ->
RoPE + K/V scatter -> paged verify attention -> O-proj (+residual, fused in
the GEMM epilogue) -> RMSNorm -> gate|up -> SwiGLU -> down (+residual); final
RMSNorm -> lm_head.  Only the R new rows of each sequence are computed; the
cached context is read from the paged pool.
"""
from __future__ import annotations

import dataclasses
from typing import List, Optional

import torch

from . import ops
from .gemm import dense_gemm, w4a16_gemm


@dataclasses.dataclass(frozen=True)
class LlamaConfig:
    layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_base: float = 10000.0
    eps: float = 1e-6
    quant: str = "int4"          # "int4" (W4A16, group 128) or "dense"
    dtype: torch.dtype = torch.bfloat16

    @property
    def qkv_dim(self):
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim

    def linear_shapes(self):
        """(name, N, K) of every per-layer projection plus the lm_head."""
        d = self.d_model
        return [("qkv", self.qkv_dim, d), ("o", d, self.n_heads * self.head_dim), ("gate_up", 2 * self.ffn, d),
                ("down", d, self.ffn)]

    def gemm_flops(self, tokens: int) -> float:
        per_layer = sum(2.0 * n * k for _, n, k in self.linear_shapes())
        return tokens * (self.layers * per_layer + 2.0 * self.vocab * self.d_model)

    def weight_bytes(self) -> float:
        """Bytes of the GEMM weights as stored (INT4 + fp16 group scales, or 16-bit dense)."""
        params = self.layers * sum(n * k for _, n, k in self.linear_shapes()) + self.vocab * self.d_model
        return params * (0.5 + 2.0 / 128) if self.quant == "int4" else params * 2.0


# BASELINE configurations
TINY_TARGET = LlamaConfig(4, 512, 8, 8, 64, 1408, 32000, quant="dense", dtype=torch.float16)
TINY_DRAFT = LlamaConfig(1, 256, 4, 4, 64, 704, 32000, quant="dense", dtype=torch.float16)
LLAMA_8B = LlamaConfig(32, 4096, 32, 8, 128, 14336, 128256)
DRAFT_1B = LlamaConfig(16, 2048, 32, 8, 64, 8192, 128256)
LLAMA_70B = LlamaConfig(80, 8192, 64, 8, 128, 28672, 128256)


class Linear:
    """One projection y = x W^T: INT4 (kernel-packed [K/8, N] + fp16 scales
    [K/128, N]) or dense 16-bit [N, K]."""

    def __init__(self, n: int, k: int, cfg: LlamaConfig, gen: torch.Generator, device, std=0.02,
                 int4_scale=0.002):
        self.n, self.k, self.quant = n, k, cfg.quant
        if cfg.quant == "int4":
            # every nibble uniform in 0..15 (value = nibble - 8 in [-8, 7]); uniform random
            # words are uniform in any nibble order, so they serve directly as kernel-packed weights
            self.wq = torch.randint(-2**31, 2**31 - 1, (k // 8, n), generator=gen, device=device, dtype=torch.int32)
            self.scales = (torch.randn(k // 128, n, generator=gen, device=device).abs() * int4_scale).to(torch.float16)
        else:
            self.w = (torch.randn(n, k, generator=gen, device=device) * std).to(cfg.dtype)

    @classmethod
    def _wrap(cls, quant, n, k, wq=None, scales=None, w=None):
        lin = cls.__new__(cls)
        lin.n, lin.k, lin.quant = n, k, quant
        if quant == "int4":
            lin.wq, lin.scales = wq.contiguous(), scales.contiguous()
        else:
            lin.w = w.contiguous()
        return lin

    def take_columns(self, cols: torch.Tensor, pad_to: int = 0) -> "Linear":
        """Column-parallel shard: output features `cols` (zero columns appended
        up to pad_to, for the GEMM's 128-wide N tiles)."""
        n = max(int(cols.numel()), pad_to)
        if self.quant == "int4":
            wq, sc = self.wq[:, cols], self.scales[:, cols]
            if n > cols.numel():  # nibble 8 is zero; scale 0 makes the padded outputs exactly 0
                wq = torch.cat([wq, torch.full((wq.shape[0], n - cols.numel()), -2004318072, dtype=wq.dtype,
                                                device=wq.device)], 1)
                sc = torch.cat([sc, torch.zeros((sc.shape[0], n - cols.numel()), dtype=sc.dtype, device=sc.device)], 1)
            return Linear._wrap("int4", n, self.k, wq=wq, scales=sc)
        w = self.w[cols]
        if n > cols.numel():
            w = torch.cat([w, torch.zeros((n - cols.numel(), self.k), dtype=w.dtype, device=w.device)], 0)
        return Linear._wrap(self.quant, n, self.k, w=w)

    def take_rows(self, k0: int, k1: int) -> "Linear":
        """Row-parallel shard: input features [k0, k1) (multiples of 128)."""
        if self.quant == "int4":
            return Linear._wrap("int4", self.n, k1 - k0, wq=self.wq[k0 // 8: k1 // 8], scales=self.scales[k0 // 128: k1 // 128])
        return Linear._wrap(self.quant, self.n, k1 - k0, w=self.w[:, k0:k1])

    def __call__(self, x, out=None, residual=None, workspace=None, partials=False, status=None):
        """y = x W^T (+ residual) into `out`; with partials=True a K-split plan returns
        (fp32 partials, splits) for an ops.splitk_* consumer instead (out untouched)."""
        if self.quant == "int4":
            return w4a16_gemm(x, self.wq, self.scales, out=out, residual=residual, workspace=workspace,
                              partials=partials, status=status)
        return dense_gemm(x, self.w, out=out, residual=residual, workspace=workspace, partials=partials,
                          status=status)


@dataclasses.dataclass(frozen=True)
class TensorParallel:
    """Megatron-style tensor parallelism over `size` ranks (one process per
    GPU, NCCL): QKV and gate|up column-parallel (heads / FFN features split),
    O and down row-parallel with an all-reduce of the residual stream after
    each, lm_head column-parallel over the vocabulary with an all-gather of
    the logits (acceptance then runs on the full rows, identically on every
    rank).  `group` is a torch.distributed process group (None = default)."""

    rank: int
    size: int
    group: object = None


def tp_local_config(cfg: LlamaConfig, size: int) -> LlamaConfig:
    """The per-rank shapes of a `size`-way tensor-parallel model."""
    if size == 1:
        return cfg
    if cfg.n_heads % size or cfg.n_kv_heads % size or cfg.ffn % size or cfg.vocab % size:
        raise ValueError(f"{cfg} does not split {size} ways")
    if (cfg.n_heads // size) * cfg.head_dim % 128 or (cfg.ffn // size) % 128:
        raise ValueError("row-parallel K shards must be multiples of 128 (INT4 groups / GEMM tiles)")
    return dataclasses.replace(cfg, n_heads=cfg.n_heads // size, n_kv_heads=cfg.n_kv_heads // size,
                               ffn=cfg.ffn // size, vocab=cfg.vocab // size)


def tp_columns(cfg: LlamaConfig, name: str, rank: int, size: int, device) -> torch.Tensor:
    """Output-feature indices of rank `rank`'s column-parallel shard."""
    D = cfg.head_dim
    ar = lambda a, b: torch.arange(a, b, device=device)  # noqa: E731
    if name == "qkv":
        hq, hk = cfg.n_heads // size, cfg.n_kv_heads // size
        q0, k0, v0 = 0, cfg.n_heads * D, (cfg.n_heads + cfg.n_kv_heads) * D
        return torch.cat([ar(q0 + rank * hq * D, q0 + (rank + 1) * hq * D),
                          ar(k0 + rank * hk * D, k0 + (rank + 1) * hk * D),
                          ar(v0 + rank * hk * D, v0 + (rank + 1) * hk * D)])
    if name == "gate_up":
        f = cfg.ffn // size
        return torch.cat([ar(rank * f, (rank + 1) * f), ar(cfg.ffn + rank * f, cfg.ffn + (rank + 1) * f)])
    if name == "lm_head":
        v = cfg.vocab // size
        return ar(rank * v, (rank + 1) * v)
    raise KeyError(name)


def tp_rows(cfg: LlamaConfig, name: str, rank: int, size: int):
    """Input-feature range [k0, k1) of rank `rank`'s row-parallel shard."""
    if name == "o":
        w = cfg.n_heads // size * cfg.head_dim
    elif name == "down":
        w = cfg.ffn // size
    else:
        raise KeyError(name)
    return rank * w, (rank + 1) * w


class _NullCtx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def _null_timer(kind):
    return _NullCtx()


class LlamaModel:
    """Random-init Llama-shaped model (seeded), resident on one device."""

    def __init__(self, cfg: LlamaConfig, device="cuda", seed: int = 0, tp: Optional[TensorParallel] = None):
        """With `tp`, every rank draws the full model from the same seeded
        stream (so a TP model equals the single-GPU model of that seed) and
        keeps its shards; `cfg` stays the global shape, `lcfg` is per rank."""
        self.cfg = cfg
        self.tp = tp if (tp is not None and tp.size > 1) else None
        self.lcfg = tp_local_config(cfg, self.tp.size) if self.tp else cfg
        self.device = torch.device(device)
        g = torch.Generator(device=self.device).manual_seed(seed)
        dt = cfg.dtype
        self.embed = (torch.randn(cfg.vocab, cfg.d_model, generator=g, device=self.device) * 0.02).to(dt)
        self.layers = []
        for _ in range(cfg.layers):
            lay = {
                "attn_norm": (torch.randn(cfg.d_model, generator=g, device=self.device) * 0.02 + 1.0).to(dt),
                "ffn_norm": (torch.randn(cfg.d_model, generator=g, device=self.device) * 0.02 + 1.0).to(dt),
            }
            for name, n, k in cfg.linear_shapes():
                lay[name] = self._shard(name, Linear(n, k, cfg, g, self.device))
            self.layers.append(lay)
        self.final_norm = (torch.randn(cfg.d_model, generator=g, device=self.device) * 0.02 + 1.0).to(dt)
        self.lm_head = self._shard("lm_head", Linear(cfg.vocab, cfg.d_model, cfg, g, self.device))
        self._bufs = {}
        self.fuse_splitk = True  # split-K reductions fused into the consuming op (bit-identical)

    def _shard(self, name: str, lin: Linear) -> Linear:
        if self.tp is None:
            return lin
        r, n = self.tp.rank, self.tp.size
        if name in ("o", "down"):
            return lin.take_rows(*tp_rows(self.cfg, name, r, n))
        cols = tp_columns(self.cfg, name, r, n, lin.wq.device if lin.quant == "int4" else lin.w.device)
        pad = ((cols.numel() + 127) // 128) * 128 if name == "lm_head" else 0
        return lin.take_columns(cols, pad_to=pad)

    def _all_reduce(self, x: torch.Tensor, group=None) -> None:
        import torch.distributed as dist
        dist.all_reduce(x, group=group if group is not None else self.tp.group)

    # ---- scratch buffers, sized once per (B, R) and reused (graph friendly) ----
    def buffers(self, B: int, R: int, tag: int = 0):
        """`tag` keeps separate buffer sets for work of the same shape that runs
        concurrently (micro-batches on two streams)."""
        key = (B, R) if tag == 0 else (B, R, tag)
        if key not in self._bufs:
            c, M, dev, dt = self.lcfg, B * R, self.device, self.cfg.dtype
            self._bufs[key] = {
                "h": torch.empty(M, c.d_model, dtype=dt, device=dev),
                "xn": torch.empty(M, c.d_model, dtype=dt, device=dev),
                "qkv": torch.empty(M, c.qkv_dim, dtype=dt, device=dev),
                "attn": torch.empty(M, c.n_heads * c.head_dim, dtype=dt, device=dev),
                "gu": torch.empty(M, 2 * c.ffn, dtype=dt, device=dev),
                "act": torch.empty(M, c.ffn, dtype=dt, device=dev),
                "logits": torch.empty(M, self.cfg.vocab, dtype=dt, device=dev),
                "k_new": torch.empty(c.layers, B, R, c.n_kv_heads, c.head_dim, dtype=dt, device=dev),
                "v_new": torch.empty(c.layers, B, R, c.n_kv_heads, c.head_dim, dtype=dt, device=dev),
            }
            if self.tp is not None:
                n = self.lm_head.n
                self._bufs[key]["logits_local"] = torch.empty(M, n, dtype=dt, device=dev)
                self._bufs[key]["logits_gather"] = torch.empty(self.tp.size, M, n, dtype=dt, device=dev)
        return self._bufs[key]

    def forward_rows(self, cache, tokens: torch.Tensor, positions: torch.Tensor, block_tables: torch.Tensor,
                     context_lens: torch.Tensor, max_context: int, tree_mask: Optional[torch.Tensor] = None,
                     status: Optional[torch.Tensor] = None, timer=None, bufs_tag: int = 0,
                     group=None) -> torch.Tensor:
        """tokens [B, R] int32 (row 0 = last emitted token, then drafts / tree
        nodes), positions [B*R] int32, block tables / context lengths from the
        cache (context = tokens already in the pool).  Returns logits [B*R, V]
        (a reused buffer) and leaves this step's K/V rows in buffers()["k_new"/"v_new"].
        bufs_tag selects the buffer set (buffers(B, R, bufs_tag)); group overrides the
        tensor-parallel process group of the collectives (one per concurrent stream).
        `timer(kind)` (optional) returns a context manager wrapped around each
        launch group ("gemm", "attn", "other") for per-kernel timing."""
        c = self.lcfg
        tp = self.tp
        B, R = tokens.shape
        bf = self.buffers(B, R, bufs_tag)
        h, xn, qkv, attn, gu, act = bf["h"], bf["xn"], bf["qkv"], bf["attn"], bf["gu"], bf["act"]
        T = timer or _null_timer
        # Split-K GEMMs hand their fp32 partials to the next op, which forms the GEMM output
        # exactly as the reduction would and fuses its own work (RoPE, residual + RMSNorm,
        # SwiGLU): no reduction launch.  Not under TP, where an all-reduce sits in between.
        fuse = tp is None and self.fuse_splitk
        split = lambda r: isinstance(r, tuple)  # noqa: E731
        with T("other"):
            ops.embedding(tokens.reshape(-1), self.embed, out=h)
        pending = None  # partials of the previous down projection (+ residual h) not yet reduced
        for li, lay in enumerate(self.layers):
            with T("other"):
                if pending is not None:
                    ops.splitk_rmsnorm(pending, lay["attn_norm"], y=h, out=xn, residual=h, eps=c.eps)
                else:
                    ops.rmsnorm(h, lay["attn_norm"], c.eps, out=xn)
            with T("gemm"):
                r = lay["qkv"](xn, out=qkv, partials=fuse, status=status)
            with T("other"):
                if split(r):
                    ops.splitk_rope_qkv(r, qkv, positions, c.n_heads, c.n_kv_heads, c.head_dim, bf["k_new"][li],
                                        bf["v_new"][li], base=c.rope_base)
                else:
                    ops.rope_qkv(qkv, positions, c.n_heads, c.n_kv_heads, c.head_dim, bf["k_new"][li],
                                 bf["v_new"][li], base=c.rope_base)
            with T("attn"):
                ops.verify_attention(cache, li, qkv, bf["k_new"][li], bf["v_new"][li], block_tables, context_lens,
                                     max_context, rows=R, num_q_heads=c.n_heads, out=attn, tree_mask=tree_mask,
                                     status=status)
            with T("gemm"):  # TP: rank 0 carries the residual, the all-reduce sums the partial outputs
                r = lay["o"](attn, out=h, residual=h if tp is None or tp.rank == 0 else None, partials=fuse,
                               status=status)
            if tp is not None:
                with T("comm"):
                    self._all_reduce(h, group)
            with T("other"):
                if split(r):
                    ops.splitk_rmsnorm(r, lay["ffn_norm"], y=h, out=xn, residual=h, eps=c.eps)
                else:
                    ops.rmsnorm(h, lay["ffn_norm"], c.eps, out=xn)
            with T("gemm"):
                r = lay["gate_up"](xn, out=gu, partials=fuse, status=status)
            with T("other"):
                if split(r):
                    ops.splitk_silu_mul(r, c.ffn, out=act)
                else:
                    ops.silu_mul(gu, c.ffn, out=act)
            with T("gemm"):
                r = lay["down"](act, out=h, residual=h if tp is None or tp.rank == 0 else None, partials=fuse,
                                  status=status)
            if tp is not None:
                with T("comm"):
                    self._all_reduce(h, group)
            pending = r if split(r) else None
        with T("other"):
            if pending is not None:
                ops.splitk_rmsnorm(pending, self.final_norm, y=h, out=xn, residual=h, eps=c.eps)
            else:
                ops.rmsnorm(h, self.final_norm, c.eps, out=xn)
        if tp is None:
            with T("gemm"):
                self.lm_head(xn, out=bf["logits"], status=status)
            return bf["logits"]
        import torch.distributed as dist
        with T("gemm"):
            self.lm_head(xn, out=bf["logits_local"], status=status)
        with T("comm"):
            dist.all_gather_into_tensor(bf["logits_gather"], bf["logits_local"],
                                        group=group if group is not None else tp.group)
            v = c.vocab  # this rank's true vocabulary slice (the shard is padded to 128 columns)
            bf["logits"].view(-1, tp.size, v).copy_(bf["logits_gather"][:, :, :v].permute(1, 0, 2))
        return bf["logits"]

    def make_cache(self, total_blocks: int, max_batch: int = 256, max_blocks_per_seq: int = 512,
                   prefix_caching: bool = False):
        from .kv_cache import KVCacheConfig, PagedKVCache
        c = self.lcfg
        kc = KVCacheConfig(num_layers=c.layers, num_kv_heads=c.n_kv_heads, head_dim=c.head_dim, block_size=16,
                           element_size_bytes=2, total_gpu_blocks=total_blocks,
                           enable_prefix_caching=prefix_caching, max_supported_batch_size=max_batch,
                           max_blocks_per_sequence=max_blocks_per_seq)
        return PagedKVCache(kc, dtype=c.dtype)


def dequant_int4_kernel_packed(wq: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 [K, N] weights of a kernel-packed INT4 Linear (for the fp32 oracle):
    kernel nibble position p holds k = 2p (p < 4) or 2(p-4)+1 (p >= 4)."""
    Kp, N = wq.shape
    w = wq.to(torch.int64) & 0xFFFFFFFF
    order = [0, 2, 4, 6, 1, 3, 5, 7]
    q = torch.empty(Kp, 8, N, dtype=torch.float32, device=wq.device)
    for pos in range(8):
        q[:, order[pos], :] = ((w >> (4 * pos)) & 0xF).float()
    q = q.reshape(Kp * 8, N)
    return (q - 8.0) * scales.float().repeat_interleave(128, dim=0)


def linear_weight_fp32(lin: Linear) -> torch.Tensor:
    """[N, K] fp32 view of a projection's weights (exact dequantisation)."""
    if lin.quant == "int4":
        return dequant_int4_kernel_packed(lin.wq, lin.scales).T.contiguous()
    return lin.w.float()
