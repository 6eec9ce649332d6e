"""BatchVerifier: the device-resident verify + accept + commit step.

This is the hot path of one speculative-decoding round for a fixed batch of
sequences (the work cudaforge/speculative.py:136-195 does per step, with the
reference's native acceptance semantics, speculative.cpp:50-103):

  1. target verify forward over R = K+1 rows per sequence (row 0 = the last
     emitted token, rows 1..K = the drafts) against the paged KV cache;
  2. fused acceptance sampling on the target / draft logits;
  3. commit: the page tables grow by num_accepted+1 tokens per sequence in
     batch order (cf_kvcache_append_batch, reference PagedKVCache semantics),
     the new tables go to the device, and cf_kv_commit copies the accepted
     rows' K/V of every layer into the pool.

All per-step state (token rows, positions, context lengths, block tables,
acceptance outputs) lives in preallocated device buffers; the only host
round trip is the num_accepted read-back the page tables need.  With
`use_graph=True` the step runs as two CUDA graphs (verify forward +
acceptance; KV commit + state update) captured on the second call, around
that read-back and the page-table upload; block tables therefore have a
fixed width (max_blocks_per_seq) on the device.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import ops
from .accept import AcceptResult, accept_sample
from .model import LlamaModel


class BatchVerifier:
    def __init__(self, model: LlamaModel, cache, seq_ids: Sequence[int], k: int, *, temperature: float = 1.0,
                 greedy: bool = False, eos_token_id: int = -1, max_blocks_per_seq: int = 512,
                 use_graph: bool = False, device_tables: bool = False, micro_batches: int = 1):
        """device_tables=True keeps the page tables on the device (DeviceTables):
        the page-table growth runs as a kernel inside the step, the whole step
        is one CUDA graph in graph mode and the host never waits for it; the
        host cache and ctx_host catch up lazily (sync() / check_status()).
        micro_batches=2 (tensor-parallel models, even batch): the two halves of the
        batch run on two CUDA streams with one process group each, so one half's
        all-reduces overlap the other half's kernels; acceptance and commit run
        per half (the same per-sequence results)."""
        self.model, self.cache = model, cache
        self.seq_ids = list(seq_ids)
        self.B, self.K, self.R = len(self.seq_ids), k, k + 1
        self.temperature, self.greedy, self.eos = max(temperature, 1e-5), greedy, eos_token_id
        dev = model.device
        B, R = self.B, self.R
        self.tokens = torch.zeros(B, R, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(B * R, dtype=torch.int32, device=dev)
        self.ctx = torch.zeros(B, dtype=torch.int32, device=dev)
        self.ctx_host = [0] * B
        self.ar = torch.arange(R, dtype=torch.int32, device=dev).view(1, R)
        self.tables_pinned = torch.full((B * max_blocks_per_seq,), -1, dtype=torch.int32).pin_memory()
        self.ctx_pinned = torch.zeros(B, dtype=torch.int32).pin_memory()
        self.cap = max_blocks_per_seq
        self.tables_fixed = torch.full((B, max_blocks_per_seq), -1, dtype=torch.int32).pin_memory()
        self.tables_dev = torch.full((B, max_blocks_per_seq), -1, dtype=torch.int32, device=dev)
        self.max_blocks = 0
        self.n_pinned = torch.zeros(B, dtype=torch.int32).pin_memory()
        self.res = AcceptResult(tokens=torch.zeros(B, R, dtype=torch.int32, device=dev),
                                num_accepted=torch.zeros(B, dtype=torch.int32, device=dev),
                                eos=torch.zeros(B, dtype=torch.bool, device=dev))
        from . import _lib as _l
        self.ws = torch.empty(_l.lib().cf_accept_workspace_bytes(B, k) + 256, dtype=torch.uint8, device=dev)
        from . import _lib
        self.st = _lib.DeviceStatus(dev)  # every kernel of the step records CF_ETIMEOUT / CF_ERANGE here
        self.status = self.st.dev
        self.model.buffers(B, R)
        # CUDA graphs (single-GPU models only: the TP collectives stay eager)
        self.use_graph = use_graph and getattr(model, "tp", None) is None
        self.graphs = None
        self.g_in = None          # static inputs of the captured forward: (draft tokens, draft logits, uniforms)
        self.start = torch.zeros(B, dtype=torch.int32, device=dev)
        self.kernels_per_step = 0
        self._keep = []
        self.device_tables = device_tables
        self.dtab = None
        self.mb = 1
        if micro_batches == 2 and getattr(model, "tp", None) is not None and B % 2 == 0:
            import torch.distributed as dist
            self.mb = 2
            # one communicator per stream: collectives of the two halves never share an NCCL queue
            self.groups = [dist.new_group(backend="nccl"), dist.new_group(backend="nccl")]
            self.side = torch.cuda.Stream(device=dev)
            self.ws_mb = [torch.empty(_l.lib().cf_accept_workspace_bytes(B // 2, k) + 256, dtype=torch.uint8,
                                      device=dev) for _ in range(2)]
            for t in (0, 1):
                model.buffers(B // 2, R, tag=t + 1)

    # ---- state ----
    def _upload_tables(self, stream=None):
        mb = self.cache.prepare_batch_into(self.seq_ids, self.tables_pinned, self.ctx_pinned)
        if mb > self.cap:
            raise ValueError(f"a sequence needs {mb} blocks > max_blocks_per_seq={self.cap}")
        self.max_blocks = mb
        # fixed-width device tables (-1 past each row's blocks): the captured graphs keep one stride
        self.tables_fixed[:, :mb].copy_(self.tables_pinned[: self.B * mb].view(self.B, mb))
        self.tables_dev.copy_(self.tables_fixed, non_blocking=True)

    def tables(self) -> torch.Tensor:
        return self.dtab.tables if self.dtab is not None else self.tables_dev

    def register_context(self, prompts, last_tokens, registered: bool = False) -> None:
        """Register each sequence's cached prompt (page tables) and set row 0
        (the last emitted token, not yet cached).  Pool contents come from a
        prefill or from fill_synthetic_kv().  registered=True adopts sequences
        already in the cache with exactly len(prompts[b]) tokens (e.g. after
        PagedRunner.prefill)."""
        if not registered:
            for sid, p in zip(self.seq_ids, prompts):
                self.cache.register_sequence_with_prefix(sid, p)
        self.ctx_host = [len(p) for p in prompts]
        self.ctx.copy_(torch.tensor(self.ctx_host, dtype=torch.int32))
        self.tokens[:, 0].copy_(torch.as_tensor(last_tokens, dtype=torch.int32))
        self._upload_tables()
        if self.device_tables:
            from .device_tables import DeviceTables
            self.dtab = DeviceTables(self.cache, self.seq_ids, self.cap, self.model.device)
            self.dtab.upload(self.ctx)


    def fill_synthetic_kv(self, gen: torch.Generator, std: float = 1.0) -> None:
        """Seeded random K/V for every pool slot (stands in for a prefill of
        random prompts: the verify step reads the same bytes either way)."""
        for pool in (self.cache.key_pool, self.cache.value_pool):
            flat = pool.view(-1)
            chunk = 1 << 28
            for i in range(0, flat.numel(), chunk):
                seg = flat[i: i + chunk]
                seg.copy_((torch.randn(seg.numel(), generator=gen, device=seg.device) * std).to(seg.dtype))

    # ---- the step ----
    def _halves(self):
        h = self.B // 2
        return [slice(0, h), slice(h, self.B)]

    def _forward_accept_mb(self, draft_tokens, draft_logits, uniforms, timer, max_context) -> AcceptResult:
        """Two micro-batches; concurrently on two streams unless a timer wants
        per-kernel events (then one after the other on the current stream)."""
        from .model import _null_timer
        B, R, Bm = self.B, self.R, self.B // 2
        main = torch.cuda.current_stream(self.model.device)
        self.tokens[:, 1:].copy_(draft_tokens)
        torch.add(self.ctx.view(B, 1), self.ar, out=self.pos.view(B, R))
        concurrent = timer is None
        if concurrent:
            self.side.wait_stream(main)
        mctx = max_context if max_context is not None else max(self.ctx_host)
        for i, sl in enumerate(self._halves()):
            st = self.side if (concurrent and i == 1) else main
            with torch.cuda.stream(st):
                lg = self.model.forward_rows(self.cache, self.tokens[sl], self.pos[sl.start * R: sl.stop * R],
                                             self.tables()[sl], self.ctx[sl], mctx, status=self.status, timer=timer,
                                             bufs_tag=i + 1, group=self.groups[i])
                part = AcceptResult(tokens=self.res.tokens[sl], num_accepted=self.res.num_accepted[sl],
                                    eos=self.res.eos[sl])
                with (timer or _null_timer)("accept"):
                    accept_sample(None if draft_logits is None else draft_logits[sl], lg.view(Bm, R, -1),
                                  draft_tokens[sl], None if uniforms is None else uniforms[sl],
                                  temperature=self.temperature, eos_token_id=self.eos, greedy=self.greedy,
                                  workspace=self.ws_mb[i], out=part)
        if concurrent:
            main.wait_stream(self.side)
        return self.res

    def _forward_accept(self, draft_tokens, draft_logits, uniforms, timer=None, max_context=None) -> AcceptResult:
        if self.mb == 2:
            return self._forward_accept_mb(draft_tokens, draft_logits, uniforms, timer, max_context)
        B, R = self.B, self.R
        self.tokens[:, 1:].copy_(draft_tokens)
        torch.add(self.ctx.view(B, 1), self.ar, out=self.pos.view(B, R))
        logits = self.model.forward_rows(self.cache, self.tokens, self.pos, self.tables(), self.ctx,
                                         max_context if max_context is not None else max(self.ctx_host),
                                         status=self.status, timer=timer)
        from .model import _null_timer
        with (timer or _null_timer)("accept"):
            return accept_sample(draft_logits, logits.view(B, R, -1), draft_tokens, uniforms,
                                 temperature=self.temperature, eos_token_id=self.eos, greedy=self.greedy,
                                 workspace=self.ws, out=self.res)

    def _commit_update(self, res: AcceptResult, timer=None) -> None:
        from .model import _null_timer
        B, R = self.B, self.R
        bf = self.model.buffers(B, R)
        self.start.copy_(self.ctx)
        with (timer or _null_timer)("commit"):
            if self.dtab is not None:  # the page tables grow on the device first
                self.dtab.append(res.num_accepted, self.ctx, 1, status=self.status)
            if self.mb == 2:  # each half's K/V rows are in its own buffer set
                for i, sl in enumerate(self._halves()):
                    bfi = self.model.buffers(self.B // 2, R, tag=i + 1)
                    ops.kv_commit(self.cache, bfi["k_new"], bfi["v_new"], res.num_accepted[sl], self.start[sl],
                                  self.tables()[sl], n_commit_add=1, status=self.status)
            else:
                ops.kv_commit(self.cache, bf["k_new"], bf["v_new"], res.num_accepted, self.start, self.tables(),
                              n_commit_add=1, status=self.status)
        # next round: context grows by n, row 0 = the final token
        self.ctx.add_(res.num_accepted.clamp_min(0) + 1)
        idx = res.num_accepted.clamp_min(0).long().view(B, 1)
        self.tokens[:, :1].copy_(res.tokens.gather(1, idx))

    def _capture(self, draft_tokens, draft_logits, uniforms) -> None:
        from . import gemm as _gemm
        g_tok = draft_tokens.to(dtype=torch.int32).clone()
        g_uni = None if uniforms is None else uniforms.clone()
        self.g_in = (g_tok, draft_logits, g_uni)  # draft logits are captured by address
        max_ctx = self.cap * self.cache.get_config().block_size
        if self.dtab is not None:  # the whole step, page-table growth included, is one graph
            g1 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g1):
                self._forward_accept(g_tok, draft_logits, g_uni, max_context=max_ctx)
                self._commit_update(self.res)
            self.graphs = (g1, None)
        else:
            g1, g2 = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            with torch.cuda.graph(g1):
                self._forward_accept(g_tok, draft_logits, g_uni, max_context=max_ctx)
            with torch.cuda.graph(g2):
                self._commit_update(self.res)
            self.graphs = (g1, g2)
        # hold every workspace the captured kernels address: the capture plans for
        # max_context, which can grow a cached workspace inside the capture, and a
        # later call may replace the cache entry while this graph still uses it
        self._keep = [dict(ops._Ws.bufs), dict(_gemm._Ws.bufs)]

    @torch.no_grad()
    def step(self, draft_tokens: torch.Tensor, draft_logits: Optional[torch.Tensor],
             uniforms: Optional[torch.Tensor], timer=None) -> AcceptResult:
        """draft_tokens [B, K] int32 and draft_logits [B, K, V] (device),
        uniforms [B, K+1] fp32 (device; unused when greedy).  Returns the
        acceptance result (device tensors, reused across steps).  In graph
        mode the captured forward reads the draft logits at the address seen
        at capture; a different tensor is copied there first."""
        from . import _lib
        graph = self.use_graph and timer is None
        l0 = _lib.LAUNCHES[0]
        if graph and self.graphs is None and self.kernels_per_step:
            self._capture(draft_tokens, draft_logits, uniforms)
            _lib.LAUNCHES[0] = l0  # capture records launches without running them
        if graph and self.graphs is not None:
            g_tok, g_dlog, g_uni = self.g_in
            g_tok.copy_(draft_tokens)
            if g_uni is not None:
                g_uni.copy_(uniforms)
            if draft_logits is not None and draft_logits.data_ptr() != g_dlog.data_ptr():
                g_dlog.copy_(draft_logits)
            self.graphs[0].replay()
            res = self.res
        elif self.dtab is not None:
            max_ctx = self.cap * self.cache.get_config().block_size
            res = self._forward_accept(draft_tokens, draft_logits, uniforms, timer=timer, max_context=max_ctx)
        else:
            res = self._forward_accept(draft_tokens, draft_logits, uniforms, timer=timer)
        if self.dtab is not None:
            return self._finish_device_step(res, graph, timer, l0)
        self.n_pinned.copy_(res.num_accepted, non_blocking=True)
        self.st.snapshot()
        torch.cuda.current_stream(self.model.device).synchronize()
        # a bounded wait that ran out or a bad page id makes the step's results meaningless
        self.st.check("BatchVerifier.step")
        n = [max(0, int(x)) + 1 for x in self.n_pinned.tolist()]
        self.cache.append_batch(self.seq_ids, n)
        self._upload_tables()
        if graph and self.graphs is not None:
            self.graphs[1].replay()
            _lib.count(self.kernels_per_step)
        else:
            self._commit_update(res, timer=timer)
            if not self.kernels_per_step:
                self.kernels_per_step = _lib.LAUNCHES[0] - l0
        self.ctx_host = [c + x for c, x in zip(self.ctx_host, n)]
        return res

    def _finish_device_step(self, res, graph, timer, l0) -> AcceptResult:
        from . import _lib
        if graph and self.graphs is not None:
            _lib.count(self.kernels_per_step)
        else:
            self._commit_update(res, timer=timer)
            if not self.kernels_per_step:
                self.kernels_per_step = _lib.LAUNCHES[0] - l0
        # host bookkeeping trails the device: queue this step's counts, replay finished steps
        self.dtab.record(res.num_accepted, 1)
        self._catch_up(False)
        # errors of earlier steps surface here (the status copy lands asynchronously)
        self.st.check("BatchVerifier.step")
        self.st.snapshot()
        return res

    def _catch_up(self, block: bool) -> None:
        if self.dtab.catch_up(block_all=block):
            self.ctx_host = self._host_ctx()  # the host cache now holds every replayed step

    def _host_ctx(self):
        tables = torch.zeros(self.B * self.cap, dtype=torch.int32)
        ctx = torch.zeros(self.B, dtype=torch.int32)
        self.cache.prepare_batch_into(self.seq_ids, tables, ctx)
        return ctx.tolist()

    def sync(self) -> None:
        """Device-table mode: wait for every queued step and bring the host
        cache (page tables, ctx_host) up to date."""
        if self.dtab is not None:
            self._catch_up(True)

    def check_status(self) -> None:
        """Synchronise and raise DeviceError if a kernel since the last check
        (e.g. the last step's KV commit) recorded an error."""
        self.sync()
        self.st.sync_check("BatchVerifier")
