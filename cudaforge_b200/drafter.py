"""BatchDrafter: the device-resident K-step chain draft loop.

The reference drafts one token at a time from the host: per step it runs the
draft runner over the whole prefix, takes the last row, applies
softmax(logits / T) and samples (cudaforge/speculative.py:113-123).  Here the
K steps of a round run back to back on the device for a fixed batch, with no
host round trip inside the loop, and can be replayed as one CUDA graph:

  step 0    rows (token at position P-1, last emitted token at P), R = 2,
            attending to the pool positions < P-1;
  step j>0  row (draft token j-1 at position P+j), R = 1, attending to the
            pool positions < P+j;

where P is the position of the last emitted token.  Every step writes its
rows' K/V straight into the draft model's paged pool (cf_kv_commit), so the
next step reads them from there, and samples draft token j from its last row
with the acceptance kernel's K = 0 path (inverse CDF of softmax(row / T) with
uniform U[b, j]; argmax when greedy).

Step 0 recomputes position P-1 on purpose: when a round accepted all K drafts,
the draft model never saw draft K-1 (it is at P-1 in the next round), and the
two-row step covers that case and the others with one rectangular launch.

Page tables follow the reference PagedKVCache (append_tokens in batch order):
the draft cache holds P + K tokens per sequence, i.e. the tables always cover
the K positions a round writes; after acceptance advance() appends the n+1
emitted tokens.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from . import ops
from .accept import AcceptResult, accept_sample
from .model import LlamaModel


class BatchDrafter:
    def __init__(self, model: LlamaModel, cache, seq_ids: Sequence[int], k: int, *, temperature: float = 1.0,
                 greedy: bool = False, max_blocks_per_seq: int = 512, use_graph: bool = False):
        if k < 1:
            raise ValueError("a draft round needs k >= 1")
        self.model, self.cache = model, cache
        self.seq_ids = list(seq_ids)
        self.B, self.K = len(self.seq_ids), k
        self.temperature, self.greedy = max(temperature, 1e-5), greedy
        dev = model.device
        B, V = self.B, model.cfg.vocab
        self.last = torch.zeros(B, dtype=torch.int32, device=dev)   # last emitted token (position P)
        self.prev = torch.zeros(B, dtype=torch.int32, device=dev)   # token at position P-1
        self.base = torch.zeros(B, dtype=torch.int32, device=dev)   # P
        self.rows0 = torch.zeros(B, 2, dtype=torch.int32, device=dev)
        self.pos0 = torch.zeros(B * 2, dtype=torch.int32, device=dev)
        self.ctx0 = torch.zeros(B, dtype=torch.int32, device=dev)
        self.rows1 = torch.zeros(B, 1, dtype=torch.int32, device=dev)
        self.pos1 = torch.zeros(B, dtype=torch.int32, device=dev)
        self.ar2 = torch.tensor([[-1, 0]], dtype=torch.int32, device=dev)
        self.zero_n = torch.zeros(B, dtype=torch.int32, device=dev)
        self.tokens = torch.zeros(B, k, dtype=torch.int32, device=dev)
        self.logits = torch.zeros(B, k, V, dtype=model.cfg.dtype, device=dev)
        self.uniforms = torch.zeros(k, B, 1, dtype=torch.float32, device=dev)  # [j] = U[:, j], contiguous
        self.empty = torch.zeros(B, 0, dtype=torch.int32, device=dev)
        self.res = AcceptResult(tokens=torch.zeros(B, 1, dtype=torch.int32, device=dev),
                                num_accepted=torch.zeros(B, dtype=torch.int32, device=dev),
                                eos=torch.zeros(B, dtype=torch.bool, device=dev))
        from . import _lib as _l
        self.ws = torch.empty(_l.lib().cf_accept_workspace_bytes(B, 0) + 256, dtype=torch.uint8, device=dev)
        from . import _lib
        self.st = _lib.DeviceStatus(dev)
        self.status = self.st.dev
        self.cap = max_blocks_per_seq
        self.tables_pinned = torch.full((B * max_blocks_per_seq,), -1, dtype=torch.int32).pin_memory()
        self.ctx_pinned = torch.zeros(B, dtype=torch.int32).pin_memory()
        self.tables_fixed = torch.full((B, max_blocks_per_seq), -1, dtype=torch.int32).pin_memory()
        self.tables_dev = torch.full((B, max_blocks_per_seq), -1, dtype=torch.int32, device=dev)
        self.base_host = [0] * B
        self.uploaded = None  # event after the last table upload (the pinned staging is reused)
        model.buffers(B, 2)
        model.buffers(B, 1)
        self.use_graph = use_graph and getattr(model, "tp", None) is None
        self.graph = None
        self.calls = 0
        self.kernels_per_round = 0
        self._keep = []

    # ---- state ----
    def _upload_tables(self) -> None:
        if self.uploaded is not None:
            self.uploaded.synchronize()  # the previous copy out of the pinned staging has finished
        mb = self.cache.prepare_batch_into(self.seq_ids, self.tables_pinned, self.ctx_pinned)
        if mb > self.cap:
            raise ValueError(f"a sequence needs {mb} blocks > max_blocks_per_seq={self.cap}")
        self.tables_fixed[:, :mb].copy_(self.tables_pinned[: self.B * mb].view(self.B, mb))
        self.tables_dev.copy_(self.tables_fixed, non_blocking=True)
        self.uploaded = torch.cuda.Event()
        self.uploaded.record()

    def register_context(self, prompts, last_tokens, registered: bool = False) -> None:
        """prompts[b]: the tokens whose K/V are (or will be, by a prefill or a
        synthetic fill) in the draft pool, at least one per sequence;
        last_tokens[b]: the last emitted token (position len(prompts[b])).
        registered=True adopts sequences already in the cache with exactly
        len(prompts[b]) tokens (e.g. after PagedRunner.prefill)."""
        if any(len(p) < 1 for p in prompts):
            raise ValueError("every sequence needs at least one cached token")
        if not registered:
            for sid, p in zip(self.seq_ids, prompts):
                self.cache.register_sequence_with_prefix(sid, p)
        self.cache.append_batch(self.seq_ids, [self.K] * self.B)  # room for the round's K positions
        self.base_host = [len(p) for p in prompts]
        self.base.copy_(torch.tensor(self.base_host, dtype=torch.int32))
        self.prev.copy_(torch.tensor([p[-1] for p in prompts], dtype=torch.int32))
        self.last.copy_(torch.as_tensor(last_tokens, dtype=torch.int32))
        self._upload_tables()

    # ---- the round ----
    def _sample(self, lg: torch.Tensor, j: int) -> None:
        u = None if self.greedy else self.uniforms[j]
        accept_sample(None, lg, self.empty, u, temperature=self.temperature, greedy=self.greedy,
                      workspace=self.ws, out=self.res)
        self.tokens[:, j: j + 1].copy_(self.res.tokens)
        self.logits[:, j: j + 1].copy_(lg)

    def _round(self, max_context: int) -> None:
        B, m = self.B, self.model
        tables = self.tables_dev
        bf2, bf1 = m.buffers(B, 2), m.buffers(B, 1)
        # step 0: rows (P-1, P)
        self.rows0[:, 0].copy_(self.prev)
        self.rows0[:, 1].copy_(self.last)
        torch.add(self.base.view(B, 1), self.ar2, out=self.pos0.view(B, 2))
        torch.sub(self.base, 1, out=self.ctx0)
        lg = m.forward_rows(self.cache, self.rows0, self.pos0, tables, self.ctx0, max_context, status=self.status)
        ops.kv_commit(self.cache, bf2["k_new"], bf2["v_new"], self.zero_n, self.ctx0, tables, n_commit_add=2,
                      status=self.status)
        self._sample(lg.view(B, 2, -1)[:, 1:2], 0)
        # steps 1..K-1: one row at P + j
        for j in range(1, self.K):
            self.rows1.copy_(self.tokens[:, j - 1: j])
            torch.add(self.base, j, out=self.pos1)
            lg = m.forward_rows(self.cache, self.rows1, self.pos1, tables, self.pos1, max_context,
                                status=self.status)
            ops.kv_commit(self.cache, bf1["k_new"], bf1["v_new"], self.zero_n, self.pos1, tables, n_commit_add=1,
                          status=self.status)
            self._sample(lg.view(B, 1, -1), j)

    @torch.no_grad()
    def draft(self, uniforms: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """One round: K draft tokens per sequence.  uniforms [B, K] fp32 in
        [0, 1) (device; unused when greedy): U[b, j] draws draft token j.
        Returns (draft_tokens [B, K] int32, draft_logits [B, K, V]) --
        buffers reused by the next round."""
        from . import _lib
        if not self.greedy:
            if uniforms is None or tuple(uniforms.shape) != (self.B, self.K):
                raise ValueError(f"uniforms must be [{self.B}, {self.K}]")
            self.uniforms.copy_(uniforms.t().unsqueeze(-1))
        l0 = _lib.LAUNCHES[0]
        if self.graph is not None:
            self.graph.replay()
            _lib.count(self.kernels_per_round)
        elif self.use_graph and self.calls >= 1:
            from . import gemm as _gemm
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._round(self.cap * self.cache.get_config().block_size)
            self.graph = g
            # workspaces the graph addresses, taken after capture (a capture can grow them)
            self._keep = [dict(ops._Ws.bufs), dict(_gemm._Ws.bufs)]
            _lib.LAUNCHES[0] = l0  # capture records launches without running them
            g.replay()
            _lib.count(self.kernels_per_round)
        else:
            self._round(max(self.base_host) + self.K)
            self.kernels_per_round = _lib.LAUNCHES[0] - l0
        self.calls += 1
        self.st.snapshot()  # checked by advance(), after the verifier's step has synchronised the stream
        return self.tokens, self.logits

    @torch.no_grad()
    def advance(self, res: AcceptResult, n_emitted: Sequence[int]) -> None:
        """After acceptance: res.tokens[b, :n] are the accepted drafts and
        res.tokens[b, n] the final token (n = res.num_accepted[b]);
        n_emitted[b] = n + 1 on the host (the value the target's page tables
        already needed).  Grows the draft tables by n + 1 tokens per sequence
        and moves (P-1, P) to the last two emitted tokens."""
        B = self.B
        self.st.check("BatchDrafter.draft")
        ext = torch.cat([self.last.view(B, 1), res.tokens], 1)   # ext[b, i + 1] = emitted token i
        n = res.num_accepted.clamp_min(0).long().view(B, 1)
        self.prev.copy_(ext.gather(1, n).view(B))                # emitted token n-1 (old last when n = 0)
        self.last.copy_(ext.gather(1, n + 1).view(B))             # the final token
        self.base.add_(res.num_accepted.clamp_min(0) + 1)
        self.base_host = [b + e for b, e in zip(self.base_host, n_emitted)]
        self.cache.append_batch(self.seq_ids, list(n_emitted))
        self._upload_tables()
