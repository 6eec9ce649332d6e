"""Paged runner: a model + its paged KV cache, speaking the reference's runner
protocol `.forward(input_ids, kv_cache_handles) -> logits` (the duck type
cudaforge/speculative.py:30-55 expects), but incremental: only the rows not
yet in the cache are computed.

State per sequence: `committed[b]` tokens have K/V in the pool (page tables
grown with PagedKVCache.append_tokens in batch order, so the tables equal the
reference PagedKVCache's for the same call sequence).  A forward over a
[B, S] id batch computes R = max_b(S - committed[b]) rows per sequence; a
sequence with fewer uncommitted rows recomputes some committed tail tokens
(identical K/V; the attention context is shortened accordingly), which keeps
every launch rectangular.  `commit(n)` moves the first n[b] rows' K/V of the
last forward into the pool (cf_kv_commit) and appends the new tokens to the
page tables.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from . import ops
from .model import LlamaModel


class PagedRunner:
    def __init__(self, model: LlamaModel, cache, seq_ids: Sequence[int]):
        self.model = model
        self.cache = cache
        self.seq_ids = list(seq_ids)
        self.committed = [0] * len(self.seq_ids)
        self.registered = False
        self.last = None  # (start[b], R) of the last forward
        from . import _lib
        self.st = _lib.DeviceStatus(model.device)
        self.status = self.st.dev

    @property
    def device(self):
        return self.model.device

    def register(self, prompts: List[List[int]]):
        """Register the sequences' prompts (page tables only; K/V come from a
        forward + commit, i.e. a prefill, or are filled synthetically)."""
        for sid, p in zip(self.seq_ids, prompts):
            self.cache.register_sequence_with_prefix(sid, p)
        self.committed = [len(p) for p in prompts]
        self.registered = True

    def register_empty(self):
        self.register([[] for _ in self.seq_ids])
        self.committed = [0] * len(self.seq_ids)

    @torch.no_grad()
    def forward(self, input_ids, kv_cache_handles=None, tree=None) -> torch.Tensor:
        """input_ids: [B, S] tensor or a list of B token lists (full prefixes,
        possibly ragged).  Returns logits [B, R, V] for the last R tokens of
        every sequence (R = max uncommitted count); callers slice from the
        end, as speculative.py:118, :143 do.
        tree: optional (tokens [B, N+1], depth [B, N+1], mask words [B, N+1, W])
        for tree verification over the committed prefix; input_ids is then
        ignored."""
        B = len(self.seq_ids)
        dev = self.device
        if tree is not None:
            tokens, depth, mask = tree
            R = tokens.shape[1]
            start = list(self.committed)
            pos = torch.tensor(start, dtype=torch.int32, device=dev).view(B, 1) + depth.to(dev, torch.int32)
            rows = tokens.to(device=dev, dtype=torch.int32).contiguous()
        else:
            seqs = input_ids.tolist() if torch.is_tensor(input_ids) else [list(x) for x in input_ids]
            lens = [len(x) for x in seqs]
            R = max(1, max(n - c for n, c in zip(lens, self.committed)))
            start = [n - R for n in lens]
            if min(start) < 0:
                raise ValueError("a sequence is shorter than the rows to compute")
            rows = torch.tensor([x[n - R:] for x, n in zip(seqs, lens)], dtype=torch.int32).to(dev, non_blocking=True)
            pos = (torch.arange(R, dtype=torch.int32).view(1, R)
                   + torch.tensor(start, dtype=torch.int32).view(B, 1)).to(dev, non_blocking=True)
            mask = None
        tables, _ = self.cache.prepare_batch_metadata(self.seq_ids)
        ctx = torch.tensor(start, dtype=torch.int32).to(dev, non_blocking=True)
        logits = self.model.forward_rows(self.cache, rows, pos.reshape(-1).contiguous(), tables, ctx, max(start),
                                         tree_mask=mask, status=self.status)
        self.last = (start, R)
        return logits.view(B, R, -1)

    def commit_upto(self, lengths, row_index: Optional[torch.Tensor] = None) -> None:
        """Make positions < lengths[b] resident: commit the rows of the last
        forward that cover positions [start[b], lengths[b]) (row_index[b] lists
        the source rows for a tree path) and grow the page tables in batch
        order."""
        start, R = self.last
        n = [max(0, min(int(L) - s, R)) for L, s in zip(lengths, start)]
        for b, sid in enumerate(self.seq_ids):
            grow = start[b] + n[b] - self.committed[b]
            if grow > 0:
                self.cache.append_tokens(sid, grow)
                self.committed[b] += grow
        tables, _ = self.cache.prepare_batch_metadata(self.seq_ids)
        bf = self.model.buffers(len(self.seq_ids), R)
        dev = self.device
        ops.kv_commit(self.cache, bf["k_new"], bf["v_new"], torch.tensor(n, dtype=torch.int32).to(dev),
                      torch.tensor(start, dtype=torch.int32).to(dev), tables, row_index=row_index,
                      status=self.status)

    def prefill(self, prompts: List[List[int]], chunk: int = 0) -> None:
        """Register empty tables, run the prompts through the model and commit
        their K/V (one forward; ragged prompts are right-aligned)."""
        self.register_empty()
        self.forward(prompts)
        self.commit_upto([len(p) for p in prompts])
