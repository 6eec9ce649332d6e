"""Speculative decoding engine -- the `cudaforge.speculative` API on B200.

Keeps the reference's public surface (cudaforge/speculative.py:15-217):
`SpeculativeBatchResult`, `SpeculativeEngine(draft_runner, target_runner,
num_speculative_tokens=5, temperature=1.0, top_p=0.9)`, `.step(input_ids,
kv_cache_handles)` and `.get_aggregate_acceptance_rate()`, and adds the
split phases `draft()`, `verify()`, `accept()`.

Acceptance follows the reference's deterministic native verifier
(SpeculativeEngine::verify_candidates, csrc/src/scheduler/speculative.cpp:
50-103) per sequence, on the GPU (cf_accept_sample), with explicit uniforms
so results are reproducible; the Python reference's batch-coupled loop
(speculative.py:155-185) is not reproducible bit-for-bit (global torch RNG)
and is not followed.  With our paged runners, step() also commits the
accepted tokens' K/V to both models' caches.
"""
from __future__ import annotations

import dataclasses
import time
from typing import Any, Dict, List, Optional, Tuple

import torch

from .accept import AcceptResult, accept_sample


@dataclasses.dataclass
class SpeculativeBatchResult:
    """Same fields as the reference (speculative.py:15-24).  accepted_tokens is
    [B, max_emitted] (-1 padded) and num_accepted the batch total of emitted
    tokens; per-sequence detail is in `per_sequence`."""

    accepted_tokens: torch.Tensor
    num_accepted: int
    draft_tokens_generated: int
    acceptance_rate: float
    draft_latency_ms: float
    target_latency_ms: float
    per_sequence: Optional[AcceptResult] = None


class SpeculativeEngine:
    def __init__(self, draft_runner: Any, target_runner: Any, num_speculative_tokens: int = 5,
                 temperature: float = 1.0, top_p: float = 0.9, eos_token_id: int = -1,
                 greedy: bool = False, seed: int = 0, nucleus_bonus: bool = False) -> None:
        """The reference's constructor (speculative.py:28-50) plus: eos_token_id,
        greedy verification, the seed of the device uniforms, and
        nucleus_bonus -- True applies top_p to the bonus draw as the reference
        Python engine does (speculative.py:188-195); False (default) follows
        the reference C++ verifier, which ignores top_p (speculative.h:17),
        so that decisions stay bit-exact with it."""
        self.draft_runner = draft_runner
        self.target_runner = target_runner
        self.k = num_speculative_tokens
        self.temperature = max(temperature, 1e-5)  # speculative.py:50
        self.top_p = top_p
        self.nucleus_bonus = nucleus_bonus
        self.eos_token_id = eos_token_id
        self.greedy = greedy
        self.total_draft_tokens = 0
        self.total_accepted_tokens = 0
        self._gen = None
        self._seed = seed

    def _generator(self, device):
        if self._gen is None:
            self._gen = torch.Generator(device=device).manual_seed(self._seed)
        return self._gen

    def _uniforms(self, B, n, device):
        return torch.rand((B, n), generator=self._generator(device), device=device)

    @staticmethod
    def _as_lists(input_ids):
        return input_ids.tolist() if torch.is_tensor(input_ids) else [list(x) for x in input_ids]

    def _device(self):
        r = self.target_runner
        return getattr(r, "device", torch.device("cuda"))

    @torch.no_grad()
    def draft(self, input_ids, kv_cache_handles: Optional[Dict] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """K autoregressive draft tokens (speculative.py:113-123), sampled on the
        GPU by the acceptance kernel's bonus path (K=0: inverse-CDF draw from
        softmax(row / T)).  input_ids: [B, S] or B token lists.  Returns
        (draft_tokens [B, K] int32, draft_logits [B, K, V])."""
        seqs = self._as_lists(input_ids)
        B = len(seqs)
        dev = self._device()
        toks, logits = [], []
        empty = torch.zeros((B, 0), dtype=torch.int32, device=dev)
        for _ in range(self.k):
            lg = self.draft_runner.forward(seqs, kv_cache_handles)[:, -1:, :]
            u = None if self.greedy else self._uniforms(B, 1, dev)
            r = accept_sample(None, lg, empty, u, temperature=self.temperature, greedy=self.greedy)
            t = r.tokens[:, :1]
            toks.append(t)
            logits.append(lg.clone())
            tl = t.view(-1).tolist()
            seqs = [x + [tl[b]] for b, x in enumerate(seqs)]
        return torch.cat(toks, 1), torch.cat(logits, 1)

    @torch.no_grad()
    def verify(self, input_ids, draft_tokens: torch.Tensor, kv_cache_handles: Optional[Dict] = None) -> torch.Tensor:
        """Target forward over prefix + drafts; returns target logits
        [B, K+1, V] (speculative.py:138-145, without the softmax, which the
        acceptance kernel fuses)."""
        seqs = self._as_lists(input_ids)
        d = draft_tokens.tolist()
        lg = self.target_runner.forward([x + d[b] for b, x in enumerate(seqs)], kv_cache_handles)
        return lg[:, -(draft_tokens.shape[1] + 1):, :]

    @torch.no_grad()
    def accept(self, draft_logits: Optional[torch.Tensor], target_logits: torch.Tensor, draft_tokens: torch.Tensor,
               uniforms: Optional[torch.Tensor] = None, greedy: Optional[bool] = None, **kw) -> AcceptResult:
        """Per-sequence modified rejection sampling (speculative.cpp:50-150)."""
        greedy = self.greedy if greedy is None else greedy
        B, K = draft_tokens.shape
        if not greedy and uniforms is None:
            uniforms = self._uniforms(B, K + 1, target_logits.device)
        if self.nucleus_bonus and "top_p" not in kw:
            kw["top_p"] = self.top_p
        return accept_sample(draft_logits, target_logits, draft_tokens, uniforms, temperature=self.temperature,
                             eos_token_id=self.eos_token_id, greedy=greedy, **kw)

    @torch.no_grad()
    def step(self, input_ids, kv_cache_handles: Optional[Dict] = None) -> SpeculativeBatchResult:
        """One draft -> verify -> accept round.  input_ids: [B, S] or B token
        lists (per-sequence acceptance makes lengths ragged after a step).
        Runners with `commit_upto` (PagedRunner) get the accepted tokens' K/V
        committed: positions < len(prefix) - 1 + num_accepted + 1."""
        dev = self._device()
        seqs = self._as_lists(input_ids)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        draft_tokens, draft_logits = self.draft(seqs, kv_cache_handles)
        torch.cuda.synchronize(dev)
        t1 = time.perf_counter()
        target_logits = self.verify(seqs, draft_tokens, kv_cache_handles)
        res = self.accept(draft_logits, target_logits, draft_tokens)
        n_host = (res.num_accepted.clamp_min(0) + 1).tolist()
        upto = [len(x) - 1 + n for x, n in zip(seqs, n_host)]
        for runner in (self.target_runner, self.draft_runner):
            if hasattr(runner, "commit_upto"):
                runner.commit_upto(upto)
        torch.cuda.synchronize(dev)
        t2 = time.perf_counter()
        for runner in (self.target_runner, self.draft_runner):
            st = getattr(runner, "st", None)
            if st is not None:  # a bounded wait that ran out or a bad page id voids the step
                st.sync_check(type(runner).__name__)
        B, K = draft_tokens.shape
        width = max(n_host)
        tok = res.tokens.cpu()
        acc = torch.full((B, width), -1, dtype=torch.int64)
        for b in range(B):
            acc[b, : n_host[b]] = tok[b, : n_host[b]].to(torch.int64)
        total = int(sum(n_host))
        self.total_draft_tokens += K * B
        self.total_accepted_tokens += total
        return SpeculativeBatchResult(accepted_tokens=acc.to(dev), num_accepted=total, draft_tokens_generated=K,
                                      acceptance_rate=total / max(1, K * B), draft_latency_ms=(t1 - t0) * 1e3,
                                      target_latency_ms=(t2 - t1) * 1e3, per_sequence=res)

    def get_aggregate_acceptance_rate(self) -> float:
        if self.total_draft_tokens == 0:
            return 0.0
        return self.total_accepted_tokens / self.total_draft_tokens
