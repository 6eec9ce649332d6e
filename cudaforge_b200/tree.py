"""Tree speculative decoding: draft-tree builder, tree verify and tree
acceptance on top of the paged runners.

The reference drafts and verifies chains only (cudaforge/speculative.py:
113-195, speculative.cpp:50-150).  The tree mode here is defined by this
package and reduces to the chain rule for a branching-1 tree:

* shape: a top-k tree, branching (4, 4, 4) truncated breadth-first to 64
  nodes (4 + 16 + 44) by default; node 0 is the root (the last emitted,
  not yet cached token); nodes are numbered breadth-first and the children
  of a node are consecutive, in draft-rank order;
* drafting: the children of a node are the k highest draft logits of the
  node's draft row (cf_topk_rows; ties to the lower token id).  One regular
  draft forward gives the root row, then one tree forward per inner level;
* verification: one target forward over all N+1 nodes with the ancestor
  mask (cf_verify_attention tree mask);
* acceptance: cf_accept_tree (siblings tried in rank order, residual after
  each rejected sibling; greedy = follow the target argmax);
* commit: the accepted root-to-node path's K/V rows go to the pool
  (cf_kv_commit with a row map).
"""
from __future__ import annotations

import ctypes
import dataclasses
import time
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from .accept import _DT, TreeAcceptResult, accept_tree


def topk_rows(logits: torch.Tensor, k: int, out: Optional[torch.Tensor] = None,
              values: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Row-wise top-k indices of a [rows, V] CUDA tensor with unit stride on V
    (descending, ties to the lower index), via cf_topk_rows."""
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be [rows, V] with unit stride on V")
    if logits.device.type != "cuda":
        raise ValueError("topk_rows runs on CUDA tensors only (no CPU fallback)")
    rows, V = logits.shape
    if out is None:
        out = torch.empty((rows, k), dtype=torch.int32, device=logits.device)
    s = stream or torch.cuda.current_stream(logits.device)
    _lib.check(_lib.lib().cf_topk_rows(logits.data_ptr(), logits.stride(0), rows, V, _DT[logits.dtype], k,
                                       out.data_ptr(), values.data_ptr() if values is not None else None,
                                       ctypes.c_void_p(s.cuda_stream)), "cf_topk_rows")
    _lib.count()
    return out


@dataclasses.dataclass(frozen=True)
class TreeShape:
    """Static topology shared by every sequence of a batch."""

    branching: Tuple[int, ...]
    parent: Tuple[int, ...]        # parent[0] = 0 (the root's own entry is unused)
    depth: Tuple[int, ...]
    levels: Tuple[Tuple[int, ...], ...]  # node ids per depth; level 0 = (0,)

    @property
    def nodes(self) -> int:
        return len(self.parent)

    def mask_words(self) -> torch.Tensor:
        """[N+1, W] int64 bit rows: bit j of row r set iff node j is r or an
        ancestor of r (the attention tree mask)."""
        n = self.nodes
        W = (n + 63) // 64
        rows = []
        for r in range(n):
            words = [0] * W
            j = r
            while True:
                words[j // 64] |= 1 << (j % 64)
                if j == 0:
                    break
                j = self.parent[j]
            rows.append([w - (1 << 64) if w >= (1 << 63) else w for w in words])
        return torch.tensor(rows, dtype=torch.int64)


def topk_tree_shape(branching: Sequence[int] = (4, 4, 4), max_nodes: int = 64) -> TreeShape:
    """Breadth-first top-k tree: level d+1 lists, for each level-d node in
    order, its branching[d] children in rank order, until max_nodes non-root
    nodes exist."""
    parent, depth, levels = [0], [0], [(0,)]
    for d, k in enumerate(branching):
        nxt = []
        for p in levels[-1]:
            for _ in range(k):
                if len(parent) - 1 >= max_nodes:
                    break
                nxt.append(len(parent))
                parent.append(p)
                depth.append(d + 1)
        if not nxt:
            break
        levels.append(tuple(nxt))
    return TreeShape(tuple(branching), tuple(parent), tuple(depth), tuple(levels))


@dataclasses.dataclass
class TreeStepResult:
    emitted: List[List[int]]          # per sequence: accepted tokens + the final token
    accept: TreeAcceptResult
    tree_tokens: torch.Tensor         # [B, N+1] int32
    draft_latency_ms: float
    target_latency_ms: float


class TreeSpeculativeEngine:
    """draft tree -> tree verify -> tree accept -> commit, for PagedRunner
    draft and target runners over the same sequences."""

    def __init__(self, draft_runner, target_runner, shape: Optional[TreeShape] = None, temperature: float = 1.0,
                 eos_token_id: int = -1, greedy: bool = False, seed: int = 0):
        self.draft_runner, self.target_runner = draft_runner, target_runner
        self.shape = shape or topk_tree_shape()
        self.temperature = max(temperature, 1e-5)
        self.eos_token_id, self.greedy = eos_token_id, greedy
        dev = target_runner.device
        self.dev = dev
        self._gen = torch.Generator(device=dev).manual_seed(seed)
        self.mask = self.shape.mask_words().to(dev)
        self.depth = torch.tensor(self.shape.depth, dtype=torch.int32, device=dev)
        self.parent = torch.tensor(self.shape.parent, dtype=torch.int32, device=dev)
        self.total_nodes = 0
        self.total_emitted = 0

    def _tree(self, tokens: torch.Tensor, n: int):
        B = tokens.shape[0]
        return (tokens[:, :n], self.depth[:n].view(1, n).expand(B, n),
                self.mask[:n].view(1, n, -1).expand(B, n, self.mask.shape[1]).contiguous())

    @torch.no_grad()
    def draft_tree(self, seqs: List[List[int]]) -> Tuple[torch.Tensor, torch.Tensor]:
        """Returns (tree tokens [B, N+1] int32 with the roots in column 0,
        draft logits [B, N+1, V]; rows of leaves are zero)."""
        sh = self.shape
        B, N1 = len(seqs), sh.nodes
        lg0 = self.draft_runner.forward(seqs)[:, -1, :]  # the root's draft row
        self.draft_runner.commit_upto([len(x) - 1 for x in seqs])
        V = lg0.shape[-1]
        tokens = torch.zeros((B, N1), dtype=torch.int32, device=self.dev)
        tokens[:, 0] = torch.tensor([x[-1] for x in seqs], dtype=torch.int32, device=self.dev)
        dlog = torch.zeros((B, N1, V), dtype=lg0.dtype, device=self.dev)
        dlog[:, 0] = lg0
        for d in range(len(sh.levels) - 1):
            lv, nxt = sh.levels[d], sh.levels[d + 1]
            if d > 0:  # the draft rows of level d come from a tree forward over levels 0..d
                n = lv[-1] + 1
                lg = self.draft_runner.forward(None, tree=self._tree(tokens, n))
                dlog[:, lv[0]: n] = lg[:, lv[0]: n]
            k = sh.branching[d]
            rows = dlog[:, lv[0]: lv[-1] + 1].reshape(B * len(lv), V)
            kids = topk_rows(rows, k).view(B, len(lv) * k)
            tokens[:, nxt[0]: nxt[-1] + 1] = kids[:, : len(nxt)]
        return tokens, dlog

    @torch.no_grad()
    def step(self, seqs: List[List[int]]) -> TreeStepResult:
        torch.cuda.synchronize(self.dev)
        t0 = time.perf_counter()
        tokens, dlog = self.draft_tree(seqs)
        torch.cuda.synchronize(self.dev)
        t1 = time.perf_counter()
        B, N1 = tokens.shape
        tlog = self.target_runner.forward(None, tree=self._tree(tokens, N1))
        u = None if self.greedy else torch.rand((B, N1), generator=self._gen, device=self.dev)
        par = self.parent.view(1, N1).expand(B, N1).contiguous()
        res = accept_tree(None if self.greedy else dlog, tlog, par, tokens, u, temperature=self.temperature,
                          eos_token_id=self.eos_token_id, greedy=self.greedy)
        na = (res.num_accepted.clamp_min(0)).tolist()
        self.target_runner.commit_upto([len(x) + n for x, n in zip(seqs, na)], row_index=res.path)
        torch.cuda.synchronize(self.dev)
        t2 = time.perf_counter()
        emitted = [res.emitted(b) for b in range(B)]
        self.total_nodes += B * (N1 - 1)
        self.total_emitted += sum(len(e) for e in emitted)
        return TreeStepResult(emitted, res, tokens, (t1 - t0) * 1e3, (t2 - t1) * 1e3)


class TreeVerifier:
    """Device-resident tree verify + accept + commit for a fixed batch (the
    tree counterpart of verifier.BatchVerifier, whose page-table and buffer
    handling it reuses): one target forward over the N+1 tree nodes with the
    ancestor mask, cf_accept_tree, then the accepted path's K/V rows committed
    through cf_kv_commit's row map.  The only host round trip is the
    num_accepted read-back the page tables need."""

    def __init__(self, model, cache, seq_ids: Sequence[int], shape: Optional[TreeShape] = None, *,
                 temperature: float = 1.0, greedy: bool = False, eos_token_id: int = -1,
                 max_blocks_per_seq: int = 512):
        from .verifier import BatchVerifier

        self.shape = shape or topk_tree_shape()
        N1 = self.shape.nodes
        self.base = BatchVerifier(model, cache, seq_ids, N1 - 1, temperature=temperature, greedy=greedy,
                                  eos_token_id=eos_token_id, max_blocks_per_seq=max_blocks_per_seq)
        b = self.base
        dev = model.device
        self.depth = torch.tensor(self.shape.depth, dtype=torch.int32, device=dev).view(1, N1)
        self.mask = self.shape.mask_words().to(dev).view(1, N1, -1).expand(b.B, N1, -1).contiguous()
        self.parent = torch.tensor(self.shape.parent, dtype=torch.int32, device=dev).view(1, N1).expand(b.B, N1)
        self.parent = self.parent.contiguous()
        V = model.cfg.vocab
        self.ws = torch.empty(_lib.lib().cf_accept_tree_workspace_bytes(b.B, N1, V) + 256, dtype=torch.uint8,
                              device=dev)

    @property
    def seq_ids(self):
        return self.base.seq_ids

    def register_context(self, prompts, last_tokens) -> None:
        self.base.register_context(prompts, last_tokens)

    def fill_synthetic_kv(self, gen: torch.Generator, std: float = 1.0) -> None:
        self.base.fill_synthetic_kv(gen, std)

    @property
    def ctx_host(self):
        return self.base.ctx_host

    @property
    def n_pinned(self):
        return self.base.n_pinned

    @torch.no_grad()
    def step(self, tree_tokens: torch.Tensor, draft_logits: Optional[torch.Tensor], uniforms: Optional[torch.Tensor],
             timer=None) -> TreeAcceptResult:
        """tree_tokens [B, N+1] int32 (column 0 ignored: the root is the last
        emitted token), draft_logits [B, N+1, V], uniforms [B, N+1] fp32."""
        b = self.base
        B, N1 = b.B, b.R
        b.tokens[:, 1:].copy_(tree_tokens[:, 1:])
        torch.add(b.ctx.view(B, 1), self.depth, out=b.pos.view(B, N1))
        logits = b.model.forward_rows(b.cache, b.tokens, b.pos, b.tables(), b.ctx, max(b.ctx_host),
                                      tree_mask=self.mask, status=b.status, timer=timer)
        res = accept_tree(None if b.greedy else draft_logits, logits.view(B, N1, -1), self.parent, b.tokens, uniforms,
                          temperature=b.temperature, eos_token_id=b.eos, greedy=b.greedy, workspace=self.ws)
        b.n_pinned.copy_(res.num_accepted, non_blocking=True)
        b.st.snapshot()
        torch.cuda.current_stream(b.model.device).synchronize()
        b.st.check("TreeVerifier.step")
        n = [max(0, int(x)) + 1 for x in b.n_pinned.tolist()]
        start = b.ctx.clone()
        b.cache.append_batch(b.seq_ids, n)
        b._upload_tables()
        bf = b.model.buffers(B, N1)
        from . import ops
        ops.kv_commit(b.cache, bf["k_new"], bf["v_new"], res.num_accepted, start, b.tables(), n_commit_add=1,
                      row_index=res.path, status=b.status)
        b.ctx.add_(res.num_accepted.clamp_min(0) + 1)
        b.ctx_host = [c + x for c, x in zip(b.ctx_host, n)]
        idx = res.num_accepted.clamp_min(0).long().view(B, 1)
        b.tokens[:, :1].copy_(res.tokens.gather(1, idx))
        return res

    def check_status(self) -> None:
        self.base.check_status()
