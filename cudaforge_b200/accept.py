"""Batched acceptance sampling through the C ABI (cf_accept_sample).

Semantics follow the reference's native verifier
SpeculativeEngine::verify_candidates / verify_candidates_greedy
(csrc/src/scheduler/speculative.cpp:50-150) applied per sequence, with the
softmax(logits / T) of cudaforge/speculative.py:118, :145 fused in.
"""
from __future__ import annotations

import ctypes
import dataclasses
from typing import Optional

import torch

from . import _lib


@dataclasses.dataclass
class AcceptResult:
    """Per-sequence outcome.  tokens[b, :num_accepted[b]] are the accepted
    drafts and tokens[b, num_accepted[b]] the final (resampled / bonus) token,
    matching SpeculativeVerificationResult{accepted_tokens, final_token,
    num_accepted, end_of_sequence} (speculative.h:24-31)."""

    tokens: torch.Tensor        # [B, K+1] int32
    num_accepted: torch.Tensor  # [B] int32
    eos: torch.Tensor           # [B] bool
    probs_draft: Optional[torch.Tensor] = None   # [B, K, V] f32 (parity export)
    probs_target: Optional[torch.Tensor] = None  # [B, K+1, V] f32 (parity export)

    def emitted(self, b: int) -> list:
        n = int(self.num_accepted[b])
        return self.tokens[b, : n + 1].tolist()


_DT = {torch.float32: _lib.CF_F32, torch.bfloat16: _lib.CF_BF16, torch.float16: _lib.CF_F16}


def _rows_view(x: torch.Tensor, name: str):
    """Accept [B, R, V] with unit stride on V; return (seq_stride, row_stride)."""
    if x.dim() != 3:
        raise ValueError(f"{name} must be [B, rows, V], got {tuple(x.shape)}")
    if x.stride(2) != 1:
        raise ValueError(f"{name} must be contiguous along the vocabulary")
    return x.stride(0), x.stride(1)


def accept_sample(
    draft_logits: Optional[torch.Tensor],
    target_logits: torch.Tensor,
    draft_tokens: torch.Tensor,
    uniforms: Optional[torch.Tensor] = None,
    *,
    temperature: float = 1.0,
    eos_token_id: int = -1,
    greedy: bool = False,
    export_probs: bool = False,
    workspace: Optional[torch.Tensor] = None,
    out: Optional[AcceptResult] = None,
    stream: Optional[torch.cuda.Stream] = None,
    top_p: Optional[float] = None,
) -> AcceptResult:
    """Run the fused acceptance kernel.

    draft_logits [B, K, V] and target_logits [B, K+1, V] (fp32 / bf16 / fp16,
    same dtype, on one CUDA device), draft_tokens [B, K] (int32/int64),
    uniforms [B, K+1] fp32 in [0, 1) (required unless greedy).
    top_p in (0, 1) applies the nucleus filter of the reference Python engine
    (speculative.py:58-84, :188-195) to the bonus draw (all K accepted); None
    (default) follows the reference C++ verifier, which has no top-p.
    Raises ValueError on shape mismatch, as the reference raises
    std::invalid_argument (speculative.cpp:59-62).
    """
    if target_logits.dim() != 3:
        raise ValueError("target_logits must be [B, K+1, V]")
    B, R, V = target_logits.shape
    K = R - 1
    dev = target_logits.device
    if dev.type != "cuda":
        raise ValueError("accept_sample runs on CUDA tensors only (no CPU fallback)")
    if draft_tokens.shape != (B, K):
        raise ValueError(f"Incompatible draft and target tensor dimensions: draft_tokens {tuple(draft_tokens.shape)} vs target {tuple(target_logits.shape)}")
    if greedy and draft_logits is None:
        pass  # greedy verification reads only the target (speculative.cpp:105-150)
    elif K > 0:
        if draft_logits is None or draft_logits.shape != (B, K, V):
            raise ValueError("Incompatible draft and target tensor dimensions in SpeculativeEngine.")
        if draft_logits.dtype != target_logits.dtype or draft_logits.device != dev:
            raise ValueError("draft and target logits must share dtype and device")
    if target_logits.dtype not in _DT:
        raise ValueError(f"unsupported logits dtype {target_logits.dtype}")
    if not greedy:
        if uniforms is None or uniforms.shape != (B, K + 1):
            raise ValueError("uniforms [B, K+1] required for stochastic acceptance")
        uniforms = uniforms.to(device=dev, dtype=torch.float32).contiguous()
    dt = draft_tokens.to(device=dev, dtype=torch.int32).contiguous()
    ts, tr = _rows_view(target_logits, "target_logits")
    if K > 0 and draft_logits is not None:
        ds, dr = _rows_view(draft_logits, "draft_logits")
    else:
        ds, dr = 0, V
    L = _lib.lib()
    ws_bytes = L.cf_accept_workspace_bytes(B, K)
    if workspace is None or workspace.numel() * workspace.element_size() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    if out is None:
        out = AcceptResult(
            tokens=torch.full((B, K + 1), -1, dtype=torch.int32, device=dev),
            num_accepted=torch.zeros(B, dtype=torch.int32, device=dev),
            eos=torch.zeros(B, dtype=torch.bool, device=dev),
        )
    if export_probs:
        out.probs_draft = torch.empty((B, K, V), dtype=torch.float32, device=dev)
        out.probs_target = torch.empty((B, K + 1, V), dtype=torch.float32, device=dev)
    a = _lib.CfAcceptArgs(
        batch=B, k=K, vocab=V, logits_dtype=_DT[target_logits.dtype],
        draft_logits=draft_logits.data_ptr() if (K > 0 and draft_logits is not None) else None,
        draft_seq_stride=ds, draft_row_stride=dr,
        target_logits=target_logits.data_ptr(), target_seq_stride=ts, target_row_stride=tr,
        draft_tokens=dt.data_ptr() if K > 0 else None,
        uniforms=uniforms.data_ptr() if not greedy else None,
        temperature=float(temperature), eos_token_id=int(eos_token_id), greedy=int(bool(greedy)),
        out_tokens=out.tokens.data_ptr(), out_num_accepted=out.num_accepted.data_ptr(),
        out_eos=out.eos.data_ptr(), workspace=workspace.data_ptr(),
        probs_draft=out.probs_draft.data_ptr() if export_probs else None,
        probs_target=out.probs_target.data_ptr() if export_probs else None,
        top_p=float(top_p) if top_p is not None else 0.0,
    )
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    with torch.cuda.device(dev):
        _lib.check(L.cf_accept_sample(ctypes.byref(a), ctypes.c_void_p(s.cuda_stream)), "cf_accept_sample")
    nucleus = top_p is not None and 0.0 < top_p < 1.0
    # row statistics (+ parity export), then the greedy decision or the five-launch stochastic draw
    _lib.count(1 + int(export_probs) + (1 if greedy else 5 + int(nucleus)))
    return out


@dataclasses.dataclass
class TreeAcceptResult:
    """Per-sequence outcome of tree acceptance: path[b, :num_accepted[b]+1]
    the accepted node ids (path[b, 0] = 0, the root), tokens[b,
    :num_accepted[b]] their tokens and tokens[b, num_accepted[b]] the final
    token."""

    path: torch.Tensor          # [B, N+1] int32
    tokens: torch.Tensor        # [B, N+1] int32
    num_accepted: torch.Tensor  # [B] int32
    eos: torch.Tensor           # [B] bool
    probs_draft: Optional[torch.Tensor] = None   # [B, N+1, V] f32 (parity export)
    probs_target: Optional[torch.Tensor] = None  # [B, N+1, V] f32 (parity export)

    def emitted(self, b: int) -> list:
        n = int(self.num_accepted[b])
        return self.tokens[b, : n + 1].tolist()


def accept_tree(
    draft_logits: Optional[torch.Tensor],
    target_logits: torch.Tensor,
    parent: torch.Tensor,
    tree_tokens: torch.Tensor,
    uniforms: Optional[torch.Tensor] = None,
    *,
    temperature: float = 1.0,
    eos_token_id: int = -1,
    greedy: bool = False,
    export_probs: bool = False,
    workspace: Optional[torch.Tensor] = None,
    stream: Optional[torch.cuda.Stream] = None,
) -> TreeAcceptResult:
    """Tree acceptance (cf_accept_tree).  The reference verifies chains only
    (speculative.cpp:50-150); a tree whose every node has one child gives its
    results exactly.  Node 0 is the root (last emitted token); parent[b, i] < i
    for i > 0; siblings are tried in increasing node index.

    draft_logits / target_logits [B, N+1, V]: row u is the distribution after
    node u (draft: the one node u's children were drawn from).  parent and
    tree_tokens [B, N+1] (entry 0 ignored), uniforms [B, N+1] fp32 (one per
    acceptance test in walk order, then one for the final draw).
    """
    if target_logits.dim() != 3:
        raise ValueError("target_logits must be [B, N+1, V]")
    B, NN, V = target_logits.shape
    dev = target_logits.device
    if dev.type != "cuda":
        raise ValueError("accept_tree runs on CUDA tensors only (no CPU fallback)")
    if parent.shape != (B, NN) or tree_tokens.shape != (B, NN):
        raise ValueError("parent and tree_tokens must be [B, N+1]")
    if target_logits.dtype not in _DT:
        raise ValueError(f"unsupported logits dtype {target_logits.dtype}")
    if not greedy:
        if draft_logits is None or draft_logits.shape != (B, NN, V):
            raise ValueError("draft_logits [B, N+1, V] required for stochastic tree acceptance")
        if draft_logits.dtype != target_logits.dtype or draft_logits.device != dev:
            raise ValueError("draft and target logits must share dtype and device")
        if uniforms is None or uniforms.shape != (B, NN):
            raise ValueError("uniforms [B, N+1] required for stochastic acceptance")
        uniforms = uniforms.to(device=dev, dtype=torch.float32).contiguous()
    par = parent.to(device=dev, dtype=torch.int32).contiguous()
    tk = tree_tokens.to(device=dev, dtype=torch.int32).contiguous()
    ts, tr = _rows_view(target_logits, "target_logits")
    ds, dr = _rows_view(draft_logits, "draft_logits") if draft_logits is not None else (0, V)
    L = _lib.lib()
    ws_bytes = L.cf_accept_tree_workspace_bytes(B, NN, V)
    if workspace is None or workspace.numel() * workspace.element_size() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    out = TreeAcceptResult(
        path=torch.full((B, NN), -1, dtype=torch.int32, device=dev),
        tokens=torch.full((B, NN), -1, dtype=torch.int32, device=dev),
        num_accepted=torch.zeros(B, dtype=torch.int32, device=dev),
        eos=torch.zeros(B, dtype=torch.bool, device=dev),
    )
    if export_probs:
        out.probs_draft = torch.empty((B, NN, V), dtype=torch.float32, device=dev) if draft_logits is not None else None
        out.probs_target = torch.empty((B, NN, V), dtype=torch.float32, device=dev)
    a = _lib.CfAcceptTreeArgs(
        batch=B, nodes=NN, vocab=V, logits_dtype=_DT[target_logits.dtype],
        draft_logits=draft_logits.data_ptr() if draft_logits is not None else None,
        draft_seq_stride=ds, draft_row_stride=dr,
        target_logits=target_logits.data_ptr(), target_seq_stride=ts, target_row_stride=tr,
        parent=par.data_ptr(), tokens=tk.data_ptr(),
        uniforms=uniforms.data_ptr() if not greedy else None,
        temperature=float(temperature), eos_token_id=int(eos_token_id), greedy=int(bool(greedy)),
        out_path=out.path.data_ptr(), out_tokens=out.tokens.data_ptr(),
        out_num_accepted=out.num_accepted.data_ptr(), out_eos=out.eos.data_ptr(),
        workspace=workspace.data_ptr(),
        probs_draft=out.probs_draft.data_ptr() if out.probs_draft is not None else None,
        probs_target=out.probs_target.data_ptr() if out.probs_target is not None else None,
    )
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    with torch.cuda.device(dev):
        _lib.check(L.cf_accept_tree(ctypes.byref(a), ctypes.c_void_p(s.cuda_stream)), "cf_accept_tree")
    _lib.count(3 if export_probs else 2)
    return out
