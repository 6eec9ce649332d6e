"""TEST INFRASTRUCTURE ONLY: torch fp32 restatement of the verify forward.

The reference ships no model forward (its ModelRunner::step is a stub,
csrc/src/engine/model_runner.cpp:106-173), so logits / attention parity is
against this fp32 restatement of the reference kernels' semantics:
  RMSNorm     csrc/kernels/cuda/fused_rmsnorm.cu:53-144 (fp32 math, eps 1e-6)
  RoPE        csrc/include/cudaforge/kernels/rope.cuh:13-31 (half split),
              tests/unit/test_fused_primitives.py:6-21; base 10000
  attention   csrc/kernels/triton/flash_attn_triton.py:7-110 (scale D^-1/2)
  INT4 GEMM   tests/unit/test_int4_dequant.py:41-47 (w = nibble*scale, here
              with zero point 8)
  SwiGLU, GQA and the Llama wiring from the benchmark configuration.
"""
from __future__ import annotations

import math

import torch


def rmsnorm(x, w, eps=1e-6):
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def rope(x, pos, base=10000.0):
    """x [..., D] fp32, pos broadcastable to x[..., 0]."""
    D = x.shape[-1]
    half = D // 2
    i = torch.arange(half, dtype=torch.float32, device=x.device)
    inv = torch.exp2(-(2.0 * i / D) * math.log2(base))
    ang = pos.float().unsqueeze(-1) * inv
    c, s = torch.cos(ang), torch.sin(ang)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


def gather_context(pool, layer, table, ctx, bs=16):
    """pool [blocks, L, Hkv, bs, D] -> [ctx, Hkv, D] fp32 for one sequence."""
    if ctx == 0:
        return pool.new_zeros((0, pool.shape[2], pool.shape[4]), dtype=torch.float32)
    pages = [int(b) for b in table[: (ctx + bs - 1) // bs]]
    kv = torch.stack([pool[p, layer] for p in pages])  # [P, Hkv, bs, D]
    kv = kv.permute(0, 2, 1, 3).reshape(-1, pool.shape[2], pool.shape[4])
    return kv[:ctx].float()


def verify_attention(q, k_pool, v_pool, layer, tables, ctx_lens, k_new, v_new, tree_mask=None, bs=16):
    """q [B, R, Hq, D]; k_new/v_new [B, R, Hkv, D]; tree_mask [B, R, R] bool
    (row r may see new row j) or None for causal.  Returns fp32 [B, R, Hq, D]."""
    B, R, Hq, D = q.shape
    Hkv = k_new.shape[2]
    G = Hq // Hkv
    out = torch.empty((B, R, Hq, D), dtype=torch.float32, device=q.device)
    for b in range(B):
        c = int(ctx_lens[b])
        kc = gather_context(k_pool, layer, tables[b], c, bs)
        vc = gather_context(v_pool, layer, tables[b], c, bs)
        k = torch.cat([kc, k_new[b].float()], 0)  # [c+R, Hkv, D]
        v = torch.cat([vc, v_new[b].float()], 0)
        if tree_mask is None:
            newm = torch.tril(torch.ones(R, R, dtype=torch.bool, device=q.device))
        else:
            newm = tree_mask[b].bool()
        mask = torch.cat([torch.ones(R, c, dtype=torch.bool, device=q.device), newm], 1)  # [R, c+R]
        kk = k.repeat_interleave(G, dim=1)  # [c+R, Hq, D]
        vv = v.repeat_interleave(G, dim=1)
        s = torch.einsum("rhd,thd->hrt", q[b].float(), kk) / math.sqrt(D)
        s = s.masked_fill(~mask.unsqueeze(0), float("-inf"))
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("hrt,thd->rhd", p, vv)
    return out
