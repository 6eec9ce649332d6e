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


def forward_full(model, tokens, tree_parent=None):
    """fp32 forward of a whole sequence batch tokens [B, S] (positions 0..S-1,
    causal) through the random-init model `model` (cudaforge_b200.model.
    LlamaModel), using exactly dequantised weights.  Returns logits [B, S, V]
    fp32.  This recomputes everything from the token ids; it shares no state
    with the paged cache."""
    from cudaforge_b200.model import linear_weight_fp32

    c = model.cfg
    B, S = tokens.shape
    dev = model.embed.device
    x = model.embed.float()[tokens.long().to(dev)]  # [B, S, d]
    pos = torch.arange(S, device=dev).view(1, S, 1)
    causal = torch.tril(torch.ones(S, S, dtype=torch.bool, device=dev))
    G = c.n_heads // c.n_kv_heads
    for lay in model.layers:
        xn = rmsnorm(x, lay["attn_norm"], c.eps)
        qkv = xn @ linear_weight_fp32(lay["qkv"]).T
        # the kernels round activations to the model dtype between ops; mirror that at op boundaries
        q = qkv[..., : c.n_heads * c.head_dim].view(B, S, c.n_heads, c.head_dim)
        k = qkv[..., c.n_heads * c.head_dim:(c.n_heads + c.n_kv_heads) * c.head_dim].view(B, S, c.n_kv_heads,
                                                                                           c.head_dim)
        v = qkv[..., (c.n_heads + c.n_kv_heads) * c.head_dim:].view(B, S, c.n_kv_heads, c.head_dim)
        q = rope(q, pos, c.rope_base)
        k = rope(k, pos, c.rope_base)
        kk = k.repeat_interleave(G, dim=2)
        vv = v.repeat_interleave(G, dim=2)
        s = torch.einsum("bqhd,bkhd->bhqk", q, kk) / math.sqrt(c.head_dim)
        s = s.masked_fill(~causal, float("-inf"))
        a = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, -1), vv).reshape(B, S, -1)
        x = x + a @ linear_weight_fp32(lay["o"]).T
        xn = rmsnorm(x, lay["ffn_norm"], c.eps)
        gu = xn @ linear_weight_fp32(lay["gate_up"]).T
        act = torch.nn.functional.silu(gu[..., : c.ffn]) * gu[..., c.ffn:]
        x = x + act @ linear_weight_fp32(lay["down"]).T
    x = rmsnorm(x, model.final_norm, c.eps)
    return x @ linear_weight_fp32(model.lm_head).T


def forward_rows(model, key_pool, value_pool, tables, ctx_lens, tokens, tree_mask=None, depth=None, bs=16):
    """fp32 restatement of the incremental verify forward (LlamaModel.forward_rows):
    the R new rows tokens [B, R] of every sequence at positions ctx_lens[b] + r
    (or ctx_lens[b] + depth[r] for a tree) attend to the cached context read
    from the paged pools ([blocks, L, Hkv, bs, D], the kernels' own inputs, so
    any cache contents serve) and to the new rows under a causal or tree mask
    (tree_mask [B, R, R] bool).  Weights are dequantised exactly.  Returns
    logits [B, R, V] fp32."""
    from cudaforge_b200.model import linear_weight_fp32

    c = model.cfg
    B, R = tokens.shape
    dev = model.embed.device
    tokens = tokens.to(dev).long()
    ctx = torch.as_tensor(ctx_lens).to(dev).long()
    off = torch.arange(R, device=dev) if depth is None else torch.as_tensor(depth, device=dev).long()
    pos = ctx.view(B, 1) + off.view(1, R)  # [B, R]
    x = model.embed.float()[tokens]  # [B, R, d]
    tables_cpu = torch.as_tensor(tables).cpu()
    ctx_cpu = ctx.cpu()
    for li, lay in enumerate(model.layers):
        xn = rmsnorm(x, lay["attn_norm"], c.eps)
        qkv = xn @ linear_weight_fp32(lay["qkv"]).T
        q = qkv[..., : c.n_heads * c.head_dim].view(B, R, c.n_heads, c.head_dim)
        k = qkv[..., c.n_heads * c.head_dim:(c.n_heads + c.n_kv_heads) * c.head_dim].view(B, R, c.n_kv_heads,
                                                                                           c.head_dim)
        v = qkv[..., (c.n_heads + c.n_kv_heads) * c.head_dim:].view(B, R, c.n_kv_heads, c.head_dim)
        q = rope(q, pos.view(B, R, 1), c.rope_base)
        k = rope(k, pos.view(B, R, 1), c.rope_base)
        a = verify_attention(q, key_pool, value_pool, li, tables_cpu, ctx_cpu, k, v, tree_mask=tree_mask, bs=bs)
        x = x + a.reshape(B, R, -1) @ linear_weight_fp32(lay["o"]).T
        xn = rmsnorm(x, lay["ffn_norm"], c.eps)
        gu = xn @ linear_weight_fp32(lay["gate_up"]).T
        act = torch.nn.functional.silu(gu[..., : c.ffn]) * gu[..., c.ffn:]
        x = x + act @ linear_weight_fp32(lay["down"]).T
    x = rmsnorm(x, model.final_norm, c.eps)
    return x @ linear_weight_fp32(model.lm_head).T
