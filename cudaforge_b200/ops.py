"""Python front ends of the verify-forward kernels (C ABI, no fallback):
paged verify attention, accepted-KV commit, embedding, RMSNorm, RoPE on the
fused QKV rows, SwiGLU."""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_DT = {torch.bfloat16: _lib.CF_BF16, torch.float16: _lib.CF_F16}


def _s(stream, dev):
    return ctypes.c_void_p((stream or torch.cuda.current_stream(dev)).cuda_stream)


def _ptr(t: Optional[torch.Tensor]):
    return t.data_ptr() if t is not None else None


def kv_layout(cache) -> _lib.CfKvLayout:
    c = cache.get_config()
    return _lib.CfKvLayout(key_pool=cache.key_pool.data_ptr(), val_pool=cache.value_pool.data_ptr(),
                           total_blocks=c.total_gpu_blocks, num_layers=c.num_layers, num_kv_heads=c.num_kv_heads,
                           head_dim=c.head_dim, block_size=c.block_size, dtype=_DT[cache.dtype])


class _Ws:
    """Cached workspaces per (purpose, device, stream): work on different
    streams may run concurrently."""
    bufs: dict = {}

    @classmethod
    def get(cls, key, dev, nbytes, stream=None):
        k = (key, dev, (stream or torch.cuda.current_stream(dev)).cuda_stream)
        b = cls.bufs.get(k)
        if b is None or b.numel() < nbytes:
            b = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8, device=dev)
            cls.bufs[k] = b
        return b


def verify_attention(cache, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                     block_tables: torch.Tensor, context_lens: torch.Tensor, max_context: int, *,
                     rows: int, num_q_heads: int, out: Optional[torch.Tensor] = None,
                     tree_mask: Optional[torch.Tensor] = None, num_splits: int = 0, status=None,
                     new_kv_all_layers: bool = False, stream=None, trace=None, timeout_ns: int = 0) -> torch.Tensor:
    """q [B*R, Hq*D] (row pitch q.stride(0)); k_new/v_new [B, R, Hkv, D] (or
    [L, B, R, Hkv, D] with new_kv_all_layers); block_tables [B, max_blocks]
    int32; context_lens [B] int32; tree_mask [B, R, W] int64 bit rows.  timeout_ns bounds
    every wait of the kernel (0 = the library default, 2 s); a wait that runs out
    records CF_ETIMEOUT in `status` and the output is then undefined."""
    B = context_lens.shape[0]
    if out is None:
        out = torch.empty_like(q)
    a = _lib.CfAttnArgs(kv=kv_layout(cache), layer=layer, batch=B, rows=rows, num_q_heads=num_q_heads,
                        q=q.data_ptr(), q_row_stride=q.stride(0), k_new=k_new.data_ptr(), v_new=v_new.data_ptr(),
                        new_kv_all_layers=int(new_kv_all_layers), block_tables=block_tables.data_ptr(),
                        max_blocks=block_tables.shape[1], context_lens=context_lens.data_ptr(),
                        max_context=int(max_context), tree_mask=_ptr(tree_mask),
                        mask_words=tree_mask.shape[-1] if tree_mask is not None else 0,
                        out=out.data_ptr(), out_row_stride=out.stride(0), scale=0.0, num_splits=num_splits,
                        status=_ptr(status), timeout_ns=timeout_ns, trace=_ptr(trace))
    L = _lib.lib()
    need = L.cf_attention_workspace_bytes(ctypes.byref(a))
    if need:
        ws = _Ws.get("attn", q.device, need, stream)
        a.workspace, a.workspace_bytes = ws.data_ptr(), need
    _lib.check(L.cf_verify_attention(ctypes.byref(a), _s(stream, q.device)), "cf_verify_attention")
    _lib.count(2 if need else 1)
    return out


def kv_commit(cache, k_new: torch.Tensor, v_new: torch.Tensor, n_commit: torch.Tensor, start_pos: torch.Tensor,
              block_tables: torch.Tensor, *, n_commit_add: int = 0, row_index: Optional[torch.Tensor] = None,
              layer_begin: int = 0, layer_count: Optional[int] = None, status=None, stream=None) -> None:
    """Copy committed scratch rows ([L, B, R, Hkv, D]) into the paged pools."""
    L_, B, R = k_new.shape[0], k_new.shape[1], k_new.shape[2]
    a = _lib.CfKvCommitArgs(kv=kv_layout(cache), batch=B, rows=R, layer_begin=layer_begin,
                            layer_count=L_ - layer_begin if layer_count is None else layer_count,
                            k_new=k_new.data_ptr(), v_new=v_new.data_ptr(), n_commit=n_commit.data_ptr(),
                            n_commit_add=n_commit_add, row_index=_ptr(row_index), start_pos=start_pos.data_ptr(),
                            block_tables=block_tables.data_ptr(), max_blocks=block_tables.shape[1],
                            status=_ptr(status))
    _lib.check(_lib.lib().cf_kv_commit(ctypes.byref(a), _s(stream, k_new.device)), "cf_kv_commit")
    _lib.count()


def embedding(ids: torch.Tensor, table: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None):
    m = ids.numel()
    if out is None:
        out = torch.empty((m, table.shape[1]), dtype=table.dtype, device=table.device)
    _lib.check(_lib.lib().cf_embedding(ids.data_ptr(), m, table.data_ptr(), table.shape[0], table.shape[1],
                                       out.data_ptr(), _DT[table.dtype], _s(stream, table.device)), "cf_embedding")
    _lib.count()
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, out: Optional[torch.Tensor] = None, stream=None):
    if out is None:
        out = torch.empty_like(x)
    _lib.check(_lib.lib().cf_rmsnorm(x.data_ptr(), x.stride(0), w.data_ptr(), out.data_ptr(), out.stride(0),
                                     x.shape[0], x.shape[1], eps, _DT[x.dtype], _s(stream, x.device)), "cf_rmsnorm")
    _lib.count()
    return out


def rope_qkv(qkv: torch.Tensor, pos: torch.Tensor, num_q_heads: int, num_kv_heads: int, head_dim: int,
             k_new: torch.Tensor, v_new: torch.Tensor, base: float = 10000.0, stream=None) -> None:
    _lib.check(_lib.lib().cf_rope_qkv(qkv.data_ptr(), qkv.stride(0), qkv.shape[0], num_q_heads, num_kv_heads,
                                      head_dim, pos.data_ptr(), base, k_new.data_ptr(), v_new.data_ptr(),
                                      _DT[qkv.dtype], _s(stream, qkv.device)), "cf_rope_qkv")
    _lib.count()


def silu_mul(gu: torch.Tensor, ffn: int, out: Optional[torch.Tensor] = None, stream=None):
    if out is None:
        out = torch.empty((gu.shape[0], ffn), dtype=gu.dtype, device=gu.device)
    _lib.check(_lib.lib().cf_silu_mul(gu.data_ptr(), gu.stride(0), out.data_ptr(), out.stride(0), gu.shape[0], ffn,
                                      _DT[gu.dtype], _s(stream, gu.device)), "cf_silu_mul")
    _lib.count()
    return out


# ---- split-K consumers: `part` = (partials [S, M, N] fp32 view, S) from gemm.*_partials ----
def splitk_rmsnorm(part, w: torch.Tensor, y: torch.Tensor, out: torch.Tensor, residual: Optional[torch.Tensor] = None,
                   eps: float = 1e-6, stream=None):
    """y = reduce(partials) (+ residual), out = rmsnorm(y) * w (bit-identical to
    the split-K reduction followed by rmsnorm)."""
    p, S = part
    M, N = y.shape
    _lib.check(_lib.lib().cf_splitk_rmsnorm(p.data_ptr(), S, M, N, _ptr(residual),
                                            residual.stride(0) if residual is not None else 0, y.data_ptr(),
                                            y.stride(0), w.data_ptr(), out.data_ptr(), out.stride(0), eps,
                                            _DT[y.dtype], _s(stream, y.device)), "cf_splitk_rmsnorm")
    _lib.count()
    return out


def splitk_rope_qkv(part, qkv: torch.Tensor, pos: torch.Tensor, num_q_heads: int, num_kv_heads: int, head_dim: int,
                    k_new: torch.Tensor, v_new: torch.Tensor, base: float = 10000.0, stream=None) -> None:
    p, S = part
    _lib.check(_lib.lib().cf_splitk_rope_qkv(p.data_ptr(), S, qkv.shape[0], qkv.data_ptr(), qkv.stride(0),
                                             num_q_heads, num_kv_heads, head_dim, pos.data_ptr(), base,
                                             k_new.data_ptr(), v_new.data_ptr(), _DT[qkv.dtype],
                                             _s(stream, qkv.device)), "cf_splitk_rope_qkv")
    _lib.count()


def splitk_silu_mul(part, ffn: int, out: torch.Tensor, stream=None):
    p, S = part
    _lib.check(_lib.lib().cf_splitk_silu_mul(p.data_ptr(), S, out.shape[0], ffn, out.data_ptr(), out.stride(0),
                                             _DT[out.dtype], _s(stream, out.device)), "cf_splitk_silu_mul")
    _lib.count()
    return out
