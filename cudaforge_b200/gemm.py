"""W4A16 (and dense 16-bit) GEMM through the C ABI (cf_w4a16_gemm / cf_dense_gemm).

The INT4 format is the reference's: [K/8, N] 32-bit words, nibble i of word
(j, n) holding k = 8j + i (tests/unit/test_int4_dequant.py:6-15), fp16 group
scales [K/128, N], zero point 8, i.e. w = (nibble - 8) * scale.  The kernel
consumes a one-time repack of that packing (repack_int4)."""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_DT = {torch.bfloat16: _lib.CF_BF16, torch.float16: _lib.CF_F16}


def pack_int4_reference(q: torch.Tensor) -> torch.Tensor:
    """[K, N] integers in 0..15 -> [K/8, N] int32, nibble i <-> k % 8 == i
    (the packing of the reference's tests/unit/test_int4_dequant.py:6-15)."""
    K, N = q.shape
    assert K % 8 == 0
    q = q.to(torch.int64) & 0xF
    packed = torch.zeros((K // 8, N), dtype=torch.int64, device=q.device)
    for i in range(8):
        packed |= q[i::8, :] << (4 * i)
    return (packed - ((packed >> 31) << 32)).to(torch.int32)  # two's complement view of uint32


def dequant_reference(wq: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 [K, N] = (nibble - 8) * scale, from the reference packing."""
    Kp, N = wq.shape
    w = wq.to(torch.int64) & 0xFFFFFFFF
    q = torch.stack([(w >> (4 * i)) & 0xF for i in range(8)], dim=1).reshape(Kp * 8, N)
    g = scales.float().repeat_interleave(128, dim=0)[: Kp * 8]
    return (q.float() - 8.0) * g


def repack_int4(wq: torch.Tensor, stream=None) -> torch.Tensor:
    """Reference packing -> kernel nibble order (same values)."""
    assert wq.dtype in (torch.int32, torch.uint32) and wq.is_cuda and wq.is_contiguous()
    Kp, N = wq.shape
    out = torch.empty_like(wq)
    s = stream or torch.cuda.current_stream(wq.device)
    _lib.check(_lib.lib().cf_w4a16_repack(ctypes.c_void_p(wq.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                          Kp * 8, N, ctypes.c_void_p(s.cuda_stream)), "cf_w4a16_repack")
    _lib.count()
    return out


MAX_FUSED_SPLITS = 4


class _Ws:
    """Cached split-K workspace per (device, stream), grown on demand: work on
    different streams may run concurrently and must not share partials."""
    bufs: dict = {}

    @classmethod
    def get(cls, dev, nbytes, stream=None):
        key = (dev, (stream or torch.cuda.current_stream(dev)).cuda_stream)
        b = cls.bufs.get(key)
        if b is None or b.numel() < nbytes:
            b = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
            cls.bufs[key] = b
        return b


def _gemm(fn, x, w, scales, n, residual, out, split_k, workspace, status, int4, timeout_ns=0, stream=None,
          trace=None, partials_fn=None):
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be 2-D with unit inner stride")
    M, K = x.shape
    if out is None:
        out = torch.empty((M, n), dtype=x.dtype, device=x.device)
    L = _lib.lib()
    splits = L.cf_gemm_splits(M, n, K, split_k, int(int4))
    # fused consumers add the partials serially per element over fewer threads than the
    # reduction kernel: worth it for a few splits (the verify shapes), not for many
    fused = partials_fn is not None and 1 < splits <= MAX_FUSED_SPLITS
    if fused:
        fn = partials_fn
    need = L.cf_gemm_workspace_bytes(M, n, K, split_k, int(int4))
    if workspace is not None and workspace.dtype != torch.uint8:
        raise ValueError("workspace must be a uint8 (byte) tensor")
    if need and (workspace is None or workspace.numel() < need):
        workspace = _Ws.get(x.device, need, stream)
    a = _lib.CfGemmArgs(m=M, n=n, k=K, act_dtype=_DT[x.dtype], x=x.data_ptr(), ldx=x.stride(0),
                        w=w.data_ptr(), scales=scales.data_ptr() if scales is not None else None,
                        y=out.data_ptr(), ldy=out.stride(0),
                        residual=residual.data_ptr() if residual is not None else None,
                        ldr=residual.stride(0) if residual is not None else 0,
                        split_k=split_k, workspace=workspace.data_ptr() if need else None,
                        workspace_bytes=need, status=status.data_ptr() if status is not None else None,
                        timeout_ns=timeout_ns, trace=trace.data_ptr() if trace is not None else None)
    s = stream or torch.cuda.current_stream(x.device)
    _lib.check(fn(ctypes.byref(a), ctypes.c_void_p(s.cuda_stream)), fn.__name__)
    if fused:
        _lib.count(1)
        part = workspace.view(-1)[: splits * M * n * 4].view(torch.float32).view(splits, M, n)
        return part, splits
    _lib.count(2 if need else 1)
    return out


def w4a16_gemm(x: torch.Tensor, wq_kernel: torch.Tensor, scales: torch.Tensor, *, residual=None, out=None,
               split_k: int = 0, workspace=None, status=None, timeout_ns: int = 0, stream=None,
               trace=None, partials: bool = False):
    """y = x @ deq(W) (+ residual); x bf16 [M, K], wq_kernel from repack_int4, scales fp16 [K/128, N].
    partials=True: when the plan splits K into 2..MAX_FUSED_SPLITS pieces, run only the GEMM
    and return (fp32 partials [splits, M, N] in the workspace, splits) for an ops.splitk_*
    consumer (residual and out untouched); otherwise y as usual.  Without a caller
    workspace the partials live in a per-device buffer shared by every GEMM: they are
    valid only until the next GEMM call on that device and stream is enqueued."""
    n = wq_kernel.shape[1]
    L = _lib.lib()
    return _gemm(L.cf_w4a16_gemm, x, wq_kernel, scales, n, residual, out, split_k, workspace, status,
                 True, timeout_ns, stream, trace, partials_fn=L.cf_w4a16_gemm_partials if partials else None)


def dense_gemm(x: torch.Tensor, w: torch.Tensor, *, residual=None, out=None, split_k: int = 0, workspace=None,
               status=None, stream=None, partials: bool = False):
    """y = x @ w.T (+ residual); x [M, K], w [N, K] (nn.Linear layout), both bf16 or both fp16.
    partials: as w4a16_gemm."""
    if w.dtype != x.dtype or not w.is_contiguous():
        raise ValueError("w must be contiguous and share x's dtype")
    L = _lib.lib()
    return _gemm(L.cf_dense_gemm, x, w, None, w.shape[0], residual, out, split_k, workspace, status,
                 False, 0, stream, partials_fn=L.cf_dense_gemm_partials if partials else None)
