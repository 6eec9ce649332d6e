"""The names the reference's native module `cudaforge._C` exports
(csrc/bindings/pybind_module.cpp:27-239), backed by this package.

  speculative   SpeculativeConfig, SpeculativeVerificationResult,
                SpeculativeEngine (native: cf_spec_engine_* in
                libcudaforge_b200.so; the reference's per-sequence API with its
                own seeded std::mt19937 stream, plus a batched entry point on
                the GPU acceptance kernel)
  KV cache      KVCacheConfig, KVCacheStats, BlockAllocator, PagedKVCache
                (cudaforge_b200.kv_cache)
  engine        Request, RequestState, BatchStepResult, ContinuousBatcher,
                StreamOutput, TokenStreamBuffer, ModelRunner
                (cudaforge_b200.serving)

`from cudaforge_b200 import _C` is a drop-in for `from cudaforge import _C`.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import numpy as np

from . import _lib
from .kv_cache import BlockAllocator, KVCacheConfig, KVCacheStats, OutOfPagesException, PagedKVCache  # noqa: F401
from .serving import (BatchStepResult, ContinuousBatcher, ModelRunner, Request, RequestState,  # noqa: F401
                      StreamOutput, TokenStreamBuffer)

# py::enum_(...).export_values(): the states are also module attributes
WAITING, RUNNING, FINISHED, PREEMPTED = (RequestState.WAITING, RequestState.RUNNING, RequestState.FINISHED,
                                         RequestState.PREEMPTED)

_P = ctypes.c_void_p


class _CfSpecConfig(ctypes.Structure):
    _fields_ = [("gamma", ctypes.c_int64), ("temperature", ctypes.c_float), ("top_p", ctypes.c_float),
                ("rng_seed", ctypes.c_uint64)]


def _spec_lib():
    L = _lib.lib()
    if not getattr(L, "_spec_ready", False):
        L.cf_spec_engine_create.argtypes = [ctypes.POINTER(_CfSpecConfig), ctypes.POINTER(_P)]
        L.cf_spec_engine_destroy.argtypes = [_P]
        L.cf_spec_engine_set_config.argtypes = [_P, ctypes.POINTER(_CfSpecConfig)]
        L.cf_spec_engine_get_config.argtypes = [_P, ctypes.POINTER(_CfSpecConfig)]
        L.cf_spec_engine_verify.argtypes = [_P, ctypes.c_int32, _P, _P, _P, ctypes.c_int32, _P, _P, ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_int32, _P, _P, _P, _P]
        L.cf_spec_engine_draw_uniforms.argtypes = [_P, ctypes.c_int64, _P]
        L._spec_ready = True
    return L


class SpeculativeConfig:
    """SpeculativeConfig (speculative.h:14-19): gamma=5, temperature=1.0,
    top_p=1.0, rng_seed=42."""

    def __init__(self):
        self.gamma = 5
        self.temperature = 1.0
        self.top_p = 1.0
        self.rng_seed = 42

    def _native(self) -> _CfSpecConfig:
        g, seed = int(self.gamma), int(self.rng_seed)
        if g < 0 or seed < 0 or seed >= 1 << 64:
            raise TypeError("gamma and rng_seed are unsigned integers")
        return _CfSpecConfig(g, float(self.temperature), float(self.top_p), seed)

    @classmethod
    def _from_native(cls, c: _CfSpecConfig) -> "SpeculativeConfig":
        o = cls()
        o.gamma, o.temperature, o.top_p, o.rng_seed = int(c.gamma), float(c.temperature), float(c.top_p), int(c.rng_seed)
        return o

    def __repr__(self):
        return (f"SpeculativeConfig(gamma={self.gamma}, temperature={self.temperature}, top_p={self.top_p}, "
                f"rng_seed={self.rng_seed})")


class SpeculativeVerificationResult:
    """SpeculativeVerificationResult (speculative.h:24-31)."""

    def __init__(self):
        self.accepted_tokens: List[int] = []
        self.final_token = 0
        self.num_accepted = 0
        self.end_of_sequence = False

    def __repr__(self):
        return (f"SpeculativeVerificationResult(accepted_tokens={self.accepted_tokens}, final_token="
                f"{self.final_token}, num_accepted={self.num_accepted}, end_of_sequence={self.end_of_sequence})")


def _rows(rows: Sequence[Sequence[float]]):
    arrs = [np.ascontiguousarray(np.asarray(r, dtype=np.float32).reshape(-1)) for r in rows]
    ptrs = (_P * max(1, len(arrs)))(*[a.ctypes.data for a in arrs])
    lens = (ctypes.c_int64 * max(1, len(arrs)))(*[a.size for a in arrs])
    return arrs, ptrs, lens


class SpeculativeEngine:
    """SpeculativeEngine(config) (speculative.h:36-85): verify_candidates,
    verify_candidates_greedy, set_config, get_config -- the reference's
    semantics and random stream -- plus verify_batch, the batched GPU entry
    point over logits."""

    def __init__(self, config: SpeculativeConfig):
        self._h = _P()
        L = _spec_lib()
        c = config._native()
        _lib.check(L.cf_spec_engine_create(ctypes.byref(c), ctypes.byref(self._h)), "SpeculativeEngine")

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                _spec_lib().cf_spec_engine_destroy(h)
            except Exception:  # interpreter shutdown
                pass
            self._h = None

    def set_config(self, config: SpeculativeConfig) -> None:
        c = config._native()
        _lib.check(_spec_lib().cf_spec_engine_set_config(self._h, ctypes.byref(c)), "set_config")

    def get_config(self) -> SpeculativeConfig:
        c = _CfSpecConfig()
        _lib.check(_spec_lib().cf_spec_engine_get_config(self._h, ctypes.byref(c)), "get_config")
        return SpeculativeConfig._from_native(c)

    def _verify(self, draft_tokens, draft_probs, target_probs, eos_token_id, greedy):
        toks = np.ascontiguousarray(np.asarray(list(draft_tokens), dtype=np.int64))
        if toks.size and (toks.min() < -(1 << 31) or toks.max() >= 1 << 31):
            raise TypeError("draft tokens are int32")
        toks = toks.astype(np.int32)
        K = int(toks.size)
        d_arrs, d_ptrs, d_lens = _rows(draft_probs if draft_probs is not None else [])
        t_arrs, t_ptrs, t_lens = _rows(target_probs)
        out_acc = (ctypes.c_int32 * max(1, K))()
        na, fin, eos = ctypes.c_int32(0), ctypes.c_int32(0), ctypes.c_int32(0)
        rc = _spec_lib().cf_spec_engine_verify(self._h, K, toks.ctypes.data, d_ptrs, d_lens, len(d_arrs), t_ptrs,
                                               t_lens, len(t_arrs), int(eos_token_id), int(greedy), out_acc,
                                               ctypes.byref(na), ctypes.byref(fin), ctypes.byref(eos))
        if rc == _lib.CF_EINVAL:
            raise ValueError("Incompatible draft and target tensor dimensions in SpeculativeEngine.")
        _lib.check(rc, "verify_candidates")
        r = SpeculativeVerificationResult()
        r.num_accepted = int(na.value)
        r.accepted_tokens = [int(out_acc[i]) for i in range(r.num_accepted)]
        r.final_token = int(fin.value)
        r.end_of_sequence = bool(eos.value)
        return r

    def verify_candidates(self, draft_tokens: Sequence[int], draft_probs: Sequence[Sequence[float]],
                          target_probs: Sequence[Sequence[float]], eos_token_id: int) -> SpeculativeVerificationResult:
        """Modified rejection sampling of K draft tokens (speculative.cpp:50-103)."""
        return self._verify(draft_tokens, draft_probs, target_probs, eos_token_id, False)

    def verify_candidates_greedy(self, draft_tokens: Sequence[int], target_probs: Sequence[Sequence[float]],
                                 eos_token_id: int) -> SpeculativeVerificationResult:
        """Greedy verification (speculative.cpp:105-150)."""
        return self._verify(draft_tokens, None, target_probs, eos_token_id, True)

    def draw_uniforms(self, n: int) -> np.ndarray:
        """The next n values of this engine's stream (float32)."""
        out = np.empty(int(n), dtype=np.float32)
        _lib.check(_spec_lib().cf_spec_engine_draw_uniforms(self._h, int(n), out.ctypes.data), "draw_uniforms")
        return out

    def verify_batch(self, draft_logits, target_logits, draft_tokens, eos_token_id: int = -1, greedy: bool = False,
                     uniforms=None, **kw):
        """Batched verification on the GPU (cf_accept_sample): draft_logits
        [B, K, V] and target_logits [B, K+1, V] (CUDA tensors, any of fp32 /
        bf16 / fp16) are softmaxed at the configured temperature inside the
        kernel; draft_tokens [B, K].  Sequence b uses uniforms[b, :] ([B, K+1]
        fp32): test i uses U[b, i] and the final draw U[b, tests done], the
        per-sequence order of verify_candidates.  When `uniforms` is None they
        are the next B*(K+1) values of this engine's stream, sequence-major
        (the whole block is consumed).  Returns cudaforge_b200.accept.AcceptResult
        (device tensors)."""
        import torch

        from .accept import accept_sample
        B, K = int(draft_tokens.shape[0]), int(draft_tokens.shape[1])
        if uniforms is None and not greedy:
            u = self.draw_uniforms(B * (K + 1)).reshape(B, K + 1)
            uniforms = torch.from_numpy(u).pin_memory().to(target_logits.device, non_blocking=True)
        cfg = self.get_config()
        return accept_sample(draft_logits, target_logits, draft_tokens, uniforms, temperature=cfg.temperature,
                             eos_token_id=eos_token_id, greedy=greedy, **kw)


__all__ = ["SpeculativeConfig", "SpeculativeVerificationResult", "SpeculativeEngine", "KVCacheConfig",
           "KVCacheStats", "BlockAllocator", "PagedKVCache", "OutOfPagesException", "Request", "RequestState",
           "BatchStepResult", "ContinuousBatcher", "StreamOutput", "TokenStreamBuffer", "ModelRunner",
           "WAITING", "RUNNING", "FINISHED", "PREEMPTED"]
