"""TEST INFRASTRUCTURE ONLY: ctypes front end to the CPU oracle.

`liboracle.so` is this repository's C restatement of the reference acceptance
algorithm (CUDAForge csrc/src/scheduler/speculative.cpp:12-150).
`_ref/libspec_ref.so` is the unmodified reference code compiled from its own
sources.  Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline /
reference arm may import this package; the product path never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_P = ctypes.c_void_p


def build(reference_root=None) -> None:
    """Build liboracle.so and, when a reference checkout is given (argument or
    the CF_REFERENCE_ROOT environment variable), the compiled-reference
    checkers under oracle/_ref."""
    ref = reference_root or os.environ.get("CF_REFERENCE_ROOT", "")
    cmd = ["make", "-s", "-C", HERE]
    if ref and os.path.isdir(ref):
        cmd.append(f"REF={ref}")
    subprocess.run(cmd, check=True)


def _load(path):
    if not os.path.exists(path):
        build()
    return ctypes.CDLL(path)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load(os.path.join(HERE, "liboracle.so"))
    return _lib


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libspec_ref.so"))


def ref():
    global _ref
    if _ref is None:
        _ref = ctypes.CDLL(os.path.join(HERE, "_ref", "libspec_ref.so"))
    return _ref


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_P)


def accept(draft_tokens, draft_probs, target_probs, uniforms, eos):
    """Batched restatement.  draft_tokens [B,K] int32, draft_probs [B,K,V] f32,
    target_probs [B,K+1,V] f32, uniforms [B,K+1] f32.
    Returns (tokens [B,K+1] int32, num_accepted [B] int32, eos [B] uint8)."""
    dt = np.ascontiguousarray(draft_tokens, dtype=np.int32)
    dp = np.ascontiguousarray(draft_probs, dtype=np.float32)
    tp = np.ascontiguousarray(target_probs, dtype=np.float32)
    u = np.ascontiguousarray(uniforms, dtype=np.float32)
    B, K = dt.shape
    V = tp.shape[-1]
    tok = np.full((B, K + 1), -1, np.int32)
    na = np.zeros(B, np.int32)
    ef = np.zeros(B, np.uint8)
    rc = lib().oref_accept_batch(ctypes.c_int32(B), ctypes.c_int32(K), ctypes.c_int64(V),
                                 _ptr(dt), _ptr(dp), _ptr(tp), ctypes.c_int32(eos), _ptr(u),
                                 _ptr(tok), _ptr(na), _ptr(ef))
    assert rc == 0
    return tok, na, ef


def accept_greedy(draft_tokens, target_probs, eos):
    dt = np.ascontiguousarray(draft_tokens, dtype=np.int32)
    tp = np.ascontiguousarray(target_probs, dtype=np.float32)
    B, K = dt.shape
    V = tp.shape[-1]
    tok = np.full((B, K + 1), -1, np.int32)
    na = np.zeros(B, np.int32)
    ef = np.zeros(B, np.uint8)
    lib().oref_accept_greedy_batch(ctypes.c_int32(B), ctypes.c_int32(K), ctypes.c_int64(V),
                                   _ptr(dt), _ptr(tp), ctypes.c_int32(eos),
                                   _ptr(tok), _ptr(na), _ptr(ef))
    return tok, na, ef


def accept_tree(parent, tokens, draft_probs, target_probs, uniforms, eos, greedy=False):
    """Tree restatement for one sequence.  parent/tokens [N+1] (node 0 = root),
    draft_probs / target_probs [N+1, V], uniforms [N+1].  Returns
    (path [na+1], emitted tokens [na+1], na, eos)."""
    par = np.ascontiguousarray(parent, dtype=np.int32)
    tk = np.ascontiguousarray(tokens, dtype=np.int32)
    tp = np.ascontiguousarray(target_probs, dtype=np.float32)
    N = par.shape[0] - 1
    V = tp.shape[-1]
    path = np.full(N + 1, -1, np.int32)
    out = np.full(N + 1, -1, np.int32)
    na = np.zeros(1, np.int32)
    ef = np.zeros(1, np.uint8)
    if greedy:
        lib().oref_accept_tree_greedy_one(ctypes.c_int32(N), ctypes.c_int64(V), _ptr(par), _ptr(tk), _ptr(tp),
                                          ctypes.c_int32(eos), _ptr(path), _ptr(out), _ptr(na), _ptr(ef))
    else:
        dp = np.ascontiguousarray(draft_probs, dtype=np.float32)
        u = np.ascontiguousarray(uniforms, dtype=np.float32)
        rc = lib().oref_accept_tree_one(ctypes.c_int32(N), ctypes.c_int64(V), _ptr(par), _ptr(tk), _ptr(dp),
                                        _ptr(tp), ctypes.c_int32(eos), _ptr(u), _ptr(path), _ptr(out),
                                        _ptr(na), _ptr(ef))
        assert rc == 0
    n = int(na[0])
    return path[: n + 1].tolist(), out[: n + 1].tolist(), n, int(ef[0])


def softmax_rows(x: np.ndarray, T: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    V = x.shape[-1]
    flat_x = x.reshape(-1, V)
    flat_o = out.reshape(-1, V)
    for i in range(flat_x.shape[0]):
        lib().oref_softmax_row(_ptr(flat_x[i]), ctypes.c_int64(V), ctypes.c_float(T), _ptr(flat_o[i]))
    return out


# ---- the unmodified reference (compiled) --------------------------------

def ref_uniforms(seed: int, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    ref().ref_uniforms(ctypes.c_uint64(seed), ctypes.c_int32(n), _ptr(out))
    return out


def ref_verify(seed, draft_tokens, draft_probs, target_probs, eos):
    """One sequence through SpeculativeEngine(rng_seed=seed).verify_candidates."""
    dt = np.ascontiguousarray(draft_tokens, dtype=np.int32)
    dp = np.ascontiguousarray(draft_probs, dtype=np.float32)
    tp = np.ascontiguousarray(target_probs, dtype=np.float32)
    K = dt.shape[0]
    V = tp.shape[-1]
    tok = np.full(K + 1, -1, np.int32)
    na = np.zeros(1, np.int32)
    ef = np.zeros(1, np.uint8)
    rc = ref().ref_verify(ctypes.c_uint64(seed), ctypes.c_int32(K), ctypes.c_int64(V),
                          _ptr(dt), _ptr(dp), _ptr(tp), ctypes.c_int32(eos),
                          _ptr(tok), _ptr(na), _ptr(ef))
    if rc != 0:
        raise ValueError("reference verify_candidates raised")
    return tok, int(na[0]), int(ef[0])


def ref_verify_stream(seed, draft_tokens, draft_probs, target_probs, eos):
    """B consecutive verify_candidates calls on one reference engine seeded
    with `seed` (its random stream carries over).  draft_tokens [B,K],
    draft_probs [B,K,V], target_probs [B,K+1,V].  Returns (tokens [B,K+1],
    num_accepted [B], eos [B])."""
    dt = np.ascontiguousarray(draft_tokens, dtype=np.int32)
    dp = np.ascontiguousarray(draft_probs, dtype=np.float32)
    tp = np.ascontiguousarray(target_probs, dtype=np.float32)
    B, K = dt.shape
    V = tp.shape[-1]
    tok = np.full((B, K + 1), -1, np.int32)
    na = np.zeros(B, np.int32)
    ef = np.zeros(B, np.uint8)
    rc = ref().ref_verify_stream(ctypes.c_uint64(seed), ctypes.c_int32(B), ctypes.c_int32(K), ctypes.c_int64(V),
                                 _ptr(dt), _ptr(dp), _ptr(tp), ctypes.c_int32(eos), _ptr(tok), _ptr(na), _ptr(ef))
    if rc != 0:
        raise ValueError("reference verify_candidates raised")
    return tok, na, ef


def ref_verify_greedy(draft_tokens, target_probs, eos):
    dt = np.ascontiguousarray(draft_tokens, dtype=np.int32)
    tp = np.ascontiguousarray(target_probs, dtype=np.float32)
    K = dt.shape[0]
    V = tp.shape[-1]
    tok = np.full(K + 1, -1, np.int32)
    na = np.zeros(1, np.int32)
    ef = np.zeros(1, np.uint8)
    ref().ref_verify_greedy(ctypes.c_int32(K), ctypes.c_int64(V), _ptr(dt), _ptr(tp),
                            ctypes.c_int32(eos), _ptr(tok), _ptr(na), _ptr(ef))
    return tok, int(na[0]), int(ef[0])


# ---- the unmodified reference PagedKVCache (compiled with a host-memory runtime) ----

class RefKV:
    """ctypes front end to oracle/_ref/libkv_ref.so (reference PagedKVCache)."""

    _L = None

    @classmethod
    def available(cls) -> bool:
        return os.path.exists(os.path.join(HERE, "_ref", "libkv_ref.so"))

    @classmethod
    def lib(cls):
        if cls._L is None:
            L = ctypes.CDLL(os.path.join(HERE, "_ref", "libkv_ref.so"))
            L.refkv_create.restype = _P
            L.refkv_create.argtypes = [ctypes.c_uint32] * 4 + [ctypes.c_uint64, ctypes.c_int, ctypes.c_uint64,
                                                               ctypes.c_uint64]
            for n, a in (("refkv_destroy", [_P]), ("refkv_register", [_P, ctypes.c_uint64, _P, ctypes.c_uint32, _P]),
                         ("refkv_append", [_P, ctypes.c_uint64, ctypes.c_uint32]),
                         ("refkv_unregister", [_P, ctypes.c_uint64]),
                         ("refkv_fork", [_P, ctypes.c_uint64, ctypes.c_uint64]),
                         ("refkv_table", [_P, ctypes.c_uint64, _P, ctypes.c_uint32, _P]),
                         ("refkv_prepare", [_P, _P, ctypes.c_uint32, _P, ctypes.c_uint32, _P, _P]),
                         ("refkv_stats", [_P, _P])):
                getattr(L, n).argtypes = a
            cls._L = L
        return cls._L

    def __init__(self, layers, heads, dim, bs, total, prefix=True, max_batch=256, max_blocks=512):
        self.h = self.lib().refkv_create(layers, heads, dim, bs, total, int(prefix), max_batch, max_blocks)

    def __del__(self):
        if getattr(self, "h", None):
            self.lib().refkv_destroy(self.h)
            self.h = None

    def register(self, seq, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        m = ctypes.c_uint32(0)
        rc = self.lib().refkv_register(self.h, seq, _ptr(t) if t.size else None, t.size, ctypes.byref(m))
        return rc, m.value

    def append(self, seq, n):
        return self.lib().refkv_append(self.h, seq, n)

    def unregister(self, seq):
        return self.lib().refkv_unregister(self.h, seq)

    def fork(self, p, c):
        return self.lib().refkv_fork(self.h, p, c)

    def table(self, seq):
        buf = np.zeros(4096, np.int32)
        n = ctypes.c_uint32(0)
        rc = self.lib().refkv_table(self.h, seq, _ptr(buf), buf.size, ctypes.byref(n))
        return rc, buf[: n.value].tolist()

    def prepare(self, seqs):
        ids = np.ascontiguousarray(seqs, dtype=np.uint64)
        tab = np.zeros(len(seqs) * 4096, np.int32)
        ctx = np.zeros(max(1, len(seqs)), np.int32)
        mb = ctypes.c_uint32(0)
        rc = self.lib().refkv_prepare(self.h, _ptr(ids), len(seqs), _ptr(tab), tab.size, _ptr(ctx), ctypes.byref(mb))
        return rc, tab[: len(seqs) * mb.value].reshape(len(seqs), mb.value), ctx[: len(seqs)]

    def stats(self):
        out = np.zeros(8, np.uint64)
        self.lib().refkv_stats(self.h, _ptr(out))
        return out.tolist()


class RefSched:
    """ctypes front end to oracle/_ref/libsched_ref.so (the reference
    ContinuousBatcher + ModelRunner)."""

    _L = None

    @classmethod
    def available(cls) -> bool:
        return os.path.exists(os.path.join(HERE, "_ref", "libsched_ref.so"))

    @classmethod
    def _lib(cls):
        if cls._L is None:
            L = ctypes.CDLL(os.path.join(HERE, "_ref", "libsched_ref.so"))
            L.rs_create.restype = ctypes.c_void_p
            L.rs_create.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int32]
            L.rs_destroy.argtypes = [ctypes.c_void_p]
            L.rs_add.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                 ctypes.c_int32]
            L.rs_cancel.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
            L.rs_update.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32]
            L.rs_step.restype = ctypes.c_uint64
            L.rs_step.argtypes = [ctypes.c_void_p]
            L.rs_pop.restype = ctypes.c_int32
            L.rs_pop.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32]
            L.rs_pending.restype = ctypes.c_uint64
            L.rs_pending.argtypes = [ctypes.c_void_p]
            L.rs_running.restype = ctypes.c_uint64
            L.rs_running.argtypes = [ctypes.c_void_p]
            cls._L = L
        return cls._L

    def __init__(self, max_seqs, max_tokens, vocab, eos):
        self.h = self._lib().rs_create(max_seqs, max_tokens, vocab, eos)

    def __del__(self):
        if getattr(self, "h", None):
            self._lib().rs_destroy(self.h)
            self.h = None

    def add(self, rid, prompt, max_tokens, priority):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        return bool(self._lib().rs_add(self.h, rid, _ptr(p) if p.size else None, p.size, max_tokens, priority))

    def cancel(self, rid):
        self._lib().rs_cancel(self.h, rid)

    def update(self, ids):
        a = np.ascontiguousarray(ids, dtype=np.uint64)
        self._lib().rs_update(self.h, _ptr(a) if a.size else None, a.size)

    def step(self):
        return int(self._lib().rs_step(self.h))

    def pop(self):
        cap = 4096
        ids = np.zeros(cap, np.uint64)
        tok = np.zeros(cap, np.int32)
        fin = np.zeros(cap, np.uint8)
        n = self._lib().rs_pop(self.h, _ptr(ids), _ptr(tok), _ptr(fin), cap)
        return [(int(ids[i]), int(tok[i]), bool(fin[i])) for i in range(min(n, cap))]

    def counts(self):
        return int(self._lib().rs_pending(self.h)), int(self._lib().rs_running(self.h))
