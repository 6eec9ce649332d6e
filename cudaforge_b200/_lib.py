"""ctypes binding of the cudaforge_b200 C ABI (include/cf_api.h).

The shared library is built in-tree (cudaforge_b200/csrc/libcudaforge_b200.so)
and loaded once.  There is no fallback: if the library is missing or a call
returns a non-zero status, a RuntimeError / ValueError is raised.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_PATH = os.path.join(CSRC, "libcudaforge_b200.so")

CF_OK, CF_EINVAL, CF_ERANGE, CF_ETIMEOUT, CF_ECUDA, CF_ENOMEM, CF_EUNSUPPORTED = 0, -1, -2, -3, -4, -5, -6
CF_F32, CF_BF16, CF_F16 = 0, 1, 2

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F32 = ctypes.c_float


class CfAcceptArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _I32), ("k", _I32), ("vocab", _I64), ("logits_dtype", _I32),
        ("draft_logits", _P), ("draft_seq_stride", _I64), ("draft_row_stride", _I64),
        ("target_logits", _P), ("target_seq_stride", _I64), ("target_row_stride", _I64),
        ("draft_tokens", _P), ("uniforms", _P), ("temperature", _F32),
        ("eos_token_id", _I32), ("greedy", _I32),
        ("out_tokens", _P), ("out_num_accepted", _P), ("out_eos", _P),
        ("workspace", _P), ("probs_draft", _P), ("probs_target", _P),
    ]


class CfGemmArgs(ctypes.Structure):
    _fields_ = [
        ("m", _I32), ("n", _I32), ("k", _I32), ("act_dtype", _I32),
        ("x", _P), ("ldx", _I64), ("w", _P), ("scales", _P), ("y", _P), ("ldy", _I64),
        ("residual", _P), ("ldr", _I64), ("split_k", _I32), ("workspace", _P),
        ("workspace_bytes", ctypes.c_size_t), ("status", _P), ("timeout_ns", ctypes.c_uint64),
    ]


def build() -> None:
    """Compile libcudaforge_b200.so for sm_100a (nvcc cross-compiles on CPU)."""
    subprocess.run(["make", "-s", "-j8", "-C", CSRC], check=True)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"cudaforge_b200 native library not found at {LIB_PATH}; "
                "run cudaforge_b200._lib.build() (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        L.cf_status_string.restype = ctypes.c_char_p
        L.cf_version.restype = ctypes.c_char_p
        L.cf_accept_workspace_bytes.restype = ctypes.c_size_t
        L.cf_accept_workspace_bytes.argtypes = [_I32, _I32]
        L.cf_accept_sample.argtypes = [ctypes.POINTER(CfAcceptArgs), _P]
        L.cf_gemm_workspace_bytes.restype = ctypes.c_size_t
        L.cf_gemm_workspace_bytes.argtypes = [_I32, _I32, _I32, _I32, _I32]
        for fn in ("cf_w4a16_gemm", "cf_dense_gemm"):
            getattr(L, fn).argtypes = [ctypes.POINTER(CfGemmArgs), _P]
        L.cf_w4a16_repack.argtypes = [_P, _P, _I32, _I32, _P]
        _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != CF_OK:
        msg = lib().cf_status_string(rc).decode()
        if rc in (CF_EINVAL, CF_ERANGE):
            raise ValueError(f"{what}: {msg}")
        raise RuntimeError(f"{what}: {msg}")


def declared_symbols() -> list[str]:
    """Every function name declared in include/*.h (for the export test)."""
    import re
    inc = os.path.join(os.path.dirname(HERE), "include")
    names = []
    for fn in sorted(os.listdir(inc)):
        if fn.endswith(".h"):
            src = open(os.path.join(inc, fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**\s*(cf_[a-z0-9_]+)\s*\(", src, flags=re.M)
    return names
