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
        ("workspace", _P), ("probs_draft", _P), ("probs_target", _P), ("top_p", _F32),
    ]


class CfAcceptTreeArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _I32), ("nodes", _I32), ("vocab", _I64), ("logits_dtype", _I32),
        ("draft_logits", _P), ("draft_seq_stride", _I64), ("draft_row_stride", _I64),
        ("target_logits", _P), ("target_seq_stride", _I64), ("target_row_stride", _I64),
        ("parent", _P), ("tokens", _P), ("uniforms", _P), ("temperature", _F32),
        ("eos_token_id", _I32), ("greedy", _I32),
        ("out_path", _P), ("out_tokens", _P), ("out_num_accepted", _P), ("out_eos", _P),
        ("workspace", _P), ("probs_draft", _P), ("probs_target", _P),
    ]


class CfGemmArgs(ctypes.Structure):
    _fields_ = [
        ("m", _I32), ("n", _I32), ("k", _I32), ("act_dtype", _I32),
        ("x", _P), ("ldx", _I64), ("w", _P), ("scales", _P), ("y", _P), ("ldy", _I64),
        ("residual", _P), ("ldr", _I64), ("split_k", _I32), ("workspace", _P),
        ("workspace_bytes", ctypes.c_size_t), ("status", _P), ("timeout_ns", ctypes.c_uint64),
        ("trace", _P),
    ]


class CfKvLayout(ctypes.Structure):
    _fields_ = [("key_pool", _P), ("val_pool", _P), ("total_blocks", _I64), ("num_layers", _I32),
                ("num_kv_heads", _I32), ("head_dim", _I32), ("block_size", _I32), ("dtype", _I32)]


class CfAttnArgs(ctypes.Structure):
    _fields_ = [
        ("kv", CfKvLayout), ("layer", _I32), ("batch", _I32), ("rows", _I32), ("num_q_heads", _I32),
        ("q", _P), ("q_row_stride", _I64), ("k_new", _P), ("v_new", _P), ("new_kv_all_layers", _I32),
        ("block_tables", _P), ("max_blocks", _I32), ("context_lens", _P), ("max_context", _I32),
        ("tree_mask", _P), ("mask_words", _I32), ("out", _P), ("out_row_stride", _I64), ("scale", _F32),
        ("num_splits", _I32), ("workspace", _P), ("workspace_bytes", ctypes.c_size_t), ("status", _P),
        ("timeout_ns", ctypes.c_uint64), ("trace", _P),
    ]


class CfKvCommitArgs(ctypes.Structure):
    _fields_ = [
        ("kv", CfKvLayout), ("batch", _I32), ("rows", _I32), ("layer_begin", _I32), ("layer_count", _I32),
        ("k_new", _P), ("v_new", _P), ("n_commit", _P), ("n_commit_add", _I32), ("row_index", _P),
        ("start_pos", _P), ("block_tables", _P), ("max_blocks", _I32), ("status", _P),
    ]


def build() -> None:
    """Compile libcudaforge_b200.so for sm_100a (nvcc cross-compiles on CPU)."""
    subprocess.run(["make", "-s", "-j8", "-C", CSRC], check=True)


_lib = None

# Kernel launches issued through this binding (for the bench's gpu_launches claim).
LAUNCHES = [0]


def count(n: int = 1) -> None:
    LAUNCHES[0] += n


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
        L.cf_accept_tree_workspace_bytes.restype = ctypes.c_size_t
        L.cf_accept_tree_workspace_bytes.argtypes = [_I32, _I32, _I64]
        L.cf_accept_tree.argtypes = [ctypes.POINTER(CfAcceptTreeArgs), _P]
        L.cf_topk_rows.argtypes = [_P, _I64, _I32, _I64, _I32, _I32, _P, _P, _P]
        L.cf_gemm_workspace_bytes.restype = ctypes.c_size_t
        L.cf_gemm_workspace_bytes.argtypes = [_I32, _I32, _I32, _I32, _I32]
        for fn in ("cf_w4a16_gemm", "cf_dense_gemm"):
            getattr(L, fn).argtypes = [ctypes.POINTER(CfGemmArgs), _P]
        L.cf_w4a16_repack.argtypes = [_P, _P, _I32, _I32, _P]
        L.cf_attention_workspace_bytes.restype = ctypes.c_size_t
        L.cf_attention_workspace_bytes.argtypes = [ctypes.POINTER(CfAttnArgs)]
        L.cf_verify_attention.argtypes = [ctypes.POINTER(CfAttnArgs), _P]
        L.cf_kv_commit.argtypes = [ctypes.POINTER(CfKvCommitArgs), _P]
        L.cf_embedding.argtypes = [_P, _I32, _P, _I32, _I32, _P, _I32, _P]
        L.cf_rmsnorm.argtypes = [_P, _I64, _P, _P, _I64, _I32, _I32, _F32, _I32, _P]
        L.cf_rope_qkv.argtypes = [_P, _I64, _I32, _I32, _I32, _I32, _P, _F32, _P, _P, _I32, _P]
        L.cf_silu_mul.argtypes = [_P, _I64, _P, _I64, _I32, _I32, _I32, _P]
        L.cf_gemm_splits.argtypes = [_I32, _I32, _I32, _I32, _I32]
        for fn in ("cf_w4a16_gemm_partials", "cf_dense_gemm_partials"):
            getattr(L, fn).argtypes = [ctypes.POINTER(CfGemmArgs), _P]
        L.cf_splitk_rmsnorm.argtypes = [_P, _I32, _I32, _I32, _P, _I64, _P, _I64, _P, _P, _I64, _F32, _I32, _P]
        L.cf_splitk_rope_qkv.argtypes = [_P, _I32, _I32, _P, _I64, _I32, _I32, _I32, _P, _F32, _P, _P, _I32, _P]
        L.cf_splitk_silu_mul.argtypes = [_P, _I32, _I32, _I32, _P, _I64, _I32, _P]
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


class DeviceError(RuntimeError):
    """A kernel recorded a non-zero status word on the device (CF_ETIMEOUT for a
    bounded wait that ran out, CF_ERANGE for an out-of-range page or row id)."""

    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: device status {code} ({lib().cf_status_string(code).decode()})")


class DeviceStatus:
    """The int32 status word the kernels of one step write on the device, with
    a pinned host mirror.  snapshot() enqueues the copy on the current stream;
    after that stream has been synchronised, check() raises DeviceError on any
    non-zero code and clears the word for the next step."""

    def __init__(self, device):
        import torch
        self.dev = torch.zeros(1, dtype=torch.int32, device=device)
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()

    def snapshot(self) -> None:
        self.host.copy_(self.dev, non_blocking=True)

    def check(self, where: str) -> None:
        code = int(self.host[0])
        if code != CF_OK:
            self.dev.zero_()
            self.host.zero_()
            raise DeviceError(code, where)

    def sync_check(self, where: str) -> None:
        import torch
        self.snapshot()
        torch.cuda.current_stream(self.dev.device).synchronize()
        self.check(where)
