"""CPU: the C-ABI library loads and exports every symbol include/*.h declares."""
import ctypes

from cudaforge_b200 import _lib


def test_library_exports_declared_symbols():
    names = _lib.declared_symbols()
    assert "cf_accept_sample" in names
    L = _lib.lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_status_strings_and_workspace_query():
    L = _lib.lib()
    assert L.cf_status_string(0) == b"CF_OK"
    assert b"EINVAL" in L.cf_status_string(-1)
    # row statistics (8 B per row, padded to 256 B) + per sequence 32 B of state and 32 chunk records of 32 B
    assert L.cf_accept_workspace_bytes(64, 5) == ((64 * 11 * 8 + 255) // 256) * 256 + 64 * (32 + 32 * 32)


def test_accept_rejects_bad_args_on_host():
    L = _lib.lib()
    a = _lib.CfAcceptArgs(batch=2, k=3, vocab=0)
    assert L.cf_accept_sample(ctypes.byref(a), None) == _lib.CF_EINVAL
    assert L.cf_accept_sample(None, None) == _lib.CF_EINVAL
    a = _lib.CfAcceptArgs(batch=0, k=3, vocab=10)
    assert L.cf_accept_sample(ctypes.byref(a), None) == _lib.CF_OK  # empty batch is a no-op


def test_accept_tree_rejects_bad_args_on_host():
    L = _lib.lib()
    assert L.cf_accept_tree_workspace_bytes(4, 65, 1000) == ((4 * 2 * 65 * 8 + 255) // 256) * 256 + 4 * 1000 * 4
    a = _lib.CfAcceptTreeArgs(batch=2, nodes=0, vocab=10)
    assert L.cf_accept_tree(ctypes.byref(a), None) == _lib.CF_EINVAL
    assert L.cf_accept_tree(None, None) == _lib.CF_EINVAL
    a = _lib.CfAcceptTreeArgs(batch=2, nodes=3, vocab=10, temperature=1.0)  # null pointers
    assert L.cf_accept_tree(ctypes.byref(a), None) == _lib.CF_EINVAL
    a = _lib.CfAcceptTreeArgs(batch=0, nodes=3, vocab=10)
    assert L.cf_accept_tree(ctypes.byref(a), None) == _lib.CF_OK


def test_gemm_plan_queries_on_host():
    """Split-K plans of the benchmark shapes (148 SMs): the cfg3 qkv / o / down projections split
    3-4 ways (fused consumers), gate_up and lm_head do not split; the draft's one-row steps split
    up to 16 ways (reduction kernel).  Workspace = splits x M x N fp32 when split."""
    from cudaforge_b200.gemm import MAX_FUSED_SPLITS
    from cudaforge_b200.model import DRAFT_1B, LLAMA_8B
    L = _lib.lib()
    got = [L.cf_gemm_splits(384, n, k, 0, 1) for _, n, k in LLAMA_8B.linear_shapes()]
    assert got == [3, 4, 1, 4]
    assert L.cf_gemm_splits(384, LLAMA_8B.vocab, LLAMA_8B.d_model, 0, 1) == 1
    assert all(1 < s <= MAX_FUSED_SPLITS for s in (got[0], got[1], got[3]))
    for _, n, k in LLAMA_8B.linear_shapes():
        s = L.cf_gemm_splits(384, n, k, 0, 1)
        assert L.cf_gemm_workspace_bytes(384, n, k, 0, 1) == (s * 384 * n * 4 if s > 1 else 0)
    draft = [L.cf_gemm_splits(64, n, k, 0, 1) for _, n, k in DRAFT_1B.linear_shapes()]
    assert draft == [11, 16, 2, 16]
    assert L.cf_gemm_splits(384, 6144, 4096, 1, 1) == 1       # split_k = 1 forces one piece
    assert L.cf_gemm_splits(384, 100, 4096, 0, 1) == 0        # n % 128 != 0: unsupported
