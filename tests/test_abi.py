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
    assert L.cf_accept_workspace_bytes(64, 5) == 64 * 11 * 8


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
