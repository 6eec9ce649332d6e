"""GPU: the allocation-free acceptance entry point, cf_accept_sample_noalloc.

It exists for callers that may not allocate device memory (allocator hooks,
runtimes that own all device memory, plugins limited to the buffers they are
handed); it keeps its scratch in a fixed array inside the library.  Called
through the C ABI, its outputs must equal the regular cf_accept_sample's
bit for bit (the tolerance of every acceptance test here: token ids, counts
and EOS flags are integers), on two calls in a row with different inputs,
since the calls share the array.  This file sorts last so a stop-at-first-
failure run has already run everything else."""
import ctypes

import pytest
import torch

from cudaforge_b200 import _lib
from cudaforge_b200.accept import accept_sample

pytestmark = pytest.mark.gpu


def _noalloc(d, t, dt, u, T, eos, greedy):
    B, R, V = t.shape
    K = R - 1
    out_tok = torch.full((B, K + 1), -7, dtype=torch.int32, device="cuda")
    out_n = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    out_e = torch.zeros(B, dtype=torch.uint8, device="cuda")
    a = _lib.CfAcceptArgs(batch=B, k=K, vocab=V, logits_dtype=_lib.CF_BF16,
                          draft_logits=d.data_ptr(), draft_seq_stride=d.stride(0), draft_row_stride=d.stride(1),
                          target_logits=t.data_ptr(), target_seq_stride=t.stride(0), target_row_stride=t.stride(1),
                          draft_tokens=dt.data_ptr(), uniforms=None if greedy else u.data_ptr(), temperature=T,
                          eos_token_id=eos, greedy=int(greedy), out_tokens=out_tok.data_ptr(),
                          out_num_accepted=out_n.data_ptr(), out_eos=out_e.data_ptr(), workspace=None)
    L = _lib.lib()
    L.cf_accept_sample_noalloc.argtypes = [ctypes.POINTER(_lib.CfAcceptArgs), ctypes.c_void_p]
    s = torch.cuda.current_stream().cuda_stream
    rc = L.cf_accept_sample_noalloc(ctypes.byref(a), ctypes.c_void_p(s))
    assert rc == _lib.CF_OK, L.cf_status_string(rc)
    torch.cuda.synchronize()
    return out_tok, out_n, out_e


def _inputs(seed, B, K, V):
    g = torch.Generator().manual_seed(seed)
    d = (torch.randn(B, K + 1, V, generator=g) * 2).to(torch.bfloat16)
    t = (d.float() + 0.5 * torch.randn(B, K + 1, V, generator=g)).to(torch.bfloat16)
    dt = torch.multinomial(torch.softmax(d[:, :K].float().reshape(-1, V), -1), 1, generator=g).reshape(B, K)
    u = torch.rand(B, K + 1, generator=g)
    return d[:, :K].cuda(), t.cuda(), dt.to(torch.int32).cuda(), u.cuda()


def test_noalloc_matches_regular_entry_point_twice():
    for call, (seed, B, K, V, T, greedy) in enumerate([(1, 16, 5, 32000, 1.0, False), (2, 9, 3, 4099, 0.8, False),
                                                         (3, 5, 4, 1000, 1.0, True), (4, 64, 5, 128256, 1.0, False)]):
        d, t, dt, u = _inputs(seed, B, K, V)
        eos = int(dt[0, 0])
        ref = accept_sample(d, t, dt, None if greedy else u, temperature=T, eos_token_id=eos, greedy=greedy)
        tok, n, e = _noalloc(d, t, dt, u, T, eos, greedy)
        assert torch.equal(n, ref.num_accepted), call
        assert torch.equal(e.bool(), ref.eos), call
        for b in range(B):
            k = int(ref.num_accepted[b])
            assert torch.equal(tok[b, : k + 1], ref.tokens[b, : k + 1]), (call, b)


def test_noalloc_rejects_oversized_batch():
    L = _lib.lib()
    L.cf_accept_sample_noalloc.argtypes = [ctypes.POINTER(_lib.CfAcceptArgs), ctypes.c_void_p]
    L.cf_accept_noalloc_max_bytes.restype = ctypes.c_size_t
    cap = L.cf_accept_noalloc_max_bytes()
    K = 5
    B = 1
    while L.cf_accept_workspace_bytes(B, K) <= cap:
        B *= 2
    a = _lib.CfAcceptArgs(batch=B, k=K, vocab=10)
    assert L.cf_accept_sample_noalloc(ctypes.byref(a), None) == _lib.CF_ERANGE
