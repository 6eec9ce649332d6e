"""GPU: the CUDA-graph verifier step equals the eager step.

Two BatchVerifiers over the same model and identical caches run the same
drafts and uniforms for several steps (contexts grow across block
boundaries); the graph-captured one must give bit-identical acceptance
results, context lengths, page tables and pool contents."""
import pytest
import torch

from cudaforge_b200 import _lib
from cudaforge_b200.model import LlamaConfig, LlamaModel
from cudaforge_b200.verifier import BatchVerifier

pytestmark = pytest.mark.gpu


def test_graph_step_matches_eager():
    cfg = LlamaConfig(2, 512, 8, 2, 128, 768, 2048)
    m = LlamaModel(cfg, seed=8)
    B, K, P = 5, 4, 29
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, cfg.vocab, (B, P), generator=g)
    vs = []
    for use_graph in (False, True):
        cache = m.make_cache(B * 12, max_batch=B)
        v = BatchVerifier(m, cache, list(range(B)), K, max_blocks_per_seq=10, use_graph=use_graph)
        v.register_context(prompts[:, :-1].tolist(), prompts[:, -1])
        v.fill_synthetic_kv(torch.Generator(device="cuda").manual_seed(2))
        vs.append(v)
    gd = torch.Generator(device="cuda").manual_seed(3)
    dlog = torch.randn(B, K, cfg.vocab, generator=gd, device="cuda").to(cfg.dtype)
    for step in range(6):
        dtok = torch.randint(0, cfg.vocab, (B, K), generator=gd, device="cuda", dtype=torch.int32)
        # make some drafts acceptable: copy the target's own greedy choice is not available here, so
        # use low temperature-free randomness; acceptance counts still vary across sequences
        u = torch.rand(B, K + 1, generator=gd, device="cuda") * 0.05
        outs = []
        for v in vs:
            l0 = _lib.LAUNCHES[0]
            r = v.step(dtok, dlog, u)
            torch.cuda.synchronize()
            outs.append((r.num_accepted.cpu().clone(), r.tokens.cpu().clone(), list(v.ctx_host),
                         v.tables().cpu().clone(), v.ctx.cpu().clone(), _lib.LAUNCHES[0] - l0))
        a, b = outs
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]), step
        assert a[2] == b[2] and torch.equal(a[3], b[3]) and torch.equal(a[4], b[4]), step
        assert a[5] == b[5] > 0  # the graph replay reports the same kernel count
    assert vs[1].graphs is not None
    for pa, pb in ((vs[0].cache.key_pool, vs[1].cache.key_pool), (vs[0].cache.value_pool, vs[1].cache.value_pool)):
        assert torch.equal(pa, pb)


def test_graph_workspaces_outlive_later_captures():
    """Each captured graph holds every cached workspace it addresses: after the
    verifier captures, and then a drafter captures (and may grow the shared
    workspace caches), the verifier's graph still replays correctly and every
    buffer present in the caches right after each capture is held by that
    graph's owner."""
    from cudaforge_b200 import gemm as _gemm
    from cudaforge_b200 import ops
    from cudaforge_b200.drafter import BatchDrafter

    cfg = LlamaConfig(2, 512, 8, 2, 128, 768, 2048)
    m = LlamaModel(cfg, seed=8)
    B, K, P = 5, 4, 200
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, cfg.vocab, (B, P), generator=g)
    cache = m.make_cache(B * 40, max_batch=B)
    v = BatchVerifier(m, cache, list(range(B)), K, max_blocks_per_seq=30, use_graph=True)
    v.register_context(prompts[:, :-1].tolist(), prompts[:, -1])
    v.fill_synthetic_kv(torch.Generator(device="cuda").manual_seed(2))
    gd = torch.Generator(device="cuda").manual_seed(3)
    dlog = torch.randn(B, K, cfg.vocab, generator=gd, device="cuda").to(cfg.dtype)
    dtok = torch.randint(0, cfg.vocab, (B, K), generator=gd, device="cuda", dtype=torch.int32)
    u = torch.rand(B, K + 1, generator=gd, device="cuda")
    v.step(dtok, dlog, u)
    v.step(dtok, dlog, u)  # capture + replay
    assert v.graphs is not None

    def held(keep):
        ids = {id(b) for d in keep for b in d.values()}
        return all(id(b) in ids for b in list(ops._Ws.bufs.values()) + list(_gemm._Ws.bufs.values()))

    assert held(v._keep)
    dcache = m.make_cache(B * 40, max_batch=B)
    dr = BatchDrafter(m, dcache, list(range(B)), K, max_blocks_per_seq=30, use_graph=True)
    dr.register_context(prompts[:, :-1].tolist(), prompts[:, -1])
    dr.draft(u[:, :K].contiguous())
    dr.draft(u[:, :K].contiguous())  # the drafter captures its graph
    assert dr.graph is not None and held(dr._keep)
    # the verifier's graph replays after the drafter's capture, still bit-identical to eager
    ve = BatchVerifier(m, m.make_cache(B * 40, max_batch=B), list(range(B)), K, max_blocks_per_seq=30)
    ve.register_context(prompts[:, :-1].tolist(), prompts[:, -1])
    ve.fill_synthetic_kv(torch.Generator(device="cuda").manual_seed(2))
    ve.step(dtok, dlog, u)
    ve.step(dtok, dlog, u)
    a = v.step(dtok, dlog, u)
    b = ve.step(dtok, dlog, u)
    torch.cuda.synchronize()
    assert torch.equal(a.num_accepted, b.num_accepted) and torch.equal(a.tokens, b.tokens)
    v.check_status()


def test_gemm_graph_replays_after_smaller_plan():
    """A captured GEMM (large token slice, large dynamic shared memory) must
    still replay after an eager GEMM with a smaller plan ran on the same
    kernel function (the per-function shared-memory limit is never lowered)."""
    from cudaforge_b200.gemm import w4a16_gemm
    g = torch.Generator(device="cuda").manual_seed(4)
    N, K = 1024, 1024
    wq = torch.randint(-2**31, 2**31 - 1, (K // 8, N), generator=g, device="cuda", dtype=torch.int32)
    sc = (torch.rand(K // 128, N, generator=g, device="cuda") * 0.002).half()
    xb = torch.randn(384, K, generator=g, device="cuda").to(torch.bfloat16)
    xs = torch.randn(16, K, generator=g, device="cuda").to(torch.bfloat16)
    yb = torch.empty(384, N, dtype=torch.bfloat16, device="cuda")
    w4a16_gemm(xb, wq, sc, out=yb)
    ref = yb.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        w4a16_gemm(xb, wq, sc, out=yb)
    yb.zero_()
    w4a16_gemm(xs, wq, sc)  # smaller plan, same kernel function
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(yb, ref)
