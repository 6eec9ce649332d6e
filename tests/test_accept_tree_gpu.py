"""GPU parity of tree acceptance (cf_accept_tree).

1. A branching-1 tree must give exactly the chain kernel's results (which are
   themselves pinned to the reference verify_candidates).
2. Random trees: fed the fp32 probabilities the kernel exports, the CPU tree
   restatement oracle.accept_tree must give bit-identical paths, tokens,
   accepted counts and EOS flags (stochastic and greedy)."""
import numpy as np
import pytest
import torch

import oracle
from cudaforge_b200.accept import accept_sample, accept_tree

pytestmark = pytest.mark.gpu


def _random_tree(g, B, N, V, probs_d, mode):
    """parent[i] < i; tokens drawn from the parent's draft row (so some are
    accepted); 'collide' duplicates sibling tokens."""
    par = torch.zeros(B, N + 1, dtype=torch.int32)
    tok = torch.zeros(B, N + 1, dtype=torch.int32)
    for b in range(B):
        for i in range(1, N + 1):
            par[b, i] = int(torch.randint(0, i, (1,), generator=g)) if mode != "chain" else i - 1
            p = int(par[b, i])
            tok[b, i] = int(torch.multinomial(probs_d[b, p], 1, generator=g))
            if mode == "collide" and i > 1 and int(par[b, i - 1]) == p:
                tok[b, i] = tok[b, i - 1]
    return par, tok


def _check_tree(res, par, tok, u, eos, greedy):
    B = par.shape[0]
    tp = res.probs_target.cpu().numpy()
    dp = res.probs_draft.cpu().numpy() if res.probs_draft is not None else None
    for b in range(B):
        path, toks, na, ef = oracle.accept_tree(par[b].numpy(), tok[b].numpy(),
                                                None if dp is None else dp[b], tp[b],
                                                None if u is None else u[b].numpy(), eos, greedy=greedy)
        n = int(res.num_accepted[b])
        assert n == na, (b, n, na)
        assert res.path[b, : n + 1].cpu().tolist() == path, b
        assert res.emitted(b) == toks, b
        assert int(res.eos[b]) == ef, b


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,N,V", [(1, 1, 7), (4, 6, 1000), (3, 20, 32000), (2, 64, 4099)])
@pytest.mark.parametrize("mode", ["random", "collide"])
def test_tree_parity(dtype, B, N, V, mode):
    g = torch.Generator().manual_seed(B * 100 + N * 7 + V)
    d = torch.randn(B, N + 1, V, generator=g) * 2.0
    t = d + 0.5 * torch.randn(B, N + 1, V, generator=g)
    probs_d = torch.softmax(d.to(dtype).float(), -1)
    par, tok = _random_tree(g, B, N, V, probs_d, mode)
    u = torch.rand(B, N + 1, generator=g)
    for eos in (-1, int(tok[0, 1])):
        res = accept_tree(d.to(dtype).cuda(), t.to(dtype).cuda(), par.cuda(), tok.cuda(), u.cuda(),
                          temperature=0.9, eos_token_id=eos, export_probs=True)
        torch.cuda.synchronize()
        _check_tree(res, par, tok, u, eos, greedy=False)
        resg = accept_tree(None, t.to(dtype).cuda(), par.cuda(), tok.cuda(), greedy=True,
                           eos_token_id=eos, export_probs=True)
        torch.cuda.synchronize()
        _check_tree(resg, par, tok, None, eos, greedy=True)


def test_tree_greedy_follows_argmax_children():
    B, N, V = 2, 5, 300
    g = torch.Generator().manual_seed(3)
    t = torch.randn(B, N + 1, V, generator=g) * 4
    am = t.argmax(-1)
    # root has children 1,2 ; node 2 has children 3,4 ; node 4 has child 5
    par = torch.tensor([[0, 0, 0, 2, 2, 4]] * B, dtype=torch.int32)
    tok = torch.zeros(B, N + 1, dtype=torch.int32)
    tok[:, 1] = (am[:, 0] + 1) % V
    tok[:, 2] = am[:, 0]
    tok[:, 3] = am[:, 2]
    tok[:, 4] = am[:, 2]  # sibling duplicate: the first (node 3) wins
    tok[:, 5] = am[:, 4]
    tok[1, 3] = (am[1, 2] + 2) % V  # sequence 1 goes through node 4 instead
    res = accept_tree(None, t.cuda(), par.cuda(), tok.cuda(), greedy=True)
    torch.cuda.synchronize()
    assert res.path[0, :3].cpu().tolist() == [0, 2, 3] and int(res.num_accepted[0]) == 2
    assert res.emitted(0) == [int(am[0, 0]), int(am[0, 2]), int(am[0, 3])]
    assert res.path[1, :4].cpu().tolist() == [0, 2, 4, 5] and int(res.num_accepted[1]) == 3
    assert res.emitted(1) == [int(am[1, 0]), int(am[1, 2]), int(am[1, 4]), int(am[1, 5])]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("mode", ["close", "far", "same"])
def test_branching_one_tree_equals_chain(dtype, mode):
    B, K, V = 6, 5, 32000
    g = torch.Generator().manual_seed(17)
    d = torch.randn(B, K + 1, V, generator=g) * 2.0
    t = d + 0.3 * torch.randn(B, K + 1, V, generator=g) if mode == "close" else (
        torch.randn(B, K + 1, V, generator=g) * 3 if mode == "far" else d.clone())
    dtoks = torch.multinomial(torch.softmax(d[:, :K].reshape(-1, V), -1), 1, generator=g).reshape(B, K)
    u = torch.rand(B, K + 1, generator=g)
    dc, tc = d.to(dtype).cuda(), t.to(dtype).cuda()
    chain = accept_sample(dc[:, :K], tc, dtoks.cuda(), u.cuda(), temperature=0.7)
    par = torch.arange(-1, K, dtype=torch.int32).clamp(min=0).expand(B, K + 1).contiguous()
    tok = torch.cat([torch.zeros(B, 1, dtype=torch.int64), dtoks], 1)
    tree = accept_tree(dc, tc, par.cuda(), tok.cuda(), u.cuda(), temperature=0.7)
    torch.cuda.synchronize()
    assert torch.equal(chain.num_accepted, tree.num_accepted)
    assert torch.equal(chain.eos, tree.eos)
    for b in range(B):
        assert chain.emitted(b) == tree.emitted(b), b
        n = int(tree.num_accepted[b])
        assert tree.path[b, : n + 1].cpu().tolist() == list(range(n + 1))


def test_tree_shape_errors():
    t = torch.randn(2, 4, 10).cuda()
    with pytest.raises(ValueError):
        accept_tree(t, t, torch.zeros(2, 3, dtype=torch.int32), torch.zeros(2, 4, dtype=torch.int32), torch.rand(2, 4))
    with pytest.raises(ValueError):
        accept_tree(None, t, torch.zeros(2, 4, dtype=torch.int32), torch.zeros(2, 4, dtype=torch.int32), torch.rand(2, 4))
