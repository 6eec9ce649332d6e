"""GPU: row top-k against a stable CPU ranking, and the tree speculative step
end to end (draft tree -> tree verify -> tree accept -> path commit) against
a full fp32 recompute of the target (oracle/llama_ref.forward_full)."""
import pytest
import torch

from cudaforge_b200.model import TINY_DRAFT, TINY_TARGET, LlamaModel
from cudaforge_b200.runner import PagedRunner
from cudaforge_b200.tree import TreeSpeculativeEngine, topk_rows, topk_tree_shape
from oracle import llama_ref

pytestmark = pytest.mark.gpu


def _stable_topk(x: torch.Tensor, k: int):
    order = sorted(range(x.numel()), key=lambda i: (-float(x[i]), i))
    return order[:k]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("V,k", [(7, 4), (1000, 1), (32000, 4), (128256, 8), (4099, 5)])
def test_topk_rows_matches_stable_ranking(dtype, V, k):
    g = torch.Generator().manual_seed(V + k)
    x = (torch.randn(6, V, generator=g) * 3).to(dtype)
    x[1, 10 % V] = x[1].float().max().to(dtype)  # a tie with the row maximum
    x[2] = 0  # all equal: lowest ids first
    got = topk_rows(x.cuda(), k).cpu()
    for r in range(6):
        assert got[r].tolist() == _stable_topk(x[r].float(), k), r


def test_topk_rows_strided_view():
    x = torch.randn(5, 3000).cuda()
    got = topk_rows(x[:, 1:2001], 3).cpu()
    for r in range(5):
        assert got[r].tolist() == _stable_topk(x[r, 1:2001].cpu(), 3)


@pytest.mark.parametrize("branching", [(4, 4, 4), (2, 2), (1, 1, 1)])
def test_greedy_tree_step_matches_target_argmax(branching):
    tgt = LlamaModel(TINY_TARGET, seed=0)
    drf = LlamaModel(TINY_DRAFT, seed=1)
    B, S0 = 3, 20
    ids = list(range(B))
    tr = PagedRunner(tgt, tgt.make_cache(64), ids)
    dr = PagedRunner(drf, drf.make_cache(64), ids)
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, TINY_TARGET.vocab, (B, S0), generator=g)
    tr.prefill(prompt[:, :-1].tolist())
    dr.prefill(prompt[:, :-1].tolist())
    eng = TreeSpeculativeEngine(dr, tr, topk_tree_shape(branching, 64), greedy=True)
    seqs = prompt.tolist()
    checked = 0
    for _ in range(3):
        res = eng.step(seqs)
        for b in range(B):
            emitted = res.emitted[b]
            assert 1 <= len(emitted) <= len(branching) + 1
            # the accepted path follows parent links and carries the tree tokens
            path = res.accept.path[b, : len(emitted)].tolist()
            assert path[0] == 0
            for j in range(1, len(path)):
                assert eng.shape.parent[path[j]] == path[j - 1]
                assert int(res.tree_tokens[b, path[j]]) == emitted[j - 1]
            ref = llama_ref.forward_full(tgt, torch.tensor([seqs[b] + emitted]).cuda())[0]
            S = len(seqs[b])
            for j, tok in enumerate(emitted):
                row = ref[S - 1 + j]
                top2 = row.topk(2).values
                if (top2[0] - top2[1]).item() > 2e-2 * max(1.0, row.abs().max().item()):
                    assert tok == int(row.argmax()), (b, j)
                    checked += 1
            seqs[b] = seqs[b] + emitted
        assert tr.committed == [len(x) - 1 for x in seqs]
    assert checked > 0


def test_stochastic_tree_step_runs_and_commits():
    tgt = LlamaModel(TINY_TARGET, seed=0)
    drf = LlamaModel(TINY_DRAFT, seed=1)
    B, S0 = 4, 16
    ids = list(range(B))
    tr = PagedRunner(tgt, tgt.make_cache(64), ids)
    dr = PagedRunner(drf, drf.make_cache(64), ids)
    prompt = torch.randint(0, TINY_TARGET.vocab, (B, S0), generator=torch.Generator().manual_seed(6))
    tr.prefill(prompt[:, :-1].tolist())
    dr.prefill(prompt[:, :-1].tolist())
    eng = TreeSpeculativeEngine(dr, tr, temperature=0.8, seed=3)
    seqs = prompt.tolist()
    for _ in range(2):
        res = eng.step(seqs)
        for b in range(B):
            seqs[b] = seqs[b] + res.emitted[b]
        assert tr.committed == [len(x) - 1 for x in seqs]
        assert int(tr.status.item()) == 0
